"""Edge cases of the GPU path against the oracle: empty input, empty and one-token
sequences in a pack, no landmarks (k = 0), more landmarks than positions, width 1 and
widths beyond the sequence, block-causal blocks that do not divide the sequence, and the
log-sum-exp output."""
import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O

pytestmark = pytest.mark.gpu


def _dev():
    return torch.device("cuda", 0)


@pytest.fixture(scope="module")
def ops():
    from dsalt_b200 import ops as _ops
    return _ops


def _rand(cu, H, Hkv, D, w_hi, seed, dtype=torch.bfloat16, w_lo=1):
    g = torch.Generator().manual_seed(seed)
    T = cu[-1]
    q = torch.randn(T, H, D, generator=g).to(dtype)
    k = torch.randn(T, Hkv, D, generator=g).to(dtype)
    v = torch.randn(T, Hkv, D, generator=g).to(dtype)
    w = torch.randint(w_lo, w_hi + 1, (T,), generator=g, dtype=torch.int32)
    xn = (20 + torch.randn(T, generator=g)).float()
    vn = (1 + 0.2 * torch.randn(T, Hkv, generator=g)).float()
    return q, k, v, w, xn, vn


def _check_attention(ops, q, k, v, w, lmk, cu, lmk_block=0, rows=None):
    H, Hkv = q.shape[1], k.shape[1]
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    out, lse = ops.dsalt_attention(q.to(_dev()), k.to(_dev()), v.to(_dev()), lmk.to(_dev()), None, w.to(_dev()), cu_t,
                                   lmk_block=lmk_block, cu_list=cu, out_dtype=torch.float32, return_lse=True)
    T = cu[-1]
    if T == 0:
        assert out.shape[0] == 0
        return
    rows = np.arange(T) if rows is None else rows
    kr = k.repeat_interleave(H // Hkv, dim=1)
    vr = v.repeat_interleave(H // Hkv, dim=1)
    ref, ref_lse = O.attention_forward(q.float().numpy(), kr.float().numpy(), vr.float().numpy(), w.numpy(),
                                       lmk.numpy(), cu, lmk_block=lmk_block, rows=rows)
    got = out.cpu().numpy()[rows]
    # P is rounded to the input type before P·V (as the reference's tl.dot(p.to(bf16), v)),
    # so each weight carries a relative error up to the type's unit roundoff u and the
    # output an error up to u·Σp|v|/l: the oracle run on |v|. The inputs here are N(0, 1),
    # so that bound is wider than the fixed tolerance used for the model's projections.
    u = 2.0 ** -8 if q.dtype == torch.bfloat16 else 2.0 ** -11
    mag, _ = O.attention_forward(q.float().numpy(), kr.float().numpy(), np.abs(vr.float().numpy()), w.numpy(),
                                 lmk.numpy(), cu, lmk_block=lmk_block, rows=rows)
    err = np.abs(got - ref[rows])
    assert (err <= u * mag[rows] + 1e-4).all(), float((err - u * mag[rows]).max())
    gl = lse.cpu().numpy()[rows]
    rl = ref_lse[rows]
    fin = np.isfinite(rl)
    assert np.array_equal(np.isfinite(gl), fin)
    assert np.abs(gl[fin] - rl[fin]).max() <= 1e-3


def test_empty_input(ops):
    q, k, v, w, xn, vn = _rand([0, 0], 2, 2, 64, 10, 1)
    lmk = torch.full((2, 1, 8), -1, dtype=torch.int32)
    _check_attention(ops, q, k, v, w, lmk, [0, 0])


def test_pack_with_empty_and_one_token_sequences(ops):
    cu = [0, 0, 1, 130, 130, 600]
    H, Hkv, k = 4, 2, 16
    q, k_, v, w, xn, vn = _rand(cu, H, Hkv, 64, 200, 2)
    alpha = torch.tensor([0.2, 0.5, 0.7, 0.9])
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    lmk = ops.select_landmarks(xn.to(_dev()), vn.to(_dev()), w.to(_dev()), alpha.to(_dev()), cu_t, k, H, "global",
                               cu_list=cu)
    ref, *_ = O.select_global(xn.numpy(), vn.numpy(), alpha.numpy(), w.numpy(), cu, k, H)
    np.testing.assert_array_equal(lmk.cpu().numpy(), ref)
    _check_attention(ops, q, k_, v, w, lmk.cpu(), cu)
    lmkb = ops.select_landmarks(xn.to(_dev()), vn.to(_dev()), w.to(_dev()), alpha.to(_dev()), cu_t, k, H,
                                "block_causal", 128, cu_list=cu)
    parts = [O.select_block_causal(xn[cu[i]:cu[i + 1]].numpy(), vn[cu[i]:cu[i + 1]].numpy(), alpha.numpy(),
                                   w[cu[i]:cu[i + 1]].numpy(), cu[i + 1] - cu[i], k, H, 128)
             for i in range(len(cu) - 1)]
    np.testing.assert_array_equal(lmkb.cpu().numpy(), np.concatenate(parts, axis=1))
    _check_attention(ops, q, k_, v, w, lmkb.cpu(), cu, lmk_block=128)


def test_no_landmarks(ops):
    cu = [0, 700]
    q, k, v, w, *_ = _rand(cu, 2, 2, 64, 300, 3)
    _check_attention(ops, q, k, v, w, torch.zeros(2, 1, 0, dtype=torch.int32), cu, rows=np.arange(0, 700, 3))


def test_more_landmarks_than_positions(ops):
    cu = [0, 90]
    H, k = 2, 128
    q, kk, v, w, xn, vn = _rand(cu, H, H, 64, 40, 4)
    alpha = torch.tensor([0.3, 0.8])
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    lmk = ops.select_landmarks(xn.to(_dev()), vn.to(_dev()), w.to(_dev()), alpha.to(_dev()), cu_t, k, H, "global",
                               cu_list=cu)
    ref, *_ = O.select_global(xn.numpy(), vn.numpy(), alpha.numpy(), w.numpy(), cu, k, H)
    np.testing.assert_array_equal(lmk.cpu().numpy(), ref)
    assert (lmk.cpu().numpy() == -1).any()
    _check_attention(ops, q, kk, v, w, lmk.cpu(), cu)


@pytest.mark.parametrize("w_lo,w_hi", [(1, 1), (5000, 5000)])
def test_extreme_widths(ops, w_lo, w_hi):
    """Width 1 (the diagonal only, plus landmarks) and widths beyond the sequence (full
    causal window, no landmark can be used)."""
    cu = [0, 1000]
    H, k = 2, 32
    q, kk, v, w, xn, vn = _rand(cu, H, H, 64, w_hi, 5, w_lo=w_lo)
    alpha = torch.tensor([0.4, 0.6])
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    lmk = ops.select_landmarks(xn.to(_dev()), vn.to(_dev()), w.to(_dev()), alpha.to(_dev()), cu_t, k, H,
                               "block_causal", 256, cu_list=cu)
    ref = O.select_block_causal(xn.numpy(), vn.numpy(), alpha.numpy(), w.numpy(), 1000, k, H, 256)
    np.testing.assert_array_equal(lmk.cpu().numpy(), ref)
    _check_attention(ops, q, kk, v, w, lmk.cpu(), cu, lmk_block=256, rows=np.arange(0, 1000, 5))


def test_fp16_block_causal_ragged_blocks(ops):
    cu = [0, 1300, 1301, 1800]
    H, Hkv, k = 4, 1, 24
    q, kk, v, w, xn, vn = _rand(cu, H, Hkv, 64, 350, 6, dtype=torch.float16)
    alpha = torch.tensor([0.1, 0.5, 0.9, 1.0])
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    lmk = ops.select_landmarks(xn.to(_dev()), vn.to(_dev()), w.to(_dev()), alpha.to(_dev()), cu_t, k, H,
                               "block_causal", 384, cu_list=cu)
    parts = [O.select_block_causal(xn[cu[i]:cu[i + 1]].numpy(), vn[cu[i]:cu[i + 1]].numpy(), alpha.numpy(),
                                   w[cu[i]:cu[i + 1]].numpy(), cu[i + 1] - cu[i], k, H, 384)
             for i in range(len(cu) - 1)]
    np.testing.assert_array_equal(lmk.cpu().numpy(), np.concatenate(parts, axis=1))
    _check_attention(ops, q, kk, v, w, lmk.cpu(), cu, lmk_block=384, rows=np.arange(0, 1800, 4))


@pytest.mark.parametrize("d_model,n_kv,head_dim,T", [(1024, 16, 64, 1000), (1024, 16, 64, 5003),
                                                     (2048, 16, 128, 3001)])
def test_signals_bulk_and_fallback_paths(ops, d_model, n_kv, head_dim, T):
    """Widths and norms bit-exact against the oracle on both 16-bit paths: rows that fit
    in shared memory (bulk copies, d_model 1024) and rows that do not (plain loads,
    d_model 2048 with 16 x 128 value heads), with token counts that leave warps idle or
    give them two tokens."""
    g0 = torch.Generator().manual_seed(d_model + T)
    x = torch.randn(T, d_model, generator=g0).bfloat16()
    gw = (0.05 * torch.randn(d_model, generator=g0)).bfloat16()
    gb = torch.tensor([0.1]).bfloat16()
    v = torch.randn(T, n_kv * head_dim, generator=g0).bfloat16()
    w, xn, vn, lg = ops.window_signals(x.to(_dev()), gw.to(_dev()), gb.to(_dev()), 16, 512, v.to(_dev()), head_dim,
                                       False, return_logit=True)
    lo = O.window_logit(x.float().numpy(), gw.float().numpy(), float(gb.float()[0]), "bf16")
    np.testing.assert_array_equal(lg.cpu().numpy(), lo)
    wo, amb = O.window_sizes_from_logit(lo, 16, 512, "bf16")
    assert not ((w.cpu().numpy() != wo) & ~amb).any()
    np.testing.assert_array_equal(xn.cpu().numpy(), O.row_norms(x.float().numpy(), None))
    np.testing.assert_array_equal(vn.cpu().numpy(),
                                  O.row_norms(v.float().numpy().reshape(T, n_kv, head_dim), None))


@pytest.mark.parametrize("gate_scale", [0.05, 0.0])
def test_signals_rows_outside_the_fast_range(ops, gate_scale):
    """Rows whose squares or gate products would underflow or overflow in fp32, zero rows,
    a single tiny element and a zero gate: the kernel's exact sums must not pass through
    fp32 intermediates, so widths, logits and norms stay bit-exact with the oracle's
    float64 sums (an overflowing norm is inf on both sides)."""
    g0 = torch.Generator().manual_seed(11)
    T, d_model, n_kv, head_dim = 640, 1024, 16, 64
    x = torch.randn(T, d_model, generator=g0)
    v = torch.randn(T, n_kv * head_dim, generator=g0)
    x[0] = 0.0
    x[1] *= 2.0 ** -70  # squares underflow fp32
    x[2] *= 2.0 ** 70  # squares overflow fp32 (norm inf)
    x[3, 5] = 2.0 ** -100  # one tiny element among normal ones
    x[4, :512] = 0.0
    v[0] = 0.0
    v[1, :64] *= 2.0 ** -70  # one value head underflows
    v[2, 64:128] *= 2.0 ** 66  # one value head overflows
    x, v = x.bfloat16(), v.bfloat16()
    gw = (gate_scale * torch.randn(d_model, generator=g0)).bfloat16()
    gb = torch.tensor([0.1]).bfloat16()
    for rnd in (False, True):
        w, xn, vn, lg = ops.window_signals(x.to(_dev()), gw.to(_dev()), gb.to(_dev()), 16, 512, v.to(_dev()),
                                           head_dim, rnd, return_logit=True)
        lo = O.window_logit(x.float().numpy(), gw.float().numpy(), float(gb.float()[0]), "bf16")
        np.testing.assert_array_equal(lg.cpu().numpy(), lo)
        wo, amb = O.window_sizes_from_logit(lo, 16, 512, "bf16")
        assert not ((w.cpu().numpy() != wo) & ~amb).any()
        np.testing.assert_array_equal(xn.cpu().numpy(), O.row_norms(x.float().numpy(), "bf16" if rnd else None))
        np.testing.assert_array_equal(
            vn.cpu().numpy(), O.row_norms(v.float().numpy().reshape(T, n_kv, head_dim), "bf16" if rnd else None))
