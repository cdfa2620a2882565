"""head_dim 128 (the Qwen-shaped configuration: 16 query heads over 2 kv heads) on the
tensor-core path, against the fp64 oracle.

The attention tolerance is the bound of the reference's own bf16/fp16 rounding of P before
the P·V product (``tl.dot(p.to(bf16), v)``, ``dsalt/kernels/dsalt_triton_attn.py:116,148``):
``u · Σ p|v| / Σ p`` per element with u = 2^-8 (bf16) or 2^-11 (fp16), plus 1e-4 for the fp32
accumulations; the landmark sets are bit-exact.
"""
import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from dsalt_b200 import ops as _ops
    return _ops


def _dev():
    return torch.device("cuda", 0)


def _inputs(cu, H, Hkv, D, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = cu[-1]
    q = (torch.randn(T, H, D, device=_dev(), generator=g) * 0.5).to(dt)
    k = (torch.randn(T, Hkv, D, device=_dev(), generator=g) * 0.5).to(dt)
    v = torch.randn(T, Hkv, D, device=_dev(), generator=g).to(dt)
    w = torch.randint(1, 700, (T,), device=_dev(), generator=g, dtype=torch.int32)
    xn = 30 + torch.randn(T, device=_dev(), generator=g)
    vn = 1 + 0.1 * torch.randn(T, Hkv, device=_dev(), generator=g)
    return q, k, v, w, xn, vn


def _check(out32, q, k, v, w, lmk, cu, lmk_block, dt, rows):
    H, Hkv = q.shape[1], k.shape[1]
    kr = k.repeat_interleave(H // Hkv, dim=1).float().cpu().numpy()
    vr = v.repeat_interleave(H // Hkv, dim=1).float().cpu().numpy()
    ref, _, mag = O.attention_forward(q.float().cpu().numpy(), kr, vr, w.cpu().numpy(), lmk.cpu().numpy(), cu,
                                      lmk_block=lmk_block, rows=rows, return_mag=True)
    u = 2.0 ** -8 if dt == torch.bfloat16 else 2.0 ** -11
    err = np.abs(out32.cpu().numpy()[rows] - ref[rows])
    bound = (u + 2.0 ** -12) * mag[rows] + 1e-4
    assert (err <= bound).all(), float((err / bound).max())


@pytest.mark.parametrize("mode", ["global", "block_causal"])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_attention_head_dim_128_gqa(ops, mode, dt):
    cu = [0, 1500, 1537, 4096]
    H, Hkv, D, k_lmk, B = 16, 2, 128, 128, 512
    q, k, v, w, xn, vn = _inputs(cu, H, Hkv, D, dt, 31)
    alpha = torch.full((H,), 0.6, device=_dev())
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    lmk = ops.select_landmarks(xn, vn, w, alpha, cu_t, k_lmk, H, mode, B, cu_list=cu)
    lb = 0 if mode == "global" else B
    out32 = ops.dsalt_attention(q, k, v, lmk, None, w, cu_t, lmk_block=lb, cu_list=cu, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    rng = np.random.default_rng(5)
    rows = np.unique(np.concatenate([rng.choice(cu[-1], 200, replace=False), [0, 1499, 1500, 1536, 4095]]))
    _check(out32, q, k, v, w, lmk, cu, lb, dt, rows)


def test_core_forward_head_dim_128(ops):
    """Widths, signals, block-causal selection and attention in one call at D = 128, GQA."""
    g = torch.Generator(device="cuda").manual_seed(8)
    cu = [0, 3072]
    T, H, Hkv, D, dm, k_lmk, B = cu[-1], 16, 2, 128, 512, 64, 512
    x = torch.randn(T, dm, device=_dev(), generator=g).bfloat16()
    Wv = (torch.randn(Hkv * D, dm, device=_dev(), generator=g) * 0.05).bfloat16()
    v = (x @ Wv.T).view(T, Hkv, D).contiguous()
    q = (torch.randn(T, H, D, device=_dev(), generator=g) * 0.5).bfloat16()
    k = (torch.randn(T, Hkv, D, device=_dev(), generator=g) * 0.5).bfloat16()
    gw = (torch.randn(dm, device=_dev(), generator=g) * 0.05).bfloat16()
    gb = torch.zeros(1, device=_dev()).bfloat16()
    alpha = torch.full((H,), 0.6, device=_dev())
    cu_t = torch.tensor(cu, dtype=torch.int32, device=_dev())
    out, w, lmk = ops.core_forward(x, gw, gb, 16, 512, alpha, q, k, v, k_lmk, cu_t, mode="block_causal", block=B,
                                   cu_list=cu, return_aux=True, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    xn, vn = O.token_signals(x.float().cpu().numpy(), v.float().cpu().numpy().reshape(T, -1), Hkv, D, None)
    lo = O.select_block_causal(xn, vn, alpha.cpu().numpy(), w.cpu().numpy(), T, k_lmk, H, B)
    np.testing.assert_array_equal(lmk.cpu().numpy(), lo)
    rows = np.arange(0, T, 23)
    _check(out, q, k, v, w, lmk, cu, B, torch.bfloat16, rows)


def test_sharded_attention_head_dim_128_on_emulated_shards(ops):
    """The sharded attention (pre-gathered landmark tiles, halo-extended K/V) at D = 128
    equals the whole-sequence kernel bit for bit."""
    from dsalt_b200.sharded import shard_plan
    L, H, Hkv, D, k_lmk, B, P, n_max = 8192, 8, 2, 128, 64, 512, 4, 300
    q, kk, v, w, xn, vn = _inputs([0, L], H, Hkv, D, torch.bfloat16, 12)
    w = w.clamp(max=n_max)
    alpha = torch.full((H,), 0.6, device=_dev())
    cu = torch.tensor([0, L], dtype=torch.int32, device=_dev())
    full_sets = ops.select_landmarks(xn, vn, w, alpha, cu, k_lmk, H, mode="block_causal", block=B, cu_list=[0, L])
    full_out = ops.dsalt_attention(q, kk, v, full_sets, None, w, cu, lmk_block=B, out_dtype=torch.bfloat16,
                                   cu_list=[0, L])
    T = L // P
    stride = kk.stride(0) * kk.element_size()
    k_src = torch.tensor([kk.data_ptr() + r * T * stride for r in range(P)], dtype=torch.int64, device=_dev())
    v_src = torch.tensor([v.data_ptr() + r * T * stride for r in range(P)], dtype=torch.int64, device=_dev())
    outs = []
    for r in range(P):
        plan = shard_plan(L, P, r, n_max, B)
        s = full_sets[:, plan.set_lo:plan.set_hi].contiguous()
        outs.append(ops.attention_sharded(q[plan.q_pos0:plan.q_pos0 + T], kk[plan.kv_pos0:plan.q_pos0 + T],
                                          v[plan.kv_pos0:plan.q_pos0 + T], plan.q_pos0, plan.kv_pos0, L, w, s, B,
                                          k_src, v_src, T))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(torch.cat(outs), full_out)
