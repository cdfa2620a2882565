"""The oracle's soft-selector training attention (``oracle.dsalt_oracle.train_attention_*``,
a restatement of ``dsalt/kernels/dsalt_triton_train.py``): its backward against float64
autograd of its forward, in q, k, v, the landmark log-weights and the continuous widths
(through the soft window edge ``log σ((w̃ − d)/τ)``)."""
import math

import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O


def _dense_train_forward(q, k, v, logw, wc, lmk, cu, tau, edge):
    T, H, D = q.shape
    rep = H // k.shape[1]
    scale = float(np.float32(1.0 / math.sqrt(D)))
    out = torch.zeros_like(q)
    wcn = wc.detach().numpy()
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        L = b - a
        for i in range(L):
            t = a + i
            j = np.arange(0, i + 1)
            d = (i - j).astype(np.float64)
            band = d <= wcn[t]
            j, d = j[band], torch.tensor(d[band])
            core = torch.tensor((d.numpy() <= wcn[t] - edge))
            z = (wc[t] - d) / tau
            wbias = torch.where(core, torch.zeros_like(z), torch.nn.functional.logsigmoid(z))
            for h in range(H):
                g = h // rep
                P = lmk[h, s]
                ok = (P >= 0) & (P < L) & (P <= i) & (P.astype(np.float64) < i - wcn[t])
                slots = np.nonzero(ok)[0]
                rows = np.concatenate([a + j, a + P[slots]])
                lg = k[rows, g] @ q[t, h] * scale
                lg = lg + torch.cat([wbias, logw[h, s, slots]])
                out[t, h] = torch.softmax(lg, 0) @ v[rows, g]
    return out


@pytest.mark.parametrize("H,Hkv", [(2, 2), (4, 2)])
def test_oracle_train_backward_matches_autograd(H, Hkv):
    rng = np.random.default_rng(11)
    cu = [0, 90, 150]
    T, D, k_lmk, tau, edge = cu[-1], 8, 5, 1.0, 4
    q = rng.standard_normal((T, H, D))
    k = rng.standard_normal((T, Hkv, D))
    v = rng.standard_normal((T, Hkv, D))
    wc = (rng.uniform(2.0, 30.0, T)).astype(np.float32)
    lmk = np.full((H, 2, k_lmk), -1, dtype=np.int32)
    for h in range(H):
        for s in range(2):
            lmk[h, s, :k_lmk - 1] = rng.choice(55, size=k_lmk - 1, replace=False)  # any slot order
    logw = rng.standard_normal(lmk.shape) * 0.5
    out, lse = O.train_attention_forward(q, k, v, lmk, logw, wc, cu, tau, edge)
    dout = rng.standard_normal(out.shape)
    dq, dk, dv, dlw, dw = O.train_attention_backward(q, k, v, out, dout, lse, lmk, logw, wc, cu, tau, edge)
    tq, tk, tv = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
    tl = torch.tensor(logw, requires_grad=True)
    tw = torch.tensor(wc.astype(np.float64), requires_grad=True)
    o = _dense_train_forward(tq, tk, tv, tl, tw, lmk, cu, tau, edge)
    np.testing.assert_allclose(o.detach().numpy(), out, atol=1e-12)
    (o * torch.tensor(dout)).sum().backward()
    for got, ref in ((dq, tq.grad), (dk, tk.grad), (dv, tv.grad), (dlw, tl.grad), (dw, tw.grad)):
        np.testing.assert_allclose(got, ref.numpy(), atol=1e-10)


_GOLDEN = __import__("pathlib").Path(__file__).parent / "golden" / "train_ref.npz"


@pytest.mark.parametrize("case", ["mha", "gqa"])
def test_oracle_train_matches_reference_fixture(case):
    """The oracle against the reference's own dense training attention
    (``_dense_logbias_from_kernel`` + SDPA, as ``_packed_train`` runs it) on the reference's
    own selectors (``_train_selectors``): output, and the gradients of q, k, v (per kv
    head), the continuous widths and the landmark log-weights (fixture from
    ``tests/golden/make_golden_train.py``, fp32 on CPU; the oracle is float64)."""
    z = np.load(_GOLDEN)
    f = lambda n: z[f"{case}/{n}"]  # noqa: E731
    cu = f("cu").tolist()
    tau, edge = float(f("tau")), float(f("edge"))
    q, k, v = (f(n).astype(np.float64) for n in ("q", "k", "v"))
    lmk, logw, w = f("lmk_pos"), f("lmk_logw").astype(np.float64), f("w_cont")
    out, lse = O.train_attention_forward(q, k, v, lmk, logw, w, cu, tau, edge)
    ref = f("out")
    assert np.abs(out - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
    got = O.train_attention_backward(q, k, v, out, f("dout").astype(np.float64), lse, lmk, logw, w, cu, tau, edge)
    for name, g in zip(("dq", "dk", "dv", "d_logw", "d_w"), got):
        r = f(name)
        err = float(np.abs(g - r).max())
        assert err <= 1e-4 * max(1.0, float(np.abs(r).max())), f"{case} {name}: {err:.3e}"


@pytest.mark.parametrize("case", ["mha", "gqa"])
def test_module_landmark_logw_matches_reference_fixture(case):
    """The training module's hybrid scores and landmark log-weights (the torch half of
    ``DSALTAttention._train_selectors``; the positions come from the CUDA selection) equal
    the reference's on its own inputs and positions, bit for bit."""
    from dsalt_b200.module import DSALTAttention, hybrid_scores_per_head
    z = np.load(_GOLDEN)
    f = lambda n: torch.from_numpy(z[f"{case}/{n}"])  # noqa: E731
    scores_ref, lmk = f("scores"), f("lmk_pos")
    H = scores_ref.shape[1]
    dm = f("x").shape[1]
    sc = hybrid_scores_per_head(f("x"), f("v_proj_weight"), f("alpha"), H, dm // H)
    assert torch.equal(sc, scores_ref)
    m = DSALTAttention(dm, H, 1, 2, lmk.shape[-1], 8, n_kv_heads=f("v").shape[1])
    assert m.tau_lmk == float(f("tau_lmk"))
    assert torch.equal(m._landmark_logw(scores_ref, lmk, f("cu").tolist()), f("lmk_logw"))


def test_module_landmark_logw_empty_slots():
    """Empty slots (-1) get log-weight -inf; positions index their own sequence's rows."""
    from dsalt_b200.module import DSALTAttention
    m = DSALTAttention(16, 2, 1, 8, 3, 8)
    scores = torch.arange(20, dtype=torch.float32).view(10, 2) / 10  # [T, H], T = 4 + 6
    lmk = torch.tensor([[[0, 3, -1], [1, -1, -1]], [[2, 2, 0], [5, 0, -1]]])  # [H, S, k]
    got = m._landmark_logw(scores, lmk, [0, 4, 10])
    starts = [0, 4]
    for h in range(2):
        for s in range(2):
            for c in range(3):
                p = int(lmk[h, s, c])
                if p < 0:
                    assert got[h, s, c] == float("-inf")
                else:
                    ref = math.log(1.0 / (1.0 + math.exp(-float(scores[starts[s] + p, h]) / m.tau_lmk)))
                    assert abs(float(got[h, s, c]) - ref) < 1e-6


def test_oracle_train_small_widths_match_autograd():
    """Widths below the edge width (the whole band is soft edge, w̃ < 1 keeps only the
    diagonal), landmarks out of range and empty slots: backward against float64 autograd."""
    rng = np.random.default_rng(5)
    cu = [0, 40, 70]
    T, H, D, k_lmk, tau, edge = cu[-1], 2, 8, 6, 0.7, 4
    q, k, v = (rng.standard_normal((T, H, D)) for _ in range(3))
    wc = rng.uniform(0.2, 6.0, T).astype(np.float32)
    lmk = np.full((H, 2, k_lmk), -1, dtype=np.int32)
    for h in range(H):
        for s in range(2):
            lmk[h, s, :4] = rng.choice(30, size=4, replace=False)
    lmk[0, 1, 4] = 45  # beyond the second sequence's length: never a key
    logw = rng.standard_normal(lmk.shape) * 0.5
    out, lse = O.train_attention_forward(q, k, v, lmk, logw, wc, cu, tau, edge)
    dout = rng.standard_normal(out.shape)
    got = O.train_attention_backward(q, k, v, out, dout, lse, lmk, logw, wc, cu, tau, edge)
    tq, tk, tv = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
    tl = torch.tensor(logw, requires_grad=True)
    tw = torch.tensor(wc.astype(np.float64), requires_grad=True)
    o = _dense_train_forward(tq, tk, tv, tl, tw, lmk, cu, tau, edge)
    np.testing.assert_allclose(o.detach().numpy(), out, atol=1e-12)
    (o * torch.tensor(dout)).sum().backward()
    for g, r in zip(got, (tq.grad, tk.grad, tv.grad, tl.grad, tw.grad)):
        np.testing.assert_allclose(g, r.numpy(), atol=1e-10)
