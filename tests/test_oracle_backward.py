"""The oracle's backward (``oracle.dsalt_oracle.attention_backward``, a restatement of
``dsalt/kernels/dsalt_triton_bwd.py``) against float64 autograd of the forward it
differentiates: each row's softmax over its window and its causal, de-duplicated
landmarks, with the landmark bias on the landmark logits."""
import math

import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O


def _dense_forward(q, k, v, bias, w, lmk, cu, lmk_block):
    """``out = softmax(mask(q kᵀ scale + bias)) v`` with the kernel's key sets, as a dense
    masked softmax in float64 (autograd-able in q, k, v and the bias)."""
    T, H, D = q.shape
    rep = H // k.shape[1]
    scale = float(np.float32(1.0 / math.sqrt(D)))
    out = torch.zeros_like(q)
    set_base = 0
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        L = b - a
        nsets = 1 if lmk_block == 0 else (L + lmk_block - 1) // lmk_block
        for i in range(L):
            t = a + i
            lo = i - int(max(w[t], 1)) + 1
            sid = set_base if lmk_block == 0 else set_base + i // lmk_block
            for h in range(H):
                g = h // rep
                P = lmk[h, sid]
                ok = (P >= 0) & (P < L) & (P <= i) & (P < lo)
                slots = np.nonzero(ok)[0]
                rows = np.concatenate([np.arange(a + max(lo, 0), t + 1), a + P[slots]])
                lg = k[rows, g] @ q[t, h] * scale
                nw = t + 1 - (a + max(lo, 0))
                lg = torch.cat([lg[:nw], lg[nw:] + bias[h, sid, slots]])
                out[t, h] = torch.softmax(lg, 0) @ v[rows, g]
        set_base += nsets
    return out


@pytest.mark.parametrize("H,Hkv,lmk_block,with_bias", [(2, 2, 0, True), (4, 2, 64, False), (2, 1, 0, False)])
def test_oracle_backward_matches_autograd(H, Hkv, lmk_block, with_bias):
    rng = np.random.default_rng(7)
    cu = [0, 150, 230]
    T, D, k_lmk = cu[-1], 16, 6
    q = rng.standard_normal((T, H, D))
    k = rng.standard_normal((T, Hkv, D))
    v = rng.standard_normal((T, Hkv, D))
    w = rng.integers(1, 40, T).astype(np.int32)
    n_sets = 2 if lmk_block == 0 else sum((cu[s + 1] - cu[s] + lmk_block - 1) // lmk_block for s in range(2))
    lmk = np.full((H, n_sets, k_lmk), -1, dtype=np.int32)
    for h in range(H):
        for sid in range(n_sets):
            pos = np.sort(rng.choice(80, size=k_lmk - 1, replace=False))
            lmk[h, sid, :k_lmk - 1] = pos
    bias = rng.standard_normal(lmk.shape) * 0.3 if with_bias else np.zeros(lmk.shape)
    out, lse = O.attention_forward(q, np.repeat(k, H // Hkv, 1), np.repeat(v, H // Hkv, 1), w, lmk, cu,
                                   lmk_block=lmk_block, lmk_bias=bias if with_bias else None)
    dout = rng.standard_normal(out.shape)
    dq, dk, dv, db = O.attention_backward(q, k, v, out, dout, lse, w, lmk, cu, lmk_block=lmk_block,
                                          lmk_bias=bias if with_bias else None)
    tq, tk, tv = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
    tb = torch.tensor(bias, requires_grad=True)
    o = _dense_forward(tq, tk, tv, tb, w, lmk, cu, lmk_block)
    np.testing.assert_allclose(o.detach().numpy(), out, atol=1e-12)
    (o * torch.tensor(dout)).sum().backward()
    np.testing.assert_allclose(dq, tq.grad.numpy(), atol=1e-10)
    np.testing.assert_allclose(dk, tk.grad.numpy(), atol=1e-10)
    np.testing.assert_allclose(dv, tv.grad.numpy(), atol=1e-10)
    np.testing.assert_allclose(db, tb.grad.numpy(), atol=1e-10)


def test_oracle_backward_matches_reference_fixture():
    """The oracle's backward against autograd through the reference's PyTorch restatement
    of its kernel (``_block_attention``, one landmark set per query block; fixture from
    ``tests/golden/make_golden_backward.py``, fp32 on CPU; the oracle is float64)."""
    import pathlib
    z = np.load(pathlib.Path(__file__).parent / "golden" / "bwd_ref.npz")
    q, k, v = (z[n].astype(np.float64) for n in ("q", "k", "v"))
    L = q.shape[0]
    block = int(z["block"])
    out, lse = O.attention_forward(q, k, v, z["w"], z["lmk"], [0, L], lmk_block=block)
    ref = z["out"]
    assert np.abs(out - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())
    dq, dk, dv, _ = O.attention_backward(q, k, v, out, z["dout"].astype(np.float64), lse, z["w"], z["lmk"], [0, L],
                                         lmk_block=block)
    for name, g in (("dq", dq), ("dk", dk), ("dv", dv)):
        r = z[name]
        err = float(np.abs(g - r).max())
        assert err <= 1e-4 * max(1.0, float(np.abs(r).max())), f"{name}: {err:.3e}"
