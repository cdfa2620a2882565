"""Soft-selector training attention (``dsalt_train_attention_fwd`` / ``_bwd``; reference
``dsalt/kernels/dsalt_triton_train.py``) against the float64 oracle
(``oracle.dsalt_oracle.train_attention_*``, itself checked against autograd in
``tests/test_oracle_train.py``), and the autograd function built on them."""
import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


def _case(seed, cu, H, Hkv, D, k_lmk, dtype):
    g = torch.Generator().manual_seed(seed)
    T = cu[-1]
    q = torch.randn(T, H, D, generator=g).to(dtype)
    k = torch.randn(T, Hkv, D, generator=g).to(dtype)
    v = torch.randn(T, Hkv, D, generator=g).to(dtype)
    w = (torch.rand(T, generator=g) * 250 + 1.5).float()  # continuous widths, fractional
    S = len(cu) - 1
    lmk = torch.full((H, S, k_lmk), -1, dtype=torch.int32)
    Lmin = min(cu[s + 1] - cu[s] for s in range(S))
    for h in range(H):
        for s in range(S):
            n = int(torch.randint(k_lmk // 2, k_lmk + 1, (1,), generator=g))
            lmk[h, s, :n] = torch.randperm(Lmin, generator=g)[:n].to(torch.int32)  # any slot order
    logw = torch.nn.functional.logsigmoid(torch.randn(H, S, k_lmk, generator=g) * 2)
    return q, k, v, w, lmk, logw


def _check(got, ref, tol, what):
    scale = max(1.0, float(np.abs(ref).max()))
    err = float(np.abs(np.asarray(got, dtype=np.float64) - ref).max())
    assert err <= tol * scale, f"{what}: max error {err:.3e} (scale {scale:.2e})"


@pytest.mark.parametrize("H,Hkv,D,dtype", [(4, 4, 64, torch.bfloat16), (4, 2, 64, torch.float32),
                                            (2, 1, 128, torch.float16)])
def test_train_forward_backward_match_oracle(H, Hkv, D, dtype):
    from dsalt_b200 import ops
    dev = _dev()
    cu = [0, 600, 1001]
    tau, edge = 1.0, 4.0
    q, k, v, w, lmk, logw = _case(3, cu, H, Hkv, D, 20, dtype)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    args = [t.to(dev) for t in (q, k, v, lmk, logw, w)]
    out, lse = ops.train_attention_forward(*args[:3], args[3], args[4], args[5], cu_t, tau, edge,
                                           out_dtype=torch.float32, cu_list=cu)
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref_out, ref_lse = O.train_attention_forward(qn, kn, vn, lmk.numpy(), logw.numpy(), w.numpy(), cu, tau, edge)
    _check(out.cpu().numpy(), ref_out, 2e-5, "out")
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lse.cpu().numpy()), fin)
    _check(lse.cpu().numpy()[fin], ref_lse[fin], 2e-5, "lse")
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(4)).to(dtype)
    got = ops.train_attention_backward(dout.to(dev), *args[:3], out, lse, args[3], args[4], args[5], cu_t, tau, edge,
                                       cu_list=cu)
    ref = O.train_attention_backward(qn, kn, vn, out.cpu().numpy(), dout.float().numpy(),
                                     lse.cpu().numpy().astype(np.float64), lmk.numpy(), logw.numpy(), w.numpy(), cu,
                                     tau, edge)
    for name, g_, r in zip(("dq", "dk", "dv", "d_logw", "d_w"), got, ref):
        _check(g_.cpu().numpy(), r, 2e-4, name)


def test_train_autograd_function():
    """``dsalt_train_attention`` (the reference's ``dsalt_triton_train_attention``) carries the
    gradients of q, k, v, the landmark log-weights and the continuous widths through
    ``.backward()``."""
    from dsalt_b200 import ops
    dev = _dev()
    cu = [0, 512, 800]
    q, k, v, w, lmk, logw = _case(5, cu, 4, 2, 64, 16, torch.bfloat16)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    tq, tk, tv = (t.to(dev).requires_grad_(True) for t in (q, k, v))
    tl = logw.to(dev).requires_grad_(True)
    tw = w.to(dev).requires_grad_(True)
    out = ops.dsalt_train_attention(tq, tk, tv, lmk.to(dev), tl, tw, cu_t, cu_list=cu)
    assert out.dtype == torch.float32
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(6)).to(dev)
    out.backward(dout)
    o2, lse = ops.train_attention_forward(tq.detach(), tk.detach(), tv.detach(), lmk.to(dev), tl.detach(), tw.detach(),
                                          cu_t, 1.0, 4.0, cu_list=cu)
    ref = O.train_attention_backward(q.float().numpy(), k.float().numpy(), v.float().numpy(), o2.float().cpu().numpy(),
                                     dout.to(torch.bfloat16).float().cpu().numpy(),
                                     lse.cpu().numpy().astype(np.float64), lmk.numpy(), logw.numpy(), w.numpy(), cu,
                                     1.0, 4.0)
    for name, got, r in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), ref[:3]):
        _check(got.float().cpu().numpy(), r, 2 ** -7, name)
    _check(tl.grad.cpu().numpy(), ref[3], 2e-4, "d_logw")
    _check(tw.grad.cpu().numpy(), ref[4], 2e-4, "d_w")
