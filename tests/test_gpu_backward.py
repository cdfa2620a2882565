"""Backward of the sparse attention (``dsalt_attention_bwd``; reference
``dsalt/kernels/dsalt_triton_bwd.py``) against the float64 oracle
(``oracle.dsalt_oracle.attention_backward``, itself checked against autograd of the forward
in ``tests/test_oracle_backward.py``), and the autograd function built on it."""
import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda", 0)


def _case(seed, cu, H, Hkv, D, k_lmk, lmk_block, dtype, with_bias):
    g = torch.Generator().manual_seed(seed)
    T = cu[-1]
    q = torch.randn(T, H, D, generator=g).to(dtype)
    k = torch.randn(T, Hkv, D, generator=g).to(dtype)
    v = torch.randn(T, Hkv, D, generator=g).to(dtype)
    w = torch.randint(1, 300, (T,), generator=g, dtype=torch.int32)
    n_sets = len(cu) - 1 if lmk_block == 0 else sum((cu[s + 1] - cu[s] + lmk_block - 1) // lmk_block
                                                   for s in range(len(cu) - 1))
    lmk = torch.full((H, n_sets, k_lmk), -1, dtype=torch.int32)
    for h in range(H):
        for sid in range(n_sets):
            n = int(torch.randint(k_lmk // 2, k_lmk + 1, (1,), generator=g))
            pos = torch.randperm(min(cu[1] - cu[0], cu[-1] - cu[-2]), generator=g)[:n].sort().values
            lmk[h, sid, :n] = pos.to(torch.int32)
    bias = (0.3 * torch.randn(H, n_sets, k_lmk, generator=g)) if with_bias else None
    return q, k, v, w, lmk, bias


def _check(got, ref, what):
    scale = max(1.0, float(np.abs(ref).max()))
    err = float(np.abs(got - ref).max())
    assert err <= 2e-4 * scale, f"{what}: max error {err:.3e} (scale {scale:.2e})"


@pytest.mark.parametrize("H,Hkv,D,lmk_block,dtype,with_bias", [
    (4, 4, 64, 0, torch.bfloat16, True),
    (4, 2, 64, 128, torch.bfloat16, False),
    (2, 1, 128, 0, torch.float16, True),
    (4, 2, 64, 512, torch.float32, False),
])
def test_backward_matches_oracle(H, Hkv, D, lmk_block, dtype, with_bias):
    from dsalt_b200 import ops
    dev = _dev()
    cu = [0, 700, 1213]
    q, k, v, w, lmk, bias = _case(1, cu, H, Hkv, D, 24, lmk_block, dtype, with_bias)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    qd, kd, vd, wd, ld = (t.to(dev) for t in (q, k, v, w, lmk))
    bd = bias.to(dev) if bias is not None else None
    out, lse = ops.dsalt_attention(qd, kd, vd, ld, bd, wd, cu_t, lmk_block=lmk_block, out_dtype=dtype,
                                   cu_list=cu, return_lse=True)
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(2)).to(dtype)
    dq, dk, dv, db = ops.dsalt_attention_backward(dout.to(dev), qd, kd, vd, out, lse, ld, bd, wd, cu_t,
                                                  lmk_block=lmk_block, cu_list=cu)
    ref = O.attention_backward(q.float().numpy(), k.float().numpy(), v.float().numpy(), out.float().cpu().numpy(),
                               dout.float().numpy(), lse.cpu().numpy().astype(np.float64), w.numpy(), lmk.numpy(),
                               cu, lmk_block=lmk_block, lmk_bias=bias.numpy() if bias is not None else None)
    for name, got, r in zip(("dq", "dk", "dv", "d_bias"), (dq, dk, dv, db), ref):
        if name == "d_bias" and bias is None:
            continue
        _check(got.cpu().numpy().astype(np.float64), r, name)


def test_autograd_function_and_unsorted_sets():
    """``dsalt_attention_autograd`` gives the backward's gradients through ``.backward()``,
    for landmark sets given in any slot order (the bias gradient follows the caller's slots)."""
    from dsalt_b200 import ops
    dev = _dev()
    cu = [0, 512, 900]
    H, Hkv, D = 4, 2, 64
    q, k, v, w, lmk, bias = _case(3, cu, H, Hkv, D, 16, 0, torch.bfloat16, True)
    perm = torch.randperm(16, generator=torch.Generator().manual_seed(4))
    lmk, bias = lmk[..., perm].contiguous(), bias[..., perm].contiguous()
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    qd, kd, vd = (t.to(dev).requires_grad_(True) for t in (q, k, v))
    bd = bias.to(dev).requires_grad_(True)
    out = ops.dsalt_attention_autograd(qd, kd, vd, lmk.to(dev), bd, w.to(dev), cu_t, cu_list=cu)
    assert out.dtype == torch.float32
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(5)).to(dev)
    out.backward(dout)
    o2, lse = ops.dsalt_attention(qd.detach(), kd.detach(), vd.detach(), lmk.to(dev), bd.detach(), w.to(dev), cu_t,
                                  out_dtype=torch.bfloat16, cu_list=cu, return_lse=True)
    ref = O.attention_backward(q.float().numpy(), k.float().numpy(), v.float().numpy(), o2.float().cpu().numpy(),
                               dout.to(torch.bfloat16).float().cpu().numpy(), lse.cpu().numpy().astype(np.float64),
                               w.numpy(), lmk.numpy(), cu, lmk_bias=bias.numpy())
    # gradients come back in the input dtypes (bf16 for q, k, v; fp32 for the bias)
    for name, got, r in zip(("dq", "dk", "dv"), (qd.grad, kd.grad, vd.grad), ref[:3]):
        scale = max(1.0, float(np.abs(r).max()))
        assert float(np.abs(got.float().cpu().numpy() - r).max()) <= 2 ** -7 * scale, name
    _check(bd.grad.cpu().numpy().astype(np.float64), ref[3], "d_bias")
