"""Soft-selector training attention (``dsalt_train_attention_fwd`` / ``_bwd``; reference
``dsalt/kernels/dsalt_triton_train.py``) against the float64 oracle
(``oracle.dsalt_oracle.train_attention_*``, itself checked against autograd in
``tests/test_oracle_train.py``), and the autograd function built on them."""
import math

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
                                            (2, 1, 128, torch.float16), (4, 2, 128, torch.bfloat16)])
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
    # fp32 inputs: CUDA cores, P in fp32. bf16 / fp16: tensor cores, P rounded to the input
    # dtype for P·V (|error| <= u·Σp|v|/Σp <= u·max|v|, u the dtype's unit roundoff) and part
    # of the exponentials from a polynomial 2^x (relative error 7.5e-5)
    u = {torch.float32: 0.0, torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}[dtype]
    vmax = float(np.abs(vn).max())
    err = float(np.abs(out.cpu().numpy() - ref_out).max())
    assert err <= (u + 2e-4) * vmax if u else err <= 2e-5 * max(1.0, float(np.abs(ref_out).max())), f"out: {err:.3e}"
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lse.cpu().numpy()), fin)
    _check(lse.cpu().numpy()[fin], ref_lse[fin], 3e-4 if u else 2e-5, "lse")
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


def _dense_module_train(m, x, cu, lmk_pos, w_gpu):
    """Float64 dense restatement of the module's training forward (``_packed_train_triton`` with
    ``_train_selectors``, ``dsalt_attention.py:438-487``, and the kernel's bias
    ``_dense_logbias_from_kernel`` ``:513-563``) on the same landmark positions. The hard masks
    (band ``d ≤ w̃``, core ``d ≤ w̃ − win_edge``, landmark ``p < i − w̃``) use the GPU's fp32
    widths ``w_gpu`` so that a width within rounding of an integer cannot flip a mask; the soft
    biases use the float64 widths, so their gradients flow."""
    from dsalt_b200.module import hybrid_scores_per_head
    T = x.shape[0]
    H, Hkv, D = m.n_heads, m.n_kv_heads, m.head_dim
    q, k, v = m._qkv(x, cu, T, x.device, None)
    w64 = m.n_min + torch.sigmoid(m.win_gate(x).squeeze(-1)) * (m.n_max - m.n_min)
    scores = hybrid_scores_per_head(x, m.v_proj.weight, m._alpha(), H, D)
    outs = []
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        L = b - a
        i = torch.arange(L, dtype=torch.float64)[:, None]
        d = i - torch.arange(L, dtype=torch.float64)[None, :]
        wf, wd = w_gpu[a:b, None], w64[a:b, None]
        band = (d >= 0) & (d <= wf)
        core = d <= wf - m.win_edge
        wb = torch.where(core, torch.zeros_like(d), torch.log(torch.sigmoid((wd - d) / m.tau_win).clamp(min=1e-20)))
        wb = wb.masked_fill(~band, float("-inf"))
        heads = []
        for h in range(H):
            g = h // (H // Hkv)
            p = lmk_pos[h, s]
            pc = p.clamp(min=0)
            logw = torch.log(torch.sigmoid(scores[a + pc, h] / m.tau_lmk).clamp(min=1e-20))
            pf = pc.double()[None, :]
            ok = (p >= 0)[None, :] & (pf <= i) & (pf < i - wf)
            lb = torch.where(ok, logw[None, :], torch.full_like(pf.expand(L, -1), float("-inf")))
            lg = torch.cat([q[a:b, h] @ k[a:b, g].T / math.sqrt(D) + wb, q[a:b, h] @ k[a + pc, g].T / math.sqrt(D) + lb], 1)
            heads.append(torch.softmax(lg, 1) @ torch.cat([v[a:b, g], v[a + pc, g]], 0))
        outs.append(torch.stack(heads, 1))
    return m.out_proj(torch.cat(outs, 0).reshape(T, m.d_model))


def test_module_training_matches_dense():
    """``DSALTAttention`` in training mode: output and the gradients of every parameter
    (``win_gate`` through the soft window edge, ``alpha_w`` through the landmark weights)
    against the float64 dense restatement."""
    import copy
    from dsalt_b200 import ops
    from dsalt_b200.module import DSALTAttention
    dev = _dev()
    torch.manual_seed(0)
    m = DSALTAttention(d_model=256, n_heads=4, n_min=8, n_max=64, k_lmk=8, max_seq_len=512, n_kv_heads=2).to(dev)
    with torch.no_grad():
        m.win_gate.weight.mul_(4.0)  # spread the widths over [n_min, n_max]
    m.train()
    cu = [0, 200, 330]
    x = torch.randn(cu[-1], 256, device=dev)
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    out, aux = m(x, cu_t, cu_list=cu)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(1)).to(dev)
    out.backward(gout)
    with torch.no_grad():
        w_gpu = m.n_min + torch.sigmoid(m.win_gate(x).squeeze(-1)) * (m.n_max - m.n_min)
        lmk_pos, _, _ = ops.compute_landmark_indices(x, m.v_proj.weight, m._alpha().float(), w_gpu.floor().clamp(min=1),
                                                     cu_t, m.k_lmk, m.n_min, cu[-1], cu, head_dim=m.head_dim)
    mc = copy.deepcopy(m).cpu().double()
    mc.zero_grad()
    ref = _dense_module_train(mc, x.cpu().double(), cu, lmk_pos.cpu(), w_gpu.cpu().double())
    _check(out.detach().cpu().double().numpy(), ref.detach().numpy(), 1e-4, "out")
    ref.backward(gout.cpu().double())
    for (name, p), (_, pc) in zip(m.named_parameters(), mc.named_parameters()):
        r = pc.grad.numpy()
        err = float(np.abs(p.grad.double().cpu().numpy() - r).max())
        assert err <= 1e-3 * float(np.abs(r).max()) + 1e-6, f"grad {name}: {err:.3e} vs max {np.abs(r).max():.3e}"
    assert float(m.alpha_w.grad.abs().max()) > 0 and float(m.win_gate.weight.grad.abs().max()) > 0


def test_module_training_bf16_autocast():
    """Training step under bf16 autocast (the trainer's setting): finite loss and gradients."""
    from dsalt_b200.module import DSALTAttention
    dev = _dev()
    torch.manual_seed(2)
    m = DSALTAttention(d_model=512, n_heads=8, n_min=16, n_max=128, k_lmk=16, max_seq_len=2048).to(dev).train()
    cu = [0, 700, 1024, 1500]
    x = torch.randn(cu[-1], 512, device=dev)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out, _ = m(x, torch.tensor(cu, dtype=torch.int32, device=dev), cu_list=cu)
        loss = out.float().pow(2).mean()
    loss.backward()
    assert torch.isfinite(loss)
    for name, p in m.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
