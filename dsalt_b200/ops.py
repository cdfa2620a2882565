"""Torch-facing operators over the C ABI, mirroring the reference's functions.

* :func:`window_signals`            — ``DSALTAttention._window_sizes(x, floor=True)``
  (``dsalt/modules/dsalt_attention.py:270-284``) fused with the selection norms of
  ``hybrid_scores_per_head`` (``dsalt/kernels/landmark_tokens_ker.py:47,52``)
* :func:`compute_landmark_indices`  — ``_compute_landmark_indices``
  (``dsalt/kernels/selectors.py:75-134``), same arguments and return values
* :func:`select_landmarks`          — whole-sequence or block-causal selection from the
  signals (block-causal: ``results/causal_landmark_check.py:82-113``)
* :func:`dsalt_attention`           — ``dsalt_triton_attention``
  (``dsalt/kernels/dsalt_triton_attn.py:337-349``), same arguments; returns fp32 like the
  reference unless ``out_dtype`` is given
* :func:`core_forward`              — widths + selection + attention in one C call.

Tensors must be CUDA tensors; every call launches on the current stream. There is no
CPU path: a CPU tensor raises.
"""
from __future__ import annotations

import math

import torch

from . import _lib as L

_DT = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.float16: L.F16}


def _dt(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("dsalt_b200 operators need CUDA tensors (no CPU path)")


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _host_cu(cu_seqlens: torch.Tensor, cu_list):
    if cu_list is not None:
        return [int(c) for c in cu_list]
    return [int(c) for c in cu_seqlens.detach().to("cpu").tolist()]


def _cu_i32(cu_seqlens: torch.Tensor) -> torch.Tensor:
    cu = cu_seqlens if cu_seqlens.dtype == torch.int32 else cu_seqlens.to(torch.int32)
    return cu.contiguous()


def n_block_sets(cu_list, block: int) -> int:
    return sum((cu_list[i + 1] - cu_list[i] + block - 1) // block for i in range(len(cu_list) - 1))


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


# --------------------------------------------------------------------------- widths
def window_signals(x, gate_weight, gate_bias, n_min: int, n_max: int, v, head_dim: int, norm_round: bool = False,
                   return_logit: bool = False, logit=None):
    """Widths ``w [T] int32``, ``‖x‖ [T] fp32`` and value norms ``[T, n_kv] fp32``.

    ``gate_weight``/``gate_bias`` are ``win_gate``'s parameters already in the dtype the
    logit is computed in (the autocast dtype under autocast). ``v`` is ``x·W_Vᵀ``
    (``[T, n_kv·head_dim]``, or a ``[T, n_kv, head_dim]`` view). ``norm_round`` rounds the
    norms to the input dtype (a half-precision ``norm`` outside autocast).

    ``logit`` (``[T]`` or ``[T, 1]`` in ``gate_weight``'s dtype) is ``win_gate(x)`` as the
    caller computed it, e.g. by the same library GEMV the reference's
    ``_window_continuous`` calls (``dsalt/modules/dsalt_attention.py:275``); the widths are
    then taken from it, which makes them equal to the reference's on the same GPU. Without
    it the kernel forms the logit itself (float64 dot product rounded once), which can
    round to the neighbouring value of an fp32-accumulating GEMV.
    """
    _cuda(x, gate_weight, gate_bias, v, logit)
    T, dm = x.shape
    v2 = v.reshape(T, -1)
    if v2.stride(1) != 1:
        v2 = v2.contiguous()
    if x.stride(1) != 1:
        x = x.contiguous()
    n_kv = v2.shape[1] // head_dim
    gw = gate_weight.reshape(-1).contiguous()
    gb = gate_bias.reshape(-1).to(gw.dtype).contiguous()
    w = torch.empty(T, dtype=torch.int32, device=x.device)
    xn = torch.empty(T, dtype=torch.float32, device=x.device)
    vn = torch.empty(T, n_kv, dtype=torch.float32, device=x.device)
    lg = torch.empty(T, dtype=torch.float32, device=x.device) if return_logit else None
    lin = _logit_in(logit, T, gw.dtype)
    L.call("dsalt_token_signals", _ptr(x), _dt(x), T, dm, x.stride(0), _ptr(gw), _ptr(gb), _dt(gw), int(n_min),
           int(n_max), _ptr(v2), _dt(v2), v2.stride(0), n_kv, int(head_dim),
           L.NORM_INPUT if norm_round else L.NORM_F32, _ptr(w), _ptr(xn), _ptr(vn), _ptr(lg), _ptr(lin), _stream())
    if return_logit:
        return w, xn, vn, lg
    return w, xn, vn


def _logit_in(logit, T, dtype):
    """The caller's ``win_gate`` logit as a contiguous ``[T]`` tensor in the gate dtype."""
    if logit is None:
        return None
    lg = logit.reshape(-1)
    if lg.numel() != T:
        raise ValueError(f"logit has {lg.numel()} entries for {T} tokens")
    if lg.dtype != dtype:
        raise TypeError(f"logit dtype {lg.dtype} differs from the gate dtype {dtype}")
    return lg.contiguous()


# --------------------------------------------------------------------------- selection
def select_landmarks(xnorm, vnorm, w, alpha, cu_seqlens, k_lmk: int, n_heads: int, mode: str = "global",
                     block: int = 512, cu_list=None, return_z: bool = False):
    """Landmark sets ``[H, n_sets, k] int32`` (ascending positions within the sequence,
    ``-1`` padded). ``mode`` is ``"global"`` (one set per sequence) or ``"block_causal"``
    (one set per ``block`` queries, drawn from earlier positions)."""
    _cuda(xnorm, vnorm, w, alpha, cu_seqlens)
    cu_h = _host_cu(cu_seqlens, cu_list)
    S = len(cu_h) - 1
    T = int(xnorm.shape[0])
    n_kv = int(vnorm.shape[1])
    maxL = max([cu_h[i + 1] - cu_h[i] for i in range(S)] + [0])
    m = L.SELECT_GLOBAL if mode == "global" else L.SELECT_BLOCK_CAUSAL
    n_sets = S if m == L.SELECT_GLOBAL else n_block_sets(cu_h, block)
    dev = xnorm.device
    lmk = torch.empty(n_heads, n_sets, k_lmk, dtype=torch.int32, device=dev)
    zx = torch.empty(T, dtype=torch.float32, device=dev) if (return_z and m == L.SELECT_GLOBAL) else None
    zv = torch.empty(T, n_kv, dtype=torch.float32, device=dev) if (return_z and m == L.SELECT_GLOBAL) else None
    if T == 0 or k_lmk == 0:
        lmk.fill_(-1)
        return (lmk, zx, zv) if return_z else lmk
    ws_n = L.query("dsalt_select_workspace_bytes", m, T, S, maxL, n_heads, n_kv, k_lmk, block)
    ws = _workspace(ws_n, dev)
    a = alpha.float().contiguous()
    L.call("dsalt_select_landmarks", m, _ptr(xnorm.contiguous()), _ptr(vnorm.contiguous()),
           _ptr(w.to(torch.int32).contiguous()), _ptr(a), _ptr(_cu_i32(cu_seqlens)), S, T, maxL, n_heads, n_kv,
           k_lmk, block, _ptr(lmk), _ptr(zx), _ptr(zv), _ptr(ws), ws.numel(), _stream())
    return (lmk, zx, zv) if return_z else lmk


def compute_landmark_indices(x, W_V, alpha, w_sizes, cu_seqlens, k_lmk, n_min, total_len, cu_list=None,
                             head_dim=None, *, v=None, norm_round=None):
    """Drop-in for ``_compute_landmark_indices`` (``dsalt/kernels/selectors.py:75-86``).

    Returns ``(lmk [H, S, k] int64, z_x [T], z_v [T, H])``. The value norms use ``v`` if
    given (the ``v_proj`` output, equal to ``x @ W_Vᵀ`` without bias), else ``x @ W_Vᵀ``
    computed here with a library GEMM. ``norm_round`` defaults to the reference's dtype
    behaviour: fp32 norms under CUDA autocast or for fp32 inputs, input-dtype norms for a
    half-precision ``x`` outside autocast.
    """
    del n_min, total_len
    H = int(alpha.shape[0])
    dh = head_dim if head_dim is not None else W_V.shape[0] // H
    if v is None:
        v = x @ W_V.T
    if norm_round is None:
        norm_round = x.dtype != torch.float32 and not torch.is_autocast_enabled("cuda")
    w = w_sizes.to(torch.int32)
    n_kv = v.reshape(x.shape[0], -1).shape[1] // dh
    vn = _norms_only(x, v, dh, norm_round)
    xn = vn[0]
    lmk, zx, zv = select_landmarks(xn, vn[1], w, alpha, cu_seqlens, int(k_lmk), H, "global", cu_list=cu_list,
                                   return_z=True)
    if n_kv != H:
        zv = zv.repeat_interleave(H // n_kv, dim=1)
    return lmk.long(), zx, zv


def _norms_only(x, v, head_dim, norm_round):
    T, dm = x.shape
    gw = torch.zeros(dm, dtype=x.dtype, device=x.device)
    gb = torch.zeros(1, dtype=x.dtype, device=x.device)
    _, xn, vn = window_signals(x, gw, gb, 1, 1, v, head_dim, norm_round)
    return xn, vn


# --------------------------------------------------------------------------- attention
def normalize_landmarks(lmk_indices, lmk_bias=None):
    """Each landmark set in the kernel's format: valid positions ascending, ``-1`` last
    (the reference leaves the order unspecified). The bias follows its landmark."""
    lmk = lmk_indices.to(torch.int32)
    key = torch.where(lmk < 0, torch.full_like(lmk, torch.iinfo(torch.int32).max), lmk)
    key, order = torch.sort(key, dim=-1, stable=True)
    lmk = torch.where(key == torch.iinfo(torch.int32).max, torch.full_like(key, -1), key).contiguous()
    bias = None
    if lmk_bias is not None:
        bias = torch.gather(lmk_bias.to(torch.float32), -1, order).contiguous()
    return lmk, bias


def dsalt_attention(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, *, lmk_block: int = 0, out_dtype=None,
                    cu_list=None, return_lse: bool = False):
    """Drop-in for ``dsalt_triton_attention(q, k, v, lmk_indices, lmk_bias, w_sizes,
    cu_seqlens)`` (``dsalt/kernels/dsalt_triton_attn.py:337-349``).

    ``q [T, H, D]``; ``k, v [T, H or H_kv, D]`` (grouped heads are indexed, not
    repeated); ``lmk_indices [H, n_sets, k]`` positions within the sequence (any order,
    ``-1`` = none); ``lmk_block`` > 0 gives one set per ``lmk_block`` queries. The result
    is fp32 like the reference (values rounded to the input dtype when the input is
    bf16/fp16, as the reference stores its output before widening); pass ``out_dtype``
    to skip the widening. fp32 inputs run in fp32 on CUDA cores.
    """
    _cuda(q, k, v, lmk_indices, w_sizes, cu_seqlens)
    T, H, D = q.shape
    if k.shape[-1] != D or v.shape != k.shape:
        raise ValueError("k and v must be [T, H_kv, D] with the head_dim of q")
    n_kv = k.shape[1]
    dt = q.dtype
    if k.dtype != dt or v.dtype != dt:
        raise TypeError("q, k, v must share a dtype")
    qc = q if (q.stride(2) == 1 and q.stride(1) == D) else q.contiguous()
    kc = k.contiguous() if not (k.stride(2) == 1 and k.stride(1) == D) else k
    vc = v.contiguous() if not (v.stride(2) == 1 and v.stride(1) == D) else v
    if kc.stride(0) != vc.stride(0):
        kc, vc = kc.contiguous(), vc.contiguous()
    cu_h = _host_cu(cu_seqlens, cu_list)
    S = len(cu_h) - 1
    maxL = max([cu_h[i + 1] - cu_h[i] for i in range(S)] + [0])
    lmk, bias = normalize_landmarks(lmk_indices, lmk_bias)
    kl = int(lmk.shape[-1])
    odt = out_dtype if out_dtype is not None else (dt if dt != torch.float32 else torch.float32)
    out = torch.empty(T, H, D, dtype=odt, device=q.device)
    lse = torch.empty(T, H, dtype=torch.float32, device=q.device) if return_lse else None
    ws_n = L.query("dsalt_attention_workspace_bytes", T, S, H, kl, int(lmk_block))
    ws = _workspace(ws_n, q.device)
    L.call("dsalt_attention_fwd", _ptr(qc), _ptr(kc), _ptr(vc), _dt(qc), T, H, n_kv, D, qc.stride(0), kc.stride(0),
           _ptr(w_sizes.to(torch.int32).contiguous()), _ptr(lmk), _ptr(bias), kl, int(lmk_block),
           _ptr(_cu_i32(cu_seqlens)), S, maxL, _ptr(out), _dt(out), _ptr(lse), _ptr(ws), ws.numel(), _stream())
    if out_dtype is None:
        out = out.float()
    return (out, lse) if return_lse else out


def dsalt_attention_backward(grad_out, q, k, v, out, lse, lmk_indices, lmk_bias, w_sizes, cu_seqlens, *,
                             lmk_block: int = 0, cu_list=None):
    """Drop-in for ``dsalt_triton_backward`` (``dsalt/kernels/dsalt_triton_bwd.py:219-323``):
    ``(dq [T,H,D], dk [T,H_kv,D], dv [T,H_kv,D], d_bias [H,n_sets,k])``, all fp32.

    ``out`` is the forward's output (its values in the input dtype, as the reference keeps
    them) and ``lse`` its log-sum-exp (``dsalt_attention(..., return_lse=True)``);
    ``grad_out`` is taken in the input dtype for bf16/fp16 inputs, as the reference's
    ``do_f``. ``d_bias`` follows the caller's slot order of ``lmk_indices``."""
    _cuda(q, k, v, out, grad_out, lse, lmk_indices, w_sizes, cu_seqlens)
    T, H, D = q.shape
    n_kv = k.shape[1]
    dt = q.dtype
    qc = q if (q.stride(2) == 1 and q.stride(1) == D) else q.contiguous()
    kc = k.contiguous() if not (k.stride(2) == 1 and k.stride(1) == D) else k
    vc = v.contiguous() if not (v.stride(2) == 1 and v.stride(1) == D) else v
    if kc.stride(0) != vc.stride(0):
        kc, vc = kc.contiguous(), vc.contiguous()
    do = grad_out.to(dt if dt != torch.float32 else torch.float32).contiguous()
    oc = out.contiguous()
    cu_h = _host_cu(cu_seqlens, cu_list)
    S = len(cu_h) - 1
    lmk, bias = normalize_landmarks(lmk_indices, lmk_bias)
    kl = int(lmk.shape[-1])
    n_sets = int(lmk.shape[1])
    dq = torch.empty(T, H, D, dtype=torch.float32, device=q.device)
    dk = torch.empty(T, n_kv, D, dtype=torch.float32, device=q.device)
    dv = torch.empty(T, n_kv, D, dtype=torch.float32, device=q.device)
    db = torch.empty(H, n_sets, kl, dtype=torch.float32, device=q.device)
    ws = _workspace(L.query("dsalt_attention_bwd_workspace_bytes", T, S), q.device)
    L.call("dsalt_attention_bwd", _ptr(qc), _ptr(kc), _ptr(vc), _dt(qc), T, H, n_kv, D, qc.stride(0), kc.stride(0),
           _ptr(oc), _dt(oc), _ptr(do), _dt(do), _ptr(lse.contiguous()), _ptr(w_sizes.to(torch.int32).contiguous()),
           _ptr(lmk), _ptr(bias), kl, int(lmk_block), n_sets, _ptr(_cu_i32(cu_seqlens)), S, _ptr(dq), _ptr(dk),
           _ptr(dv), _ptr(db), _ptr(ws), ws.numel(), _stream())
    # back to the caller's slot order (normalize_landmarks sorted each set)
    raw = lmk_indices.to(torch.int32)
    key = torch.where(raw < 0, torch.full_like(raw, torch.iinfo(torch.int32).max), raw)
    order = torch.sort(key, dim=-1, stable=True).indices
    d_bias = torch.empty_like(db).scatter_(-1, order, db)
    return dq, dk, dv, d_bias


class DSALTAttentionFunction(torch.autograd.Function):
    """Autograd of the sparse attention (``DSALTAttentionFunction``,
    ``dsalt/kernels/dsalt_triton_attn.py:257-327``): the forward kernel with its
    log-sum-exp, the backward kernel for ``q``, ``k``, ``v`` and the landmark bias."""

    @staticmethod
    def forward(ctx, q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, lmk_block, cu_list):
        out_raw, lse = dsalt_attention(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, lmk_block=lmk_block,
                                       out_dtype=q.dtype, cu_list=cu_list, return_lse=True)
        ctx.save_for_backward(q, k, v, out_raw, lse, lmk_indices, lmk_bias if lmk_bias is not None else q.new_empty(0),
                              w_sizes, cu_seqlens)
        ctx.has_bias = lmk_bias is not None
        ctx.lmk_block, ctx.cu_list = lmk_block, cu_list
        return out_raw.float()

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out_raw, lse, lmk, bias, w, cu = ctx.saved_tensors
        dq, dk, dv, db = dsalt_attention_backward(grad_out, q, k, v, out_raw, lse, lmk, bias if ctx.has_bias else None,
                                                  w, cu, lmk_block=ctx.lmk_block, cu_list=ctx.cu_list)
        d_bias = db.to(bias.dtype) if ctx.has_bias else None
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, d_bias, None, None, None, None


def dsalt_attention_autograd(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, *, lmk_block: int = 0,
                             cu_list=None):
    """``dsalt_triton_attention`` with gradients (``dsalt_triton_attn.py:337-349``): fp32
    output, differentiable in ``q``, ``k``, ``v`` and ``lmk_bias``."""
    return DSALTAttentionFunction.apply(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, int(lmk_block), cu_list)


def train_attention_forward(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win: float, win_edge: float, *,
                            out_dtype=None, cu_list=None):
    """Forward of the soft-selector training attention (``_train_fwd_kernel``,
    ``dsalt/kernels/dsalt_triton_train.py:74-217``): ``(out [T,H,D], lse [T,H])``. ``w_cont [T]``
    continuous widths, ``lmk_pos [H, S, k]`` one landmark set per sequence (any order, ``-1``
    = none), ``lmk_logw [H, S, k]`` their log-weights. ``out`` is in ``out_dtype`` (default:
    the input dtype). bf16 / fp16 inputs with ``win_edge <= 4`` run on the tensor cores (P
    rounded to the input dtype for P·V, as the reference's ``tl.dot``), fp32 inputs on CUDA
    cores in fp32."""
    _cuda(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens)
    T, H, D = q.shape
    n_kv = k.shape[1]
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    cu_h = _host_cu(cu_seqlens, cu_list)
    S = len(cu_h) - 1
    kl = int(lmk_pos.shape[-1])
    out = torch.empty(T, H, D, dtype=out_dtype or q.dtype, device=q.device)
    lse = torch.empty(T, H, dtype=torch.float32, device=q.device)
    ws = _workspace(L.query("dsalt_train_attention_fwd_workspace_bytes", T, H, S, kl), q.device)
    L.call("dsalt_train_attention_fwd", _ptr(qc), _ptr(kc), _ptr(vc), _dt(qc), T, H, n_kv, D, qc.stride(0),
           kc.stride(0), _ptr(w_cont.float().contiguous()), _ptr(lmk_pos.to(torch.int32).contiguous()),
           _ptr(lmk_logw.float().contiguous()), kl, _ptr(_cu_i32(cu_seqlens)), S, float(tau_win), float(win_edge),
           _ptr(out), _dt(out), _ptr(lse), _ptr(ws), ws.numel(), _stream())
    return out, lse


def train_attention_backward(grad_out, q, k, v, out, lse, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win: float,
                             win_edge: float, *, cu_list=None):
    """Backward of :func:`train_attention_forward` (``_train_bwd_*``,
    ``dsalt_triton_train.py:220-490``): ``(dq, dk [T,H_kv,D], dv, d_logw [H,S,k], d_w [T])``,
    fp32; ``d_w`` is the gradient of the continuous widths summed over heads."""
    _cuda(q, k, v, out, grad_out, lse, lmk_pos, lmk_logw, w_cont, cu_seqlens)
    T, H, D = q.shape
    n_kv = k.shape[1]
    dt = q.dtype
    qc, kc, vc, oc = q.contiguous(), k.contiguous(), v.contiguous(), out.contiguous()
    do = grad_out.to(dt).contiguous()
    cu_h = _host_cu(cu_seqlens, cu_list)
    S = len(cu_h) - 1
    kl = int(lmk_pos.shape[-1])
    dq = torch.empty(T, H, D, dtype=torch.float32, device=q.device)
    dk = torch.empty(T, n_kv, D, dtype=torch.float32, device=q.device)
    dv = torch.empty(T, n_kv, D, dtype=torch.float32, device=q.device)
    dlw = torch.empty(H, S, kl, dtype=torch.float32, device=q.device)
    dw = torch.empty(T, dtype=torch.float32, device=q.device)
    ws = _workspace(L.query("dsalt_attention_bwd_workspace_bytes", T, S), q.device)
    L.call("dsalt_train_attention_bwd", _ptr(qc), _ptr(kc), _ptr(vc), _dt(qc), T, H, n_kv, D, qc.stride(0),
           kc.stride(0), _ptr(oc), _dt(oc), _ptr(do), _dt(do), _ptr(lse.contiguous()),
           _ptr(w_cont.float().contiguous()), _ptr(lmk_pos.to(torch.int32).contiguous()),
           _ptr(lmk_logw.float().contiguous()), kl, _ptr(_cu_i32(cu_seqlens)), S, float(tau_win), float(win_edge),
           _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dlw), _ptr(dw), _ptr(ws), ws.numel(), _stream())
    return dq, dk, dv, dlw, dw


class DSALTTrainFunction(torch.autograd.Function):
    """``DSALTTrainFunction`` (``dsalt_triton_train.py:583-762``): fp32 output,
    gradients for ``q``, ``k``, ``v``, the landmark log-weights (to alpha) and the continuous
    widths (to ``win_gate``)."""

    @staticmethod
    def forward(ctx, q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge, n_max, cu_list=None):
        del n_max  # the reference's tile bound; the band here comes from w_cont itself
        out, lse = train_attention_forward(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge,
                                           cu_list=cu_list)
        ctx.save_for_backward(q, k, v, out, lse, lmk_pos, lmk_logw, w_cont, cu_seqlens)
        ctx.tau_win, ctx.win_edge, ctx.cu_list = float(tau_win), float(win_edge), cu_list
        return out.float()

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out, lse, lmk_pos, lmk_logw, w_cont, cu = ctx.saved_tensors
        dq, dk, dv, dlw, dw = train_attention_backward(grad_out, q, k, v, out, lse, lmk_pos, lmk_logw, w_cont, cu,
                                                       ctx.tau_win, ctx.win_edge, cu_list=ctx.cu_list)
        od = q.dtype
        return (dq.to(od), dk.to(k.dtype), dv.to(v.dtype), None, dlw.to(lmk_logw.dtype), dw.to(w_cont.dtype),
                None, None, None, None, None)


def dsalt_train_attention(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win=1.0, win_edge=4.0, n_max=256,
                          cu_list=None):
    """Drop-in for ``dsalt_triton_train_attention`` (``dsalt_triton_train.py:771-782``): differentiable
    in ``q``, ``k``, ``v``, ``lmk_logw`` and ``w_cont``."""
    return DSALTTrainFunction.apply(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge,
                                             n_max, cu_list)


# --------------------------------------------------------------------------- fused core
def core_forward(x, gate_weight, gate_bias, n_min, n_max, alpha, q, k, v, k_lmk, cu_seqlens, *, mode="global",
                 block=512, norm_round=False, out_dtype=None, cu_list=None, return_aux=False, workspace=None,
                 out=None, logit=None):
    """Widths, selection and attention in one C call (``dsalt_core_forward``).

    ``v`` ([T, n_kv, D]) is used both as attention values and for the value norms, so
    it must equal ``x·W_Vᵀ`` (no ``v_proj`` bias). ``logit`` is the optional caller-computed
    ``win_gate`` logit of :func:`window_signals`. Returns the attention output
    ``[T, H, D]`` (``out_dtype``, default the input dtype) and, with ``return_aux``, the
    widths and landmark sets.
    """
    _cuda(x, gate_weight, gate_bias, alpha, q, k, v, cu_seqlens, logit)
    T, H, D = q.shape
    n_kv = k.shape[1]
    cu_h = _host_cu(cu_seqlens, cu_list)
    S = len(cu_h) - 1
    maxL = max([cu_h[i + 1] - cu_h[i] for i in range(S)] + [0])
    m = L.SELECT_GLOBAL if mode == "global" else L.SELECT_BLOCK_CAUSAL
    n_sets = S if m == L.SELECT_GLOBAL else n_block_sets(cu_h, block)
    dev = q.device
    gw = gate_weight.reshape(-1).contiguous()
    gb = gate_bias.reshape(-1).to(gw.dtype).contiguous()
    odt = out_dtype or q.dtype
    if out is None:
        out = torch.empty(T, H, D, dtype=odt, device=dev)
    w = torch.empty(T, dtype=torch.int32, device=dev) if return_aux else None
    lmk = torch.empty(H, n_sets, k_lmk, dtype=torch.int32, device=dev) if return_aux else None
    need = L.query("dsalt_core_workspace_bytes", m, T, S, maxL, H, n_kv, D, k_lmk, block)
    ws = workspace if (workspace is not None and workspace.numel() >= need) else _workspace(need, dev)
    lin = _logit_in(logit, T, gw.dtype)
    L.call("dsalt_core_forward", m, _ptr(x), _dt(x), x.shape[1], x.stride(0), _ptr(gw), _ptr(gb), _dt(gw), _ptr(lin),
           int(n_min), int(n_max), _ptr(alpha.float().contiguous()), L.NORM_INPUT if norm_round else L.NORM_F32,
           _ptr(q), _ptr(k), _ptr(v), _dt(q), H, n_kv, D, q.stride(0), k.stride(0), int(k_lmk), int(block),
           _ptr(_cu_i32(cu_seqlens)), S, T, maxL, _ptr(out), _dt(out), _ptr(w), _ptr(lmk), _ptr(ws), ws.numel(),
           _stream())
    if return_aux:
        return out, w, lmk
    return out


def core_workspace_bytes(T, n_seqs, max_seqlen, n_heads, n_kv, head_dim, k_lmk, mode="global", block=512) -> int:
    m = L.SELECT_GLOBAL if mode == "global" else L.SELECT_BLOCK_CAUSAL
    return L.query("dsalt_core_workspace_bytes", m, T, n_seqs, max_seqlen, n_heads, n_kv, head_dim, k_lmk, block)


def device_status(clear: bool = True) -> int:
    import ctypes
    st = ctypes.c_int(0)
    L.call("dsalt_device_status", ctypes.byref(st), 1 if clear else 0, _stream())
    return int(st.value)


def scale_for(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# --------------------------------------------------------------------------- sequence shards
def select_block_range(xnorm, vnorm, w, alpha, k_lmk: int, n_heads: int, block: int, set_lo: int, set_hi: int,
                       workspace=None):
    """Block-causal landmark sets ``[set_lo, set_hi)`` of one sequence whose per-position
    signals (``xnorm [L]``, ``vnorm [L, n_kv]``, ``w [L]``) are all given (``dsalt_select_block_range``).
    Returns ``[n_heads, set_hi - set_lo, k_lmk]`` int32, the same sets as
    :func:`select_landmarks` in ``block_causal`` mode."""
    _cuda(xnorm, vnorm, w, alpha)
    Lseq = xnorm.shape[0]
    n_kv = vnorm.shape[1]
    out = torch.empty(n_heads, set_hi - set_lo, k_lmk, dtype=torch.int32, device=xnorm.device)
    n = L.query("dsalt_select_block_range_workspace_bytes", Lseq, n_heads, n_kv, k_lmk, block, set_hi)
    ws = workspace if workspace is not None and workspace.numel() >= n else _workspace(n, xnorm.device)
    L.call("dsalt_select_block_range", _ptr(xnorm.contiguous()), _ptr(vnorm.contiguous()),
           _ptr(w.to(torch.int32).contiguous()), _ptr(alpha.float().contiguous()), Lseq, n_heads, n_kv, k_lmk, block,
           set_lo, set_hi, _ptr(out), _ptr(ws), ws.numel(), _stream())
    return out


def select_shard_workspace_bytes(seq_len: int, n_heads: int, n_kv: int, k_lmk: int, block: int) -> int:
    return L.query("dsalt_select_shard_workspace_bytes", seq_len, n_heads, n_kv, k_lmk, block)


def select_shard(phase: int, xnorm, vnorm, w, alpha, k_lmk: int, n_heads: int, block: int, rank: int, n_ranks: int,
                 workspace, peer_workspaces, lmk_out=None):
    """One phase (1-4) of the rank-distributed block-causal selection (``dsalt_select_shard``).

    ``xnorm [L]``, ``vnorm [L, n_kv]``, ``w [L]`` are whole-sequence arrays holding (at least)
    this rank's shard; ``workspace`` is this rank's, ``peer_workspaces`` an int64 device
    tensor of every rank's workspace pointer. Phases run in order with a cross-GPU barrier
    between them; phase 4 writes ``lmk_out [n_heads, blocks per rank, k_lmk]`` (allocated
    when not given) and returns it."""
    _cuda(xnorm, vnorm, w, alpha, workspace, peer_workspaces)
    Lseq = int(xnorm.shape[0])
    n_kv = int(vnorm.shape[1])
    if phase == 4 and lmk_out is None:
        cpr = Lseq // block // n_ranks
        lmk_out = torch.empty(n_heads, cpr, k_lmk, dtype=torch.int32, device=xnorm.device)
    L.call("dsalt_select_shard", int(phase), _ptr(xnorm), _ptr(vnorm), _ptr(w), _ptr(alpha), Lseq, n_heads, n_kv,
           int(k_lmk), int(block), int(rank), int(n_ranks), _ptr(workspace), workspace.numel(), _ptr(peer_workspaces),
           _ptr(lmk_out), _stream())
    return lmk_out


def attention_sharded(q, k, v, q_pos0: int, kv_pos0: int, seq_len: int, w, lmk, lmk_block: int, lmk_k_src,
                      lmk_v_src, rows_per_src: int, *, lmk_bias=None, out=None, workspace=None):
    """One rank's share of a sequence-sharded attention (``dsalt_attention_fwd_sharded``).

    ``q [q_rows, H, D]`` are positions ``[q_pos0, q_pos0 + q_rows)``; ``k, v [kv_rows, H_kv, D]``
    positions ``[kv_pos0, kv_pos0 + kv_rows)`` (the shard plus its window halo); ``w [seq_len]``;
    ``lmk [H, n_local_sets, k]`` ascending with -1 last; ``lmk_k_src`` / ``lmk_v_src``: int64
    device tensors of the ranks' K / V shard base pointers. Returns ``out [q_rows, H, D]``
    in the input dtype."""
    _cuda(q, k, v, w, lmk, lmk_k_src, lmk_v_src)
    q_rows, H, D = q.shape
    n_kv = k.shape[1]
    if q.stride(2) != 1 or q.stride(1) != D or k.stride(2) != 1 or k.stride(1) != D or k.stride(0) != v.stride(0):
        raise ValueError("q, k, v must have contiguous heads and k, v the same token stride")
    if out is None:
        out = torch.empty(q_rows, H, D, dtype=q.dtype, device=q.device)
    n = L.query("dsalt_attention_sharded_workspace_bytes", q_rows, H, int(lmk.shape[-1]), int(lmk_block), D)
    ws = workspace if workspace is not None and workspace.numel() >= n else _workspace(n, q.device)
    bias = None if lmk_bias is None else lmk_bias.float().contiguous()
    L.call("dsalt_attention_fwd_sharded", _ptr(q), _ptr(k), _ptr(v), _dt(q), q_rows, H, n_kv, D, q.stride(0),
           k.stride(0), q_pos0, kv_pos0, k.shape[0], seq_len, _ptr(w), _ptr(lmk), _ptr(bias), int(lmk.shape[-1]),
           int(lmk_block), _ptr(lmk_k_src), _ptr(lmk_v_src), rows_per_src, _ptr(out), _dt(out), None, _ptr(ws),
           ws.numel(), _stream())
    return out


def ipc_export(t: torch.Tensor):
    """(64-byte CUDA IPC handle, byte offset) of a CUDA tensor's data pointer."""
    import ctypes
    h = (ctypes.c_char * 64)()
    off = ctypes.c_int64(0)
    L.call("dsalt_ipc_export", ctypes.c_void_p(t.data_ptr()), h, ctypes.byref(off))
    return bytes(h), int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Device pointer (int) of another process's tensor on this node (plain peer mapping)."""
    import ctypes
    p = ctypes.c_void_p(0)
    buf = ctypes.create_string_buffer(handle, 64)
    L.call("dsalt_ipc_open", buf, offset, ctypes.byref(p))
    return int(p.value)


def ipc_close(ptr: int, offset: int) -> None:
    import ctypes
    L.call("dsalt_ipc_close", ctypes.c_void_p(ptr), offset)
