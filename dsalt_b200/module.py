"""``DSALTAttention`` with the reference's constructor, parameters and forward signature
(``dsalt/modules/dsalt_attention.py:147-369``), whose packed path (inference and
training) runs on the B200 kernels of this package.

Same state-dict keys (``q_proj``, ``k_proj``, ``v_proj``, ``out_proj``, ``win_gate``,
``alpha_w``), same RoPE cache and half-split rotation, same ``(out, aux)`` return. The
packed path (``cu_seqlens`` given) replaces ``_packed``'s inference branch
(``:610-641``): widths, landmark selection and the sparse attention run in CUDA, the
projections, RoPE and ``out_proj`` stay library GEMMs/elementwise ops. Grouped kv heads
are indexed by the kernels instead of being repeated (``_repeat_kv``, ``:254-268``).

``selection="block_causal"`` selects per ``block`` queries from earlier positions only,
as ``results/causal_landmark_check.py``'s ``"block"`` mode does.

In eval mode ``_last_P`` holds the dense attention matrix ``[H, T0, T0]`` of the first
packed sequence, rebuilt as the reference does for its analysis metrics (``:636-704``:
landmarks of that sequence alone by ``compute_landmark_indices``, the window ∪ landmark
mask, softmax of the masked scores in the caller's dtype). As in the reference it is
collected unless ``_collect_last_P`` is set to False; it costs O(T0²) memory, so callers
that need only the output (the decoder stack in :mod:`dsalt_b200.model`) turn it off.

In training mode the packed path is the reference's Triton training branch
(``_packed_train_triton`` / ``_train_selectors``, ``:438-487``): continuous widths
``w̃ = n_min + σ(win_gate(x))·(n_max − n_min)``, landmarks selected without gradient on
``floor(w̃)`` by the global selection, their log-weights ``log σ(s/τ_lmk)`` from the hybrid
scores (differentiable in ``alpha_w``, ``x`` and ``v_proj``), and the soft-selector attention
of :func:`dsalt_b200.ops.dsalt_train_attention`, whose backward carries the gradients of the
soft window edge to ``win_gate`` and of the landmark weights to ``alpha_w``.

Out of scope (raise): the batched ``[B, T, d]`` path, and training with
``selection="block_causal"`` (the training kernel takes one landmark set per sequence, as
the reference's does).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import library  # noqa: F401  (registers torch.ops.dsalt_b200.*)
from . import ops


def hybrid_scores_per_head(x, W_V, alpha, n_heads, dh):
    """Per-head hybrid score ``α·z_v + (1 − α)·z_x`` over all ``T`` rows of ``x``
    (``dsalt/kernels/landmark_tokens_ker.py:19-61``), differentiable in ``x``, ``W_V`` and
    ``alpha``: the training path's landmark weights. The hard selection uses the CUDA
    selection kernels instead."""
    T = x.shape[0]
    x_norm = x.norm(dim=-1).float()
    z_x = (x_norm - x_norm.mean()) / x_norm.std().clamp(min=1e-6)
    n_kv = W_V.shape[0] // dh
    xwv = (x @ W_V.T).view(T, n_kv, dh).norm(dim=-1).float()
    z_v = (xwv - xwv.mean(0, keepdim=True)) / xwv.std(0, keepdim=True).clamp(min=1e-6)
    if n_kv != n_heads:
        z_v = z_v.repeat_interleave(n_heads // n_kv, dim=1)
    return alpha * z_v + (1.0 - alpha) * z_x.unsqueeze(1)


def build_rope_cache(seq_len, head_dim, device, dtype=torch.float32, base=10000.0, scale=1.0):
    """RoPE ``(cos, sin)`` ``[seq_len, head_dim]`` (same numbers as the reference's
    ``build_rope_cache``, ``dsalt/kernels/window_utils.py:91-106``)."""
    theta = 1.0 / (base ** (torch.arange(0, head_dim, 2, device=device, dtype=dtype) / head_dim))
    positions = torch.arange(seq_len, device=device, dtype=dtype) / scale
    emb = torch.cat([torch.outer(positions, theta)] * 2, dim=-1)
    return emb.cos(), emb.sin()


def apply_rotary_emb(q, k, cos, sin):
    """Half-split rotary embedding, op for op as the reference's ``apply_rotary_emb``
    (``dsalt/kernels/window_utils.py:73-88``)."""
    half = q.shape[-1] // 2

    def rot(x):
        return torch.cat([-x[..., half:], x[..., :half]], dim=-1)

    return q * cos + rot(q) * sin, k * cos + rot(k) * sin


class DSALTAttention(nn.Module):
    def __init__(self, d_model, n_heads, n_min, n_max, k_lmk, max_seq_len, dropout=0.0, yarn_scale=1.0,
                 layer_idx=0, n_kv_heads=None, qkv_bias=False, rope_base=10000.0, selection="global", block=512):
        super().__init__()
        assert d_model % n_heads == 0
        if selection not in ("global", "block_causal"):
            raise ValueError("selection must be 'global' or 'block_causal'")
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.n_kv_heads = n_kv_heads if n_kv_heads is not None else n_heads
        assert n_heads % self.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads"
        self.n_rep = n_heads // self.n_kv_heads
        self.kv_dim = self.n_kv_heads * self.head_dim
        self.n_min, self.n_max, self.k_lmk = n_min, n_max, k_lmk
        self.max_seq_len = max_seq_len
        self.dropout = dropout
        self.yarn_scale = yarn_scale
        self.rope_base = rope_base
        self.layer_idx = layer_idx
        self.selection = selection
        self.block = block
        self.q_proj = nn.Linear(d_model, d_model, bias=qkv_bias)
        self.k_proj = nn.Linear(d_model, self.kv_dim, bias=qkv_bias)
        self.v_proj = nn.Linear(d_model, self.kv_dim, bias=qkv_bias)
        self.out_proj = nn.Linear(d_model, d_model, bias=False)
        self.win_gate = nn.Linear(d_model, 1, bias=True)
        self.alpha_w = nn.Parameter(torch.full((n_heads,), math.log(0.6 / 0.4)))
        self.tau_win, self.tau_lmk, self.win_edge = 1.0, 2.0, 4
        self._last_P = None
        self._collect_last_P = True  # the reference's default (dsalt_attention.py:639)
        cos, sin = build_rope_cache(max_seq_len, self.head_dim, torch.device("cpu"), base=rope_base, scale=yarn_scale)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def _alpha(self):
        return torch.sigmoid(self.alpha_w)

    def forward(self, x, cu_seqlens=None, max_seqlen=None, rope_cs=None, cu_list=None):
        """Packed forward ``-> (out [T, d_model], aux 0)``: the inference kernels in eval
        mode, the differentiable soft-selector attention in training mode. ``max_seqlen`` is
        accepted for signature compatibility and not needed: the kernels derive every
        sequence length from ``cu_seqlens`` (or ``cu_list``). Under ``torch.compile`` pass
        ``cu_list`` (the host list of ``cu_seqlens``): reading it from the device tensor is a
        host synchronisation, which a compiled graph cannot contain."""
        if cu_seqlens is None:
            raise NotImplementedError("dsalt_b200 implements the packed path; pass cu_seqlens")
        if self.training:
            return self._packed_train(x, cu_seqlens, x.shape[0], x.device, rope_cs, cu_list)
        return self._packed(x, cu_seqlens, x.shape[0], x.device, rope_cs, cu_list)

    def _qkv(self, x, cu_h, total_len, device, rope_cs):
        """Projections and RoPE (``_packed`` ``:566-589``); kv heads stay grouped."""
        T, H, Hkv, D = total_len, self.n_heads, self.n_kv_heads, self.head_dim
        q = self.q_proj(x).view(T, H, D)
        k = self.k_proj(x).view(T, Hkv, D)
        v = self.v_proj(x).view(T, Hkv, D)
        if rope_cs is None:
            pos = torch.cat([torch.arange(cu_h[i + 1] - cu_h[i], device=device) for i in range(len(cu_h) - 1)])
            cos, sin = self.rope_cos.to(device)[pos], self.rope_sin.to(device)[pos]
        else:
            cos, sin = rope_cs
        cos, sin = cos.to(q.dtype), sin.to(q.dtype)
        q, k = apply_rotary_emb(q, k, cos.unsqueeze(1), sin.unsqueeze(1))
        return q, k, v

    def _packed_train(self, x, cu_seqlens, total_len, device, rope_cs=None, cu_list=None):
        """Training forward (``_packed`` ``:596-605`` → ``_packed_train_triton`` ``:438-455``)."""
        if self.selection != "global":
            raise NotImplementedError("training takes one landmark set per sequence: selection='global'")
        T = total_len
        cu_h = ops._host_cu(cu_seqlens, cu_list)
        q, k, v = self._qkv(x, cu_h, T, device, rope_cs)
        w_cont, lmk_pos, lmk_logw = self._train_selectors(x, cu_seqlens, T, cu_h)
        out = ops.dsalt_train_attention(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win=self.tau_win,
                                        win_edge=float(self.win_edge), n_max=self.n_max, cu_list=cu_h)
        self._last_P = None
        aux = torch.zeros((), device=x.device, dtype=x.dtype)
        return self.out_proj(out.view(T, self.d_model).to(self.out_proj.weight.dtype)), aux

    def _train_selectors(self, x, cu_seqlens, total_len, cu_h):
        """``(w_cont [T], lmk_pos [H, S, k], lmk_logw [H, S, k])`` (``_train_selectors``
        ``:457-487``): the continuous widths and the landmark log-weights carry gradients, the
        landmark positions do not."""
        H, D = self.n_heads, self.head_dim
        w_cont = self.n_min + torch.sigmoid(self.win_gate(x).squeeze(-1)) * (self.n_max - self.n_min)
        alpha = self._alpha()
        with torch.no_grad():
            w_disc = w_cont.floor().clamp(min=1)
            lmk_pos, _, _ = ops.compute_landmark_indices(x.detach(), self.v_proj.weight.detach(),
                                                         alpha.detach().float(), w_disc, cu_seqlens, self.k_lmk,
                                                         self.n_min, total_len, cu_h, head_dim=D)
        scores = hybrid_scores_per_head(x, self.v_proj.weight, alpha, H, D)              # [T, H]
        return w_cont, lmk_pos, self._landmark_logw(scores, lmk_pos, cu_h)

    def _landmark_logw(self, scores, lmk_pos, cu_h):
        """``log σ(s/τ_lmk)`` of each selected landmark's hybrid score, ``-inf`` in empty slots
        (``_train_selectors`` ``:481-486``): ``scores [T, H]``, ``lmk_pos [H, S, k]`` positions
        within each sequence, ``cu_h`` the host list of ``cu_seqlens``."""
        H = self.n_heads
        starts = torch.tensor(cu_h[:-1], dtype=torch.long, device=scores.device)
        abs_pos = starts[None, :, None] + lmk_pos.long().clamp(min=0)                    # [H, S, k]
        s_sel = scores[abs_pos, torch.arange(H, device=scores.device)[:, None, None]]
        lmk_logw = torch.log(torch.sigmoid(s_sel / self.tau_lmk).clamp(min=1e-20))
        return torch.where(lmk_pos >= 0, lmk_logw, torch.full_like(lmk_logw, float("-inf")))

    @torch.no_grad()
    def _packed(self, x, cu_seqlens, total_len, device, rope_cs=None, cu_list=None):
        T, H, Hkv, D = total_len, self.n_heads, self.n_kv_heads, self.head_dim
        cu_h = ops._host_cu(cu_seqlens, cu_list)
        q, k, v = self._qkv(x, cu_h, T, device, rope_cs)
        amp = torch.is_autocast_enabled("cuda") if x.is_cuda else False
        # the width logit comes from the same library op as the reference's
        # _window_continuous (win_gate(x), :275), so that the widths equal the reference's
        logit = self.win_gate(x).squeeze(-1)
        gdt = logit.dtype
        gw = self.win_gate.weight.to(gdt)
        gb = self.win_gate.bias.to(gdt)
        # value norms use x·W_Vᵀ, which is the v_proj output when there is no bias
        vs = v if self.v_proj.bias is None else F.linear(x, self.v_proj.weight.to(v.dtype))
        norm_round = (x.dtype != torch.float32) and not amp
        # the operators as registered torch.library ops: opaque nodes under torch.compile
        w, xn, vn = torch.ops.dsalt_b200.window_signals(x, gw, gb, self.n_min, self.n_max, vs, D, norm_round, logit)
        alpha = self._alpha().detach().float()
        mode = "global" if self.selection == "global" else "block_causal"
        lmk = torch.ops.dsalt_b200.select_landmarks(xn, vn, w, alpha, cu_seqlens, self.k_lmk, H, mode, self.block,
                                                    cu_h)
        out = torch.ops.dsalt_b200.dsalt_attention(q.contiguous(), k.contiguous(), v.contiguous(), lmk, None, w,
                                                   cu_seqlens, 0 if mode == "global" else self.block, cu_h, q.dtype)
        self._last_P = self._rebuild_last_P(x, q, k, w, alpha, cu_h) if self._collect_last_P else None
        aux = torch.zeros((), device=x.device, dtype=x.dtype)
        return self.out_proj(out.view(T, self.d_model).to(self.out_proj.weight.dtype)), aux

    @torch.no_grad()
    def _rebuild_last_P(self, x, q, k, w, alpha, cu_h):
        """Dense attention ``[H, T0, T0]`` of the first sequence (``dsalt_attention.py:643-702``):
        its landmarks selected on that sequence alone, query ``i`` attending to its window
        ``[i - w(i) + 1, i]`` and to every landmark ``j <= i``, softmax of the masked scaled
        scores. ``q`` / ``k`` are the post-RoPE projections in the compute dtype."""
        s0, e0 = int(cu_h[0]), int(cu_h[1])
        T0, H, dev = e0 - s0, self.n_heads, x.device
        q0 = q[s0:e0].transpose(0, 1)
        k0 = k[s0:e0].repeat_interleave(self.n_rep, dim=1).transpose(0, 1)
        w0 = w[s0:e0]
        cu0 = torch.tensor([0, T0], dtype=torch.int32, device=dev)
        lmk_idx, _, _ = ops.compute_landmark_indices(x[s0:e0].float(), self.v_proj.weight.float(), alpha.float(), w0,
                                                     cu0, self.k_lmk, self.n_min, T0, [0, T0],
                                                     head_dim=self.head_dim)
        rows = torch.arange(T0, device=dev)
        causal = rows.unsqueeze(0) <= rows.unsqueeze(1)                          # key j <= query i
        in_win = (rows.unsqueeze(0) >= rows.unsqueeze(1) - w0.long().unsqueeze(1) + 1) & causal
        lmk0 = lmk_idx[:, 0, :]                                                  # [H, k], -1 padded
        col_is_lmk = torch.zeros(H, T0 + 1, dtype=torch.bool, device=dev)
        col_is_lmk.scatter_(1, torch.where(lmk0 >= 0, lmk0, T0), True)          # -1 slots land in column T0
        full_mask = in_win.unsqueeze(0) | (col_is_lmk[:, :T0].unsqueeze(1) & causal.unsqueeze(0))
        sc = torch.matmul(q0, k0.transpose(-2, -1)) * (1.0 / math.sqrt(self.head_dim))
        additive = sc.new_full((H, T0, T0), float("-inf")).masked_fill_(full_mask, 0.0)
        return torch.softmax(sc + additive, dim=-1).detach()
