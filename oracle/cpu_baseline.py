"""Timed CPU baselines: the reference's CPU paths restated with torch CPU ops.

TEST/BENCH INFRASTRUCTURE ONLY (imported by ``bench.py``'s CPU-baseline legs).

``masked_sdpa_step`` is the reference's non-Triton inference branch of ``_packed``
(``dsalt/modules/dsalt_attention.py:619-625``): widths, hybrid scores, the ``[T, T]``
window ∪ landmark mask and masked SDPA. ``BlockCausalCPU`` below is its block-causal path.

Follows ``results/causal_landmark_check.py``: token signals (``_token_signals``
``:68-79``: ``‖x‖``, value norms) and window widths
(``dsalt/modules/dsalt_attention.py:270-284``), prefix statistics in float64 cumsums
(``_prefix_stats`` ``:82-85``, ``_std_at`` ``:88-92``), per-block top-k over the prefix
(``_select`` ``:95-113``) and the fp32 masked attention of ``_block_attention``
(``:119-147``), per 512-query block (``:183-186``). The masked-SDPA fallback of the
reference needs ``[T, T]`` masks and is infeasible at L=131072, so this is the CPU path
that is timed for that configuration.

The sequence is processed as a stream of blocks: a step over blocks ``[b0, b1)`` computes
the signals and widths of those blocks' tokens, extends the prefix sums, then selects
and attends each block, so every step is charged exactly the work of its own tokens.
"""
from __future__ import annotations

import math
import time

import torch


class BlockCausalCPU:
    def __init__(self, x, gate_w, gate_b, n_min, n_max, q, k, v, alpha, k_lmk, block=512):
        self.x = x                      # [T, d_model] (bf16 as given)
        self.gw = gate_w.float()
        self.gb = float(gate_b.float().reshape(-1)[0])
        self.n_min, self.n_max = n_min, n_max
        self.q = q.float()
        self.k = k.float()
        self.v = v.float()
        self.alpha = alpha.float()
        self.k_lmk = k_lmk
        self.B = block
        self.T, self.H, self.D = self.q.shape
        self.n_kv = self.k.shape[1]
        self.scale = 1.0 / math.sqrt(self.D)
        self.reset()

    def reset(self):
        T = self.T
        self.w = torch.empty(T, dtype=torch.long)
        self.xn = torch.empty(T, dtype=torch.float64)
        self.vn = torch.empty(T, self.n_kv, dtype=torch.float64)
        self.sx = (torch.empty(T, dtype=torch.float64), torch.empty(T, dtype=torch.float64))
        self.sv = (torch.empty(T, self.n_kv, dtype=torch.float64), torch.empty(T, self.n_kv, dtype=torch.float64))
        self.covered = torch.empty(T, dtype=torch.bool)
        self.done = 0  # tokens whose signals and prefix sums exist

    def signals(self, t1):
        """Signals, widths and prefix sums of tokens [done, t1)."""
        t0 = self.done
        if t1 <= t0:
            return
        xs = self.x[t0:t1].float()
        logit = xs @ self.gw + self.gb
        w = torch.floor(self.n_min + torch.sigmoid(logit) * (self.n_max - self.n_min)).clamp(min=1).long()
        self.w[t0:t1] = w
        self.covered[t0:t1] = torch.arange(t0, t1) < w
        xn = xs.norm(dim=-1).double()
        vn = self.v[t0:t1].norm(dim=-1).double()
        self.xn[t0:t1] = xn
        self.vn[t0:t1] = vn
        for (S1, S2), val in ((self.sx, xn), (self.sv, vn)):
            c1 = torch.cumsum(val, 0)
            c2 = torch.cumsum(val * val, 0)
            if t0 > 0:
                c1 += S1[t0 - 1]
                c2 += S2[t0 - 1]
            S1[t0:t1] = c1
            S2[t0:t1] = c2
        self.done = t1

    @staticmethod
    def _std_at(S1, S2, n):
        mean = S1[n - 1] / n
        var = (S2[n - 1] - n * mean * mean) / max(n - 1, 1)
        return mean, var.clamp(min=0).sqrt().clamp(min=1e-6)

    def select(self, n):
        H, k = self.H, self.k_lmk
        out = torch.full((H, k), -1, dtype=torch.long)
        if n < 2:
            return out
        mx, sdx = self._std_at(*self.sx, n)
        mv, sdv = self._std_at(*self.sv, n)
        z_x = ((self.xn[:n] - mx) / sdx).float()
        z_v = ((self.vn[:n] - mv) / sdv).float()
        if z_v.shape[1] != H:
            z_v = z_v.repeat_interleave(H // z_v.shape[1], dim=1)
        scores = self.alpha * z_v + (1.0 - self.alpha) * z_x.unsqueeze(1)
        scores = scores.masked_fill(self.covered[:n].unsqueeze(1), float("-inf"))
        kk = min(k, n)
        val, idx = torch.topk(scores.T, kk, dim=1, sorted=False)
        out[:, :kk] = torch.where(torch.isfinite(val), idx, torch.full_like(idx, -1))
        return out

    def attend(self, lmk, b0, b1):
        H = self.H
        wb = self.w[b0:b1]
        lo = max(0, b0 - int(wb.max()) + 1)
        qb = self.q[b0:b1].transpose(0, 1)
        kw = self.k[lo:b1].transpose(0, 1)
        vw = self.v[lo:b1].transpose(0, 1)
        i = torch.arange(b0, b1).unsqueeze(1)
        j = torch.arange(lo, b1).unsqueeze(0)
        win_lo = i - wb.unsqueeze(1) + 1
        in_win = (j >= win_lo) & (j <= i)
        s_w = torch.matmul(qb, kw.transpose(-1, -2)) * self.scale
        s_w = s_w.masked_fill(~in_win.unsqueeze(0), float("-inf"))
        hidx = torch.arange(H).unsqueeze(1)
        safe = lmk.clamp(min=0)
        lk = self.k[safe, hidx]
        lv = self.v[safe, hidx]
        s_l = torch.einsum("hbd,hkd->hbk", qb, lk) * self.scale
        pos = lmk.unsqueeze(1)
        ok = (lmk >= 0).unsqueeze(1) & (pos <= i.unsqueeze(0)) & (pos < win_lo.unsqueeze(0))
        s_l = s_l.masked_fill(~ok, float("-inf"))
        p = torch.softmax(torch.cat([s_w, s_l], dim=-1), dim=-1)
        Kw = kw.shape[1]
        out = torch.matmul(p[..., :Kw], vw) + torch.matmul(p[..., Kw:], lv)
        return out.transpose(0, 1)

    def run_block(self, b):
        b0 = b * self.B
        b1 = min(self.T, b0 + self.B)
        self.signals(b1)
        return self.attend(self.select(b0), b0, b1)

    def time_blocks(self, b0, b1):
        """Stream blocks [b0, b1) (restarting the stream when b0 == 0); (tokens, seconds)."""
        if b0 == 0:
            self.reset()
        t0 = time.perf_counter()
        for b in range(b0, b1):
            self.run_block(b)
        dt = time.perf_counter() - t0
        return min(self.T, b1 * self.B) - b0 * self.B, dt


def masked_sdpa_step(x, gate_w, gate_b, n_min, n_max, xwv, alpha, q, k, v, k_lmk, cu):
    """The reference's masked-SDPA inference path on CPU, op for op in torch:

    * widths ``clamp(floor(n_min + σ(x·g + b)·(n_max − n_min)), min=1)``
      (``_window_sizes``, ``dsalt_attention.py:270-284``);
    * hybrid scores: ``z_x`` of ``‖x‖`` and ``z_v`` of the value norms over all packed tokens
      (unbiased std, clamp 1e-6), ``s = α·z_v + (1 − α)·z_x``
      (``hybrid_scores_per_head``, ``dsalt/kernels/landmark_tokens_ker.py:44-60``);
      ``xwv`` is ``x·W_Vᵀ`` ``[T, n_kv·D]`` (the value projection without bias);
    * the mask of ``_build_mask_packed`` (``dsalt_attention.py:96-144``): the causal window
      of each row (``build_local_window_mask_packed``, ``window_utils.py:40-70``) plus, for
      every row of a sequence, the union over heads of the sequence's top-k positions
      among tokens outside their own window;
    * ``sparse_attention_forward_packed`` (``dsalt/kernels/sparse_attn.py:29-56``): SDPA
      with the additive ``-inf`` mask.

    ``q, k, v`` are ``[T, H, D]`` (kv heads already repeated). Returns ``[T, H, D]``."""
    T, H, D = q.shape
    xf = x.float()
    w = torch.floor(n_min + torch.sigmoid(xf @ gate_w.float() + gate_b.float()) * (n_max - n_min)).clamp(min=1)
    x_norm = xf.norm(dim=-1)
    z_x = (x_norm - x_norm.mean()) / x_norm.std().clamp(min=1e-6)
    n_kv = xwv.shape[1] // D
    vn = xwv.float().view(T, n_kv, D).norm(dim=-1)
    z_v = (vn - vn.mean(0, keepdim=True)) / vn.std(0, keepdim=True).clamp(min=1e-6)
    if n_kv != H:
        z_v = z_v.repeat_interleave(H // n_kv, dim=1)
    scores = alpha * z_v + (1.0 - alpha) * z_x.unsqueeze(1)
    lens = torch.tensor([cu[i + 1] - cu[i] for i in range(len(cu) - 1)])
    starts = torch.tensor(cu[:-1])
    seq_ids = torch.repeat_interleave(torch.arange(len(cu) - 1), lens)
    seq_off = torch.arange(T) - starts[seq_ids]
    wl = w.long()
    lo = (seq_off - wl + 1).clamp(min=0) + starts[seq_ids]
    col = torch.arange(T)
    mask = (seq_ids[:, None] == seq_ids[None, :]) & (col[None, :] >= lo[:, None]) & (col[None, :] <= col[:, None])
    # the landmark columns as _build_mask_packed forms them (:119-142): scores padded per
    # sequence, top-k along positions, the union over heads scattered into every row
    s_masked = scores.masked_fill((seq_off < wl)[:, None], float("-inf"))
    n_seqs, max_len = len(cu) - 1, int(lens.max())
    score_pad = torch.full((n_seqs, max_len, H), float("-inf"))
    score_pad[seq_ids, seq_off] = s_masked
    vals, top = torch.topk(score_pad, min(k_lmk, max_len), dim=1, sorted=False)
    valid = vals > float("-inf")
    abs_lmk = (starts[:, None, None] + top).clamp(max=T - 1)
    for b in range(n_seqs):
        if not valid[b].any():
            continue
        a, e = cu[b], cu[b + 1]
        idx = abs_lmk[b][valid[b]].reshape(-1).unique()
        row_idx = torch.arange(a, e).unsqueeze(1).expand(-1, idx.shape[0])
        col_idx = idx.unsqueeze(0).expand(e - a, -1)
        mask[row_idx, col_idx] = True
    additive = torch.zeros(T, T, dtype=q.dtype).masked_fill(~mask, float("-inf"))
    o = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                         v.transpose(0, 1)[None], attn_mask=additive[None, None])
    return o[0].transpose(0, 1)
