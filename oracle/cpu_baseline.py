"""Timed CPU baseline: the reference's block-causal forward restated with torch CPU ops.

TEST/BENCH INFRASTRUCTURE ONLY (imported by ``bench.py``'s CPU-baseline legs).

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
