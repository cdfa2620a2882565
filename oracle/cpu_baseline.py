"""Timed CPU baseline: the reference's block-causal forward restated with torch CPU ops.

TEST/BENCH INFRASTRUCTURE ONLY (imported by ``bench.py``'s CPU-baseline legs).

Follows ``results/causal_landmark_check.py``: prefix statistics in float64 cumsums
(``_prefix_stats`` ``:82-85``, ``_std_at`` ``:88-92``), per-block top-k over the prefix
(``_select`` ``:95-113``) and the fp32 masked attention of ``_block_attention``
(``:119-147``), per 512-query block (``:183-186``). The masked-SDPA fallback of the
reference needs ``[T, T]`` masks and is infeasible at L=131072, so this is the CPU path
that is timed for that configuration.
"""
from __future__ import annotations

import math
import time

import torch


class BlockCausalCPU:
    def __init__(self, q, k, v, w, xn, vn, alpha, k_lmk, block=512):
        self.q = q.float()
        self.k = k.float()
        self.v = v.float()
        self.w = w.long()
        self.xn = xn.double()
        self.vn = vn.double()
        self.alpha = alpha.float()
        self.k_lmk = k_lmk
        self.B = block
        self.T, self.H, self.D = self.q.shape
        self.sx = (torch.cumsum(self.xn, 0), torch.cumsum(self.xn * self.xn, 0))
        self.sv = (torch.cumsum(self.vn, 0), torch.cumsum(self.vn * self.vn, 0))
        self.covered = torch.arange(self.T) < self.w
        self.scale = 1.0 / math.sqrt(self.D)

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
        return self.attend(self.select(b0), b0, b1)

    def time_sample(self, blocks):
        t0 = time.perf_counter()
        for b in blocks:
            self.run_block(b)
        dt = time.perf_counter() - t0
        tokens = sum(min(self.T, (b + 1) * self.B) - b * self.B for b in blocks)
        return tokens, dt
