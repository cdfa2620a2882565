"""CPU oracle for the DSALT attention-forward hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
baseline legs of ``bench.py`` may import this module, and only as the checker or the
timed CPU baseline. The product path (``dsalt_b200``) never calls it and fails loudly
when its CUDA library is missing.

It restates, in numpy, the algorithm of the reference (LeonardoCofone/dsalt) for:

* the adaptive window width        (``dsalt/modules/dsalt_attention.py:270-284``)
* the per-token selection signals  (``dsalt/kernels/landmark_tokens_ker.py:47-52``)
* whole-sequence landmark scores   (``dsalt/kernels/landmark_tokens_ker.py:47-60``)
* whole-sequence landmark top-k    (``dsalt/kernels/selectors.py:75-134``)
* block-causal landmark selection  (``results/causal_landmark_check.py:68-113``)
* the sparse attention forward     (``dsalt/kernels/dsalt_triton_attn.py:27-169``,
  restated in PyTorch by the reference at ``results/causal_landmark_check.py:119-147``)
* the masked-SDPA CPU fallback     (``dsalt/modules/dsalt_attention.py:96-144`` and
  ``dsalt/kernels/sparse_attn.py:29-56``), used only as the timed CPU baseline.

Floating-point contract (what "bit-exact" means for the integer outputs):

* Sums whose order the reference leaves to a library (``x.norm``, ``mean``, ``std``,
  ``cumsum``) are defined here as correctly rounded: sums of squares are accumulated
  in float64 and rounded once to float32; the statistics use the correctly rounded
  float64 value of the exact sum (``math.fsum`` / exact integers here, double-double
  on the GPU). The reference's own reductions differ from these by a few ulps; the
  golden tests quantify that.
* Every other step replays the reference's op chain one IEEE operation at a time
  (no fused multiply-add), in the reference's dtypes.
* ``torch.topk(sorted=False)`` leaves the order and the tie-break unspecified; here the
  k largest scores are taken with ties broken towards the lower position, and the set
  is returned sorted by position with ``-1`` padding.
* The bf16 window chain uses CUDA's fp32 sigmoid ``1/(1+expf(-x))``; for the three bf16
  logits whose bf16 sigmoid depends on the last bit of ``expf`` the value measured on a
  B200 is used (``tests/golden/sigmoid_bf16_cuda.npz``) when it is available, and those
  logits are otherwise reported as ambiguous.

Parity of this oracle against the reference is pinned by ``tests/golden/`` (fixtures
produced by running the reference itself on CPU, see ``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np

F32 = np.float32
F64 = np.float64

_HERE = os.path.dirname(os.path.abspath(__file__))
_SIGMOID_TABLE_PATH = os.path.join(os.path.dirname(_HERE), "tests", "golden", "sigmoid_bf16_cuda.npz")


# --------------------------------------------------------------------------- #
# bf16 helpers
# --------------------------------------------------------------------------- #
def bf16_rne(a) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    a = np.asarray(a, dtype=F32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(F32)
    return np.where(np.isnan(a), a, out).astype(F32)


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(F32)


def f32_to_bf16_bits(a) -> np.ndarray:
    return (bf16_rne(a).view(np.uint32) >> 16).astype(np.uint16)


# --------------------------------------------------------------------------- #
# (a2) adaptive window width  -- dsalt/modules/dsalt_attention.py:270-284
# --------------------------------------------------------------------------- #
def window_logit(x: np.ndarray, g: np.ndarray, b: float, dtype: str) -> np.ndarray:
    """``win_gate(x)`` (``nn.Linear(d_model, 1)``, ``dsalt_attention.py:223,274``).

    The dot product is accumulated in float64 and rounded once to ``dtype`` (bf16 under
    autocast, else fp32) with the bias added before that rounding, as a GEMM epilogue
    does. ``x``, ``g`` and ``b`` already hold values of ``dtype``.
    """
    acc = np.asarray(x, dtype=F64) @ np.asarray(g, dtype=F64).reshape(-1) + F64(b)
    out = acc.astype(F32)
    if dtype == "bf16":
        # round the float64 value straight to bf16: first to the nearest float32 that
        # keeps the bf16 decision (the float64 -> float32 step is exact enough except
        # at float32 ties, which cannot straddle a bf16 tie), then to bf16.
        out = _f64_to_bf16(acc)
    return out


def _f64_to_bf16(acc: np.ndarray) -> np.ndarray:
    """Correct rounding of float64 values to bf16 (no double rounding)."""
    acc = np.asarray(acc, dtype=F64)
    f = acc.astype(F32)
    b = bf16_rne(f)
    # double rounding can only go wrong when f sits exactly on a bf16 midpoint
    u = f.view(np.uint32)
    on_mid = (u & 0xFFFF) == 0x8000
    if np.any(on_mid):
        lo = (u & 0xFFFF0000).view(F32).astype(F64)
        hi = ((u & 0xFFFF0000) + 0x10000).astype(np.uint32).view(F32).astype(F64)
        # compare in magnitude: for negatives the roles of lo/hi swap, the test is symmetric
        d_lo = np.abs(acc - lo)
        d_hi = np.abs(acc - hi)
        pick = np.where(d_lo < d_hi, lo, np.where(d_hi < d_lo, hi, b.astype(F64))).astype(F32)
        b = np.where(on_mid, pick, b).astype(F32)
    return b


def _load_sigmoid_table() -> dict:
    if os.path.exists(_SIGMOID_TABLE_PATH):
        d = np.load(_SIGMOID_TABLE_PATH)
        return {int(k): int(v) for k, v in zip(d["logit_bits"].tolist(), d["sigmoid_bits"].tolist())}
    return {}


_SIG_TABLE: dict | None = None


def _sigmoid_exact(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=F64)
    with np.errstate(over="ignore"):
        return 1.0 / (1.0 + np.exp(-x))


def sigmoid_ambiguous_f32(x: np.ndarray, s_exact: np.ndarray, ulps: float = 4.0) -> np.ndarray:
    """True where an fp32 sigmoid with a few ulps of error may round to a different bf16
    value than the exact sigmoid (the exact value is near a bf16 midpoint)."""
    s32 = s_exact.astype(F32)
    u = s32.view(np.uint32)
    base = u & 0xFFFF0000
    mids = []
    for off in (-0x10000, 0, 0x10000):
        m = (base.astype(np.int64) + off) | 0x8000
        m = np.clip(m, 0, 0xFFFFFFFF).astype(np.uint32).view(F32).astype(F64)
        mids.append(np.abs(s_exact - m))
    d = np.minimum(np.minimum(mids[0], mids[1]), mids[2])
    ulp = np.spacing(np.abs(s32)).astype(F64)
    return d <= ulps * ulp


def sigmoid_bf16(logit_bf16: np.ndarray):
    """``torch.sigmoid`` of a bf16 tensor: fp32 ``1/(1+exp(-x))`` rounded to bf16.

    Returns ``(s, ambiguous)``. ``ambiguous`` marks logits whose result depends on the
    last bit of the fp32 ``exp``; where the B200 measurement table is present those are
    resolved from it and reported as not ambiguous.
    """
    global _SIG_TABLE
    if _SIG_TABLE is None:
        _SIG_TABLE = _load_sigmoid_table()
    x = np.asarray(logit_bf16, dtype=F32)
    s_exact = _sigmoid_exact(x)
    s = bf16_rne(s_exact.astype(F32))
    amb = sigmoid_ambiguous_f32(x, s_exact)
    if np.any(amb) and _SIG_TABLE:
        bits = (x.view(np.uint32) >> 16).astype(np.int64)
        idx = np.nonzero(amb)
        for i in zip(*idx):
            key = int(bits[i])
            if key in _SIG_TABLE:
                s[i] = bf16_bits_to_f32(_SIG_TABLE[key])
                amb[i] = False
    return s.astype(F32), amb


def window_sizes_from_logit(logit: np.ndarray, n_min: int, n_max: int, dtype: str):
    """``_window_sizes(floor=True)``: ``clamp(floor(n_min + σ(l)·(n_max−n_min)), min=1)``.

    Follows ``dsalt_attention.py:275`` (``n_min + torch.sigmoid(l) * (n_max - n_min)``)
    and ``:282-284`` (floor, clamp). In bf16 every op rounds its fp32 result to bf16.
    Returns ``(w int32, ambiguous bool)``.
    """
    rng = F32(n_max - n_min)
    if dtype == "bf16":
        s, amb = sigmoid_bf16(logit)
        m = bf16_rne((s * rng).astype(F32))
        c = bf16_rne((m + F32(n_min)).astype(F32))
        w = np.maximum(np.floor(c), F32(1)).astype(np.int32)
        return w, amb
    # fp32: the sigmoid is fp32 with a few ulps of error; results whose floor depends
    # on those ulps are reported as ambiguous.
    x = np.asarray(logit, dtype=F32)
    s_exact = _sigmoid_exact(x)
    s = s_exact.astype(F32)
    m = (s * rng).astype(F32)
    c = (m + F32(n_min)).astype(F32)
    c_exact = F64(n_min) + s_exact * F64(n_max - n_min)
    amb = np.abs(c_exact - np.round(c_exact)) <= 16 * np.spacing(np.abs(c)).astype(F64)
    w = np.maximum(np.floor(c), F32(1)).astype(np.int32)
    return w, amb


def window_sizes(x, g, b, n_min, n_max, dtype):
    """Width of every token: logit then integerisation (``dsalt_attention.py:278-284``)."""
    logit = window_logit(x, g, b, dtype)
    w, amb = window_sizes_from_logit(logit, n_min, n_max, dtype)
    return w, logit, amb


# --------------------------------------------------------------------------- #
# (a3) per-token selection signals -- landmark_tokens_ker.py:47,52 ;
#      causal_landmark_check.py:68-79
# --------------------------------------------------------------------------- #
def row_norms(a: np.ndarray, round_to: str | None) -> np.ndarray:
    """L2 norm over the last axis: float64 sum of squares rounded once to fp32, fp32
    sqrt; rounded to bf16 when ``round_to == 'bf16'`` (a bf16 ``Tensor.norm`` outside
    autocast). Under CUDA autocast ``norm`` runs in fp32 (``round_to=None``)."""
    s = np.sum(np.square(np.asarray(a, dtype=F64)), axis=-1)
    n = np.sqrt(s.astype(F32)).astype(F32)
    if round_to == "bf16":
        n = bf16_rne(n)
    return n


def token_signals(x: np.ndarray, v: np.ndarray, n_kv: int, head_dim: int, round_to):
    """``x_norm = ‖x_i‖`` and ``xwv = ‖(x W_Vᵀ)_{i,g}‖`` per kv group.

    ``v`` is the value projection ``x @ W_Vᵀ`` in its compute dtype; without a bias it is
    the ``v_proj`` output (``landmark_tokens_ker.py:52`` recomputes the same product).
    """
    T = x.shape[0]
    xn = row_norms(x, round_to)
    vn = row_norms(np.asarray(v, dtype=F32).reshape(T, n_kv, head_dim), round_to)
    return xn, vn


# --------------------------------------------------------------------------- #
# exact sums
# --------------------------------------------------------------------------- #
def exact_sum(values: np.ndarray) -> float:
    """Correctly rounded float64 value of the exact sum."""
    return math.fsum(np.asarray(values, dtype=F64).ravel().tolist())


class ExactPrefix:
    """Exact running sums of fp32 values and of their squares (Python integers)."""

    S1_SHIFT = 149      # every fp32 value is an integer multiple of 2**-149
    S2_SHIFT = 298      # every square of an fp32 value is a multiple of 2**-298

    def __init__(self):
        self.a1 = 0
        self.a2 = 0

    def add(self, vals: np.ndarray):
        v = np.asarray(vals, dtype=F32).astype(F64)
        for x in v.tolist():
            self.a1 += int(math.ldexp(x, self.S1_SHIFT))
            self.a2 += int(math.ldexp(x * x, self.S2_SHIFT))

    def sums(self):
        from fractions import Fraction
        return (float(Fraction(self.a1, 1 << self.S1_SHIFT)),
                float(Fraction(self.a2, 1 << self.S2_SHIFT)))


# --------------------------------------------------------------------------- #
# whole-sequence statistics and scores -- landmark_tokens_ker.py:47-60
# --------------------------------------------------------------------------- #
def global_stats(vals: np.ndarray):
    """fp32 ``mean()`` and ``std().clamp(min=1e-6)`` over all tokens (unbiased std).

    mean = fl32(S1/n); var = (S2 − (S1/n)·S1)/(n−1) in float64; std = fl32(sqrt(var)).
    """
    v = np.asarray(vals, dtype=F32)
    n = v.shape[0]
    S1 = exact_sum(v)
    S2 = exact_sum(v.astype(F64) ** 2)
    m64 = S1 / n
    mean = F32(m64)
    if n > 1:
        var = (S2 - m64 * S1) / F64(n - 1)
        std = F32(math.sqrt(max(var, 0.0)))
    else:
        std = F32(np.nan)
    std = F32(max(std, F32(1e-6))) if not np.isnan(std) else std
    return mean, std


def global_scores(xn, vn, alpha, n_heads):
    """``hybrid_scores_per_head`` (``landmark_tokens_ker.py:47-60``) → (scores [T,H], z_x, z_v)."""
    xn = np.asarray(xn, dtype=F32)
    vn = np.asarray(vn, dtype=F32)
    alpha = np.asarray(alpha, dtype=F32)
    n_kv = vn.shape[1]
    mx, sx = global_stats(xn)
    z_x = ((xn - mx).astype(F32) / sx).astype(F32)
    z_v = np.empty_like(vn)
    for g in range(n_kv):
        mv, sv = global_stats(vn[:, g])
        z_v[:, g] = ((vn[:, g] - mv).astype(F32) / sv).astype(F32)
    if n_kv != n_heads:
        z_v = np.repeat(z_v, n_heads // n_kv, axis=1)
    a = alpha[None, :]
    scores = ((a * z_v).astype(F32) + ((F32(1.0) - a).astype(F32) * z_x[:, None]).astype(F32)).astype(F32)
    return scores, z_x, z_v


# --------------------------------------------------------------------------- #
# top-k with the declared tie rule
# --------------------------------------------------------------------------- #
def topk_positions(scores: np.ndarray, cand_mask: np.ndarray, k: int) -> np.ndarray:
    """The ``min(k, #candidates)`` best candidates (score descending, ties → lower
    position), returned sorted by position and padded with ``-1`` to ``k``."""
    pos = np.nonzero(cand_mask)[0]
    out = np.full(k, -1, dtype=np.int32)
    if pos.size == 0 or k == 0:
        return out
    s = np.asarray(scores, dtype=F32)[pos]
    order = np.lexsort((pos, -s.astype(F64)))
    sel = np.sort(pos[order[:k]])
    out[: sel.size] = sel
    return out


def kth_margin_sets(scores, cand_mask, k):
    """(strict set, tie-value, tie candidates) used to compare against an unspecified
    tie-break: positions strictly above the k-th value, the k-th value itself, and the
    positions holding it."""
    pos = np.nonzero(cand_mask)[0]
    if pos.size == 0:
        return set(), None, set()
    s = np.asarray(scores, dtype=F32)[pos]
    kk = min(k, pos.size)
    kth = np.sort(s)[::-1][kk - 1]
    strict = set(pos[s > kth].tolist())
    ties = set(pos[s == kth].tolist())
    return strict, kth, ties


# --------------------------------------------------------------------------- #
# (a4) whole-sequence landmark indices -- selectors.py:75-134
# --------------------------------------------------------------------------- #
def covered_mask(cu_seqlens, w):
    """``seq_off < w`` (``selectors.py:105``): tokens inside their own window."""
    T = int(cu_seqlens[-1])
    seq_off = np.empty(T, dtype=np.int64)
    for s in range(len(cu_seqlens) - 1):
        a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        seq_off[a:b] = np.arange(b - a)
    return seq_off < np.asarray(w, dtype=np.int64)


def select_global(xn, vn, alpha, w, cu_seqlens, k_lmk, n_heads):
    """Landmark positions ``[H, S, k]`` (local to each sequence, sorted, ``-1`` padded),
    plus ``(scores, z_x, z_v)``. Statistics are over all packed tokens
    (``landmark_tokens_ker.py:47-55`` is called on the packed ``x``)."""
    scores, z_x, z_v = global_scores(xn, vn, alpha, n_heads)
    cov = covered_mask(cu_seqlens, w)
    S = len(cu_seqlens) - 1
    out = np.full((n_heads, S, k_lmk), -1, dtype=np.int32)
    for s in range(S):
        a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        for h in range(n_heads):
            out[h, s] = topk_positions(scores[a:b, h], ~cov[a:b], k_lmk)
    return out, scores, z_x, z_v


# --------------------------------------------------------------------------- #
# (a5) block-causal selection -- results/causal_landmark_check.py:82-113
# --------------------------------------------------------------------------- #
def prefix_stat(S1: float, S2: float, n: int):
    """``_std_at`` (``causal_landmark_check.py:88-92``) in float64."""
    mean = S1 / F64(n)
    var = (S2 - (F64(n) * mean) * mean) / F64(max(n - 1, 1))
    sd = math.sqrt(max(var, 0.0))
    sd = max(sd, 1e-6)
    return F64(mean), F64(sd)


def block_scores(xn_pre, vn_pre, stats_x, stats_v, alpha, n_heads):
    """Scores of the candidates ``[0, n)`` for one block (``_select`` ``:102-108``)."""
    mx, sdx = stats_x
    z_x = ((np.asarray(xn_pre, dtype=F32).astype(F64) - mx) / sdx).astype(F32)
    n_kv = vn_pre.shape[1]
    z_v = np.empty(vn_pre.shape, dtype=F32)
    for g in range(n_kv):
        mv, sdv = stats_v[g]
        z_v[:, g] = ((np.asarray(vn_pre[:, g], dtype=F32).astype(F64) - mv) / sdv).astype(F32)
    if n_kv != n_heads:
        z_v = np.repeat(z_v, n_heads // n_kv, axis=1)
    a = np.asarray(alpha, dtype=F32)[None, :]
    return ((a * z_v).astype(F32) + ((F32(1.0) - a).astype(F32) * z_x[:, None]).astype(F32)).astype(F32)


def select_block_causal(xn, vn, alpha, w, L, k_lmk, n_heads, block=512, return_stats=False):
    """Landmarks of every ``block``-query block of one sequence of length ``L``:
    ``[H, ceil(L/block), k]``. Block ``b`` draws from positions ``[0, b·block)`` with the
    statistics of that prefix (``causal_landmark_check.py:95-113``, driven at
    ``:176-186``); ``n < 2`` selects nothing (``:100-101``)."""
    xn = np.asarray(xn, dtype=F32)[:L]
    vn = np.asarray(vn, dtype=F32)[:L]
    cov = np.arange(L) < np.asarray(w, dtype=np.int64)[:L]
    n_kv = vn.shape[1]
    nb = (L + block - 1) // block
    out = np.full((n_heads, nb, k_lmk), -1, dtype=np.int32)
    accx = ExactPrefix()
    accv = [ExactPrefix() for _ in range(n_kv)]
    stats = []
    for b in range(nb):
        n = b * block
        if b > 0:
            accx.add(xn[n - block:n])
            for g in range(n_kv):
                accv[g].add(vn[n - block:n, g])
        if n < 2:
            stats.append(None)
            continue
        sx = prefix_stat(*accx.sums(), n)
        sv = [prefix_stat(*accv[g].sums(), n) for g in range(n_kv)]
        stats.append((sx, sv))
        sc = block_scores(xn[:n], vn[:n], sx, sv, alpha, n_heads)
        for h in range(n_heads):
            out[h, b] = topk_positions(sc[:, h], ~cov[:n], k_lmk)
    if return_stats:
        return out, stats
    return out


# --------------------------------------------------------------------------- #
# (a8) sparse attention forward -- dsalt_triton_attn.py:27-169 /
#      causal_landmark_check.py:119-147
# --------------------------------------------------------------------------- #
def attention_forward(q, k, v, w, lmk, cu_seqlens, lmk_block=0, lmk_bias=None,
                      scale=None, rows=None, return_mag=False):
    """Reference semantics of the inference kernel, evaluated in float64.

    For query ``i`` (position within its sequence) and head ``h`` the keys are the
    window ``j ∈ [i−w(i)+1, i] ∩ [0, L)`` (``dsalt_triton_attn.py:102-105``) and every
    landmark ``p`` with ``0 ≤ p < L``, ``p ≤ i`` and ``p < i−w(i)+1``
    (``:132-135``); the logit is ``q·k·scale`` (+ ``lmk_bias`` on landmarks, ``:140``);
    a row whose softmax mass is ≤ 1e-9 is zero (``:150-154``).

    ``lmk`` is ``[H, S, k]`` (``lmk_block == 0``) or ``[H, n_sets, k]`` with one set per
    ``lmk_block`` queries of each sequence, numbered sequence after sequence.
    ``rows`` optionally restricts the evaluation to a subset of packed rows.
    Returns ``(out [T,H,D] float64 (rows not evaluated are 0), lse [T,H])``, and with
    ``return_mag`` also ``mag [T,H,D] = Σ_j p_j·|v_jd| / Σ_j p_j``: rounding every
    probability to bf16 before the P·V product (the reference's
    ``tl.dot(p.to(bf16), v)``, ``dsalt_triton_attn.py:116,148``) moves an output by at most
    ``2^-8 · mag`` (bf16 keeps 8 significant bits: round-to-nearest relative error ≤ 2^-8).
    """
    q = np.asarray(q, dtype=F64)
    k = np.asarray(k, dtype=F64)
    v = np.asarray(v, dtype=F64)
    T, H, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    scale = F64(F32(scale))
    w = np.maximum(np.asarray(w, dtype=np.int64), 1)
    out = np.zeros((T, H, D), dtype=F64)
    lse = np.full((T, H), -np.inf, dtype=F64)
    mag = np.zeros((T, H, D), dtype=F64) if return_mag else None
    S = len(cu_seqlens) - 1
    want = None if rows is None else np.zeros(T, dtype=bool)
    if want is not None:
        want[np.asarray(rows)] = True
    set_base = 0
    for s in range(S):
        a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        L = b - a
        nsets = 1 if lmk_block == 0 else max((L + lmk_block - 1) // lmk_block, 0)
        for i in range(L):
            t = a + i
            if want is not None and not want[t]:
                continue
            lo = i - int(w[t]) + 1
            j0 = max(lo, 0)
            set_id = set_base if lmk_block == 0 else set_base + i // lmk_block
            for h in range(H):
                kw = k[a + j0:a + i + 1, h]
                vw = v[a + j0:a + i + 1, h]
                lg = kw @ q[t, h] * scale
                P = lmk[h, set_id]
                ok = (P >= 0) & (P < L) & (P <= i) & (P < lo)
                pv = P[ok].astype(np.int64)
                ll = k[a + pv, h] @ q[t, h] * scale
                if lmk_bias is not None:
                    ll = ll + np.asarray(lmk_bias, dtype=F64)[h, set_id][ok]
                allg = np.concatenate([lg, ll])
                allv = np.concatenate([vw, v[a + pv, h]], axis=0)
                if allg.size == 0:
                    continue
                m = allg.max()
                p = np.exp(allg - m)
                l = p.sum()
                if l > 1e-9:
                    out[t, h] = (p @ allv) / l
                    lse[t, h] = m + math.log(l)
                    if mag is not None:
                        mag[t, h] = (p @ np.abs(allv)) / l
        set_base += nsets
    if return_mag:
        return out, lse, mag
    return out, lse


# --------------------------------------------------------------------------- #
# full core pipeline (widths -> signals -> selection -> attention)
# --------------------------------------------------------------------------- #
@dataclass
class CoreResult:
    w: np.ndarray
    xn: np.ndarray
    vn: np.ndarray
    lmk: np.ndarray
    out: np.ndarray | None


def core_forward(x, g, gb, q, k, v, alpha, cu_seqlens, n_min, n_max, k_lmk, n_kv,
                 dtype, norm_round, mode="global", block=512, rows=None, with_attention=True):
    T = x.shape[0]
    H = q.shape[1]
    D = q.shape[2]
    w, _, _ = window_sizes(x, g, gb, n_min, n_max, dtype)
    xn, vn = token_signals(x, np.asarray(v, dtype=F32).reshape(T, -1)[:, : n_kv * D], n_kv, D, norm_round)
    if mode == "global":
        lmk, _, _, _ = select_global(xn, vn, alpha, w, cu_seqlens, k_lmk, H)
        lb = 0
    else:
        parts = []
        for s in range(len(cu_seqlens) - 1):
            a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
            parts.append(select_block_causal(xn[a:b], vn[a:b], alpha, w[a:b], b - a, k_lmk, H, block))
        lmk = np.concatenate(parts, axis=1) if parts else np.zeros((H, 0, k_lmk), np.int32)
        lb = block
    out = None
    if with_attention:
        out, _ = attention_forward(q, k, v, w, lmk, cu_seqlens, lmk_block=lb, rows=rows)
    return CoreResult(w=w, xn=xn, vn=vn, lmk=lmk, out=out)


# --------------------------------------------------------------------------- #
# masked-SDPA CPU path (the reference's non-Triton inference branch), for timing
# --------------------------------------------------------------------------- #
def masked_sdpa_forward(q, k, v, x_signals_scores, w, cu_seqlens, k_lmk):
    """Restatement of ``_build_mask_packed`` (``dsalt_attention.py:96-144``) followed by
    ``sparse_attention_forward_packed`` (``sparse_attn.py:29-56``), in torch on CPU.

    ``x_signals_scores`` is the ``[T, H]`` score matrix. Landmarks are the union over
    heads of each sequence's top-k and are attended by every row of the sequence (no
    causal cut), as in the reference's fallback. Used only as the timed CPU baseline.
    """
    import torch
    qt = torch.as_tensor(np.asarray(q, dtype=F32))
    kt = torch.as_tensor(np.asarray(k, dtype=F32))
    vt = torch.as_tensor(np.asarray(v, dtype=F32))
    T = qt.shape[0]
    cu = [int(c) for c in cu_seqlens]
    wt = torch.as_tensor(np.asarray(w, dtype=np.int64))
    seq_ids = torch.repeat_interleave(torch.arange(len(cu) - 1), torch.tensor([cu[i + 1] - cu[i] for i in range(len(cu) - 1)]))
    starts = torch.tensor(cu[:-1])
    seq_off = torch.arange(T) - starts[seq_ids]
    lo = (seq_off - wt.clamp(min=1) + 1).clamp(min=0) + starts[seq_ids]
    col = torch.arange(T)
    mask = (seq_ids[:, None] == seq_ids[None, :]) & (col[None, :] >= lo[:, None]) & (col[None, :] <= torch.arange(T)[:, None])
    sc = torch.as_tensor(np.asarray(x_signals_scores, dtype=F32)).masked_fill((seq_off < wt)[:, None], float("-inf"))
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        kk = min(k_lmk, b - a)
        if kk == 0:
            continue
        vals, top = torch.topk(sc[a:b].T, kk, dim=1)
        idx = (top[torch.isfinite(vals)] + a).unique()
        if idx.numel():
            mask[a:b][:, idx] = True
    add = torch.zeros(T, T).masked_fill(~mask, float("-inf"))
    o = torch.nn.functional.scaled_dot_product_attention(
        qt.transpose(0, 1)[None], kt.transpose(0, 1)[None], vt.transpose(0, 1)[None], attn_mask=add[None, None])
    return o[0].transpose(0, 1).numpy()


# --------------------------------------------------------------------------- #
# backward of the inference kernel -- dsalt/kernels/dsalt_triton_bwd.py:18-216
# --------------------------------------------------------------------------- #
def attention_backward(q, k, v, out, dout, lse, w, lmk, cu_seqlens, lmk_block=0, lmk_bias=None, scale=None):
    """Gradients of :func:`attention_forward` in float64, with the reference backward's
    recomputation: ``delta = Σ_d O·dO`` (``_dsalt_bwd_preprocess``, ``:18-49``), and for each
    key of the row's set (window, then landmarks with the causal and de-duplicating rule)
    ``p = exp(q·k·scale (+ bias) − lse)``, ``ds = p (dO·v − delta) scale``; ``dq += ds k``,
    ``dk += ds q``, ``dv += p dO`` (``:110-212``), ``d_bias[h, set, slot] += p (dO·v − delta)``
    (``:153-155``). Rows whose ``lse`` is ``-inf`` contribute nothing. ``k`` / ``v`` may have
    fewer (grouped) heads than ``q``: head ``h`` uses kv head ``h // (H / H_kv)`` and the kv
    gradients sum over the group. Returns ``(dq [T,H,D], dk, dv [T,H_kv,D], d_bias)``."""
    q = np.asarray(q, dtype=F64)
    k = np.asarray(k, dtype=F64)
    v = np.asarray(v, dtype=F64)
    out = np.asarray(out, dtype=F64)
    dout = np.asarray(dout, dtype=F64)
    lse = np.asarray(lse, dtype=F64)
    T, H, D = q.shape
    Hkv = k.shape[1]
    rep = H // Hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    scale = F64(F32(scale))
    w = np.maximum(np.asarray(w, dtype=np.int64), 1)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    d_bias = np.zeros(np.asarray(lmk).shape, dtype=F64)
    delta = np.sum(out * dout, axis=-1)
    S = len(cu_seqlens) - 1
    set_base = 0
    for s in range(S):
        a, b = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        L = b - a
        nsets = 1 if lmk_block == 0 else max((L + lmk_block - 1) // lmk_block, 0)
        for i in range(L):
            t = a + i
            lo = i - int(w[t]) + 1
            j0 = max(lo, 0)
            set_id = set_base if lmk_block == 0 else set_base + i // lmk_block
            for h in range(H):
                if not np.isfinite(lse[t, h]):
                    continue
                g = h // rep
                rows = np.arange(a + j0, a + i + 1)
                P = np.asarray(lmk)[h, set_id]
                ok = (P >= 0) & (P < L) & (P <= i) & (P < lo)
                slots = np.nonzero(ok)[0]
                rows = np.concatenate([rows, a + P[slots].astype(np.int64)])
                lg = k[rows, g] @ q[t, h] * scale
                nw = i + 1 - j0
                if lmk_bias is not None:
                    lg[nw:] += np.asarray(lmk_bias, dtype=F64)[h, set_id][slots]
                p = np.exp(lg - lse[t, h])
                dp = v[rows, g] @ dout[t, h]
                rec = p * (dp - delta[t, h])
                ds = rec * scale
                dq[t, h] += ds @ k[rows, g]
                np.add.at(dk[:, g], rows, ds[:, None] * q[t, h][None, :])
                np.add.at(dv[:, g], rows, p[:, None] * dout[t, h][None, :])
                d_bias[h, set_id, slots] += rec[nw:]
        set_base += nsets
    return dq, dk, dv, d_bias


# --------------------------------------------------------------------------- #
# training attention with soft selectors -- dsalt/kernels/dsalt_triton_train.py
# --------------------------------------------------------------------------- #
def _train_keys(i, L, wc, P, logw_row, win_edge, tau):
    """Keys of row ``i`` (position in a sequence of length ``L``) with continuous width
    ``wc``: the band ``0 ≤ d = i − j ≤ w̃`` (``_train_fwd_kernel`` ``:131-141``) with its soft
    edge bias ``0`` in the core ``d ≤ w̃ − win_edge`` and ``log σ((w̃ − d)/τ)`` outside it,
    then the landmarks ``p`` with ``0 ≤ p < L``, ``p ≤ i``, ``p < i − w̃`` and log-weight
    bias (``:173-184``). Returns (positions, bias, is_edge, d_bias/d_w̃, landmark slots)."""
    j = np.arange(0, i + 1)
    d = (i - j).astype(F64)
    band = d <= wc
    j, d = j[band], d[band]
    z = (wc - d) / tau
    core = d <= wc - win_edge
    bias = np.where(core, 0.0, -np.log1p(np.exp(-z)))
    dbdw = np.where(core, 0.0, (1.0 - 1.0 / (1.0 + np.exp(-z))) / tau)
    ok = (P >= 0) & (P < L) & (P <= i) & (P.astype(F64) < i - wc)
    slots = np.nonzero(ok)[0]
    pos = np.concatenate([j, P[slots].astype(np.int64)])
    b = np.concatenate([bias, np.asarray(logw_row, dtype=F64)[slots]])
    return pos, b, len(j), dbdw, slots


def train_attention_forward(q, k, v, lmk, logw, w_cont, cu_seqlens, tau_win, win_edge, scale=None):
    """``_train_fwd_kernel`` (``dsalt_triton_train.py:74-217``) in float64: softmax over each
    row's soft band and log-weighted landmarks (one set per sequence), rows with mass ≤ 1e-9
    zero. Grouped kv heads are indexed. Returns ``(out [T,H,D], lse [T,H])``."""
    q, k, v = (np.asarray(a, dtype=F64) for a in (q, k, v))
    T, H, D = q.shape
    rep = H // k.shape[1]
    scale = F64(F32(1.0 / math.sqrt(D) if scale is None else scale))
    wc = np.asarray(w_cont, dtype=F32).astype(F64)
    out = np.zeros((T, H, D), dtype=F64)
    lse = np.full((T, H), -np.inf, dtype=F64)
    for s in range(len(cu_seqlens) - 1):
        a, b_ = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        L = b_ - a
        for i in range(L):
            t = a + i
            for h in range(H):
                g = h // rep
                pos, bias, _, _, _ = _train_keys(i, L, wc[t], np.asarray(lmk)[h, s], np.asarray(logw)[h, s],
                                                 win_edge, tau_win)
                if pos.size == 0:
                    continue
                lg = k[a + pos, g] @ q[t, h] * scale + bias
                m = lg.max()
                p = np.exp(lg - m)
                l = p.sum()
                if l > 1e-9:
                    out[t, h] = p @ v[a + pos, g] / l
                    lse[t, h] = m + math.log(l)
    return out, lse


def train_attention_backward(q, k, v, out, dout, lse, lmk, logw, w_cont, cu_seqlens, tau_win, win_edge,
                             scale=None):
    """``_train_bwd_kernel`` / ``_train_bwd_dkdv_kernel`` (``dsalt_triton_train.py:240-490``) in
    float64: ``p = exp(logit − lse)``, ``ds = p (dO·v − delta)``; ``dq += ds·scale k``,
    ``dk += ds·scale q``, ``dv += p dO``; ``d_logw[h, s, slot] += ds`` on landmarks;
    ``d_w̃[i] += Σ ds · (1 − σ(z))/τ`` over the band's edge keys, summed over heads
    (``:363-376``, ``:688``). Returns ``(dq, dk, dv, d_logw, d_w)``."""
    q, k, v, out, dout = (np.asarray(a, dtype=F64) for a in (q, k, v, out, dout))
    lse = np.asarray(lse, dtype=F64)
    T, H, D = q.shape
    rep = H // k.shape[1]
    scale = F64(F32(1.0 / math.sqrt(D) if scale is None else scale))
    wc = np.asarray(w_cont, dtype=F32).astype(F64)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    d_logw = np.zeros(np.asarray(logw).shape, dtype=F64)
    d_w = np.zeros(T, dtype=F64)
    delta = np.sum(out * dout, axis=-1)
    for s in range(len(cu_seqlens) - 1):
        a, b_ = int(cu_seqlens[s]), int(cu_seqlens[s + 1])
        L = b_ - a
        for i in range(L):
            t = a + i
            for h in range(H):
                if not np.isfinite(lse[t, h]):
                    continue
                g = h // rep
                pos, bias, nw, dbdw, slots = _train_keys(i, L, wc[t], np.asarray(lmk)[h, s],
                                                         np.asarray(logw)[h, s], win_edge, tau_win)
                rows = a + pos
                p = np.exp(k[rows, g] @ q[t, h] * scale + bias - lse[t, h])
                ds = p * (v[rows, g] @ dout[t, h] - delta[t, h])
                dq[t, h] += (ds * scale) @ k[rows, g]
                np.add.at(dk[:, g], rows, (ds * scale)[:, None] * q[t, h][None, :])
                np.add.at(dv[:, g], rows, p[:, None] * dout[t, h][None, :])
                d_logw[h, s, slots] += ds[nw:]
                d_w[t] += np.sum(ds[:nw] * dbdw)
    return dq, dk, dv, d_logw, d_w
