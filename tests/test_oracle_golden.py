"""Pins the CPU oracle to the reference: fixtures in ``tests/golden`` were produced by
running the reference itself (``tests/golden/make_golden.py``).

What is asserted per case:

* window widths: the oracle's integerisation of the reference's own logit equals the
  reference's width for every token (bit-exact), except logits whose bf16 sigmoid
  depends on the last bit of ``exp`` (at most three bf16 values, reported);
* the oracle's logit equals the reference's except where the exact value lies within
  the float32 accumulation error of a bf16 rounding boundary;
* signals (``‖x‖``, value norms) agree to a few ulps (the reference's reduction order is
  a library detail);
* landmark sets, given the reference's own signals, equal the reference's sets per
  (head, sequence | block), except slots decided by an exact or near tie at the k-th
  score;
* the attention output of the oracle equals the reference's ``_block_attention``
  output within 1e-5 (fp32 arithmetic on the same inputs);
* the masked-SDPA port used as the timed CPU baseline equals the reference's fallback.
"""
import json
import math
import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import dsalt_oracle as O

GOLDEN = os.path.dirname(os.path.abspath(C.__file__))
NAMES = [n for n in C.CASES if os.path.exists(os.path.join(GOLDEN, f"{n}.npz"))]


def load(name):
    d = np.load(os.path.join(GOLDEN, f"{name}.npz"), allow_pickle=False)
    cfg = json.loads(str(d["cfg"]))
    return cfg, d


def ulp_diff(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    ia = np.where(ia < 0, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


@pytest.fixture(scope="module", params=NAMES)
def case(request):
    return request.param, *load(request.param)


def test_fixtures_present():
    assert set(NAMES) == set(C.CASES), f"missing golden fixtures: {set(C.CASES) - set(NAMES)}"


def test_inputs_regenerate(case):
    name, cfg, d = case
    x = C.make_x(cfg)
    import hashlib
    h = hashlib.sha256(x.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    assert h == str(d["x_sha"]), "seeded inputs changed: fixtures no longer match"


def test_width_integerisation_bit_exact(case):
    name, cfg, d = case
    logit = d["logit"]
    w_ref = d["w"]
    w, amb = O.window_sizes_from_logit(logit, cfg["n_min"], cfg["n_max"], cfg["dtype"])
    bad = (w != w_ref) & ~amb
    assert not bad.any(), f"{bad.sum()} widths differ: idx {np.nonzero(bad)[0][:10]}"
    assert ((w != w_ref) & amb).sum() <= 3


def test_window_logit(case):
    name, cfg, d = case
    params = C.make_params(cfg)
    dt = C.torch_dtype(cfg)
    x = C.make_x(cfg).float().numpy()
    g = params["win_gate.weight"].to(dt).float().numpy()
    b = float(params["win_gate.bias"].to(dt).float()[0])
    lo = O.window_logit(x, g, b, cfg["dtype"])
    ref = d["logit"]
    diff = lo != ref
    if diff.any():
        exact = x.astype(np.float64) @ g.astype(np.float64).reshape(-1) + b
        bound = x.shape[1] * 2.0 ** -23 * (np.abs(x.astype(np.float64)) @ np.abs(g.astype(np.float64)).reshape(-1))
        if cfg["dtype"] == "bf16":
            # boundary between the two bf16 neighbours
            mid = (lo.astype(np.float64) + ref.astype(np.float64)) / 2
            near = np.abs(exact - mid) <= bound
        else:
            near = np.abs(exact - ref.astype(np.float64)) <= bound
        assert near[diff].all(), f"{(diff & ~near).sum()} logits differ beyond the accumulation bound"
    if cfg["dtype"] == "bf16":
        assert diff.mean() < 2e-3


def test_signals(case):
    name, cfg, d = case
    x = C.make_x(cfg).float().numpy()
    rnd = "bf16" if cfg["norm"] == "bf16" else None
    xn = O.row_norms(x, rnd)
    tol = 1 if rnd == "bf16" else 4
    ud = ulp_diff(xn, d["xn"]) if rnd is None else ulp_diff(xn, d["xn"]) // 65536
    assert ud.max() <= tol, f"x-norm differs by {ud.max()} ulp"
    params = C.make_params(cfg)
    _, _, _, vp = C.project(cfg, params, C.make_x(cfg))
    vn = O.row_norms(vp.float().numpy().reshape(-1, cfg["Hkv"], cfg["D"]), rnd)
    ud = ulp_diff(vn, d["vn"]) if rnd is None else ulp_diff(vn, d["vn"]) // 65536
    assert ud.max() <= tol, f"value-norm differs by {ud.max()} ulp"


def _compare_sets(ref_row, ora_row, scores, cand, k):
    """Sets equal up to slots decided at (or within a few ulps of) the k-th score."""
    R = set(int(p) for p in ref_row if p >= 0)
    Q = set(int(p) for p in ora_row if p >= 0)
    if R == Q:
        return 0
    assert len(R) == len(Q), (len(R), len(Q))
    strict, kth, ties = O.kth_margin_sets(scores, cand, k)
    s = np.asarray(scores, np.float32)
    eps = 8 * float(np.spacing(np.float32(abs(kth)))) if kth is not None else 0.0
    near = set(np.nonzero(cand & (np.abs(s.astype(np.float64) - float(kth)) <= eps))[0].tolist())
    assert strict - near <= Q, "oracle misses a landmark strictly above the k-th score"
    assert (R ^ Q) <= near, f"sets differ outside the near-tie band: {sorted(R ^ Q)[:8]}"
    return len(R ^ Q)


def test_selection_given_reference_signals(case):
    name, cfg, d = case
    H, k = cfg["H"], cfg["k"]
    cu = C.cu_seqlens(cfg)
    w = d["w"]
    if cfg["mode"] == "global":
        lmk, scores, z_x, z_v = O.select_global(d["xn"], d["vn"], d["alpha"], w, cu, k, H)
        # statistics: a few ulps (of values of order one) from the reference's fp32
        # reductions
        assert np.abs(z_x - d["z_x"]).max() <= 4e-6
        assert np.abs(z_v - d["z_v"]).max() <= 4e-6
        cov = O.covered_mask(cu, w)
        ndiff = 0
        for s in range(len(cu) - 1):
            a, b = cu[s], cu[s + 1]
            for h in range(H):
                ndiff += _compare_sets(d["lmk"][h, s], lmk[h, s], d["scores"][a:b, h], ~cov[a:b], k)
        assert ndiff <= 2 * H
    else:
        L = cu[-1]
        B = cfg["block"]
        lmk, stats = O.select_block_causal(d["xn"], d["vn"], d["alpha"], w, L, k, H, B, return_stats=True)
        cov = np.arange(L) < w
        ref_stats = d["block_stats"]
        for b, st in enumerate(stats):
            if st is None:
                assert (lmk[:, b] == -1).all() and (d["lmk"][:, b] == -1).all()
                continue
            (mx, sx), sv = st
            assert abs(mx - ref_stats[b, 0, 0]) <= 1e-12 * abs(mx)
            assert abs(sx - ref_stats[b, 1, 0]) <= 1e-9 * abs(sx)
            n = b * B
            sc = O.block_scores(d["xn"][:n], d["vn"][:n], st[0], st[1], d["alpha"], H)
            for h in range(H):
                _compare_sets(d["lmk"][h, b], lmk[h, b], sc[:, h], ~cov[:n], k)


def _qkv(cfg):
    params = C.make_params(cfg)
    q, k, v, _ = C.project(cfg, params, C.make_x(cfg))
    return q, k, v


def test_attention_matches_reference_restatement(case):
    name, cfg, d = case
    q, k, v = _qkv(cfg)
    cu = C.cu_seqlens(cfg)
    rows = d["rows"]
    lb = 0 if cfg["mode"] == "global" else cfg["block"]
    out, _ = O.attention_forward(q.float().numpy(), k.float().numpy(), v.float().numpy(), d["w"], d["lmk"], cu,
                                 lmk_block=lb, rows=rows)
    err = np.abs(out[rows] - d["out_rows"].astype(np.float64)).max()
    assert err <= 1e-5, err


def test_masked_sdpa_port_matches_reference_fallback():
    if "cfg1_fp32" not in NAMES:
        pytest.skip("fixture missing")
    cfg, d = load("cfg1_fp32")
    if "fallback_mod_rows" not in d.files:
        pytest.skip("no fallback record")
    params = C.make_params(cfg)
    x = C.make_x(cfg)
    q, k, v, _ = C.project(cfg, params, x)
    cu = C.cu_seqlens(cfg)
    scores, _, _ = O.global_scores(d["xn"], d["vn"], d["alpha"], cfg["H"])
    o = O.masked_sdpa_forward(q.numpy(), k.numpy(), v.numpy(), scores, d["w"], cu, cfg["k"])
    mod = torch.nn.functional.linear(torch.as_tensor(o).reshape(x.shape[0], -1), params["out_proj.weight"])
    err = (mod.numpy()[d["rows"]] - d["fallback_mod_rows"]).__abs__().max()
    assert err <= 1e-5, err


def test_sigmoid_table_covers_every_ambiguous_logit():
    """The B200 measurement (``tests/golden/make_sigmoid_table.py``) lists exactly the bf16
    logits whose sigmoid rounding the oracle cannot decide, so no width stays ambiguous."""
    d = np.load(os.path.join(GOLDEN, "sigmoid_bf16_cuda.npz"))
    bits = np.arange(65536, dtype=np.uint32)
    vals = O.bf16_bits_to_f32(bits)
    fin = np.isfinite(vals)
    amb = O.sigmoid_ambiguous_f32(vals[fin], O._sigmoid_exact(vals[fin]))
    assert set(bits[fin][amb].tolist()) == set(d["logit_bits"].astype(np.uint32).tolist())
    _, still = O.sigmoid_bf16(O.bf16_bits_to_f32(d["logit_bits"].astype(np.uint32)))
    assert not np.any(still)
