"""The timed CPU baseline (``oracle/cpu_baseline.py``, the reference's block-causal path
restated with torch CPU ops) computes what the oracle computes: same landmark sets as
sets (its ``topk`` order is unspecified) given its own signals, and the same attention
output within 1e-4 (fp32 against the oracle's float64)."""
import numpy as np
import torch

from oracle import dsalt_oracle as O
from oracle.cpu_baseline import BlockCausalCPU


def test_block_causal_cpu_baseline_matches_oracle():
    g = torch.Generator().manual_seed(5)
    T, H, D, dm, k, B = 1536, 2, 32, 64, 16, 512
    x = torch.randn(T, dm, generator=g).bfloat16()
    gw = (torch.randn(dm, generator=g) * 0.2).bfloat16()
    gb = torch.zeros(1).bfloat16()
    q = torch.randn(T, H, D, generator=g)
    kk = torch.randn(T, H, D, generator=g)
    v = torch.randn(T, H, D, generator=g)
    alpha = torch.tensor([0.3, 0.8])
    base = BlockCausalCPU(x, gw, gb, 16, 256, q, kk, v, alpha, k, B)
    nb = T // B
    outs, sets = [], []
    base.reset()
    for b in range(nb):
        outs.append(base.run_block(b))
        sets.append(base.select(b * B))
    out = torch.cat(outs).numpy()
    w = base.w.numpy()
    lo = O.select_block_causal(base.xn.float().numpy(), base.vn.float().numpy(), alpha.numpy(), w, T, k, H, B)
    for b in range(nb):
        for h in range(H):
            got = sorted(int(p) for p in sets[b][h] if p >= 0)
            ref = [int(p) for p in lo[h, b] if p >= 0]
            assert got == ref, (b, h)
    ref, _ = O.attention_forward(q.numpy(), kk.numpy(), v.numpy(), w, lo, [0, T], lmk_block=B)
    assert np.abs(out - ref).max() < 1e-4


def test_masked_sdpa_step_matches_golden_pinned_port():
    """The timed masked-SDPA restatement equals the oracle's port, which the golden test
    pins to the reference's own fallback (configs[0] shapes)."""
    import cases as C
    from oracle.cpu_baseline import masked_sdpa_step
    cfg = C.CASES["cfg1_fp32"]
    params = C.make_params(cfg)
    x = C.make_x(cfg)
    q, k, v, vp = C.project(cfg, params, x)
    cu = C.cu_seqlens(cfg)
    alpha = C.alpha(params)
    gw = params["win_gate.weight"].reshape(-1)
    gb = params["win_gate.bias"]
    out = masked_sdpa_step(x, gw, gb, cfg["n_min"], cfg["n_max"], vp, alpha, q, k, v, cfg["k"], cu)
    w, _, _ = O.window_sizes(x.numpy(), gw.numpy(), float(gb[0]), cfg["n_min"], cfg["n_max"], "fp32")
    xn, vn = O.token_signals(x.numpy(), vp.numpy(), cfg["Hkv"], cfg["D"], None)
    scores, _, _ = O.global_scores(xn, vn, alpha.numpy(), cfg["H"])
    ref = O.masked_sdpa_forward(q.numpy(), k.numpy(), v.numpy(), scores, w, cu, cfg["k"])
    assert np.abs(out.numpy() - ref).max() < 1e-5
