"""Benchmark of the DSALT attention forward core on B200 (BASELINE.json's metric).

Workload: one DSALT layer, B=1, L=131072, H=16, head_dim 64, d_model 1024,
window widths in [16, 512] from the random-init predictor, k=128 landmarks, block-causal
selection over 512-query blocks, bf16. Inputs are synthetic: x ~ N(0,1), weights
N(0, 0.02), seeded; q/k/v come from the layer's projections and RoPE (library GEMMs,
outside the timed region). A step is the core of the layer's inference forward: window
widths + selection signals, block-causal landmark selection, sparse attention.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

One JSON line on rank 0. ``value`` is the device-timed step throughput (tokens/s, all
ranks), ``e2e`` the same metric through the C-ABI call with host buffers (pinned
host→device copies of x, q, k, v and the device→host copy of the output inside the
timed region), ``roofline`` the attention kernel's achieved HBM bandwidth against
MEASURED_PEAKS.json, ``cpu_baseline`` the reference's CPU path on a bounded sample.
With N > 1 (torchrun, one rank per GPU) the same L=131072 sequence is split across the
ranks (``dsalt_b200.sharded``): strong scaling, ``value`` = L tokens per max-over-ranks
step time.
"""
from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(workload="dsalt_attn_fwd_core_L131072_H16_D64_k128_block512_bf16", L=131072, H=16, D=64, dm=1024,
           n_min=16, n_max=512, k=128, block=512)
METRIC = "DSALT attn fwd tokens/s at L=131072"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(T):
    """DRAM bytes (read + write) of one attention launch at this sequence length, from
    the committed ncu summary (a line ``dram_bytes_per_launch[L=<T>]: <bytes>``)."""
    import re
    path = os.path.join(ROOT, "profiles", "attn_fwd_tc.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch\[L=%d\]:\s*([0-9.eE+]+)" % T, txt)
    return float(m.group(1)) if m else None


def make_inputs(dev, seed=0):
    from dsalt_b200.module import apply_rotary_emb, build_rope_cache
    T, H, D, dm = CFG["L"], CFG["H"], CFG["D"], CFG["dm"]
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, dm, device=dev, generator=g).bfloat16()

    def w(*s):
        return (torch.randn(*s, device=dev, generator=g) * 0.02).bfloat16()

    Wq, Wk, Wv, gw = w(dm, dm), w(dm, dm), w(dm, dm), w(dm)
    gb = torch.zeros(1, device=dev).bfloat16()
    alpha = torch.sigmoid(torch.full((H,), 0.4054651081081644, device=dev)).float()
    q = (x @ Wq.T).view(T, H, D)
    k = (x @ Wk.T).view(T, H, D)
    v = (x @ Wv.T).view(T, H, D).contiguous()
    cos, sin = build_rope_cache(T, D, dev)
    q, k = apply_rotary_emb(q, k, cos.bfloat16().unsqueeze(1), sin.bfloat16().unsqueeze(1))
    return x, gw, gb, alpha, q.contiguous(), k.contiguous(), v


class ClockSampler:
    """nvidia-smi clock / throttle samples taken during the timed region: a reader thread
    collects one line per 10 ms; entering waits (up to 3 s) for the first sample, so that
    sampling is running before the timed region starts, and leaving takes one more."""

    def __init__(self, index, interval_ms=10):
        self.index = index  # None: every GPU of the node, one line per GPU and interval
        self.interval_ms = interval_ms
        self.proc = None
        self.lines = []

    def _reader(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.lines.append(ln)

    def __enter__(self):
        import threading
        try:
            sel = [] if self.index is None else ["-i", str(self.index)]
            self.proc = subprocess.Popen(
                ["nvidia-smi", *sel,
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self
        self.thread = threading.Thread(target=self._reader, daemon=True)
        self.thread.start()
        t0 = time.time()
        while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
            time.sleep(0.005)
        self.n0 = len(self.lines)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            n = len(self.lines)
            t0 = time.time()
            while len(self.lines) <= n and time.time() - t0 < 0.5 and self.proc.poll() is None:
                time.sleep(0.002)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        # the samples from the last one before the timed region to the first one after it
        lines = self.lines[max(getattr(self, "n0", 1) - 1, 0):]
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, val in zip(names, parts[3:7]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _cpu_port(x, gw, gb, alpha, q, k, v):
    from oracle.cpu_baseline import BlockCausalCPU
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    base = BlockCausalCPU(x.cpu(), gw.cpu(), gb.cpu(), CFG["n_min"], CFG["n_max"], q.cpu(), k.cpu(), v.cpu(),
                          alpha.cpu(), CFG["k"], CFG["block"])
    return base, cores


def cpu_baseline(x, gw, gb, alpha, q, k, v, min_s=10.0):
    """The reference's block-causal CPU path over the whole L=131072 sequence (signals,
    widths, prefix statistics, selection and attention of all 256 blocks), repeated until
    at least ``min_s`` seconds of CPU work have been timed."""
    base, cores = _cpu_port(x, gw, gb, alpha, q, k, v)
    nb = -(-CFG["L"] // CFG["block"])
    base.time_blocks(0, 2)  # warm-up
    tok, spent, passes = 0, 0.0, 0
    while spent < min_s:
        t, dt = base.time_blocks(0, nb)
        tok += t
        spent += dt
        passes += 1
    return {"value": tok / spent, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{passes} full pass(es) over L={CFG['L']} (signals, widths, block-causal selection and "
                      f"attention of all {nb} 512-query blocks; fp32 torch CPU restatement of the reference's "
                      f"path), {spent:.1f} s"}


def masked_sdpa_baselines(budget_s=60.0):
    """The reference's masked-SDPA CPU path (``oracle/cpu_baseline.py::masked_sdpa_step``:
    widths, hybrid scores, the ``[T, T]`` window ∪ landmark mask, masked SDPA) on all host
    cores, fp32, at configs[0] (cfg1), configs[1] (cfg2: 4 × 8192 packed) and the cfg4
    recipe (H 16, d_model 1024, n_max 512, k 128, one sequence; whole-sequence landmarks —
    the fallback has no block-causal mode) at the largest L in 8192, 16384, 32768, 65536
    that fits the time budget and half the free host memory ([T, T] masks: ~8 bytes per
    entry). Synthetic seeded inputs of each config's shapes (q, k, v from random-init
    projections, RoPE left out: it changes values, not cost). Median of 3 after one
    warm-up for cfg1; one run for the larger ones. Projections are not timed."""
    from oracle.cpu_baseline import masked_sdpa_step
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        import psutil
        free = psutil.virtual_memory().available
    except Exception:
        free = 64 << 30

    def case(T, n_seq, H, dm, n_max, k, seed):
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(T, dm, generator=g)

        def W(*sh):
            return torch.randn(*sh, generator=g) * 0.02

        q = (x @ W(H * 64, dm).T).view(T, H, 64)
        kk = (x @ W(H * 64, dm).T).view(T, H, 64)
        xwv = x @ W(H * 64, dm).T
        alpha = torch.sigmoid(torch.full((H,), 0.4054651081081644))
        cu = [i * (T // n_seq) for i in range(n_seq + 1)]
        return (x, W(dm), torch.zeros(1), 16, n_max, xwv, alpha, q, kk, xwv.view(T, H, 64), k, cu)

    def timed(args, reps):
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            masked_sdpa_step(*args)
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    out = {"cores": cores, "dtype": "f32", "unit": "tokens/s"}
    t_start = time.perf_counter()
    a1 = case(1024, 1, 4, 256, 128, 32, 1)
    timed(a1, 1)
    s1 = timed(a1, 3)
    out["cfg1"] = {"T": 1024, "seconds": s1, "value": 1024 / s1}
    a2 = case(32768, 4, 12, 768, 256, 64, 2)
    s2 = timed(a2, 1)
    out["cfg2"] = {"T": 32768, "seconds": s2, "value": 32768 / s2}
    del a2
    last = None
    for L in (8192, 16384, 32768, 65536):
        left = budget_s - (time.perf_counter() - t_start)
        if 8 * L * L > free // 2 or (last is not None and last[1] * (L / last[0]) ** 2 > left):
            break
        sL = timed(case(L, 1, 16, 1024, 512, 128, 3), 1)
        last = (L, sL)
        out["cfg4_recipe_L%d" % L] = {"seconds": sL, "value": L / sL}
    out["largest_L_cfg4_recipe"] = last[0] if last else None
    return out


def run_reference(args):
    """--impl reference: the reference's CPU path (restated, see oracle/cpu_baseline.py) on
    this host's cores. A step streams the next run of consecutive 512-query blocks of the
    same L=131072 workload, sized so that all warm-up and timed steps take about three
    minutes in total; the value is tokens over time summed over the timed steps."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else None
    if dev is None:
        print(json.dumps({"impl": "reference", "unavailable": "no CUDA device to build the synthetic inputs"}))
        return
    x, gw, gb, alpha, q, k, v = make_inputs(dev)
    base, cores = _cpu_port(x, gw, gb, alpha, q, k, v)
    nb = -(-CFG["L"] // CFG["block"])
    t, dt = base.time_blocks(0, 4)  # calibration: seconds per block
    per_block = dt / 4
    n_steps = args.warmup + args.steps
    bps = max(1, min(nb, int(min(3.0, 180.0 / n_steps) / per_block)))
    nxt, tok, spent = 4, 0, 0.0
    for i in range(n_steps):
        if nxt >= nb:
            nxt = 0
        b1 = min(nb, nxt + bps)
        t, dt = base.time_blocks(nxt, b1)
        nxt = b1
        if i >= args.warmup:
            tok += t
            spent += dt
    value = tok / spent
    sample = (f"{args.steps} timed steps of {bps} consecutive 512-query blocks each, streamed through "
              f"L={CFG['L']} (signals, widths, selection, attention), {spent:.1f} s")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": spent / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": CFG["workload"], "where": "host CPU cores"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_sharded(args, rank, world, local, dev):
    """N > 1: the L = 131072 sequence split across the ranks (dsalt_b200.sharded): each rank
    owns L/N queries, signals are all-gathered, landmark rows are read from their owners over
    NVLink, the window halo comes from the previous rank. Strong scaling: the whole job
    processes the same L tokens per step as one GPU."""
    from dsalt_b200 import ops
    from dsalt_b200.sharded import ShardedCore
    T, H, D, k, B = CFG["L"], CFG["H"], CFG["D"], CFG["k"], CFG["block"]
    x, gw, gb, alpha, q, kk, v = make_inputs(dev, seed=0)  # the same sequence on every rank
    core = ShardedCore(T, H, H, D, k, CFG["n_min"], CFG["n_max"], B)
    p = core.plan
    sl = slice(p.q_pos0, p.q_pos0 + p.t_local)
    xs, qs = x[sl].contiguous(), q[sl].contiguous()
    core.k_local.copy_(kk[sl])
    core.v_local.copy_(v[sl])
    del x, q
    torch.cuda.synchronize()

    # the step is ~25 launches: captured into CUDA graphs of one and of GRAPH_STEPS steps (a
    # Python host issues launches more slowly than the GPUs run them at small shards, and
    # eight ranks share the host's cores); the timed loop replays the multi-step graph and
    # reads the device status word once, after the loop
    GRAPH_STEPS = 4
    core.capture(xs, gw, gb, alpha, qs, steps=1)
    core.capture(xs, gw, gb, alpha, qs, steps=GRAPH_STEPS)

    def steps(n):
        for _ in range(n // GRAPH_STEPS):
            core.replay(GRAPH_STEPS, read_status=False)
        for _ in range(n % GRAPH_STEPS):
            core.replay(1, read_status=False)

    steps(args.warmup)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    # one nvidia-smi, on rank 0, samples rank 0's GPU: an nvidia-smi that queries every GPU of
    # the node stalled them (N = 2: 0.78 -> 6.1 ms per step), one per rank cost ~2 % at N = 2.
    # Host stalls (eight ranks and the sampler on one host) must not starve the GPUs inside
    # the timed region: each stream is held by a device-side sleep while the host queues every
    # timed step behind it, and the timer starts when the sleep ends. A one-element all-reduce
    # queued first makes the sleeps start together on every GPU, whatever the hosts' timing.
    align = torch.zeros(1, device=dev)
    with (ClockSampler(local) if rank == 0 else contextlib.nullcontext()) as clk:
        torch.distributed.all_reduce(align)
        torch.cuda._sleep(int(0.03 * 1.9e9))  # ~30 ms of GPU clocks, outside the timed region
        e0.record(stream)
        steps(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    status = ops.device_status()
    # per-phase breakdown of one more (uncaptured) step: CUDA events on this rank's stream,
    # max over ranks; the GPUs first sleep ~5 ms together (after an aligning all-reduce) so that
    # every launch is queued before it runs
    evs = []
    torch.distributed.all_reduce(align)
    torch.cuda._sleep(10_000_000)
    core.forward(xs, gw, gb, alpha, qs, events=evs)
    torch.cuda.synchronize()
    breakdown = {}
    for (_, a), (name, b) in zip(evs[:-1], evs[1:]):
        breakdown[name] = max_over_ranks(a.elapsed_time(b), world)

    # dominant kernel: this rank's attention alone
    w, xn, vn = None, None, None
    out, lmk = core.forward(xs, gw, gb, alpha, qs)
    w, xn, vn = core._sig  # the whole sequence's signals, gathered by the step
    n_att = max(20, args.steps // 4)
    for _ in range(3):
        ops.attention_sharded(qs, core.k_ext, core.v_ext, p.q_pos0, p.kv_pos0, T, w, lmk, B, core.k_src, core.v_src,
                              p.t_local, out=core.out, workspace=core._ws_att)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(n_att):
        ops.attention_sharded(qs, core.k_ext, core.v_ext, p.q_pos0, p.kv_pos0, T, w, lmk, B, core.k_src, core.v_src,
                              p.t_local, out=core.out, workspace=core._ws_att)
    e1.record(stream)
    torch.cuda.synchronize()
    att_ms = max_over_ranks(e0.elapsed_time(e1) / n_att, world)
    att_bytes = 4 * p.t_local * H * D * 2
    hbm, src = peaks()
    achieved = att_bytes / (att_ms / 1e3) / 1e9
    barrier(world)

    # end to end: the shard's inputs from pinned host memory, the shard's output back
    xh, qh = xs.cpu().pin_memory(), qs.cpu().pin_memory()
    kh, vh = core.k_local.cpu().pin_memory(), core.v_local.cpu().pin_memory()
    oh = torch.empty_like(core.out, device="cpu").pin_memory()

    def e2e_step():
        xs.copy_(xh, non_blocking=True)
        qs.copy_(qh, non_blocking=True)
        core.k_local.copy_(kh, non_blocking=True)
        core.v_local.copy_(vh, non_blocking=True)
        o, _ = core.replay()
        oh.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.e2e_steps, world)
    h2d = world * sum(t.numel() * t.element_size() for t in (xh, qh, kh, vh))
    d2h = world * oh.numel() * oh.element_size()
    if rank == 0:
        line = {"metric": METRIC, "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": CFG["workload"], "L": T, "heads": H, "head_dim": D, "d_model": CFG["dm"],
                           "k_lmk": k, "block": B, "n_min": CFG["n_min"], "n_max": CFG["n_max"],
                           "selection": "block_causal", "l2": "inputs larger than L2",
                           "parallelism": f"sequence-sharded x{world} (signals, halo and landmark rows over NVLink "
                                          f"peer memory between device-side barriers)"},
                "clocks": clk.summary(), "device_status": status,
                "e2e": {"value": T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                "roofline": {"bound": "hbm", "kernel": "attn_fwd_tc_kernel (one rank's shard)", "achieved": achieved,
                             "peak": hbm, "peak_source": src, "unit": "GB/s", "frac": achieved / hbm,
                             "traffic": None, "algorithmic_bytes": att_bytes, "kernel_ms": att_ms},
                "step_breakdown_ms": {"max over ranks, one step": breakdown},
                # rank 0 per step: signals 1, selection 10 (4 phases), barriers 4, attention 3
                "gpu_launches": 18 * args.steps}
        print(json.dumps(line), flush=True)
    core.close()
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()


PREFILL = {
    # 24-layer decoder, d_model 1024, 16 heads (head_dim 64), MLP 4096, vocab
    # 50257, w_max 256, k 64, whole-sequence selection; B = 1, L = 16384. The reference's
    # block is SwiGLU (configs[2] says GELU): SwiGLU with d_ff 4096 is used.
    "prefill_cfg3": dict(cfg=dict(vocab_size=50257, d_model=1024, n_layers=24, n_heads=16, n_min=16, n_max=256,
                                  k_lmk=64, max_seq_len=16384, d_ff=4096, selection="global"), L=16384),
    # Qwen2.5-3B-shaped graft: 36 layers, hidden 2048, 16 query / 2 kv heads
    # (head_dim 128), SwiGLU 11008, RMSNorm, RoPE base 1e6, q/k/v bias, vocab 151936,
    # w_max 512, k 128, block-causal; B = 1, L = 32768.
    "prefill_cfg5": dict(cfg=dict(vocab_size=151936, d_model=2048, n_layers=36, n_heads=16, n_min=16, n_max=512,
                                  k_lmk=128, max_seq_len=32768, d_ff=11008, n_kv_heads=2, qkv_bias=True,
                                  rope_base=1e6, selection="block_causal", block=512, tie_weights=False), L=32768),
}


def run_backward(args):
    """The attention backward (``dsalt_attention_bwd``, the reference's ``dsalt_triton_backward``)
    on the core's inputs at ``--seq-len``: block-causal sets of 512 queries, k = 128, H = 16,
    D = 64, bf16, one GPU. ``value`` counts query rows per second; ``useful_tflops`` counts the
    five length-D products per (query, key of A(i)) pair, landmark pairs bounded by 512 rows
    per valid slot."""
    from dsalt_b200 import ops
    dev = torch.device("cuda", 0)
    T, H, D, k, B = CFG["L"], CFG["H"], CFG["D"], CFG["k"], CFG["block"]
    x, gw, gb, alpha, q, kk, v = make_inputs(dev)
    cu = [0, T]
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    _, w, lmk = ops.core_forward(x, gw, gb, CFG["n_min"], CFG["n_max"], alpha, q, kk, v, k, cu_t,
                                 mode="block_causal", block=B, cu_list=cu, return_aux=True)
    out, lse = ops.dsalt_attention(q, kk, v, lmk, None, w, cu_t, lmk_block=B, out_dtype=torch.bfloat16, cu_list=cu,
                                   return_lse=True)
    dout = torch.randn(out.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(1)).to(out.dtype)

    def step():
        return ops.dsalt_attention_backward(dout, q, kk, v, out, lse, lmk, None, w, cu_t, lmk_block=B, cu_list=cu)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    i = torch.arange(T, device=dev)
    pairs = int(torch.minimum(w.long().clamp(min=1), i + 1).sum()) + int((lmk >= 0).sum()) * B // H
    print(json.dumps({"metric": "DSALT attention backward query rows/s", "value": T / (ms / 1e3), "unit": "rows/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "higher_is_better": True, "dtype": "bf16 inputs, fp32 arithmetic", "data": "synthetic",
                      "config": {"workload": f"dsalt_attn_bwd_L{T}_H{H}_D{D}_k{k}_block{B}", "L": T},
                      "useful_tflops": pairs * H * 10 * D / ms / 1e9, "clocks": clk.summary(),
                      "device_status": ops.device_status()}), flush=True)


def run_train(args):
    """The soft-selector training attention (``dsalt_train_attention``, the reference's
    ``dsalt_triton_train_attention``) forward and backward at BASELINE configs[1]'s shapes, the
    pack a training step sees: 4 sequences of 8192 packed, H = 12, D = 64, bf16, k = 64 landmarks
    per (head, sequence) from the global selection, continuous widths
    ``16 + σ(l)·(256 − 16)`` with ``l ~ N(0, 1.5)``, log-weights ``log σ(N(0, 1))``. A step is
    one forward (out, lse) and one backward (dq, dk, dv, d_logw, d_w) through the C ABI;
    ``value`` counts query rows per second over both. ``useful_tflops`` counts two length-D
    products per (query, key) pair in the forward and five in the backward."""
    from dsalt_b200 import ops
    dev = torch.device("cuda", 0)
    S, Ls, H, D, k = 4, 8192, 12, 64, 64
    T = S * Ls
    g = torch.Generator(device=dev).manual_seed(0)
    q, kk, v = (torch.randn(T, H, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
    w = 16.0 + torch.sigmoid(1.5 * torch.randn(T, device=dev, generator=g)) * (256.0 - 16.0)
    cu = [s * Ls for s in range(S + 1)]
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    x = torch.randn(T, 768, device=dev, generator=g).to(torch.bfloat16)
    wv = (0.02 * torch.randn(H * D, 768, device=dev, generator=g)).to(torch.bfloat16)
    alpha = torch.full((H,), 0.6, device=dev)
    lmk, _, _ = ops.compute_landmark_indices(x, wv, alpha, w.floor().clamp(min=1), cu_t, k, 16, T, cu, head_dim=D)
    logw = torch.nn.functional.logsigmoid(torch.randn(H, S, k, device=dev, generator=g))
    dout = torch.randn(T, H, D, device=dev, generator=g)
    tau, edge = 1.0, 4.0

    def fwd():
        return ops.train_attention_forward(q, kk, v, lmk, logw, w, cu_t, tau, edge, out_dtype=torch.float32, cu_list=cu)

    out, lse = fwd()

    def bwd():
        return ops.train_attention_backward(dout, q, kk, v, out, lse, lmk, logw, w, cu_t, tau, edge, cu_list=cu)

    for _ in range(args.warmup):
        fwd()
        bwd()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with ClockSampler(0) as clk:
        ms_f = ms_b = 0.0
        for _ in range(args.steps):
            ev[0].record()
            fwd()
            ev[1].record()
            bwd()
            ev[2].record()
            torch.cuda.synchronize()
            ms_f += ev[0].elapsed_time(ev[1])
            ms_b += ev[1].elapsed_time(ev[2])
    ms_f, ms_b = ms_f / args.steps, ms_b / args.steps
    i = torch.arange(Ls, device=dev).repeat(S)
    band = int(torch.minimum(w.floor().long(), i).sum() + T)
    pos = lmk.long()
    lmk_pairs = 0
    for s in range(S):  # landmark p serves the queries i > p + w̃(i) of its sequence; count them per head
        rows = torch.arange(Ls, device=dev)
        lim = rows.double() - w[cu[s]:cu[s + 1]].double()
        srt = torch.sort(lim).values
        p = pos[:, s][pos[:, s] >= 0].double()
        lmk_pairs += int((Ls - torch.searchsorted(srt, p, right=True)).sum())
    pairs = band * H + lmk_pairs
    ms = ms_f + ms_b
    print(json.dumps({"metric": "DSALT training attention fwd+bwd query rows/s", "value": T / (ms / 1e3),
                      "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                      "ms_forward": ms_f, "ms_backward": ms_b, "higher_is_better": True,
                      "dtype": "bf16 inputs, fp32 arithmetic", "data": "synthetic",
                      "config": {"workload": f"dsalt_train_attn_S{S}x{Ls}_H{H}_D{D}_k{k}_wmax256", "L": T},
                      "pairs_per_step": pairs,
                      "useful_tflops_forward": pairs * 2 * 2 * D / ms_f / 1e9,
                      "useful_tflops_backward": pairs * 5 * 2 * D / ms_b / 1e9, "clocks": clk.summary(),
                      "device_status": ops.device_status()}), flush=True)


def run_prefill(args):
    """Full-model prefill on one GPU: random-init bf16
    weights, uniform random token ids from a seed, every layer's attention on this
    package's kernels, projections / MLP / LM head as library GEMMs. A step is one forward
    of the whole pack including the logits of every token (as the reference returns them)."""
    from dsalt_b200.model import DSALTConfig, DSALTLMHeadModel
    spec = PREFILL[args.workload]
    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    cfg = DSALTConfig(**spec["cfg"])
    with torch.device(dev):
        model = DSALTLMHeadModel.from_config(cfg).to(dev, torch.bfloat16).eval()
    L = spec["L"]
    g = torch.Generator(device=dev).manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (L,), device=dev, generator=g)
    cu = [0, L]
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)

    def step():
        return model(ids, cu_t, cu_list=cu)["logits"]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(args.steps):
            out = step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    from dsalt_b200 import ops
    line = {"metric": "DSALT LM prefill tokens/s", "value": L / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random token ids, random init)",
            "config": {"workload": args.workload, "L": L, **spec["cfg"],
                       "params": sum(p.numel() for p in model.parameters())},
            "clocks": clk.summary(), "device_status": ops.device_status(),
            "logits_finite": bool(torch.isfinite(out[-1].float()).all())}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="core", choices=["core", "backward", "train", *PREFILL],
                    help="core: the DSALT attention core (the benchmark); backward: the attention backward on the "
                         "core's inputs; train: the soft-selector training attention forward + backward at "
                         "configs[1]'s shapes; prefill_cfg3 / prefill_cfg5: full-model prefill of BASELINE configs[2] / "
                         "configs[4] on one GPU")
    ap.add_argument("--seq-len", type=int, default=CFG["L"],
                    help="sequence length (131072 is the benchmark; shorter ones for profiler captures)")
    args = ap.parse_args()
    if args.seq_len != CFG["L"]:
        CFG["L"] = args.seq_len
        CFG["workload"] = CFG["workload"].replace("L131072", f"L{args.seq_len}")
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "backward":
        args.warmup = max(args.warmup, 3)
        return run_backward(args)
    if args.workload == "train":
        args.warmup = max(args.warmup, 3)
        return run_train(args)
    if args.workload != "core":
        args.warmup = max(args.warmup, 3)
        return run_prefill(args)
    args.warmup = max(args.warmup, 3)
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        return run_sharded(args, rank, world, local, dev)
    from dsalt_b200 import ops
    T, H, D, k, B = CFG["L"], CFG["H"], CFG["D"], CFG["k"], CFG["block"]
    x, gw, gb, alpha, q, kk, v = make_inputs(dev, seed=rank)
    cu = [0, T]
    cu_t = torch.tensor(cu, dtype=torch.int32, device=dev)
    out = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(ops.core_workspace_bytes(T, 1, T, H, H, D, k, "block_causal", B), dtype=torch.uint8,
                     device=dev)

    def step():
        ops.core_forward(x, gw, gb, CFG["n_min"], CFG["n_max"], alpha, q, kk, v, k, cu_t, mode="block_causal",
                         block=B, cu_list=cu, workspace=ws, out=out)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    value = T * world / (ms / 1e3)
    status = ops.device_status()

    # dominant kernel: the attention alone on the step's widths and landmark sets
    _, w_i, lmk_i = ops.core_forward(x, gw, gb, CFG["n_min"], CFG["n_max"], alpha, q, kk, v, k, cu_t,
                                     mode="block_causal", block=B, cu_list=cu, return_aux=True)
    n_att = max(20, args.steps // 4)
    for _ in range(3):
        ops.dsalt_attention(q, kk, v, lmk_i, None, w_i, cu_t, lmk_block=B, out_dtype=torch.bfloat16, cu_list=cu)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(n_att):
        ops.dsalt_attention(q, kk, v, lmk_i, None, w_i, cu_t, lmk_block=B, out_dtype=torch.bfloat16, cu_list=cu)
    e1.record(stream)
    torch.cuda.synchronize()
    att_ms = e0.elapsed_time(e1) / n_att
    att_bytes = 4 * T * H * D * 2  # q, k, v read once + output written once (bf16)
    hbm, src = peaks()
    achieved = att_bytes / (att_ms / 1e3) / 1e9
    traffic = profiled_traffic(T)

    # end to end through the C-ABI call with host buffers: every step copies its inputs in
    # from pinned host memory and its output back, as a serving loop would: the copies run
    # on their own streams with two device buffer sets, so that step i's output copy
    # (device -> host) and step i+1's input copy (host -> device) overlap step i's compute
    xh = x.cpu().pin_memory()
    qh, kh, vh = q.cpu().pin_memory(), kk.cpu().pin_memory(), v.cpu().pin_memory()
    oh = torch.empty(T, H, D, dtype=torch.bfloat16).pin_memory()
    bufs = [(torch.empty_like(x), torch.empty_like(q), torch.empty_like(kk), torch.empty_like(v),
             torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        xd, qd, kd, vd, od = bufs[b]
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_done[b])  # step i-2's compute has read this buffer set
            xd.copy_(xh, non_blocking=True)
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
            ev_in[b].record(s_in)
        stream.wait_event(ev_in[b])
        stream.wait_event(ev_out[b])  # step i-2's output has left this buffer
        ops.core_forward(xd, gw, gb, CFG["n_min"], CFG["n_max"], alpha, qd, kd, vd, k, cu_t, mode="block_causal",
                         block=B, cu_list=cu, workspace=ws, out=od)
        ev_done[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[b])
            oh.copy_(od, non_blocking=True)
            ev_out[b].record(s_out)

    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(world)
    e0.record(stream)
    s_in.wait_stream(stream)
    for i in range(args.e2e_steps):
        e2e_step(i)
    stream.wait_stream(s_out)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.e2e_steps, world)
    h2d = sum(t.numel() * t.element_size() for t in (xh, qh, kh, vh))
    d2h = oh.numel() * oh.element_size()

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": CFG["workload"], "L": T, "heads": H, "head_dim": D, "d_model": CFG["dm"],
                           "k_lmk": k, "block": B, "n_min": CFG["n_min"], "n_max": CFG["n_max"],
                           "selection": "block_causal",
                           "l2": f"inputs larger than L2 ({(T * CFG['dm'] * 2 + 3 * T * H * D * 2) / 1e9:.2f} GB per step)",
                           "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
                "clocks": clk.summary(), "device_status": status,
                "e2e": {"value": T * world / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                "roofline": {"bound": "hbm", "kernel": "attn_fwd_tc_kernel", "achieved": achieved, "peak": hbm,
                             "peak_source": src, "unit": "GB/s", "frac": achieved / hbm, "traffic": traffic,
                             "algorithmic_bytes": att_bytes, "kernel_ms": att_ms},
                "step_breakdown_ms": {"attention": att_ms, "signals_and_selection": ms - att_ms},
                "gpu_launches": 13 * args.steps}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(x, gw, gb, alpha, q, kk, v)
            line["cpu_baseline"]["masked_sdpa"] = masked_sdpa_baselines()
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
