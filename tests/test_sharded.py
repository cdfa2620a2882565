"""Sequence-sharded path.

CPU (gloo, world size 2): the exchange helpers (signal all-gather, window halo ring) and
the decomposition itself — every rank's landmark sets and attention rows computed by the
oracle from what the exchange gives it equal the oracle on the whole sequence.
GPU (one GPU): the sharded kernels on emulated shards of one sequence (landmark rows read
through per-shard pointer tables) equal the single-GPU kernels on the whole sequence,
bit for bit. Multi-GPU runs of ``ShardedCore`` are in ``test_sharded_multi_gpu`` (skipped
below 2 GPUs)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsalt_b200.sharded import exchange_halo, gather_signals, shard_plan
from oracle import dsalt_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_shard_plan():
    p = shard_plan(131072, 8, 3, 512)
    assert (p.t_local, p.q_pos0, p.halo, p.kv_pos0, p.set_lo, p.set_hi) == (16384, 49152, 511, 48641, 96, 128)
    assert shard_plan(131072, 8, 0, 512).halo == 0
    with pytest.raises(ValueError):
        shard_plan(131072, 3, 0, 512)
    with pytest.raises(ValueError):
        shard_plan(4096, 16, 0, 512)


def _problem(seed=3, L=2048, H=2, D=16, n_kv=2, k=16):
    g = np.random.default_rng(seed)
    w = g.integers(1, 200, size=L).astype(np.int32)
    xn = g.normal(1.0, 0.3, size=L).astype(np.float32)
    vn = g.normal(1.0, 0.3, size=(L, n_kv)).astype(np.float32)
    q = g.normal(size=(L, H, D)).astype(np.float32)
    kk = g.normal(size=(L, n_kv, D)).astype(np.float32)
    v = g.normal(size=(L, n_kv, D)).astype(np.float32)
    alpha = np.array([0.3, 0.7], dtype=np.float32)[:H]
    return dict(w=w, xn=xn, vn=vn, q=q, k=kk, v=v, alpha=alpha, L=L, H=H, D=D, n_kv=n_kv, k_lmk=k)


def _rank_main(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pr = _problem()
        B, n_max = 512, 200
        plan = shard_plan(pr["L"], world, rank, n_max, B)
        sl = slice(plan.q_pos0, plan.q_pos0 + plan.t_local)
        # 1-2. signals of the own shard, gathered
        w, xn, vn = gather_signals(torch.from_numpy(pr["w"][sl]), torch.from_numpy(pr["xn"][sl]),
                                   torch.from_numpy(pr["vn"][sl]))
        assert np.array_equal(w.numpy(), pr["w"]) and np.array_equal(xn.numpy(), pr["xn"])
        assert np.array_equal(vn.numpy(), pr["vn"])
        # 3. the own blocks' sets from the gathered signals
        sets = O.select_block_causal(xn.numpy(), vn.numpy(), pr["alpha"], w.numpy(), plan.set_hi * B, pr["k_lmk"],
                                     pr["H"], B)[:, plan.set_lo:plan.set_hi]
        # 4. halo ring
        nxt = shard_plan(pr["L"], world, rank + 1, n_max, B).halo if rank + 1 < world else 0
        k_ext = torch.zeros(plan.halo + plan.t_local, pr["n_kv"], pr["D"])
        v_ext = torch.zeros_like(k_ext)
        k_ext[plan.halo:] = torch.from_numpy(pr["k"][sl])
        v_ext[plan.halo:] = torch.from_numpy(pr["v"][sl])
        exchange_halo(k_ext, v_ext, plan, nxt)
        assert np.array_equal(k_ext.numpy(), pr["k"][plan.kv_pos0:plan.q_pos0 + plan.t_local])
        assert np.array_equal(v_ext.numpy(), pr["v"][plan.kv_pos0:plan.q_pos0 + plan.t_local])
        out_q.put((rank, sets))
    finally:
        dist.destroy_process_group()


def test_exchange_and_decomposition_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    pr = _problem()
    full = O.select_block_causal(pr["xn"], pr["vn"], pr["alpha"], pr["w"], pr["L"], pr["k_lmk"], pr["H"], 512)
    np.testing.assert_array_equal(np.concatenate([res[r] for r in range(world)], axis=1), full)
    # attention of the shard rows with the gathered sets equals the whole-sequence oracle
    rows = np.arange(1024, 2048, 37)
    ref, _ = O.attention_forward(pr["q"], pr["k"], pr["v"], pr["w"], full, [0, pr["L"]], lmk_block=512, rows=rows)
    got, _ = O.attention_forward(pr["q"], pr["k"], pr["v"], pr["w"], np.concatenate([res[0], res[1]], axis=1),
                                 [0, pr["L"]], lmk_block=512, rows=rows)
    np.testing.assert_array_equal(got[rows], ref[rows])


@pytest.mark.gpu
def test_sharded_kernels_equal_whole_sequence_on_emulated_shards():
    from dsalt_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    L, H, D, n_kv, k, B, P, n_max = 8192, 4, 64, 2, 64, 512, 4, 300
    q = torch.randn(L, H, D, device=dev, generator=g).bfloat16()
    kk = torch.randn(L, n_kv, D, device=dev, generator=g).bfloat16()
    v = torch.randn(L, n_kv, D, device=dev, generator=g).bfloat16()
    w = torch.randint(1, n_max + 1, (L,), device=dev, generator=g, dtype=torch.int32)
    xn = torch.rand(L, device=dev, generator=g) + 0.5
    vn = torch.rand(L, n_kv, device=dev, generator=g) + 0.5
    alpha = torch.tensor([0.2, 0.5, 0.6, 0.9], device=dev)
    cu = torch.tensor([0, L], dtype=torch.int32, device=dev)
    full_sets = ops.select_landmarks(xn, vn, w, alpha, cu, k, H, mode="block_causal", block=B, cu_list=[0, L])
    full_out = ops.dsalt_attention(q, kk, v, full_sets, None, w, cu, lmk_block=B, out_dtype=torch.bfloat16,
                                   cu_list=[0, L])
    T = L // P
    stride = kk.stride(0) * kk.element_size()
    k_src = torch.tensor([kk.data_ptr() + r * T * stride for r in range(P)], dtype=torch.int64, device=dev)
    v_src = torch.tensor([v.data_ptr() + r * T * stride for r in range(P)], dtype=torch.int64, device=dev)
    outs, sets = [], []
    for r in range(P):
        plan = shard_plan(L, P, r, n_max, B)
        s = ops.select_block_range(xn, vn, w, alpha, k, H, B, plan.set_lo, plan.set_hi)
        o = ops.attention_sharded(q[plan.q_pos0:plan.q_pos0 + T], kk[plan.kv_pos0:plan.q_pos0 + T],
                                  v[plan.kv_pos0:plan.q_pos0 + T], plan.q_pos0, plan.kv_pos0, L, w, s, B, k_src,
                                  v_src, T)
        sets.append(s)
        outs.append(o)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(torch.cat(sets, dim=1), full_sets)
    assert torch.equal(torch.cat(outs), full_out)


@pytest.mark.gpu
@pytest.mark.parametrize("P,alphas", [(2, (0.2, 0.5, 0.6, 0.9)), (4, (0.6, 0.0, 1.0, -0.5))])
def test_select_shard_phases_equal_whole_sequence_on_emulated_ranks(P, alphas):
    """The rank-distributed block-causal selection (dsalt_select_shard) with P ranks emulated
    on one GPU: every rank's workspace is a separate buffer, the peer table points at all of
    them, and the phases run phase by phase over the ranks (what the cross-GPU barriers
    order on P GPUs). The sets equal the whole-sequence selection bit for bit; alpha outside
    [0, 1] takes the unpruned path (every prefix position scored)."""
    from dsalt_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(17 + P)
    L, H, n_kv, k, B = 16384, 4, 2, 64, 512
    w = torch.randint(1, 400, (L,), device=dev, generator=g, dtype=torch.int32)
    xn = 30 + torch.randn(L, device=dev, generator=g)
    vn = 1 + 0.1 * torch.randn(L, n_kv, device=dev, generator=g)
    alpha = torch.tensor(alphas, device=dev)
    cu = torch.tensor([0, L], dtype=torch.int32, device=dev)
    full = ops.select_landmarks(xn, vn, w, alpha, cu, k, H, mode="block_causal", block=B, cu_list=[0, L])
    nbytes = ops.select_shard_workspace_bytes(L, H, n_kv, k, B)
    ws = [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(P)]
    peers = torch.tensor([t.data_ptr() for t in ws], dtype=torch.int64, device=dev)
    sets = [None] * P
    for phase in (1, 2, 3, 4):
        for r in range(P):
            out = ops.select_shard(phase, xn, vn, w, alpha, k, H, B, r, P, ws[r], peers)
            if phase == 4:
                sets[r] = out
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(torch.cat(sets, dim=1), full)


def _gpu_rank_main(rank, world, port, out_q, exchange):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    core = None
    try:
        from dsalt_b200.sharded import ShardedCore
        x, gw, gb, alpha, q, kk, v = _gpu_inputs(torch.device("cuda", rank))
        L, H, D, k, B = q.shape[0], q.shape[1], q.shape[2], 64, 512
        core = ShardedCore(L, H, H, D, k, 16, 300, B, exchange=exchange)
        p = core.plan
        sl = slice(p.q_pos0, p.q_pos0 + p.t_local)
        core.k_local.copy_(kk[sl])
        core.v_local.copy_(v[sl])
        xs, qs = x[sl].contiguous(), q[sl].contiguous()
        for _ in range(2):  # the second step reuses every buffer
            out, lmk = core.forward(xs, gw, gb, alpha, qs)
        torch.cuda.synchronize()
        out, lmk = out.clone(), lmk.clone()
        if exchange == "peer":
            # the step captured into a CUDA graph and replayed (device-side barrier epochs
            # advance on every replay): the same bits, step after step
            core.capture(xs, gw, gb, alpha, qs)
            for _ in range(3):
                o2, l2 = core.replay()
            torch.cuda.synchronize()
            assert torch.equal(o2, out) and torch.equal(l2, lmk)
            core.check()
        from dsalt_b200 import ops
        out_q.put((rank, out.cpu(), lmk.cpu(), ops.device_status()))
    finally:
        if core is not None:
            core.close()
        dist.destroy_process_group()


def _gpu_inputs(dev):
    g = torch.Generator(device=dev).manual_seed(11)
    L, H, D, dm = 8192, 4, 64, 256
    x = torch.randn(L, dm, device=dev, generator=g).bfloat16()
    Wv = (torch.randn(H * D, dm, device=dev, generator=g) * 0.05).bfloat16()
    v = (x @ Wv.T).view(L, H, D).contiguous()
    q = torch.randn(L, H, D, device=dev, generator=g).bfloat16()
    kk = torch.randn(L, H, D, device=dev, generator=g).bfloat16()
    gw = (torch.randn(dm, device=dev, generator=g) * 0.05).bfloat16()
    gb = torch.zeros(1, device=dev).bfloat16()
    alpha = torch.tensor([0.3, 0.5, 0.6, 0.8], device=dev)
    return x, gw, gb, alpha, q, kk, v


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_sharded_core_on_two_gpus_equals_single_gpu(exchange):
    from dsalt_b200 import ops
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank_main, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, out, lmk, st = q.get(timeout=300)
        res[r] = (out, lmk, st)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(res[r][2] == 0 for r in range(world))
    dev = torch.device("cuda", 0)
    x, gw, gb, alpha, qq, kk, v = _gpu_inputs(dev)
    L = qq.shape[0]
    cu = torch.tensor([0, L], dtype=torch.int32, device=dev)
    out, w, lmk = ops.core_forward(x, gw, gb, 16, 300, alpha, qq, kk, v, 64, cu, mode="block_causal", block=512,
                                   cu_list=[0, L], return_aux=True)
    assert torch.equal(torch.cat([res[r][1] for r in range(world)], dim=1), lmk.cpu())
    assert torch.equal(torch.cat([res[r][0] for r in range(world)]), out.cpu())
