"""Sequence-sharded DSALT core (block-causal selection) over the GPUs of one node, one
process per GPU (``torch.distributed``, NCCL).

One sequence of ``seq_len`` positions is split into contiguous shards of ``T_local``
positions; rank ``r`` owns queries ``[r·T_local, (r+1)·T_local)`` and computes their
projections outside this module. Per step:

1. window widths and selection signals of the rank's own tokens (``dsalt_token_signals``);
2. a device-side barrier across the GPUs, then every rank pulls the other ranks' compact
   signals (``w``, ``‖x‖``, value norms: 4·(2+H_kv) bytes per token) over NVLink, so every
   rank holds them for the whole sequence (or one grouped NCCL all-gather);
3. the block-causal landmark sets of the rank's own 512-query blocks (block ``b`` uses the
   prefix ``[0, b·512)``, as ``results/causal_landmark_check.py:176-186``). With the peer
   exchange the selection's per-block work is spread over the ranks
   (``dsalt_select_shard``): each rank sums, bins and prunes only its own blocks and reads
   the other ranks' block records from their memory between device-side barriers; with
   NCCL each rank runs ``dsalt_select_block_range`` over its whole prefix;
4. the window halo: the previous rank's last ``n_max - 1`` K/V rows, copied into the rows
   in front of the local shard;
5. the attention of the local queries (``dsalt_attention_fwd_sharded``): window tiles from
   the halo-extended local K/V, landmark rows read directly from their owner's K/V shard
   over NVLink (CUDA IPC peer mappings, plain loads — no multicast);
6. a closing barrier, so that no rank overwrites its K/V shard or signals while another
   may still read them.

The output stays sharded (``[T_local, H, D]`` per rank). Results equal the single-GPU
core on the whole sequence bit for bit (same kernels, same tiles).

The exchange helpers (:func:`shard_plan`, :func:`gather_signals`,
:func:`exchange_halo`) are device-agnostic and tested with ``gloo`` on CPU.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist


@dataclasses.dataclass(frozen=True)
class ShardPlan:
    world: int
    rank: int
    seq_len: int
    t_local: int      # queries per rank
    q_pos0: int       # first position of the rank's queries
    halo: int         # K/V rows in front of the shard (keys of earlier ranks)
    block: int        # selection block (queries per landmark set)

    @property
    def kv_pos0(self) -> int:
        return self.q_pos0 - self.halo

    @property
    def set_lo(self) -> int:
        return self.q_pos0 // self.block

    @property
    def set_hi(self) -> int:
        return (self.q_pos0 + self.t_local) // self.block


def shard_plan(seq_len: int, world: int, rank: int, n_max: int, block: int = 512) -> ShardPlan:
    """Contiguous shards of ``seq_len / world`` positions. Each shard must be a whole
    number of selection blocks and of 128-query tiles; the halo holds ``n_max - 1`` keys
    (the widest window reaches ``n_max - 1`` positions back)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    if seq_len % world:
        raise ValueError(f"seq_len {seq_len} is not divisible by {world} ranks")
    t_local = seq_len // world
    if t_local % block or t_local % 128:
        raise ValueError(f"shard of {t_local} positions is not a whole number of {block}-query blocks")
    q_pos0 = rank * t_local
    halo = min(q_pos0, max(n_max - 1, 0))
    return ShardPlan(world, rank, seq_len, t_local, q_pos0, halo, block)


def gather_signals(w_loc: torch.Tensor, xn_loc: torch.Tensor, vn_loc: torch.Tensor, group=None, out=None):
    """All-gather the per-token signals of every rank's shard.

    ``w_loc [T]`` int32, ``xn_loc [T]`` fp32, ``vn_loc [T, H_kv]`` fp32 →
    ``(w [P·T], xn [P·T], vn [P·T, H_kv])`` in position order, gathered straight into the
    output tensors (``out``, reused across steps when given); over NCCL the three
    collectives are issued as one group."""
    T = w_loc.shape[0]
    n_kv = vn_loc.shape[1]
    P = dist.get_world_size(group)
    if out is None:
        out = (torch.empty(P * T, dtype=torch.int32, device=w_loc.device),
               torch.empty(P * T, dtype=torch.float32, device=w_loc.device),
               torch.empty(P * T, n_kv, dtype=torch.float32, device=w_loc.device))
    w, xn, vn = out
    pairs = ((w, w_loc), (xn, xn_loc), (vn.view(-1), vn_loc.reshape(-1)))
    if dist.get_backend(group) == "nccl":
        with dist._coalescing_manager(group, w_loc.device, async_ops=True) as cm:
            for o, i in pairs:
                dist.all_gather_into_tensor(o, i, group=group)
        cm.wait()
    else:
        for o, i in pairs:
            dist.all_gather_into_tensor(o, i, group=group)
    return w, xn, vn


def exchange_halo(k_ext: torch.Tensor, v_ext: torch.Tensor, plan: ShardPlan, halo_next: int, group=None):
    """Ring exchange of the window halo: the last ``halo_next`` rows of this rank's shard go
    to rank+1; the previous rank's last ``plan.halo`` rows land in ``k_ext[:plan.halo]``
    (and likewise for V). ``k_ext`` / ``v_ext`` are ``[halo + T_local, H_kv, D]``."""
    ops = []
    r, P = plan.rank, plan.world
    if r + 1 < P and halo_next > 0:
        ops.append(dist.P2POp(dist.isend, k_ext[k_ext.shape[0] - halo_next:].contiguous(), r + 1, group))
        ops.append(dist.P2POp(dist.isend, v_ext[v_ext.shape[0] - halo_next:].contiguous(), r + 1, group))
    if r > 0 and plan.halo > 0:
        ops.append(dist.P2POp(dist.irecv, k_ext[:plan.halo], r - 1, group))
        ops.append(dist.P2POp(dist.irecv, v_ext[:plan.halo], r - 1, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class ShardedCore:
    """The core of one DSALT layer (widths, block-causal selection, attention) for one
    rank's shard of a sequence. ``k_local`` / ``v_local`` are the views the caller writes
    its shard's post-RoPE keys / values into before :meth:`forward`.

    ``exchange="peer"`` (default) moves the signals and the halo over NVLink peer memory
    between two device-side barriers (``dsalt_peer_barrier``); ``exchange="nccl"`` uses the
    NCCL collectives of :func:`gather_signals` / :func:`exchange_halo` and a closing
    all-reduce.

    Failure reporting: a device-side barrier that waits more than 2 s for a peer (a rank
    that died or stalled) gives up, sets the device status word and lets the step finish;
    that step's output, and every later one, is then invalid (stale signals or halo rows).
    Every step queues an asynchronous read of the status word; :meth:`forward` raises
    ``DsaltError`` (code ``ERR_DEVICE``) as soon as a completed read shows a non-zero
    status — at the latest one call later — and :meth:`check` (or ``forward(..., check=True)``)
    synchronises and raises for the step just queued."""

    def __init__(self, seq_len: int, n_heads: int, n_kv: int, head_dim: int, k_lmk: int, n_min: int, n_max: int,
                 block: int = 512, dtype=torch.bfloat16, group=None, exchange: str = "peer"):
        from . import ops
        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
        self.ops = ops
        self.exchange = exchange
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.plan = shard_plan(seq_len, self.world, self.rank, n_max, block)
        nxt = shard_plan(seq_len, self.world, self.rank + 1, n_max, block) if self.rank + 1 < self.world else None
        self.halo_next = nxt.halo if nxt is not None else 0
        self.n_heads, self.n_kv, self.head_dim = n_heads, n_kv, head_dim
        self.k_lmk, self.n_min, self.n_max, self.block = k_lmk, n_min, n_max, block
        dev = torch.device("cuda", torch.cuda.current_device())
        p = self.plan
        T = p.t_local
        self.k_ext = torch.zeros(p.halo + T, n_kv, head_dim, dtype=dtype, device=dev)
        self.v_ext = torch.zeros_like(self.k_ext)
        self.k_local = self.k_ext[p.halo:]
        self.v_local = self.v_ext[p.halo:]
        self.out = torch.empty(T, n_heads, head_dim, dtype=dtype, device=dev)
        # signals of the whole sequence; this rank writes its slice, the rest is gathered
        self._sig = (torch.empty(seq_len, dtype=torch.int32, device=dev),
                     torch.empty(seq_len, dtype=torch.float32, device=dev),
                     torch.empty(seq_len, n_kv, dtype=torch.float32, device=dev))
        sl = slice(p.q_pos0, p.q_pos0 + T)
        self._w, self._xn, self._vn = self._sig[0][sl], self._sig[1][sl], self._sig[2][sl]
        self._flag = torch.zeros(4, dtype=torch.int32, device=dev)
        self._epoch = 0
        L_ = ops.L
        nsel = L_.query("dsalt_select_block_range_workspace_bytes", seq_len, n_heads, n_kv, k_lmk, block, p.set_hi)
        nshard = ops.select_shard_workspace_bytes(seq_len, n_heads, n_kv, k_lmk, block)
        # the distributed selection's workspace: the same size on every rank, read by peers
        self._ws_shard = torch.empty(max(nshard, 1), dtype=torch.uint8, device=dev)
        self._lmk = torch.empty(n_heads, p.set_hi - p.set_lo, k_lmk, dtype=torch.int32, device=dev)
        self._alpha_key, self._alpha_unit = None, False
        natt = L_.query("dsalt_attention_sharded_workspace_bytes", T, n_heads, k_lmk, block, head_dim)
        self._ws_sel = torch.empty(max(nsel, 1), dtype=torch.uint8, device=dev)
        self._ws_att = torch.empty(max(natt, 1), dtype=torch.uint8, device=dev)
        self._peers = []
        self._open_peers()
        self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._status_event = None
        self._graph, self._graph_res = None, None
        self._graphs = {}  # steps per graph -> (graph, outputs of its last step)

    def _open_peers(self):
        """Peer pointer tables (CUDA IPC; own entries local): K / V shards, the signal
        arrays' slices, the barrier flags."""
        T, r = self.plan.t_local, self.rank
        bufs = [self.k_local, self.v_local, self._sig[0], self._sig[1], self._sig[2], self._flag, self._ws_shard]
        mine = [self.ops.ipc_export(b) for b in bufs]
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=self.group)
        tables = [[] for _ in bufs]
        for j, handles in enumerate(allh):
            for i, (h, off) in enumerate(handles):
                if j == r:
                    tables[i].append(bufs[i].data_ptr())
                else:
                    ptr = self.ops.ipc_open(h, off)
                    self._peers.append((ptr, off))
                    tables[i].append(ptr)
        dev = self.k_local.device
        self._kp, self._vp = tables[0], tables[1]
        self.k_src = torch.tensor(tables[0], dtype=torch.int64, device=dev)
        self.v_src = torch.tensor(tables[1], dtype=torch.int64, device=dev)
        # rank j's slice of each signal array
        self._w_src = torch.tensor([a + j * T * 4 for j, a in enumerate(tables[2])], dtype=torch.int64, device=dev)
        self._x_src = torch.tensor([a + j * T * 4 for j, a in enumerate(tables[3])], dtype=torch.int64, device=dev)
        self._v_src = torch.tensor([a + j * T * self.n_kv * 4 for j, a in enumerate(tables[4])], dtype=torch.int64,
                                   device=dev)
        self._flags = torch.tensor(tables[5], dtype=torch.int64, device=dev)
        self._ws_peers = torch.tensor(tables[6], dtype=torch.int64, device=dev)

    def close(self):
        # the graphs' kernels hold peer pointers: release them first
        self._graph, self._graph_res, self._graphs = None, None, {}
        for ptr, off in self._peers:
            self.ops.ipc_close(ptr, off)
        self._peers = []

    def _barrier(self):
        # the epoch comes from the device counter in _flag[1] (graph replays advance it)
        L_, ops = self.ops.L, self.ops
        L_.call("dsalt_peer_barrier", ops._ptr(self._flag), ops._ptr(self._flags), self.world, self.rank, 0,
                ops._stream())

    def _alpha_in_unit(self, alpha) -> bool:
        """Whether every head's alpha lies in [0, 1] (read once per alpha tensor version)."""
        key = (alpha.data_ptr(), alpha._version)
        if key != self._alpha_key:
            self._alpha_unit = bool(((alpha >= 0) & (alpha <= 1)).all())
            self._alpha_key = key
        return self._alpha_unit

    def _raise_if_failed(self):
        st = int(self._status_host[0])
        if st != 0:
            L_ = self.ops.L
            raise L_.DsaltError(L_.ERR_DEVICE, "ShardedCore.forward",
                                f"device status {st}: a kernel gave up a bounded wait (a peer rank stalled or "
                                f"died); the step's output is invalid")

    def check(self):
        """Waits for the last queued step and raises if a kernel of any step so far gave up
        a bounded wait (the device status word is not cleared)."""
        if self._status_event is not None:
            self._status_event.synchronize()
            self._raise_if_failed()

    def forward(self, x, gate_weight, gate_bias, alpha, q, check: bool = False, events=None):
        """``x [T_local, d_model]`` and ``q [T_local, H, D]`` of this rank's positions (``k_local`` /
        ``v_local`` already written). Returns this rank's attention output ``[T_local, H, D]``
        and its landmark sets. Raises when an earlier step's status read has completed with a
        non-zero status; ``check=True`` also waits for this step and checks it. ``events``
        (a list) receives ``(phase name, CUDA event)`` pairs recorded after each phase, for a
        per-phase time breakdown."""
        if self._status_event is not None and self._status_event.query():
            self._raise_if_failed()
        out, lmk = self._step(x, gate_weight, gate_bias, alpha, q, events)
        self._read_status()
        if check:
            self.check()
        return out, lmk

    def _read_status(self):
        # the device status word, read without stalling the stream
        self.ops.L.call("dsalt_device_status_async", self._status_host.data_ptr(), self.ops._stream())
        if self._status_event is None:
            self._status_event = torch.cuda.Event()
        self._status_event.record()

    def capture(self, x, gate_weight, gate_bias, alpha, q, steps: int = 1):
        """Record ``steps`` consecutive steps into one CUDA graph (peer exchange only): a step
        is ~25 launches, which a Python host issues more slowly than the GPUs run them once
        the shards are small, and with several steps per graph one host call queues several
        steps. The graph keeps the pointers of ``x``, ``q``, ``k_local`` / ``v_local`` and of
        the weights: write new inputs into those tensors and call :meth:`replay`. Every rank
        captures together (the capture runs one ordinary step first, with its barriers).
        Capturing again keeps the graphs captured before (see :meth:`replay`)."""
        if self.exchange != "peer":
            raise ValueError("graph capture needs exchange='peer'")
        if steps < 1:
            raise ValueError("steps must be >= 1")
        self.forward(x, gate_weight, gate_bias, alpha, q)  # first-call set-up outside the capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        # library set-up calls made outside the stream (function attributes, device queries)
        # are allowed during the capture
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            for _ in range(steps):
                res = self._step(x, gate_weight, gate_bias, alpha, q)
        self._graphs[steps] = (g, res)
        self._graph, self._graph_res = g, res

    def replay(self, steps: int = 1, read_status: bool = True):
        """``steps`` steps from the graph captured with that many steps (default: one);
        returns (out, landmark sets) of the last one like :meth:`forward`. With
        ``read_status=False`` the device status word is not read after the replay (a timed
        loop reads it once at its end with :meth:`check`-like calls of its own)."""
        if self._status_event is not None and self._status_event.query():
            self._raise_if_failed()
        if steps not in self._graphs:
            raise ValueError(f"no graph of {steps} steps captured")
        g, res = self._graphs[steps]
        g.replay()
        if read_status:
            self._read_status()
        return res

    def _step(self, x, gate_weight, gate_bias, alpha, q, events=None):
        ops, p = self.ops, self.plan
        L = ops.L
        T = p.t_local

        def mark(name):
            if events is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                events.append((name, e))

        mark("start")
        # 1. own signals, into this rank's slice of the sequence arrays
        L.call("dsalt_token_signals", ops._ptr(x), ops._dt(x), T, x.shape[1], x.stride(0),
               ops._ptr(gate_weight), ops._ptr(gate_bias), ops._dt(gate_weight), self.n_min, self.n_max,
               ops._ptr(self.v_local), ops._dt(self.v_local), self.v_local.stride(0), self.n_kv, self.head_dim,
               L.NORM_F32, ops._ptr(self._w), ops._ptr(self._xn), ops._ptr(self._vn), None, None, ops._stream())
        mark("signals")
        w, xn, vn = self._sig
        row_bytes = self.k_local.stride(0) * self.k_local.element_size()
        if self.exchange == "peer":
            H, k, B, P, r = self.n_heads, self.k_lmk, self.block, self.world, self.rank
            sel = (xn, vn, w, alpha, k, H, B, r, P, self._ws_shard, self._ws_peers)
            # chunk sums of the own blocks
            ops.select_shard(1, *sel)
            mark("select phase 1")
            # 2. every rank's signals, sums and K / V are written
            self._barrier()
            mark("barrier 1")
            # 3. the window halo over NVLink; the other ranks' signals only when some head is
            #    scored without pruning (alpha outside [0, 1] reads the whole prefix)
            if not self._alpha_in_unit(alpha):
                for dst, src, n in ((w, self._w_src, T * 4), (xn, self._x_src, T * 4),
                                    (vn, self._v_src, T * self.n_kv * 4)):
                    L.call("dsalt_peer_allgather", ops._ptr(dst), ops._ptr(src), self.world, self.rank, n,
                           ops._stream())
            if p.halo > 0:
                src_k = self._kp[self.rank - 1] + (T - p.halo) * row_bytes
                src_v = self._vp[self.rank - 1] + (T - p.halo) * row_bytes
                L.call("dsalt_peer_copy", ops._ptr(self.k_ext), src_k, p.halo * row_bytes, ops._stream())
                L.call("dsalt_peer_copy", ops._ptr(self.v_ext), src_v, p.halo * row_bytes, ops._stream())
            mark("halo")
            # 4. selection of the own blocks, its phases between barriers
            ops.select_shard(2, *sel)
            mark("select phase 2")
            self._barrier()
            mark("barrier 2")
            ops.select_shard(3, *sel)
            mark("select phase 3")
            self._barrier()
            mark("barrier 3")
            lmk = ops.select_shard(4, *sel, lmk_out=self._lmk)
            mark("select phase 4")
        else:
            gather_signals(self._w, self._xn, self._vn, self.group, out=self._sig)
            exchange_halo(self.k_ext, self.v_ext, p, self.halo_next, self.group)
            # 4. landmark sets of the own blocks
            lmk = ops.select_block_range(xn, vn, w, alpha, self.k_lmk, self.n_heads, self.block, p.set_lo, p.set_hi,
                                         workspace=self._ws_sel)
        # 5. attention of the own queries (landmark rows read from their owners)
        ops.attention_sharded(q, self.k_ext, self.v_ext, p.q_pos0, p.kv_pos0, p.seq_len, w, lmk, self.block,
                              self.k_src, self.v_src, p.t_local, out=self.out, workspace=self._ws_att)
        mark("attention")
        # 6. every rank is done reading the others' memory
        if self.exchange == "peer":
            self._barrier()
        else:
            dist.all_reduce(self._flag[:1], group=self.group)
        mark("closing barrier")
        return self.out, lmk
