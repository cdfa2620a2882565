"""dsalt_attention_fwd_noalloc: the attention forward with its scratch in a static device
array instead of a caller workspace. Compared bit for bit with dsalt_attention_fwd (the
same kernels) over calls made back to back, so that a table left over from one call
would show in the next. Kept in a file that is collected last, so that it also runs
after everything else has used the library."""
import numpy as np
import pytest
import torch

from dsalt_b200 import _lib as L
from dsalt_b200 import ops


def _ptr(t):
    return None if t is None else t.data_ptr()


def _problem(seed, lens, H, Hkv, D, k, lmk_block, dtype, bias):
    g = np.random.default_rng(seed)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    tg = torch.Generator().manual_seed(seed)
    q = torch.randn(T, H, D, generator=tg).to(dtype)
    kk = torch.randn(T, Hkv, D, generator=tg).to(dtype)
    v = torch.randn(T, Hkv, D, generator=tg).to(dtype)
    w = g.integers(1, 300, size=T).astype(np.int32)
    sets = []
    for L_ in lens:
        n = -(-L_ // lmk_block) if lmk_block else 1
        for _ in range(n):
            sets.append(L_)
    lmk = np.full((H, len(sets), k), -1, np.int32)
    for h in range(H):
        for j, L_ in enumerate(sets):
            m = min(k, L_)
            lmk[h, j, :m] = np.sort(g.choice(L_, size=m, replace=False))
    b = torch.randn(H, len(sets), k, generator=tg) if bias else None
    dev = torch.device("cuda", 0)
    return dict(q=q.to(dev), kt=kk.to(dev), v=v.to(dev), w=torch.from_numpy(w).to(dev),
                lmk=torch.from_numpy(lmk).to(dev), bias=None if b is None else b.to(dev),
                cu=torch.from_numpy(cu).to(dev), T=T, H=H, Hkv=Hkv, D=D, kl=k, lmk_block=lmk_block,
                n_seqs=len(lens), max_len=int(max(lens)), dtype=dtype)


def _args(p, out, lse):
    dt = {torch.bfloat16: L.BF16, torch.float16: L.F16, torch.float32: L.F32}[p["dtype"]]
    return [_ptr(p["q"]), _ptr(p["kt"]), _ptr(p["v"]), dt, p["T"], p["H"], p["Hkv"], p["D"], p["q"].stride(0),
            p["kt"].stride(0), _ptr(p["w"]), _ptr(p["lmk"]), _ptr(p["bias"]), p["kl"], p["lmk_block"], _ptr(p["cu"]),
            p["n_seqs"], p["max_len"], _ptr(out), dt, _ptr(lse)]


def _outputs(p):
    out = torch.full((p["T"], p["H"], p["D"]), float("nan"), dtype=p["dtype"], device="cuda")
    lse = torch.full((p["T"], p["H"]), float("nan"), dtype=torch.float32, device="cuda")
    return out, lse


def _with_workspace(p):
    out, lse = _outputs(p)
    n = L.query("dsalt_attention_workspace_bytes", p["T"], p["n_seqs"], p["H"], p["kl"], p["lmk_block"])
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device="cuda")
    L.call("dsalt_attention_fwd", *_args(p, out, lse), _ptr(ws), ws.numel(),
           torch.cuda.current_stream().cuda_stream)
    return out, lse


def _no_alloc(p):
    out, lse = _outputs(p)
    L.call("dsalt_attention_fwd_noalloc", *_args(p, out, lse), torch.cuda.current_stream().cuda_stream)
    return out, lse


def test_no_alloc_rejects_more_than_its_scratch_holds():
    # checked before any CUDA call: runs without a GPU
    lib = L.load()
    rc = lib.dsalt_attention_fwd_noalloc(None, None, None, L.BF16, 8, 1, 1, 64, 64, 64, None, None, None, 0, 0,
                                         None, L.NOALLOC_MAX_SEQS + 1, 8, None, L.BF16, None, None)
    assert rc == L.ERR_UNSUPPORTED
    assert b"static scratch limit" in lib.dsalt_last_error()
    rc = lib.dsalt_attention_fwd_noalloc(None, None, None, L.BF16, L.NOALLOC_MAX_TOKENS + 1, 1, 1, 64, 64, 64, None,
                                         None, None, 0, 0, None, 1, 8, None, L.BF16, None, None)
    assert rc == L.ERR_UNSUPPORTED


@pytest.mark.gpu
def test_no_alloc_matches_workspace_entry_point_on_calls_in_a_row():
    rng = np.random.default_rng(3)
    # call 1: bf16, ragged block-causal sets with bias, GQA; call 2: fp16, one set per
    # sequence, more sequences; call 3: the largest sequence count the scratch holds
    p1 = _problem(11, [700, 1200, 1100], H=4, Hkv=2, D=64, k=64, lmk_block=256, dtype=torch.bfloat16, bias=True)
    p2 = _problem(12, [300, 5, 2000, 129, 640], H=2, Hkv=2, D=64, k=128, lmk_block=0, dtype=torch.float16,
                  bias=False)
    p3 = _problem(13, list(rng.integers(1, 40, size=L.NOALLOC_MAX_SEQS)), H=2, Hkv=1, D=64, k=16, lmk_block=128,
                  dtype=torch.bfloat16, bias=False)
    got = [_no_alloc(p1), _no_alloc(p2), _no_alloc(p3)]
    torch.cuda.synchronize()
    ref = [_with_workspace(p1), _with_workspace(p2), _with_workspace(p3)]
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    for (o, l), (ro, rl) in zip(got, ref):
        assert not torch.isnan(o.float()).any()
        assert torch.equal(o, ro)
        assert torch.equal(torch.nan_to_num(l, neginf=-1e30), torch.nan_to_num(rl, neginf=-1e30))
    # a repeat of call 1 after the others gives the same result again
    o1, l1 = _no_alloc(p1)
    torch.cuda.synchronize()
    assert torch.equal(o1, ref[0][0]) and torch.equal(l1, ref[0][1])
