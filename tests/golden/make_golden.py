"""Generate the golden fixtures by running the reference (LeonardoCofone/dsalt) on CPU.

Run in a container where the reference is mounted (it is never read at test time):

    PYTHONPATH=/path/to/dsalt TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden.py

For each case of ``cases.py`` it records, from the reference's own functions:

* ``win_gate`` logit and ``_window_sizes(floor=True)``  (``dsalt_attention.py:270-284``)
* the selection signals ``_token_signals``            (``results/causal_landmark_check.py:68-79``)
* whole-sequence mode: ``_compute_landmark_indices`` and ``hybrid_scores_per_head``
  (``dsalt/kernels/selectors.py:75-134``, ``dsalt/kernels/landmark_tokens_ker.py:19-61``)
* block-causal mode: ``_prefix_stats`` / ``_select`` per 512-query block
  (``results/causal_landmark_check.py:82-113``)
* the attention output of ``_block_attention`` (the reference's PyTorch restatement of
  its Triton kernel, ``results/causal_landmark_check.py:119-147``) on a sample of rows
* the module output of ``DSALTAttention`` on the same rows: the real ``_packed``
  orchestration with the Triton call replaced by ``_block_attention`` (whole-sequence
  mode), or ``_packed_checked`` in ``"block"`` mode (block-causal)
* for ``cfg1_fp32`` the masked-SDPA fallback output (the reference's CPU path).

bf16 cases run under ``torch.autocast("cpu", bfloat16)``. Cases with ``norm == "fp32"``
replay CUDA autocast, whose policy runs ``norm`` in fp32 (CPU autocast keeps it in
bf16): a torch-function mode upcasts bf16 inputs of ``Tensor.norm`` to fp32, which is
what ``linalg_vector_norm(..., dtype=float32)`` computes. Nothing else is altered.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import sys

import numpy as np
import torch
from torch.overrides import TorchFunctionMode

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases as C  # noqa: E402


class CudaAutocastNormPolicy(TorchFunctionMode):
    """fp32 ``norm`` of half-precision inputs, as CUDA autocast dispatches it."""

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func in (torch.Tensor.norm, torch.norm, torch.linalg.vector_norm) and args:
            t = args[0]
            if isinstance(t, torch.Tensor) and t.dtype in (torch.bfloat16, torch.float16):
                args = (t.float(),) + tuple(args[1:])
        return func(*args, **kwargs)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def sample_rows(cu, per_seq=48, seed=0):
    rng = np.random.default_rng(seed)
    rows = []
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        L = b - a
        pick = set([0, L - 1, min(L - 1, 1), L // 2]) if L > 0 else set()
        if L > 4:
            pick |= set(rng.choice(L, size=min(per_seq, L), replace=False).tolist())
        rows += [a + i for i in sorted(pick) if 0 <= i < L]
    return np.array(sorted(set(rows)), dtype=np.int64)


def main():
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    from dsalt.modules import dsalt_attention as DA
    from dsalt.kernels import selectors as SEL
    from dsalt.kernels import landmark_tokens_ker as LTK
    import results.causal_landmark_check as CLC

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    only = sys.argv[1:]
    for name, cfg in C.CASES.items():
        if only and name not in only:
            continue
        print(f"[golden] {name}", flush=True)
        T = C.total_len(cfg)
        cu = C.cu_seqlens(cfg)
        H, Hkv, D, dm = cfg["H"], cfg["Hkv"], cfg["D"], cfg["dm"]
        params = C.make_params(cfg)
        attn = DA.DSALTAttention(dm, H, cfg["n_min"], cfg["n_max"], cfg["k"], max(cfg["seqlens"]) + 8,
                                 n_kv_heads=Hkv)
        attn.load_state_dict(params, strict=False)
        attn.eval()
        attn._collect_last_P = False
        x = C.make_x(cfg)
        dt = C.torch_dtype(cfg)
        cu_t = torch.tensor(cu, dtype=torch.int32)
        amp = torch.autocast("cpu", dtype=torch.bfloat16) if cfg["dtype"] == "bf16" else _Null()
        pol = CudaAutocastNormPolicy() if (cfg["dtype"] == "bf16" and cfg["norm"] == "fp32") else _Null()
        rec = {}
        with torch.no_grad(), amp, pol:
            logit = attn.win_gate(x).squeeze(-1)
            w = attn._window_sizes(x, floor=True)
            alpha = attn._alpha().detach().float()
            xn, xwv = CLC._token_signals(attn, x.detach())
            rec["logit"] = logit.float().numpy()
            rec["w"] = w.long().numpy().astype(np.int32)
            rec["xn"] = xn.float().numpy()
            rec["vn"] = xwv.float().numpy()
            rec["alpha"] = alpha.numpy()
            rec["logit_dtype"] = str(logit.dtype)
            rec["w_dtype"] = str(w.dtype)
            if cfg["mode"] == "global":
                lmk, z_x, z_v = SEL._compute_landmark_indices(
                    x.detach(), attn.v_proj.weight.detach(), alpha, w, cu_t, cfg["k"], cfg["n_min"], T,
                    cu, head_dim=D)
                scores, _, _ = LTK.hybrid_scores_per_head(x.detach(), attn.v_proj.weight.detach(), alpha, H, D)
                rec["lmk"] = lmk.numpy().astype(np.int32)
                rec["z_x"] = z_x.float().numpy()
                rec["z_v"] = z_v.float().numpy()
                rec["scores"] = scores.float().numpy()
                sets = [lmk[:, s] for s in range(len(cu) - 1)]
            else:
                L = T
                covered = torch.arange(T) < w.long()
                sx, sv = CLC._prefix_stats(xn), CLC._prefix_stats(xwv)
                B = cfg["block"]
                nb = (L + B - 1) // B
                lmk = torch.full((H, nb, cfg["k"]), -1, dtype=torch.long)
                stats = np.full((nb, 2, 1 + Hkv), np.nan)
                for b in range(nb):
                    b0 = b * B
                    lmk[:, b] = CLC._select(attn, xn, xwv, covered, alpha, b0, sx, sv)
                    if b0 >= 2:
                        mx, sdx = CLC._std_at(*sx, b0)
                        mv, sdv = CLC._std_at(*sv, b0)
                        stats[b, 0, 0], stats[b, 1, 0] = float(mx), float(sdx)
                        stats[b, 0, 1:], stats[b, 1, 1:] = mv.numpy(), sdv.numpy()
                rec["lmk"] = lmk.numpy().astype(np.int32)
                rec["block_stats"] = stats
                sets = None
            # q, k, v exactly as _packed (dsalt_attention.py:566-590)
            q = attn.q_proj(x).view(T, H, D)
            kk = attn.k_proj(x).view(T, Hkv, D)
            vv = attn.v_proj(x).view(T, Hkv, D)
            pos = torch.cat([torch.arange(cu[i + 1] - cu[i]) for i in range(len(cu) - 1)])
            cos, sin = attn.rope_cos[pos].to(q.dtype), attn.rope_sin[pos].to(q.dtype)
            from dsalt.kernels.window_utils import apply_rotary_emb
            q, kk = apply_rotary_emb(q, kk, cos.unsqueeze(1), sin.unsqueeze(1))
            kk = attn._repeat_kv(kk)
            vr = attn._repeat_kv(vv)
            rec["q_sha"], rec["k_sha"], rec["v_sha"] = sha(q), sha(kk), sha(vr)
            rec["vproj_sha"] = sha(vv.reshape(T, Hkv * D))
            scale = 1.0 / math.sqrt(D)
            rows = sample_rows(cu, per_seq=48 if T <= 2048 else 96, seed=cfg["seed"])
            out = torch.zeros(T, H, D)
            # the kernel accumulates q·k and P·V in fp32: evaluate the restatement with
            # autocast off (pure fp32 arithmetic on the compute-dtype q, k, v)
            noamp = torch.autocast("cpu", enabled=False)
            noamp.__enter__()
            for s in range(len(cu) - 1):
                a, b = cu[s], cu[s + 1]
                if b == a:
                    continue
                if cfg["mode"] == "global":
                    out[a:b] = CLC._block_attention(q[a:b], kk[a:b], vr[a:b], w[a:b], sets[s], 0, b - a, scale)
                else:
                    B = cfg["block"]
                    for bi, b0 in enumerate(range(0, b - a, B)):
                        b1 = min(b - a, b0 + B)
                        out[a + b0:a + b1] = CLC._block_attention(q[a:b], kk[a:b], vr[a:b], w[a:b],
                                                                  lmk[:, bi], b0, b1, scale)
            noamp.__exit__(None, None, None)
            rec["rows"] = rows
            rec["out_rows"] = out[rows].numpy()

            # module-level output
            if cfg["mode"] == "global":
                def tri_sub(q_, k_, v_, lmk_, bias_, w_, cu_):
                    o = torch.zeros(q_.shape, dtype=torch.float32)
                    cl = cu_.tolist()
                    for s in range(len(cl) - 1):
                        a, b = cl[s], cl[s + 1]
                        if b > a:
                            o[a:b] = CLC._block_attention(q_[a:b], k_[a:b], v_[a:b], w_[a:b], lmk_[:, s], 0,
                                                          b - a, scale)
                    in_dt = q_.dtype if q_.dtype in (torch.float16, torch.bfloat16) else torch.float16
                    return o.to(in_dt).float()
                saved = (DA._TRITON_OK, getattr(DA, "dsalt_triton_attention", None))
                DA._TRITON_OK = True
                DA.dsalt_triton_attention = tri_sub
                try:
                    mod_out, _ = CLC._ORIG_PACKED(attn, x, cu_t, T, x.device, None, cu)
                finally:
                    DA._TRITON_OK, DA.dsalt_triton_attention = saved
            else:
                CLC._CFG["mode"] = "block"
                CLC._CFG["block"] = cfg["block"]
                try:
                    mod_out, _ = CLC._packed_checked(attn, x, cu_t, T, x.device, None, cu)
                finally:
                    CLC._CFG["mode"] = "triton"
            rec["mod_rows"] = mod_out.float()[rows].numpy()
            if name == "cfg1_fp32":
                DA._TRITON_OK = False
                fb, _ = CLC._ORIG_PACKED(attn, x, cu_t, T, x.device, None, cu)
                rec["fallback_mod_rows"] = fb.float()[rows].numpy()
        rec["x_sha"] = sha(x)
        rec["cfg"] = json.dumps(cfg)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
        print(f"[golden] wrote {name}.npz  (T={T}, lmk {rec['lmk'].shape})", flush=True)


if __name__ == "__main__":
    main()
