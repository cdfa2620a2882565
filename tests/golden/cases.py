"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Every case is a single DSALT attention layer in the shapes of one of the reference's
benchmark configurations (reduced in length where the CPU reference would be slow).
Inputs are Gaussian, weights ``N(0, 0.02)`` with zero biases and ``alpha_w`` at the
reference's initial value ``log(0.6/0.4)`` (``dsalt/modules/dsalt_attention.py:228``).
All randomness comes from a CPU ``torch.Generator`` so the values are the same on
every machine running this torch build.
"""
from __future__ import annotations

import math

import torch

# name -> configuration
CASES = {
    # fp32, full size of the reference's CPU case, whole-sequence selection
    "cfg1_fp32": dict(seqlens=[1024], H=4, Hkv=4, D=64, dm=256, n_min=16, n_max=128, k=32,
                      dtype="fp32", mode="global", norm="none", seed=101),
    # configs[1] shapes, shorter sequences, packed uniform batch; CUDA-autocast norms
    "cfg2_bf16_packed": dict(seqlens=[512, 512, 512, 512], H=12, Hkv=12, D=64, dm=768, n_min=16,
                             n_max=256, k=64, dtype="bf16", mode="global", norm="fp32", seed=202),
    # ragged pack with degenerate sequences (a single token, shorter than k, all covered)
    "cfg2_bf16_ragged": dict(seqlens=[300, 700, 1, 47, 512], H=12, Hkv=12, D=64, dm=768, n_min=16,
                             n_max=256, k=64, dtype="bf16", mode="global", norm="fp32", seed=203),
    # bf16 norms (no autocast promotion): exercises exact score ties
    "cfg2_bf16_ties": dict(seqlens=[1024, 1024], H=12, Hkv=12, D=64, dm=768, n_min=16, n_max=256,
                           k=64, dtype="bf16", mode="global", norm="bf16", seed=204),
    # configs[3] shapes, L=4096 instead of 131072: block-causal, blocks of 512
    "cfg4_block": dict(seqlens=[4096], H=16, Hkv=16, D=64, dm=1024, n_min=16, n_max=512, k=128,
                       dtype="bf16", mode="block", norm="fp32", seed=404, block=512),
    # block-causal with bf16 norms (ties) and a ragged last block
    "cfg4_block_ties": dict(seqlens=[2500], H=16, Hkv=16, D=64, dm=1024, n_min=16, n_max=512,
                            k=128, dtype="bf16", mode="block", norm="bf16", seed=405, block=512),
    # grouped-query attention (configs[4] uses Hkv=2), both selection modes
    "gqa_global": dict(seqlens=[640, 384], H=8, Hkv=2, D=64, dm=512, n_min=16, n_max=256, k=64,
                       dtype="bf16", mode="global", norm="fp32", seed=505),
    "gqa_block": dict(seqlens=[1536], H=8, Hkv=2, D=64, dm=512, n_min=16, n_max=512, k=64,
                      dtype="bf16", mode="block", norm="fp32", seed=506, block=512),
}


def total_len(cfg) -> int:
    return int(sum(cfg["seqlens"]))


def cu_seqlens(cfg) -> list:
    cu = [0]
    for L in cfg["seqlens"]:
        cu.append(cu[-1] + int(L))
    return cu


def torch_dtype(cfg):
    return {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}[cfg["dtype"]]


def make_params(cfg) -> dict:
    """fp32 parameters of one ``DSALTAttention`` layer (state-dict names of the reference)."""
    g = torch.Generator().manual_seed(cfg["seed"])
    dm, H, Hkv, D = cfg["dm"], cfg["H"], cfg["Hkv"], cfg["D"]
    kv = Hkv * D

    def nrm(*shape):
        return torch.randn(*shape, generator=g) * 0.02

    p = {
        "q_proj.weight": nrm(dm, dm),
        "k_proj.weight": nrm(kv, dm),
        "v_proj.weight": nrm(kv, dm),
        "out_proj.weight": nrm(dm, dm),
        "win_gate.weight": nrm(1, dm),
        "win_gate.bias": torch.zeros(1),
        "alpha_w": torch.full((H,), math.log(0.6 / 0.4)),
    }
    return p


def make_x(cfg) -> torch.Tensor:
    """Block input ``x [T, d_model]`` in the case's compute dtype."""
    g = torch.Generator().manual_seed(cfg["seed"] + 7919)
    x = torch.randn(total_len(cfg), cfg["dm"], generator=g)
    return x.to(torch_dtype(cfg))


def rope_cache(L, D, base=10000.0, scale=1.0):
    """Same numbers as ``build_rope_cache`` (``dsalt/kernels/window_utils.py:91-106``)."""
    theta = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    pos = torch.arange(L, dtype=torch.float32) / scale
    emb = torch.cat([torch.outer(pos, theta)] * 2, dim=-1)
    return emb.cos(), emb.sin()


def rope(q, k, cos, sin):
    """Half-split rotary embedding, op for op as ``apply_rotary_emb``
    (``dsalt/kernels/window_utils.py:73-88``)."""
    half = q.shape[-1] // 2

    def rot(t):
        return torch.cat([-t[..., half:], t[..., :half]], dim=-1)

    return q * cos + rot(q) * sin, k * cos + rot(k) * sin


def project(cfg, params, x):
    """Post-RoPE ``q, k, v [T, H, D]`` in the compute dtype, as ``_packed``
    (``dsalt_attention.py:566-590``) under autocast: bf16 weights, bf16 GEMMs."""
    dt = torch_dtype(cfg)
    H, Hkv, D = cfg["H"], cfg["Hkv"], cfg["D"]
    T = x.shape[0]
    Wq = params["q_proj.weight"].to(dt)
    Wk = params["k_proj.weight"].to(dt)
    Wv = params["v_proj.weight"].to(dt)
    q = torch.nn.functional.linear(x, Wq).view(T, H, D)
    k = torch.nn.functional.linear(x, Wk).view(T, Hkv, D)
    v = torch.nn.functional.linear(x, Wv).view(T, Hkv, D)
    cu = cu_seqlens(cfg)
    pos = torch.cat([torch.arange(cu[i + 1] - cu[i]) for i in range(len(cu) - 1)])
    cos, sin = rope_cache(max(cfg["seqlens"]), D)
    cos = cos[pos].to(dt).unsqueeze(1)
    sin = sin[pos].to(dt).unsqueeze(1)
    q, k = rope(q, k, cos, sin)
    rep = H // Hkv
    if rep > 1:
        k = k.unsqueeze(2).expand(T, Hkv, rep, D).reshape(T, H, D)
        v_rep = v.unsqueeze(2).expand(T, Hkv, rep, D).reshape(T, H, D)
    else:
        v_rep = v
    return q.contiguous(), k.contiguous(), v_rep.contiguous(), v.reshape(T, Hkv * D).contiguous()


def alpha(params):
    return torch.sigmoid(params["alpha_w"]).float()
