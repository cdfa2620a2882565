"""The DSALT decoder stack for inference prefill on the B200 operators.

Same configuration fields, module names and state-dict keys as the reference's
``DSALTConfig`` (``dsalt/model/config.py:10-53``), ``DSALTTransformerBlock`` /
``SwiGLUFFN`` (``dsalt/modules/dsalt_transformer.py``), ``RMSENorm``
(``dsalt/kernels/RMSENorm.py``) and ``DSALTLMHeadModel`` (``dsalt/model/dsalt_lm.py:64-284``),
so a reference checkpoint loads unchanged. Every block's attention is
:class:`dsalt_b200.DSALTAttention` (widths, landmark selection and the sparse attention on
this package's kernels); norms, the SwiGLU MLP, embeddings and the LM head are library
ops. Packed input only (``input_ids [T]`` with ``cu_seqlens``), inference only: training,
the losses and the batched path are not part of this package.
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass, fields
from pathlib import Path

import torch
import torch.nn as nn
import torch.nn.functional as F

from .module import DSALTAttention


@dataclass
class DSALTConfig:
    """Hyperparameters of :class:`DSALTLMHeadModel` (the reference's fields and defaults;
    ``selection`` / ``block`` choose this package's landmark selection mode)."""
    vocab_size: int
    d_model: int
    n_layers: int
    n_heads: int
    n_min: int
    n_max: int
    k_lmk: int
    max_seq_len: int
    d_ff: int | None = None
    dropout: float = 0.0
    yarn_scale: float = 1.0
    tie_weights: bool = True
    n_kv_heads: int | None = None
    qkv_bias: bool = False
    rope_base: float = 10000.0
    padding_idx: int | None = None
    lm_head_chunk_size: int = 2048
    loss_fn: str = "chunked"
    aux_loss_weight: float = 0.0
    selection: str = "global"
    block: int = 512

    def __post_init__(self) -> None:
        if self.d_model % self.n_heads != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by n_heads ({self.n_heads})")
        if not (0 <= self.n_min <= self.n_max):
            raise ValueError(f"required 0 <= n_min <= n_max, got n_min={self.n_min} n_max={self.n_max}")
        if self.k_lmk < 0:
            raise ValueError(f"k_lmk must be >= 0, got {self.k_lmk}")
        if self.n_kv_heads is not None and (self.n_kv_heads <= 0 or self.n_heads % self.n_kv_heads != 0):
            raise ValueError(f"n_heads ({self.n_heads}) must be a positive multiple of n_kv_heads ({self.n_kv_heads})")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "DSALTConfig":
        known = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in known})

    def save(self, path) -> None:
        Path(path).write_text(json.dumps(self.to_dict(), indent=2), encoding="utf-8")

    @classmethod
    def load(cls, path) -> "DSALTConfig":
        return cls.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))


class RMSENorm(nn.Module):
    """RMSNorm with a learnable scale (``F.rms_norm``), result in the input dtype."""

    def __init__(self, d_model: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model))
        self.normalized_shape = (d_model,)

    def forward(self, x):
        return F.rms_norm(x, self.normalized_shape, self.weight, self.eps).to(x.dtype)


class SwiGLUFFN(nn.Module):
    """``down(silu(gate(x)) * up(x))``."""

    def __init__(self, d_model: int, d_ff: int, dropout: float = 0.0):
        super().__init__()
        self.gate_proj = nn.Linear(d_model, d_ff, bias=False)
        self.up_proj = nn.Linear(d_model, d_ff, bias=False)
        self.down_proj = nn.Linear(d_ff, d_model, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DSALTTransformerBlock(nn.Module):
    """Pre-norm block: RMSNorm → DSALTAttention → residual, RMSNorm → SwiGLU → residual."""

    def __init__(self, d_model, n_heads, n_min, n_max, k_lmk, max_seq_len, d_ff, dropout=0.0, yarn_scale=1.0,
                 layer_idx=0, n_kv_heads=None, qkv_bias=False, rope_base=10000.0, selection="global", block=512):
        super().__init__()
        self.layer_idx = layer_idx
        self.attn_norm = RMSENorm(d_model)
        self.ffn_norm = RMSENorm(d_model)
        self.attn = DSALTAttention(d_model, n_heads, n_min, n_max, k_lmk, max_seq_len, dropout=dropout,
                                   yarn_scale=yarn_scale, layer_idx=layer_idx, n_kv_heads=n_kv_heads,
                                   qkv_bias=qkv_bias, rope_base=rope_base, selection=selection, block=block)
        # the dense [H, T0, T0] _last_P rebuild is off in the decoder stack: at prefill lengths it
        # does not fit (set attn._collect_last_P = True on a layer whose metrics are wanted)
        self.attn._collect_last_P = False
        self.ffn = SwiGLUFFN(d_model, d_ff, dropout)

    def forward(self, x, cu_seqlens=None, max_seqlen=None, gradient_checkpointing=False, rope_cs=None, cu_list=None):
        a, aux = self.attn(self.attn_norm(x), cu_seqlens=cu_seqlens, max_seqlen=max_seqlen, rope_cs=rope_cs,
                           cu_list=cu_list)
        x = x + a
        x = x + self.ffn(self.ffn_norm(x))
        return x, aux


class DSALTLMHeadModel(nn.Module):
    """Causal LM: embeddings, ``n_layers`` DSALT blocks, a final RMSNorm and the LM head
    (tied to the embedding by default); the reference's initialisation (``N(0, 0.02)``,
    ``out_proj`` / ``down_proj`` scaled by ``1/sqrt(2·n_layers)``)."""

    def __init__(self, vocab_size, d_model, n_layers, n_heads, n_min, n_max, k_lmk, max_seq_len, d_ff=None,
                 dropout=0.0, yarn_scale=1.0, tie_weights=True, padding_idx=None, lm_head_chunk_size=2048,
                 loss_fn="chunked", aux_loss_weight=0.0, n_kv_heads=None, qkv_bias=False, rope_base=10000.0,
                 selection="global", block=512):
        super().__init__()
        del lm_head_chunk_size, loss_fn, aux_loss_weight  # training-only settings of the reference
        self.d_model, self.n_layers, self.vocab_size = d_model, n_layers, vocab_size
        if d_ff is None:
            d_ff = ((int(8 / 3 * d_model) + 127) // 128) * 128
        self.embed_tokens = nn.Embedding(vocab_size, d_model, padding_idx=padding_idx)
        self.layers = nn.ModuleList([
            DSALTTransformerBlock(d_model, n_heads, n_min, n_max, k_lmk, max_seq_len, d_ff, dropout, yarn_scale, i,
                                  n_kv_heads, qkv_bias, rope_base, selection, block)
            for i in range(n_layers)])
        self.final_norm = RMSENorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        if tie_weights:
            self.lm_head.weight = self.embed_tokens.weight
        self._init_weights()

    @classmethod
    def from_config(cls, config: DSALTConfig) -> "DSALTLMHeadModel":
        return cls(**config.to_dict())

    def _init_weights(self):
        nn.init.normal_(self.embed_tokens.weight, std=0.02)
        residual_std = 0.02 / math.sqrt(2 * self.n_layers)
        for name, module in self.named_modules():
            if isinstance(module, nn.Linear):
                std = residual_std if any(k in name for k in ("out_proj", "down_proj")) else 0.02
                nn.init.normal_(module.weight, std=std)
                if module.bias is not None:
                    nn.init.zeros_(module.bias)

    @torch.no_grad()
    def forward(self, input_ids, cu_seqlens=None, max_seqlen=None, labels=None, gradient_checkpointing=False,
                padding_mask=None, cu_list=None, logits_to_keep: int = 0):
        """Prefill of packed ``input_ids [T]`` → ``{"logits": [T, vocab], ...}`` like the
        reference's inference return. ``logits_to_keep`` > 0 computes the logits of the
        pack's last that many tokens only (the reference computes all of them)."""
        if labels is not None or self.training:
            raise NotImplementedError("dsalt_b200.DSALTLMHeadModel is inference-only")
        if cu_seqlens is None:
            raise NotImplementedError("pass packed input_ids with cu_seqlens")
        T = input_ids.shape[0]
        x = self.embed_tokens(input_ids)
        if x.is_cuda and torch.is_autocast_enabled("cuda"):
            x = x.to(torch.get_autocast_dtype("cuda"))
        cu_h = [int(c) for c in (cu_list if cu_list is not None else cu_seqlens.detach().cpu().tolist())]
        attn0 = self.layers[0].attn
        pos = torch.cat([torch.arange(cu_h[i + 1] - cu_h[i], device=x.device) for i in range(len(cu_h) - 1)])
        rope_cs = (attn0.rope_cos.to(x.device)[pos], attn0.rope_sin.to(x.device)[pos])
        for layer in self.layers:
            x, _ = layer(x, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen, rope_cs=rope_cs, cu_list=cu_h)
        x = self.final_norm(x)
        if logits_to_keep > 0:
            x = x[T - logits_to_keep:]
        return {"loss": None, "logits": self.lm_head(x), "aux_loss": None}
