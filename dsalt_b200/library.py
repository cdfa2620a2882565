"""The operators registered with ``torch.library`` (namespace ``dsalt_b200``), so that
``torch.compile`` treats each as one opaque node with a shape function, as the reference
keeps its kernels opaque (``_dynamo_opaque``, ``dsalt/kernels/dsalt_triton_attn.py:330-336``)
— here without a graph break, so ``fullgraph=True`` compiles a model that contains them.

* ``torch.ops.dsalt_b200.window_signals``   → :func:`dsalt_b200.ops.window_signals`
* ``torch.ops.dsalt_b200.select_landmarks`` → :func:`dsalt_b200.ops.select_landmarks`
* ``torch.ops.dsalt_b200.dsalt_attention``  → :func:`dsalt_b200.ops.dsalt_attention`
* ``torch.ops.dsalt_b200.core_forward``     → :func:`dsalt_b200.ops.core_forward`

``cu_list`` (the host copy of ``cu_seqlens``) is an ``int[]`` argument: the kernels size
their launches and workspaces from it, so a compiled graph is specialised on the packing.
The fake (meta) functions give the output shapes and dtypes; no real implementation runs
while tracing.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import ops


def _n_sets(cu_list: List[int], mode: str, block: int) -> int:
    return len(cu_list) - 1 if mode == "global" else ops.n_block_sets(cu_list, block)


@torch.library.custom_op("dsalt_b200::window_signals", mutates_args=())
def window_signals(x: torch.Tensor, gate_weight: torch.Tensor, gate_bias: torch.Tensor, n_min: int, n_max: int,
                   v: torch.Tensor, head_dim: int, norm_round: bool,
                   logit: Optional[torch.Tensor]) -> List[torch.Tensor]:
    w, xn, vn = ops.window_signals(x, gate_weight, gate_bias, n_min, n_max, v, head_dim, norm_round, logit=logit)
    return [w, xn, vn]


@window_signals.register_fake
def _(x, gate_weight, gate_bias, n_min, n_max, v, head_dim, norm_round, logit):
    T = x.shape[0]
    n_kv = v.reshape(T, -1).shape[1] // head_dim
    return [x.new_empty(T, dtype=torch.int32), x.new_empty(T, dtype=torch.float32),
            x.new_empty(T, n_kv, dtype=torch.float32)]


@torch.library.custom_op("dsalt_b200::select_landmarks", mutates_args=())
def select_landmarks(xnorm: torch.Tensor, vnorm: torch.Tensor, w: torch.Tensor, alpha: torch.Tensor,
                     cu_seqlens: torch.Tensor, k_lmk: int, n_heads: int, mode: str, block: int,
                     cu_list: List[int]) -> torch.Tensor:
    return ops.select_landmarks(xnorm, vnorm, w, alpha, cu_seqlens, k_lmk, n_heads, mode, block, cu_list=cu_list)


@select_landmarks.register_fake
def _(xnorm, vnorm, w, alpha, cu_seqlens, k_lmk, n_heads, mode, block, cu_list):
    return xnorm.new_empty(n_heads, _n_sets(cu_list, mode, block), k_lmk, dtype=torch.int32)


@torch.library.custom_op("dsalt_b200::dsalt_attention", mutates_args=())
def dsalt_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lmk_indices: torch.Tensor,
                    lmk_bias: Optional[torch.Tensor], w_sizes: torch.Tensor, cu_seqlens: torch.Tensor, lmk_block: int,
                    cu_list: List[int], out_dtype: torch.dtype) -> torch.Tensor:
    return ops.dsalt_attention(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, lmk_block=lmk_block,
                               out_dtype=out_dtype, cu_list=cu_list)


@dsalt_attention.register_fake
def _(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens, lmk_block, cu_list, out_dtype):
    return q.new_empty(q.shape, dtype=out_dtype)


@torch.library.custom_op("dsalt_b200::core_forward", mutates_args=())
def core_forward(x: torch.Tensor, gate_weight: torch.Tensor, gate_bias: torch.Tensor, n_min: int, n_max: int,
                 alpha: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_lmk: int,
                 cu_seqlens: torch.Tensor, mode: str, block: int, norm_round: bool, cu_list: List[int],
                 out_dtype: torch.dtype, logit: Optional[torch.Tensor]) -> torch.Tensor:
    return ops.core_forward(x, gate_weight, gate_bias, n_min, n_max, alpha, q, k, v, k_lmk, cu_seqlens, mode=mode,
                            block=block, norm_round=norm_round, out_dtype=out_dtype, cu_list=cu_list, logit=logit)


@core_forward.register_fake
def _(x, gate_weight, gate_bias, n_min, n_max, alpha, q, k, v, k_lmk, cu_seqlens, mode, block, norm_round, cu_list,
      out_dtype, logit):
    return q.new_empty(q.shape, dtype=out_dtype)
