"""dsalt_b200 — B200 (sm_100a) kernels for the DSALT sparse-attention forward.

A drop-in for the inference path of LeonardoCofone/dsalt's ``DSALTAttention``: adaptive
window widths, hybrid-score landmark selection (whole-sequence or block-causal) and the
sparse attention over ``A(i) = W(i) ∪ L(i)``, as hand-written CUDA behind a C ABI
(``include/dsalt_b200.h``). There is no CPU path: the operators need the CUDA library
(``python -m dsalt_b200.build``) and CUDA tensors.
"""
from .ops import (  # noqa: F401
    compute_landmark_indices,
    core_forward,
    core_workspace_bytes,
    device_status,
    dsalt_attention,
    select_landmarks,
    window_signals,
)
from .module import DSALTAttention  # noqa: F401
from .model import DSALTConfig, DSALTLMHeadModel, DSALTTransformerBlock  # noqa: F401
from ._lib import DsaltError  # noqa: F401

__version__ = "0.1.0"
