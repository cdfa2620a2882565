"""ctypes binding of the C-ABI library ``libdsalt_b200.so`` (``include/dsalt_b200.h``).

The library is loaded from ``dsalt_b200/_lib``; it is built by ``python -m
dsalt_b200.build`` (or ``__graft_entry__.build()``). There is no fallback: a missing
library or a missing CUDA device raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libdsalt_b200.so")

F32, BF16, F16 = 0, 1, 2
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_DEVICE = range(6)
NOALLOC_MAX_SEQS = 4096  # DSALT_NOALLOC_MAX_SEQS
NOALLOC_MAX_TOKENS = 1048576  # DSALT_NOALLOC_MAX_TOKENS
SELECT_GLOBAL, SELECT_BLOCK_CAUSAL = 0, 1
NORM_F32, NORM_INPUT = 0, 1

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_F = ctypes.c_float

# name -> (restype, argtypes); the declarations of include/dsalt_b200.h
SIGNATURES = {
    "dsalt_last_error": (ctypes.c_char_p, []),
    "dsalt_version": (_I, []),
    "dsalt_device_status": (_I, [ctypes.POINTER(_I), _I, _P]),
    "dsalt_device_status_async": (_I, [_P, _P]),
    "dsalt_token_signals": (_I, [_P, _I, _I64, _I, _I64, _P, _P, _I, _I, _I, _P, _I, _I64, _I, _I, _I,
                                 _P, _P, _P, _P, _P, _P]),
    "dsalt_select_workspace_bytes": (_SZ, [_I, _I64, _I, _I, _I, _I, _I, _I]),
    "dsalt_select_landmarks": (_I, [_I, _P, _P, _P, _P, _P, _I, _I64, _I, _I, _I, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "dsalt_attention_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I]),
    "dsalt_attention_fwd": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _I64, _P, _P, _P, _I, _I, _P, _I, _I,
                                 _P, _I, _P, _P, _SZ, _P]),
    "dsalt_attention_bwd_workspace_bytes": (_SZ, [_I64, _I]),
    "dsalt_attention_bwd": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _I64, _P, _I, _P, _I, _P, _P, _P, _P, _I, _I,
                                 _I, _P, _I, _P, _P, _P, _P, _P, _SZ, _P]),
    "dsalt_train_attention_fwd_workspace_bytes": (_SZ, [_I64, _I, _I, _I]),
    "dsalt_train_attention_fwd": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _I64, _P, _P, _P, _I, _P, _I, _F, _F,
                                       _P, _I, _P, _P, _SZ, _P]),
    "dsalt_train_attention_bwd": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _I64, _P, _I, _P, _I, _P, _P, _P, _P,
                                       _I, _P, _I, _F, _F, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "dsalt_attention_fwd_noalloc": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _I64, _P, _P, _P, _I, _I, _P, _I,
                                         _I, _P, _I, _P, _P]),
    "dsalt_select_block_range_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I]),
    "dsalt_select_block_range": (_I, [_P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "dsalt_attention_sharded_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I]),
    "dsalt_select_shard_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I]),
    "dsalt_select_shard": (_I, [_I, _P, _P, _P, _P, _I64, _I, _I, _I, _I, _I, _I, _P, _SZ, _P, _P, _P]),
    "dsalt_attention_fwd_sharded": (_I, [_P, _P, _P, _I, _I64, _I, _I, _I, _I64, _I64, _I64, _I64, _I64, _I64,
                                         _P, _P, _P, _I, _I, _P, _P, _I64, _P, _I, _P, _P, _SZ, _P]),
    "dsalt_peer_barrier": (_I, [_P, _P, _I, _I, _I, _P]),
    "dsalt_peer_allgather": (_I, [_P, _P, _I, _I, _I64, _P]),
    "dsalt_peer_copy": (_I, [_P, _P, _I64, _P]),
    "dsalt_ipc_export": (_I, [_P, _P, ctypes.POINTER(_I64)]),
    "dsalt_ipc_open": (_I, [_P, _I64, ctypes.POINTER(_P)]),
    "dsalt_ipc_close": (_I, [_P, _I64]),
    "dsalt_core_workspace_bytes": (_SZ, [_I, _I64, _I, _I, _I, _I, _I, _I, _I]),
    "dsalt_core_forward": (_I, [_I, _P, _I, _I, _I64, _P, _P, _I, _P, _I, _I, _P, _I, _P, _P, _P, _I, _I, _I, _I,
                                _I64, _I64, _I, _I, _P, _I, _I64, _I, _P, _I, _P, _P, _P, _SZ, _P]),
}

_lock = threading.Lock()
_lib = None


class DsaltError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


def load() -> ctypes.CDLL:
    """Load the library and declare its entry points (raises if it is not built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"dsalt_b200 CUDA library not built ({LIB_PATH}); run `python -m dsalt_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args):
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.dsalt_last_error().decode(errors="replace")
        raise DsaltError(rc, name, msg)
    return rc


def query(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))
