"""C-ABI library: it loads, exports every entry point declared in include/dsalt_b200.h,
and rejects bad arguments before touching a device (these calls need no GPU)."""
import ctypes
import os
import re

import pytest

from dsalt_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dsalt_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dsalt_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        from dsalt_b200 import build
        build.build()
    return L.load()


def test_header_and_binding_agree():
    assert declared_functions() == sorted(L.SIGNATURES)


def test_library_exports_every_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_workspace_queries(lib):
    assert lib.dsalt_version() >= 1
    n = lib.dsalt_select_workspace_bytes(L.SELECT_BLOCK_CAUSAL, 131072, 1, 131072, 16, 16, 128, 512)
    assert n > 0 and n % 256 == 0
    assert lib.dsalt_select_workspace_bytes(L.SELECT_GLOBAL, 4096, 4, 1024, 12, 12, 64, 0) > 0
    assert lib.dsalt_core_workspace_bytes(L.SELECT_BLOCK_CAUSAL, 131072, 1, 131072, 16, 16, 64, 128, 512) > n
    assert lib.dsalt_select_workspace_bytes(L.SELECT_BLOCK_CAUSAL, 1024, 1, 1024, 16, 16, 128, 0) == 0


def test_invalid_arguments_are_rejected(lib):
    rc = lib.dsalt_attention_fwd(None, None, None, L.BF16, -1, 16, 16, 64, 1024, 1024, None, None, None, 128, 0,
                                 None, 1, 0, None, L.BF16, None, None, 0, None)
    assert rc == L.ERR_INVALID
    assert b"bad sizes" in lib.dsalt_last_error()
    rc = lib.dsalt_attention_fwd(None, None, None, 7, 16, 16, 16, 64, 1024, 1024, None, None, None, 128, 0,
                                 None, 1, 0, None, L.BF16, None, None, 0, None)
    assert rc == L.ERR_INVALID
    rc = lib.dsalt_token_signals(None, 9, 8, 64, 64, None, None, L.BF16, 16, 128, None, L.BF16, 64, 1, 64, 0,
                                 None, None, None, None, None, None)
    assert rc == L.ERR_INVALID
    rc = lib.dsalt_select_landmarks(5, None, None, None, None, None, 1, 8, 8, 1, 1, 4, 0, None, None, None, None, 0,
                                    None)
    assert rc == L.ERR_INVALID
    rc = lib.dsalt_select_landmarks(L.SELECT_GLOBAL, None, None, None, None, None, 1, 8, 8, 1, 1, 4096, 0, None,
                                    None, None, None, 0, None)
    assert rc == L.ERR_UNSUPPORTED
    st = ctypes.c_int(0)
    assert lib.dsalt_device_status(None, 0, None) == L.ERR_INVALID


def test_training_and_backward_arguments_are_rejected(lib):
    """The training forward / backward and the inference backward validate sizes, dtypes,
    pointers and (training forward) the workspace before queuing any device work."""
    fake = ctypes.c_void_p(4096)  # never dereferenced: every call below fails before device work
    ws_need = lib.dsalt_train_attention_fwd_workspace_bytes(1024, 4, 2, 16)
    assert ws_need > lib.dsalt_attention_workspace_bytes(1024, 2, 4, 16, 0) and ws_need % 256 == 0
    assert lib.dsalt_train_attention_fwd_workspace_bytes(1024, 4, 0, 16) == 0

    def train_fwd(T=1024, H=4, Hkv=2, tau=1.0, ptr=fake, ws=fake, ws_bytes=ws_need, dtype=L.BF16):
        return lib.dsalt_train_attention_fwd(ptr, ptr, ptr, dtype, T, H, Hkv, 64, H * 64, Hkv * 64, ptr, ptr, ptr, 16,
                                             ptr, 2, tau, 4.0, ptr, L.F32, None, ws, ws_bytes, None)

    assert train_fwd(tau=0.0) == L.ERR_INVALID and b"bad sizes" in lib.dsalt_last_error()
    assert train_fwd(H=3) == L.ERR_INVALID  # heads not a multiple of the kv heads
    assert train_fwd(dtype=9) == L.ERR_INVALID
    assert train_fwd(ptr=None) == L.ERR_INVALID and b"null pointer" in lib.dsalt_last_error()
    assert train_fwd(ws=None) == L.ERR_INVALID
    assert train_fwd(ws_bytes=ws_need - 256) == L.ERR_WORKSPACE
    assert train_fwd(T=0, ptr=None, ws=None) == L.OK  # nothing to do

    rc = lib.dsalt_train_attention_bwd(fake, fake, fake, L.BF16, 1024, 4, 2, 64, 256, 128, fake, L.F32, fake, L.F32,
                                       fake, fake, fake, fake, 16, fake, 2, -1.0, 4.0, fake, fake, fake, fake, fake,
                                       fake, 4096, None)
    assert rc == L.ERR_INVALID and b"bad sizes" in lib.dsalt_last_error()
    rc = lib.dsalt_train_attention_bwd(fake, fake, fake, L.BF16, 1024, 4, 2, 64, 256, 128, fake, L.F32, fake, L.F32,
                                       fake, None, fake, fake, 16, fake, 2, 1.0, 4.0, fake, fake, fake, fake, fake,
                                       fake, 4096, None)
    assert rc == L.ERR_INVALID and b"null pointer" in lib.dsalt_last_error()
    rc = lib.dsalt_attention_bwd(fake, fake, fake, L.BF16, 1024, 4, 2, 64, 128, 128, fake, L.F32, fake, L.F32, fake,
                                 fake, fake, None, 16, 0, 2, fake, 2, fake, fake, fake, None, fake, 4096, None)
    assert rc == L.ERR_INVALID and b"token stride" in lib.dsalt_last_error()
