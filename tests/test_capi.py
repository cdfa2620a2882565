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
