"""The C-ABI library loads without a GPU and exports every entry point of include/b2tp.h."""

import ctypes
import os
import re

from pythonintern_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "b2tp.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert header_functions() == sorted(_lib.exported_symbols())


def test_library_exports_every_header_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_pure_host_entry_points():
    L = _lib.lib()
    assert L.b2_abi_version() == 1
    assert L.b2_status_name(2) == b"B2_ETIMEOUT"
    assert L.b2_comm_handle_bytes() == 64
    assert L.b2_linear_workspace_bytes(1, 4096, 4096, _lib.B2_F32) == 0
    assert L.b2_paged_attention_workspace_bytes(4, 32, 8, 128, 1) == 0
    assert L.b2_paged_attention_workspace_bytes(4, 32, 8, 128, 4) > 4 * 32 * 4 * 128 * 4


def test_argument_errors_are_reported_without_a_gpu():
    L = _lib.lib()
    rc = L.b2_rmsnorm(None, 7, None, 0, None, 0, None, 1e-5, None, 0, 1, 8, None)
    assert rc == _lib.B2_EINVAL
    assert "bad dtype" in _lib.last_error()
    rc = L.b2_paged_attention(None, 0, 1, 32, 5, 128, None, None, 0, 1, 16, None, 1, None, None, 1, 1.0, None,
                              0, 1, None, 0, 1, None, None)
    assert rc == _lib.B2_EINVAL
