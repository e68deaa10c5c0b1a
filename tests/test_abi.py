"""The C-ABI library loads and exports exactly what include/smm.h declares,
and rejects invalid arguments on the host (no kernel is launched).  CPU only."""
import ctypes
import os
import re

import pytest

from cpp1_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "smm.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(smm_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_binding_table():
    assert declared_functions() == sorted(name for name, _, _ in _lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(_lib.LIB_PATH)
    missing = [f for f in declared_functions() if not hasattr(L, f)]
    assert not missing, missing


def test_debug_bounds_library_exports_every_declared_symbol():
    """The bounds-checked build (libsmm_debug.so, -DSMM_DEBUG_BOUNDS) is a
    drop-in of the same ABI."""
    path = os.path.join(os.path.dirname(_lib.LIB_PATH), "libsmm_debug.so")
    assert os.path.exists(path), "build it with python -m cpp1_b200.build --debug-bounds"
    L = ctypes.CDLL(path)
    missing = [f for f in declared_functions() if not hasattr(L, f)]
    assert not missing, missing


def test_version_and_error_text():
    L = _lib.load()
    assert L.smm_version() >= 100
    assert isinstance(_lib.last_error(), str)


@pytest.mark.parametrize("call", [
    lambda L: L.smm_gemm(None, None, None, -1, 4, 4, 0, None, 0, None),
    lambda L: L.smm_gemm(None, None, None, 4, 4, 4, 7, None, 0, None),
    lambda L: L.smm_gemm(None, None, None, 4, 4, 4, 0, None, 0, None),
    lambda L: L.smm_diag_rows(None, None, None, -3, 2, None),
    lambda L: L.smm_diag_rows(None, None, None, 3, 2, None),
    lambda L: L.smm_upper_left(None, 5, None, None, 4, 4, 0, None, 0, None),
    lambda L: L.smm_upper_left_rows(None, 0, None, None, 8, 4, 6, 4, 0, None, 0, None),
    lambda L: L.smm_toeplitz_left(None, None, None, -1, 4, 0, None, 0, None),
    lambda L: L.smm_symm_sandwich(None, None, None, None, 4, 9, None, 0, None),
    lambda L: L.smm_add(None, None, None, -1, None),
    lambda L: L.smm_add(None, None, None, 8, None),
    lambda L: L.smm_add_struct(None, None, 9, None, 4, None),
    lambda L: L.smm_add_struct(None, None, 2, None, 4, None),
    lambda L: L.smm_unpack(None, 5, None, 4, None),
    lambda L: L.smm_pack(None, 3, None, 4, None),   # diagonal: no packed triangle
    lambda L: L.smm_pack(None, 4, None, 4, None),   # toeplitz: no packed triangle
    lambda L: L.smm_toeplitz_compact(None, None, -1, 3, None),
    lambda L: L.smm_symm_x_symm_ws(None, None, None, -2, 0, None, 0, None),
    lambda L: L.smm_lower_x_lower_ws(None, None, None, 4, 5, None, 0, None),
    lambda L: L.smm_gemm_host(None, None, None, 4, 4, 4, 0, None, 0),
    lambda L: L.smm_gemm_host(None, None, None, 4, -4, 4, 0, None, 0),
    lambda L: L.smm_upper_left_host(None, None, None, 8, 8, 3, None, 0),
    lambda L: L.smm_symm_left_host(None, None, None, 8, 8, 0, None, 0),
    lambda L: L.smm_toeplitz_left_host(None, None, None, 8, 8, 0, None, 0),
    lambda L: L.smm_symm_sandwich_host(None, None, None, None, 8, 0, None, 0),
])
def test_invalid_arguments_rejected_on_host(call):
    L = _lib.load()
    assert call(L) == _lib.SMM_ERR_INVALID
    assert _lib.last_error()


def test_empty_shapes_are_noops():
    L = _lib.load()
    assert L.smm_gemm(None, None, None, 0, 5, 5, 0, None, 0, None) == _lib.SMM_OK
    assert L.smm_diag_rows(None, None, None, 0, 0, None) == _lib.SMM_OK
    assert L.smm_toeplitz_left(None, None, None, 0, 0, 0, None, 0, None) == _lib.SMM_OK
    assert L.smm_add(None, None, None, 0, None) == _lib.SMM_OK
    assert L.smm_add_struct(None, None, 2, None, 0, None) == _lib.SMM_OK
    assert L.smm_pack(None, 1, None, 0, None) == _lib.SMM_OK
    assert L.smm_unpack(None, 4, None, 0, None) == _lib.SMM_OK
    assert L.smm_toeplitz_compact(None, None, 0, 5, None) == _lib.SMM_OK
    assert L.smm_gemm_host(None, None, None, 0, 4, 4, 0, None, 0) == _lib.SMM_OK
    assert L.smm_symm_sandwich_host(None, None, None, None, 0, 2, None, 0) == _lib.SMM_OK
    assert L.smm_symm_x_symm_ws(None, None, None, 0, 1, None, 0, None) == _lib.SMM_OK


def test_workspace_queries_are_host_only():
    L = _lib.load()
    assert L.smm_gemm_workspace_size(0, 4, 4, 0) == 0
    assert L.smm_gemm_workspace_size(128, 128, 128, 0) >= 0
    assert L.smm_symm_sandwich_workspace_size(4096, 0) >= 4096 * 4096 * 4
    assert L.smm_diag_rows_host_workspace_size(8192, 8192) >= 8192 * 4
    # host-buffer products: the left operand(s), their prepared copy and two
    # chunk buffer sets
    assert L.smm_gemm_host_workspace_size(8192, 8192, 8192, 0) >= 8192 * 8192 * 4
    assert L.smm_upper_left_host_workspace_size(8192, 8192, 2) >= 8192 * 8193 // 2 * 4 + 8192 * 8192 * 2
    assert L.smm_symm_sandwich_host_workspace_size(0, 0) == 0
    # a packed product with room for both expansions
    assert L.smm_symm_x_symm_workspace_size(1000, 0) >= 2 * 1000 * 1000 * 4
    assert L.smm_lower_x_lower_workspace_size(1000, 2) >= 2 * 1000 * 1000 * 2


def test_host_gemm_with_empty_inner_dimension_writes_zeros():
    L = _lib.load()
    C = (ctypes.c_float * 6)(*([7.0] * 6))
    rc = L.smm_gemm_host(C, C, C, 2, 3, 0, 0, None, 0)
    assert rc == _lib.SMM_OK, _lib.last_error()
    assert list(C) == [0.0] * 6


def test_host_products_reject_small_workspace_before_any_device_work():
    L = _lib.load()
    need = L.smm_gemm_host_workspace_size(64, 64, 64, 0)
    buf = ctypes.create_string_buffer(16)
    rc = L.smm_gemm_host(buf, buf, buf, 64, 64, 64, 0, buf, need - 256)
    assert rc == _lib.SMM_ERR_WORKSPACE, _lib.last_error()


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()
