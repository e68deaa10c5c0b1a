"""CPU oracle for the structured matrix-multiply path (test infrastructure).

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
(and its ``--impl reference`` arm) may import this package.  The library in
``cpp1_b200/`` never does: its CUDA path fails loudly when the extension is
missing instead of falling back to anything here.

Two back ends:

* ``liboracle.so`` (``oracle.c``): a C restatement of the reference's CPU
  kernels (bit-exact FMA order) plus fp64 ground truth on sampled rows.
* ``_ref/libref_*.so``: the reference's own CPU kernels, compiled in place
  from the reference checkout by ``oracle/Makefile`` (absent when the
  reference was not available at build time).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_F64P = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_I32P = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_c_int = ctypes.c_int

_lib = None
_ref = {}


def build(with_reference: bool = True) -> None:
    """Compile liboracle.so (and oracle/_ref when the reference is present)."""
    target = "all" if with_reference else "oracle"
    subprocess.run(["make", "-s", "-C", _HERE, target], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build(with_reference=False)
        L = ctypes.CDLL(path)
        L.orc_gemm_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int, _c_int]
        L.orc_diag_rows_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
        L.orc_diag_cols_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
        L.orc_upper_left_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
        L.orc_upper_right_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
        L.orc_symm_right_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
        L.orc_sandwich_f32.argtypes = [_F32P, _F32P, _F32P, _F32P, _c_int]
        L.orc_toeplitz_left_f32.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
        L.orc_gemm_rows_f64.argtypes = [_F32P, _F32P, _I32P, _c_int, _F64P, _c_int, _c_int]
        L.orc_upper_left_rows_f64.argtypes = [_F32P, _F32P, _I32P, _c_int, _F64P, _c_int, _c_int]
        L.orc_toeplitz_left_rows_f64.argtypes = [_F32P, _F32P, _I32P, _c_int, _F64P, _c_int, _c_int]
        L.orc_sandwich_rows_f64.argtypes = [_F32P, _F32P, _F32P, _I32P, _c_int, _F64P, _c_int]
        L.orc_symm_right_rows_f64.argtypes = [_F32P, _F32P, _I32P, _c_int, _F64P, _c_int, _c_int]
        L.orc_gemm_rows_f32.argtypes = [_F32P, _F32P, _I32P, _c_int, _F32P, _c_int, _c_int]
        L.orc_upper_left_rows_f32.argtypes = [_F32P, _F32P, _I32P, _c_int, _F32P, _c_int, _c_int]
        L.orc_toeplitz_left_rows_f32.argtypes = [_F32P, _F32P, _I32P, _c_int, _F32P, _c_int, _c_int]
        L.orc_sandwich_rows_f32.argtypes = [_F32P, _F32P, _F32P, _I32P, _c_int, _F32P, _c_int]
        L.orc_add_f32.argtypes = [_F32P, _F32P, _F32P, ctypes.c_long]
        L.orc_add_struct_f32.argtypes = [_F32P, _F32P, _c_int, _F32P, _c_int]
        L.orc_unpack_f32.argtypes = [_F32P, _c_int, _F32P, _c_int]
        L.orc_pack_f32.argtypes = [_F32P, _c_int, _F32P, _c_int]
        L.orc_toeplitz_compact_f32.argtypes = [_F32P, _F32P, _c_int, _c_int]
        L.orc_relerr.argtypes = [_F32P, _F64P, ctypes.c_size_t]
        L.orc_relerr.restype = ctypes.c_double
        _lib = L
    return _lib


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


# ---------------------------------------------------------------- fp32 restatements
def gemm_f32(A, B) -> np.ndarray:
    A, B = _f32(A), _f32(B)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    lib().orc_gemm_f32(A, B, C, M, N, K)
    return C


def diag_rows_f32(d, B) -> np.ndarray:
    d, B = _f32(d), _f32(B)
    C = np.empty_like(B)
    lib().orc_diag_rows_f32(d, B, C, B.shape[0], B.shape[1])
    return C


def diag_cols_f32(A, b) -> np.ndarray:
    A, b = _f32(A), _f32(b)
    C = np.empty_like(A)
    lib().orc_diag_cols_f32(A, b, C, A.shape[0], A.shape[1])
    return C


def upper_left_f32(Up, B) -> np.ndarray:
    Up, B = _f32(Up), _f32(B)
    N, ncols = B.shape
    C = np.empty((N, ncols), np.float32)
    lib().orc_upper_left_f32(Up, B, C, N, ncols)
    return C


def upper_right_f32(X, Up) -> np.ndarray:
    X, Up = _f32(X), _f32(Up)
    M, N = X.shape
    Y = np.empty((M, N), np.float32)
    lib().orc_upper_right_f32(X, Up, Y, M, N)
    return Y


def symm_right_f32(A, Sp) -> np.ndarray:
    A, Sp = _f32(A), _f32(Sp)
    M, N = A.shape
    W = np.empty((M, N), np.float32)
    lib().orc_symm_right_f32(A, Sp, W, M, N)
    return W


def sandwich_f32(A, Sp, B) -> np.ndarray:
    A, Sp, B = _f32(A), _f32(Sp), _f32(B)
    N = A.shape[0]
    C = np.empty((N, N), np.float32)
    lib().orc_sandwich_f32(A, Sp, B, C, N)
    return C


def toeplitz_left_f32(g, B) -> np.ndarray:
    g, B = _f32(g), _f32(B)
    N, ncols = B.shape
    C = np.empty((N, ncols), np.float32)
    lib().orc_toeplitz_left_f32(g, B, C, N, ncols)
    return C


# ---------------------------------------------------------------- elementwise / converters
STRUCTS = {"upper": 0, "lower": 1, "symm": 2, "diag": 3, "toeplitz": 4}


def struct_numel(fmt: str, N: int) -> int:
    return {"upper": N * (N + 1) // 2, "lower": N * (N + 1) // 2, "symm": N * (N + 1) // 2, "diag": N,
            "toeplitz": max(2 * N - 1, 0)}[fmt]


def add_f32(A, B) -> np.ndarray:
    A, B = _f32(A), _f32(B)
    C = np.empty_like(A)
    lib().orc_add_f32(A.reshape(-1), B.reshape(-1), C.reshape(-1), A.size)
    return C


def add_struct_f32(A, S, fmt: str) -> np.ndarray:
    A, S = _f32(A), _f32(S)
    N = A.shape[0]
    C = np.empty((N, N), np.float32)
    lib().orc_add_struct_f32(A, S, STRUCTS[fmt], C, N)
    return C


def unpack_f32(S, fmt: str, N: int) -> np.ndarray:
    S = _f32(S)
    D = np.empty((N, N), np.float32)
    lib().orc_unpack_f32(S, STRUCTS[fmt], D, N)
    return D


def pack_f32(D, fmt: str) -> np.ndarray:
    D = _f32(D)
    N = D.shape[0]
    P = np.empty(N * (N + 1) // 2, np.float32)
    lib().orc_pack_f32(D, STRUCTS[fmt], P, N)
    return P


def toeplitz_compact_f32(T) -> np.ndarray:
    T = _f32(T)
    rows, cols = T.shape
    g = np.empty(rows + cols - 1, np.float32)
    lib().orc_toeplitz_compact_f32(T, g, rows, cols)
    return g


# ---------------------------------------------------------------- fp64 sampled rows
def _rows(rows) -> np.ndarray:
    return np.ascontiguousarray(rows, dtype=np.int32)


def gemm_rows_f64(A, B, rows) -> np.ndarray:
    A, B, r = _f32(A), _f32(B), _rows(rows)
    out = np.empty((len(r), B.shape[1]), np.float64)
    lib().orc_gemm_rows_f64(A, B, r, len(r), out, B.shape[1], A.shape[1])
    return out


def upper_left_rows_f64(Up, B, rows) -> np.ndarray:
    Up, B, r = _f32(Up), _f32(B), _rows(rows)
    out = np.empty((len(r), B.shape[1]), np.float64)
    lib().orc_upper_left_rows_f64(Up, B, r, len(r), out, B.shape[0], B.shape[1])
    return out


def toeplitz_left_rows_f64(g, B, rows) -> np.ndarray:
    g, B, r = _f32(g), _f32(B), _rows(rows)
    out = np.empty((len(r), B.shape[1]), np.float64)
    lib().orc_toeplitz_left_rows_f64(g, B, r, len(r), out, B.shape[0], B.shape[1])
    return out


def sandwich_rows_f64(A, Sp, B, rows) -> np.ndarray:
    A, Sp, B, r = _f32(A), _f32(Sp), _f32(B), _rows(rows)
    out = np.empty((len(r), A.shape[0]), np.float64)
    lib().orc_sandwich_rows_f64(A, Sp, B, r, len(r), out, A.shape[0])
    return out


def symm_right_rows_f64(A, Sp, rows) -> np.ndarray:
    A, Sp, r = _f32(A), _f32(Sp), _rows(rows)
    out = np.empty((len(r), A.shape[1]), np.float64)
    lib().orc_symm_right_rows_f64(A, Sp, r, len(r), out, A.shape[0], A.shape[1])
    return out


def gemm_rows_f32(A, B, rows) -> np.ndarray:
    A, B, r = _f32(A), _f32(B), _rows(rows)
    out = np.empty((len(r), B.shape[1]), np.float32)
    lib().orc_gemm_rows_f32(A, B, r, len(r), out, B.shape[1], A.shape[1])
    return out


def upper_left_rows_f32(Up, B, rows) -> np.ndarray:
    Up, B, r = _f32(Up), _f32(B), _rows(rows)
    out = np.empty((len(r), B.shape[1]), np.float32)
    lib().orc_upper_left_rows_f32(Up, B, r, len(r), out, B.shape[0], B.shape[1])
    return out


def toeplitz_left_rows_f32(g, B, rows) -> np.ndarray:
    g, B, r = _f32(g), _f32(B), _rows(rows)
    out = np.empty((len(r), B.shape[1]), np.float32)
    lib().orc_toeplitz_left_rows_f32(g, B, r, len(r), out, B.shape[0], B.shape[1])
    return out


def sandwich_rows_f32(A, Sp, B, rows) -> np.ndarray:
    A, Sp, B, r = _f32(A), _f32(Sp), _f32(B), _rows(rows)
    out = np.empty((len(r), A.shape[0]), np.float32)
    lib().orc_sandwich_rows_f32(A, Sp, B, r, len(r), out, A.shape[0])
    return out


def relerr(X, R) -> float:
    """Normwise relative error ||X - R||_F / ||R||_F (X fp32, R fp64)."""
    X = _f32(X).ravel()
    R = np.ascontiguousarray(R, dtype=np.float64).ravel()
    return float(lib().orc_relerr(X, R, X.size))


# ---------------------------------------------------------------- reference kernels
def ref_available() -> bool:
    return all(os.path.exists(os.path.join(_HERE, "_ref", f"libref_{n}.so"))
               for n in ("gemm", "diag", "upper", "symm", "toeplitz"))


def _ref_lib(name: str) -> ctypes.CDLL:
    if name not in _ref:
        path = os.path.join(_HERE, "_ref", f"libref_{name}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: build it with `make -C oracle ref` where the reference "
                                    "checkout is present")
        L = ctypes.CDLL(path)
        d = ctypes.c_double
        if name == "gemm":
            L.ref_gemm.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int, _c_int]
            L.ref_gemm.restype = d
        elif name == "diag":
            L.ref_diag_rows.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
            L.ref_diag_rows.restype = d
            L.ref_diag_cols.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
            L.ref_diag_cols.restype = d
        elif name == "upper":
            L.ref_upper_left.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
            L.ref_upper_left.restype = d
            L.ref_upper_right.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
            L.ref_upper_right.restype = d
        elif name == "symm":
            L.ref_symm_right.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
            L.ref_symm_right.restype = d
        elif name == "toeplitz":
            L.ref_toeplitz_left.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int]
            L.ref_toeplitz_left.restype = d
            L.ref_toeplitz_right.argtypes = [_F32P, _F32P, _F32P, _c_int, _c_int, _c_int]
            L.ref_toeplitz_right.restype = d
            L.ref_toeplitz_compact.argtypes = [_F32P, _F32P, _c_int, _c_int]
            L.ref_toeplitz_compact.restype = None
        _ref[name] = L
    return _ref[name]


def _check_ms(ms: float, what: str) -> float:
    if ms < 0:
        raise ValueError(f"reference {what} kernel rejected the shape (needs tile-multiple sizes)")
    return ms


def ref_gemm(A, B) -> Tuple[np.ndarray, float]:
    A, B = _f32(A), _f32(B)
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float32)
    return C, _check_ms(_ref_lib("gemm").ref_gemm(A, B, C, M, N, K), "gemm")


def ref_diag_rows(d, B) -> Tuple[np.ndarray, float]:
    d, B = _f32(d), _f32(B)
    C = np.empty_like(B)
    return C, _check_ms(_ref_lib("diag").ref_diag_rows(d, B, C, B.shape[0], B.shape[1]), "diag")


def ref_diag_cols(A, b) -> Tuple[np.ndarray, float]:
    A, b = _f32(A), _f32(b)
    C = np.empty_like(A)
    return C, _check_ms(_ref_lib("diag").ref_diag_cols(A, b, C, A.shape[0], A.shape[1]), "diag")


def ref_upper_left(Up, B) -> Tuple[np.ndarray, float]:
    Up, B = _f32(Up), _f32(B)
    N, ncols = B.shape
    C = np.empty((N, ncols), np.float32)
    return C, _check_ms(_ref_lib("upper").ref_upper_left(Up, B, C, N, ncols), "upper")


def ref_upper_right(X, Up) -> Tuple[np.ndarray, float]:
    X, Up = _f32(X), _f32(Up)
    M, N = X.shape
    Y = np.empty((M, N), np.float32)
    return Y, _check_ms(_ref_lib("upper").ref_upper_right(X, Up, Y, M, N), "upper")


def ref_symm_right(A, Sp) -> Tuple[np.ndarray, float]:
    A, Sp = _f32(A), _f32(Sp)
    M, N = A.shape
    W = np.empty((M, N), np.float32)
    return W, _check_ms(_ref_lib("symm").ref_symm_right(A, Sp, W, M, N), "symm")


def ref_sandwich(A, Sp, B) -> Tuple[np.ndarray, float]:
    """A*S*B as the reference's graph runner executes it: A*S, then (A*S)*B."""
    W, ms1 = ref_symm_right(A, Sp)
    C, ms2 = ref_gemm(W, B)
    return C, ms1 + ms2


def ref_toeplitz_left(g, B) -> Tuple[np.ndarray, float]:
    g, B = _f32(g), _f32(B)
    N, ncols = B.shape
    C = np.empty((N, ncols), np.float32)
    return C, _check_ms(_ref_lib("toeplitz").ref_toeplitz_left(g, B, C, N, ncols), "toeplitz")


def ref_toeplitz_compact(T) -> np.ndarray:
    """The reference's build_toeplitz_compact (toeplitz_matmul2.cpp:34-41)."""
    T = _f32(T)
    rows, cols = T.shape
    g = np.zeros(rows + cols - 1, np.float32)
    _ref_lib("toeplitz").ref_toeplitz_compact(T, g, rows, cols)
    return g


def ref_toeplitz_right(X, g, N: Optional[int] = None) -> Tuple[np.ndarray, float]:
    X, g = _f32(X), _f32(g)
    M, K = X.shape
    N = N if N is not None else g.size - K + 1
    Y = np.empty((M, N), np.float32)
    return Y, _check_ms(_ref_lib("toeplitz").ref_toeplitz_right(X, g, Y, M, N, K), "toeplitz")
