"""Seeded synthetic inputs for the five structured products.

The reference ships no datasets or golden data; its drivers draw small
integers from an unseeded ``rand()``.  These generators define the workload
instead: one ``numpy.random.default_rng(seed)`` (PCG64) stream per case, values
drawn as float32 in the order listed, uniform on the stated interval:

==========  ==========================================================  ==========
op          draws (in order)                                            sizes
==========  ==========================================================  ==========
gemm        A (M x K) U[-1,1]; B (K x N) U[-1,1]                        1024^3, 8192^3
diag        d (M) U[0.5,1.5]; B (M x N) U[-1,1]                         8192^2
upper       U's upper+diagonal entries U[-1,1], drawn row-major over    8192
            i <= j, i.e. directly as the packed vector; B U[-1,1]
sandwich    A, then X, then B, each N x N U[-1,1]; S = (X + X^T)/2 in  4096
            fp32, passed packed upper
toeplitz    generator g (2N-1) U[-1,1]; B (N x ncols) U[-1,1]           16384
==========  ==========================================================  ==========

Packed upper storage is row-major over the upper triangle,
``idx(i,j) = i*N - i*(i-1)/2 + (j-i)`` (``src/dsl/layout_functions.py:8-23``),
the ``torch.triu_indices`` order the reference's driver uses
(``src/main2.py:44-45``).  A Toeplitz generator stores ``T[i][j] =
g[(N-1) + (j-i)]`` (``src/dsl/layout_functions.py:45-48``).
"""
from __future__ import annotations

from typing import Dict

import numpy as np


def _uniform(rng: np.random.Generator, shape, lo: float, hi: float) -> np.ndarray:
    u = rng.random(shape, dtype=np.float32)
    return (np.float32(lo) + np.float32(hi - lo) * u).astype(np.float32, copy=False)


def packed_size(n: int) -> int:
    return n * (n + 1) // 2


def pack_upper(M: np.ndarray) -> np.ndarray:
    """Row-major upper triangle (diagonal included) of a square matrix."""
    n = M.shape[0]
    iu = np.triu_indices(n)
    return np.ascontiguousarray(M[iu], dtype=np.float32)


def unpack_upper(p: np.ndarray, n: int) -> np.ndarray:
    """Dense upper-triangular matrix (exact zeros below) from packed storage."""
    out = np.zeros((n, n), np.float32)
    out[np.triu_indices(n)] = p
    return out


def unpack_symmetric(p: np.ndarray, n: int) -> np.ndarray:
    U = unpack_upper(p, n)
    return U + np.triu(U, 1).T


def toeplitz_dense(g: np.ndarray, n: int) -> np.ndarray:
    i = np.arange(n)[:, None]
    j = np.arange(n)[None, :]
    return np.ascontiguousarray(g[(n - 1) + (j - i)], dtype=np.float32)


def make_gemm(M: int, N: int, K: int, seed: int = 0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    A = _uniform(rng, (M, K), -1.0, 1.0)
    B = _uniform(rng, (K, N), -1.0, 1.0)
    return {"A": A, "B": B}


def make_diag(M: int, N: int, seed: int = 0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    d = _uniform(rng, (M,), 0.5, 1.5)
    B = _uniform(rng, (M, N), -1.0, 1.0)
    return {"d": d, "B": B}


def make_upper(N: int, ncols: int = None, seed: int = 0) -> Dict[str, np.ndarray]:
    ncols = N if ncols is None else ncols
    rng = np.random.default_rng(seed)
    Up = _uniform(rng, (packed_size(N),), -1.0, 1.0)
    B = _uniform(rng, (N, ncols), -1.0, 1.0)
    return {"U": Up, "B": B}


def make_sandwich(N: int, seed: int = 0) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    A = _uniform(rng, (N, N), -1.0, 1.0)
    X = _uniform(rng, (N, N), -1.0, 1.0)
    B = _uniform(rng, (N, N), -1.0, 1.0)
    S = ((X + X.T) * np.float32(0.5)).astype(np.float32)
    return {"A": A, "S": pack_upper(S), "B": B}


def make_toeplitz(N: int, ncols: int = None, seed: int = 0) -> Dict[str, np.ndarray]:
    ncols = N if ncols is None else ncols
    rng = np.random.default_rng(seed)
    g = _uniform(rng, (2 * N - 1,), -1.0, 1.0)
    B = _uniform(rng, (N, ncols), -1.0, 1.0)
    return {"g": g, "B": B}


def make_add(N: int, seed: int = 0) -> Dict[str, np.ndarray]:
    """General + symmetric (the DSL's GeneralMatrix + SymmetricMatrix): A
    (N x N) then the packed upper triangle of S, both ~ U[-1, 1]."""
    rng = np.random.default_rng(seed)
    A = _uniform(rng, (N, N), -1.0, 1.0)
    S = _uniform(rng, (packed_size(N),), -1.0, 1.0)
    return {"A": A, "S": S}
