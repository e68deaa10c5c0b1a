"""GPU: the host-buffer contractions (smm_*_host through ops.host_product)
against fp64 and against the device entry points.  Shapes give several
column chunks of B with a ragged last one, whose width is not a multiple of
4 (so the chunk is padded for TMA).  Tolerances as in test_gpu_parity."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}


def pinned(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).pin_memory()


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def relerr(C, R):
    return O.relerr(np.ascontiguousarray(C, np.float32), np.asarray(R, np.float64))


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
def test_gemm_host(cuda, mode):
    M, K, N = 300, 700, 2501
    g = W.make_gemm(M, N, K, seed=1)
    A, B = g["A"], g["B"]
    C = ops.host_product("gemm", pinned(A), pinned(B), mode=mode).numpy()
    R = A.astype(np.float64) @ B.astype(np.float64)
    assert relerr(C, R) <= TOL[mode]
    D = ops.gemm(dev(A), dev(B), mode=mode).cpu().numpy()
    assert relerr(C, D.astype(np.float64)) <= TOL[mode]


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
def test_upper_left_host(cuda, mode):
    N, ncols = 600, 2501
    w = W.make_upper(N, ncols, seed=3)
    C = ops.host_product("upper", pinned(w["U"]), pinned(w["B"]), mode=mode).numpy()
    R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(N))
    assert relerr(C, R) <= TOL[mode]


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
def test_symm_left_host(cuda, mode):
    N, ncols = 520, 2101
    s = W.make_sandwich(N, seed=4)
    B = W.make_gemm(N, 1, ncols, seed=5)["A"]  # N x ncols
    C = ops.host_product("symm", pinned(s["S"]), pinned(B), mode=mode).numpy()
    R = W.unpack_symmetric(s["S"], N).astype(np.float64) @ B.astype(np.float64)
    assert relerr(C, R) <= TOL[mode]


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
def test_toeplitz_left_host(cuda, mode):
    N, ncols = 700, 2501
    w = W.make_toeplitz(N, ncols, seed=6)
    C = ops.host_product("toeplitz", pinned(w["g"]), pinned(w["B"]), mode=mode).numpy()
    R = O.toeplitz_left_rows_f64(w["g"], w["B"], np.arange(N))
    assert relerr(C, R) <= TOL[mode]


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
def test_sandwich_host(cuda, mode):
    N = 2100
    s = W.make_sandwich(N, seed=7)
    C = ops.host_product("sandwich", pinned(s["A"]), pinned(s["S"]), pinned(s["B"]), mode=mode).numpy()
    R = O.sandwich_rows_f64(s["A"], s["S"], s["B"], np.arange(N))
    assert relerr(C, R) <= TOL[mode]


def test_host_product_accepts_pageable_buffers(cuda):
    M, K, N = 130, 257, 1100
    g = W.make_gemm(M, N, K, seed=8)
    A, B = g["A"], g["B"]
    C = ops.host_product("gemm", torch.from_numpy(A), torch.from_numpy(B),
                         out=torch.empty((M, N), dtype=torch.float32)).numpy()
    assert relerr(C, A.astype(np.float64) @ B.astype(np.float64)) <= 1e-5
