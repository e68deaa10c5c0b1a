"""The reference CPU drivers' own orientation: structured operand on the RIGHT.

C = A T with T Toeplitz (the orientation of the reference's only Toeplitz
kernels, Cuda kernels/toeplitz.cu:76-253 and toeplitz_matmul2.cpp:44-144),
on device buffers (T expanded into a dense copy, or built on chip from the
generator without room for the copy), and the host-array entries for A U,
A S, A T and A diag(b) (upper_triag_matmul.cpp:41-137,
symmetric_matmul.cpp:84-211, toeplitz_matmul2.cpp:44-144,
diag_matmul.cpp:45-111).

Random data: normwise error against an fp64 recomputation (3xTF32 1e-5,
TF32 5e-3, bf16 1e-2).  The drivers' integer data (exact fp32 sums): equal,
bit for bit, to the reference's compiled kernels (oracle/_ref) in every mode.
The column scale is one fp32 multiply: bit-exact on any data."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}
MODES = ["3xtf32", "tf32", "bf16"]


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def toeplitz_dense(g, K, N):
    k = np.arange(K)[:, None]
    n = np.arange(N)[None, :]
    return g[(K - 1) + (n - k)].astype(np.float64)


def relerr(C, R):
    C = np.asarray(C, np.float64)
    return float(np.linalg.norm(C - R) / np.linalg.norm(R))


@pytest.mark.parametrize("expand", ["1", "0"], ids=["expanded", "on_chip"])
@pytest.mark.parametrize("M,N,K", [(512, 640, 768), (300, 129, 257), (1, 7, 5), (1024, 1024, 1024)])
def test_gen_x_toeplitz_random(cuda, monkeypatch, expand, M, N, K):
    monkeypatch.setenv("SMM_EXPAND", expand)
    rng = np.random.default_rng(M + N + K)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    g = rng.uniform(-1, 1, K + N - 1).astype(np.float32)
    R = A.astype(np.float64) @ toeplitz_dense(g, K, N)
    for mode in MODES:
        C = ops.gen_x_toeplitz(dev(A), dev(g), N, mode=mode).cpu().numpy()
        ops.device_status()
        assert relerr(C, R) <= TOL[mode], (mode, relerr(C, R))


@pytest.mark.parametrize("mode", MODES)
def test_gen_x_toeplitz_integer_data_bit_exact(cuda, mode):
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(3)
    M, N, K = 512, 384, 640  # toeplitz_matmul2.cpp:303-312: rand() % 5 + 1
    X = rng.integers(1, 6, (M, K)).astype(np.float32)
    g = rng.integers(1, 6, K + N - 1).astype(np.float32)
    ref, _ = O.ref_toeplitz_right(X, g, N)
    got = ops.gen_x_toeplitz(dev(X), dev(g), N, mode=mode).cpu().numpy()
    assert np.array_equal(got, ref)


def test_gen_x_toeplitz_8192_whole_matrix(cuda):
    n = 8192
    rng = np.random.default_rng(12)
    A = dev(rng.uniform(-1, 1, (n, n)).astype(np.float32))
    g = dev(rng.uniform(-1, 1, 2 * n - 1).astype(np.float32))
    T = torch.as_strided(g.double(), (n, n), (1, 1)).flip(0)  # T[k][j] = g[(n-1) + (j-k)]
    R = A.double() @ T
    for mode in MODES:
        C = ops.gen_x_toeplitz(A, g, mode=mode)
        err = float(torch.linalg.vector_norm(C.double() - R) / torch.linalg.vector_norm(R))
        assert err <= TOL[mode], (mode, err)


# ---------------------------------------------------------------- host arrays
def _host(x):
    return torch.from_numpy(np.ascontiguousarray(x))


@pytest.mark.parametrize("mode", MODES)
def test_host_right_products_integer_data_bit_exact(cuda, mode):
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(5)
    M, N = 2560, 1024  # several row chunks on both internal streams
    # upper_triag_matmul.cpp:290-298: A rand()%10, U rand()%10+1
    A = rng.integers(0, 10, (M, N)).astype(np.float32)
    Up = rng.integers(1, 11, N * (N + 1) // 2).astype(np.float32)
    ref, _ = O.ref_upper_right(A, Up)
    assert np.array_equal(ops.host_product("gen_x_upper", _host(A), _host(Up), mode=mode).numpy(), ref)
    # symmetric_matmul.cpp:372-384: rand()%10+1
    A = rng.integers(1, 11, (M, N)).astype(np.float32)
    Sp = rng.integers(1, 11, N * (N + 1) // 2).astype(np.float32)
    ref, _ = O.ref_symm_right(A, Sp)
    assert np.array_equal(ops.host_product("gen_x_symm", _host(A), _host(Sp), mode=mode).numpy(), ref)
    # toeplitz_matmul2.cpp:303-312: rand()%5+1, rectangular T
    K, Nt = 768, 1152
    X = rng.integers(1, 6, (M, K)).astype(np.float32)
    g = rng.integers(1, 6, K + Nt - 1).astype(np.float32)
    ref, _ = O.ref_toeplitz_right(X, g, Nt)
    got = ops.host_product("gen_x_toeplitz", _host(X), _host(g), mode=mode, toeplitz_cols=Nt).numpy()
    assert np.array_equal(got, ref)


def test_host_right_products_random_data(cuda):
    rng = np.random.default_rng(6)
    M, N = 1300, 1000  # ragged row chunk and unaligned rows
    A = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    Up = rng.uniform(-1, 1, N * (N + 1) // 2).astype(np.float32)
    R = A.astype(np.float64) @ W.unpack_upper(Up, N).astype(np.float64)
    assert relerr(ops.host_product("gen_x_upper", _host(A), _host(Up)).numpy(), R) <= 1e-5
    R = A.astype(np.float64) @ W.unpack_symmetric(Up, N).astype(np.float64)
    assert relerr(ops.host_product("gen_x_symm", _host(A), _host(Up)).numpy(), R) <= 1e-5
    g = rng.uniform(-1, 1, 2 * N - 1).astype(np.float32)
    R = A.astype(np.float64) @ toeplitz_dense(g, N, N)
    assert relerr(ops.host_product("gen_x_toeplitz", _host(A), _host(g)).numpy(), R) <= 1e-5


@pytest.mark.parametrize("M,N", [(8192, 8192), (3000, 1001), (1, 5)])
def test_host_diag_cols_bit_exact(cuda, M, N):
    rng = np.random.default_rng(M)
    A = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    b = rng.uniform(0.5, 1.5, N).astype(np.float32)
    got = ops.host_product("diag_cols", _host(A), _host(b)).numpy()
    assert np.array_equal(got, A * b[None, :])  # one IEEE fp32 multiply per element
    if O.ref_available() and M % 64 == 0 and N % 64 == 0:
        ref, _ = O.ref_diag_cols(A, b)
        assert np.array_equal(got, ref)
