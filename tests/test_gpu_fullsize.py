"""GPU parity at the benchmark sizes (GEMM and U·B at 8192, A·S·B at 4096,
T·B at 16384, diag at 8192²).  A full fp64 recomputation is too slow here, so
the checks are size-independent: normwise relative error on sampled output
rows against fp64 (3xTF32 bound 1e-5), the reference's own fp32 result on the
same rows (oracle restatement, bit-identical to the reference kernels)
against the same bound, and exact agreement between the packed and dense
storage of U (the same values reach the tensor cores)."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-5


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def sample_rows(n, k=12, seed=0):
    rng = np.random.default_rng(seed)
    return np.sort(np.concatenate([[0, n - 1], rng.choice(n, k - 2, replace=False)])).astype(np.int32)


def test_gemm_8192(cuda):
    n = 8192
    w = W.make_gemm(n, n, n, seed=0)
    C = ops.gemm(dev(w["A"]), dev(w["B"])).cpu().numpy()
    r = sample_rows(n)
    R = O.gemm_rows_f64(w["A"], w["B"], r)
    assert O.relerr(C[r], R) <= TOL
    assert O.relerr(O.gemm_rows_f32(w["A"], w["B"], r), R) <= TOL  # the reference's result


def test_upper_8192_packed_and_dense(cuda):
    n = 8192
    w = W.make_upper(n, seed=0)
    B = dev(w["B"])
    Cp = ops.upper_left(dev(w["U"]), B, packed=True).cpu().numpy()
    r = sample_rows(n, seed=1)
    R = O.upper_left_rows_f64(w["U"], w["B"], r)
    assert O.relerr(Cp[r], R) <= TOL
    assert O.relerr(O.upper_left_rows_f32(w["U"], w["B"], r), R) <= TOL
    Ud = dev(W.unpack_upper(w["U"], n))
    Cd = ops.upper_left(Ud, B, packed=False).cpu().numpy()
    assert np.array_equal(Cp, Cd)


def test_sandwich_4096(cuda):
    n = 4096
    w = W.make_sandwich(n, seed=0)
    C = ops.symm_sandwich(dev(w["A"]), dev(w["S"]), dev(w["B"])).cpu().numpy()
    r = sample_rows(n, seed=2)
    R = O.sandwich_rows_f64(w["A"], w["S"], w["B"], r)
    assert O.relerr(C[r], R) <= TOL
    assert O.relerr(O.sandwich_rows_f32(w["A"], w["S"], w["B"], r), R) <= TOL


def test_toeplitz_16384(cuda):
    n = 16384
    w = W.make_toeplitz(n, seed=0)
    C = ops.toeplitz_left(dev(w["g"]), dev(w["B"])).cpu().numpy()
    r = sample_rows(n, k=8, seed=3)
    R = O.toeplitz_left_rows_f64(w["g"], w["B"], r)
    assert O.relerr(C[r], R) <= TOL
    assert O.relerr(O.toeplitz_left_rows_f32(w["g"], w["B"], r), R) <= TOL


@pytest.mark.parametrize("lo,hi", [(0.0, 1.0), (-1.0, 1.0)])
def test_gemm_same_sign_data_2048(cuda, lo, hi):
    """All-positive operands (what the reference's driver feeds, torch.rand)
    are the worst case for a truncating accumulator; the chunked 3xTF32
    accumulation keeps them inside the bound."""
    n = 2048
    rng = np.random.default_rng(5)
    A = rng.uniform(lo, hi, (n, n)).astype(np.float32)
    B = rng.uniform(lo, hi, (n, n)).astype(np.float32)
    C = ops.gemm(dev(A), dev(B)).cpu().numpy()
    r = sample_rows(n, seed=4)
    assert O.relerr(C[r], O.gemm_rows_f64(A, B, r)) <= TOL


def test_lower_left_8192(cuda):
    """L B with L packed lower (the left-side counterpart of U B) at 8192."""
    n = 8192
    rng = np.random.default_rng(7)
    Lp = rng.uniform(-1, 1, n * (n + 1) // 2).astype(np.float32)
    B = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    C = ops.lower_left(dev(Lp), dev(B)).cpu().numpy()
    r = sample_rows(n, seed=6)
    B64 = B.astype(np.float64)
    R = np.stack([Lp[i * (i + 1) // 2: i * (i + 1) // 2 + i + 1].astype(np.float64) @ B64[: i + 1] for i in r])
    assert O.relerr(C[r], R) <= TOL


@pytest.mark.parametrize("op", ["gemm", "upper"])
def test_bf16_mode_8192(cuda, op):
    """bf16 mode at the bench size: operands rounded to bf16 inside the call,
    fp32 accumulation; normwise bound 1e-2 against fp64."""
    n = 8192
    r = sample_rows(n, seed=8)
    if op == "gemm":
        w = W.make_gemm(n, n, n, seed=0)
        C = ops.gemm(dev(w["A"]), dev(w["B"]), mode="bf16").cpu().numpy()
        R = O.gemm_rows_f64(w["A"], w["B"], r)
    else:
        w = W.make_upper(n, seed=0)
        C = ops.upper_left(dev(w["U"]), dev(w["B"]), mode="bf16").cpu().numpy()
        R = O.upper_left_rows_f64(w["U"], w["B"], r)
    assert O.relerr(C[r], R) <= 1e-2
