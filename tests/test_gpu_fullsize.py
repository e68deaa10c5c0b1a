"""GPU parity at every configured size, on the WHOLE output matrix.

Configurations: GEMM 1024^3 and 8192^3, U*B at 8192 (U packed), A*S*B at 4096
(S packed symmetric), T*B at 16384 (2N-1 generator), lower-triangular L*B at
8192.  Every one runs in all three arithmetic modes, and the products whose
packed operand can be expanded or built on chip (U*B, A*S*B) run both ways
(SMM_EXPAND=0 forces the on-chip path).

Ground truth is an fp64 recomputation of the whole product on the GPU
(torch float64 matmul of the exact fp64 values of the fp32 inputs; test-only,
never part of the library).  That checker is itself spot-checked against the
oracle's fp64 rows, and the reference's own fp32 result (the oracle's
bit-exact restatement of the reference CPU kernels) is shown to meet the same
3xTF32 bound on sampled rows.  Normwise relative error bounds, per mode:
3xTF32 <= 1e-5, TF32 <= 5e-3, bf16 <= 1e-2.

The reference drivers' own input distributions (small integers:
gemm_benchmark.cpp:315-316 rand()%10, upper_triag_matmul.cpp:290-298
rand()%10 and rand()%10+1, symmetric_matmul.cpp:372-384 rand()%10+1,
toeplitz_matmul2.cpp:303-312 rand()%5+1) give exact fp32 sums at 1024, so
every mode must then equal the reference's compiled kernels (oracle/_ref)
bit for bit."""
import functools

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


def sample_rows(n, k=6, seed=0):
    rng = np.random.default_rng(seed)
    return np.sort(np.concatenate([[0, n - 1], rng.choice(n, k - 2, replace=False)])).astype(np.int32)


def relerr_dev(C: torch.Tensor, R: torch.Tensor) -> float:
    """||C - R||_F / ||R||_F over the whole matrix, in fp64 on the device."""
    C = C.reshape(R.shape).double()
    return float(torch.linalg.vector_norm(C - R) / torch.linalg.vector_norm(R))


def dense_upper64(Up: torch.Tensor, n: int) -> torch.Tensor:
    """fp64 dense upper-triangular matrix from packed storage (row-major
    upper triangle, the torch.triu_indices order)."""
    U = torch.zeros((n, n), dtype=torch.float64, device=Up.device)
    iu = torch.triu_indices(n, n, device=Up.device)
    U[iu[0], iu[1]] = Up.double()
    return U


def dense_toeplitz64(g: torch.Tensor, n: int) -> torch.Tensor:
    """T[i][j] = g[(n-1) + (j-i)] in fp64: rows of g read as overlapping
    windows (Tf[i][j] = g[i + j]), flipped top to bottom."""
    Tf = torch.as_strided(g.double(), (n, n), (1, 1))
    return Tf.flip(0).contiguous()


# ---------------------------------------------------------------- inputs + fp64 truth, cached per op
@functools.lru_cache(maxsize=1)
def _case(op: str, n: int):
    torch.cuda.empty_cache()
    if op == "gemm":
        w = W.make_gemm(n, n, n, seed=0)
        d = {"A": dev(w["A"]), "B": dev(w["B"])}
        R = d["A"].double() @ d["B"].double()
        rows = sample_rows(n, seed=1)
        spot = O.gemm_rows_f64(w["A"], w["B"], rows)
        ref32 = O.gemm_rows_f32(w["A"], w["B"], rows)
    elif op == "upper":
        w = W.make_upper(n, seed=0)
        d = {"U": dev(w["U"]), "B": dev(w["B"])}
        R = dense_upper64(d["U"], n) @ d["B"].double()
        rows = sample_rows(n, seed=2)
        spot = O.upper_left_rows_f64(w["U"], w["B"], rows)
        ref32 = O.upper_left_rows_f32(w["U"], w["B"], rows)
    elif op == "sandwich":
        w = W.make_sandwich(n, seed=0)
        d = {"A": dev(w["A"]), "S": dev(w["S"]), "B": dev(w["B"])}
        U = dense_upper64(d["S"], n)
        S = U + torch.triu(U, 1).T
        R = (d["A"].double() @ S) @ d["B"].double()
        del U, S
        rows = sample_rows(n, seed=3)
        spot = O.sandwich_rows_f64(w["A"], w["S"], w["B"], rows)
        ref32 = O.sandwich_rows_f32(w["A"], w["S"], w["B"], rows)
    elif op == "toeplitz":
        w = W.make_toeplitz(n, seed=0)
        d = {"g": dev(w["g"]), "B": dev(w["B"])}
        R = dense_toeplitz64(d["g"], n) @ d["B"].double()
        rows = sample_rows(n, seed=4)
        spot = O.toeplitz_left_rows_f64(w["g"], w["B"], rows)
        ref32 = O.toeplitz_left_rows_f32(w["g"], w["B"], rows)
    elif op == "lower":
        rng = np.random.default_rng(7)
        Lp = rng.uniform(-1, 1, n * (n + 1) // 2).astype(np.float32)
        B = rng.uniform(-1, 1, (n, n)).astype(np.float32)
        d = {"L": dev(Lp), "B": dev(B)}
        Lt = torch.zeros((n, n), dtype=torch.float64, device="cuda")
        il = torch.tril_indices(n, n, device="cuda")
        Lt[il[0], il[1]] = d["L"].double()  # row-major lower triangle: idx(i, j) = i(i+1)/2 + j
        R = Lt @ d["B"].double()
        del Lt, il
        rows = sample_rows(n, seed=5)
        B64 = B.astype(np.float64)
        spot = np.stack([Lp[i * (i + 1) // 2: i * (i + 1) // 2 + i + 1].astype(np.float64) @ B64[: i + 1]
                         for i in rows])
        ref32 = None
    else:
        raise ValueError(op)
    # the fp64 checker agrees with the oracle's fp64 rows
    got = R[torch.from_numpy(rows.astype(np.int64)).cuda()].cpu().numpy()
    assert np.max(np.abs(got - spot)) <= 1e-9 * max(1.0, np.max(np.abs(spot)))
    return d, R, rows, spot, ref32


def _run(op: str, d, mode: str) -> torch.Tensor:
    if op == "gemm":
        return ops.gemm(d["A"], d["B"], mode=mode)
    if op == "upper":
        return ops.upper_left(d["U"], d["B"], mode=mode)
    if op == "sandwich":
        return ops.symm_sandwich(d["A"], d["S"], d["B"], mode=mode)
    if op == "toeplitz":
        return ops.toeplitz_left(d["g"], d["B"], mode=mode)
    if op == "lower":
        return ops.lower_left(d["L"], d["B"], mode=mode)
    raise ValueError(op)


CASES = [("gemm", 1024), ("gemm", 8192), ("upper", 8192), ("sandwich", 4096), ("toeplitz", 16384),
         ("lower", 8192)]


@pytest.mark.parametrize("op,n", CASES, ids=[f"{o}{n}" for o, n in CASES])
def test_whole_matrix_every_mode(cuda, op, n):
    d, R, rows, spot, ref32 = _case(op, n)
    if ref32 is not None:  # the reference's own fp32 result meets the 3xTF32 bound
        assert O.relerr(ref32, spot) <= TOL["3xtf32"]
    errs = {}
    for mode in MODES:
        C = _run(op, d, mode)
        torch.cuda.synchronize()
        ops.device_status()
        assert bool(torch.isfinite(C).all()), f"{op} {n} {mode}: non-finite output"
        errs[mode] = relerr_dev(C, R)
        del C
    for mode in MODES:
        assert errs[mode] <= TOL[mode], f"{op} {n} {mode}: relerr {errs[mode]:.3e} (all: {errs})"


@pytest.mark.parametrize("op,n", [("upper", 8192), ("sandwich", 4096)], ids=["upper8192", "sandwich4096"])
def test_whole_matrix_on_chip_operand(cuda, op, n, monkeypatch):
    """The packed operand built on chip (U from packed rows; S mirrored from
    its upper half) instead of expanded into a dense copy."""
    d, R, _, _, _ = _case(op, n)
    monkeypatch.setenv("SMM_EXPAND", "0")
    for mode in MODES:
        C = _run(op, d, mode)
        torch.cuda.synchronize()
        ops.device_status()
        err = relerr_dev(C, R)
        del C
        assert err <= TOL[mode], f"{op} {n} {mode} on chip: relerr {err:.3e}"


def test_upper_packed_equals_dense_storage_8192(cuda):
    """Packed U and dense-with-zeros U feed the tensor cores the same values:
    the two storages give identical results."""
    n = 8192
    d, _, _, _, _ = _case("upper", n)
    Cp = ops.upper_left(d["U"], d["B"], packed=True)
    Ud = ops.unpack(d["U"], "upper", n)
    Cd = ops.upper_left(Ud, d["B"], packed=False)
    assert torch.equal(Cp, Cd)


@pytest.mark.parametrize("lo,hi", [(0.0, 1.0), (-1.0, 1.0)])
def test_gemm_same_sign_data_2048(cuda, lo, hi):
    """All-positive operands are the worst case for a truncating accumulator;
    the chunked 3xTF32 accumulation keeps them inside the bound."""
    n = 2048
    rng = np.random.default_rng(5)
    A = rng.uniform(lo, hi, (n, n)).astype(np.float32)
    B = rng.uniform(lo, hi, (n, n)).astype(np.float32)
    Ad, Bd = dev(A), dev(B)
    C = ops.gemm(Ad, Bd)
    assert relerr_dev(C, Ad.double() @ Bd.double()) <= TOL["3xtf32"]


# ---------------------------------------------------------------- reference drivers' integer data
def _ints(rng, shape, lo, hi):
    """Integers in [lo, hi] as float32 (the drivers' rand() % m + c)."""
    return rng.integers(lo, hi + 1, size=shape).astype(np.float32)


@pytest.mark.parametrize("mode", MODES)
def test_integer_data_bit_exact_vs_reference_kernels(cuda, mode):
    """Exact fp32 sums: every mode equals the reference's compiled kernels."""
    if not O.ref_available():
        pytest.skip("oracle/_ref (the reference CPU kernels) not built")
    n = 1024
    rng = np.random.default_rng(11)
    # gemm_benchmark.cpp:315-316
    A, B = _ints(rng, (n, n), 0, 9), _ints(rng, (n, n), 0, 9)
    ref, _ = O.ref_gemm(A, B)
    assert np.array_equal(ops.gemm(dev(A), dev(B), mode=mode).cpu().numpy(), ref)
    # upper_triag_matmul.cpp:290-298 (U entries rand()%10+1; B rand()%10)
    Up = _ints(rng, n * (n + 1) // 2, 1, 10)
    B = _ints(rng, (n, n), 0, 9)
    ref, _ = O.ref_upper_left(Up, B)
    assert np.array_equal(ops.upper_left(dev(Up), dev(B), mode=mode).cpu().numpy(), ref)
    # symmetric_matmul.cpp:372-384 (A * S, S packed symmetric)
    A, Sp = _ints(rng, (n, n), 1, 10), _ints(rng, n * (n + 1) // 2, 1, 10)
    ref, _ = O.ref_symm_right(A, Sp)
    assert np.array_equal(ops.gen_x_symm(dev(A), dev(Sp), mode=mode).cpu().numpy(), ref)
    # toeplitz_matmul2.cpp:303-312 (generator and B rand()%5+1), left orientation
    g, B = _ints(rng, 2 * n - 1, 1, 5), _ints(rng, (n, n), 1, 5)
    ref, _ = O.ref_toeplitz_left(g, B)
    assert np.array_equal(ops.toeplitz_left(dev(g), dev(B), mode=mode).cpu().numpy(), ref)
