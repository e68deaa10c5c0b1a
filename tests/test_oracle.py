"""The oracle pinned against the reference: the C restatement (oracle.c)
reproduces, bit for bit, the outputs of the reference's own CPU kernels
stored in tests/golden/golden_outputs.npz (made by tests/golden/make_golden.py
from oracle/_ref), and the storage conventions match the reference DSL's
layout functions (golden_layouts.npz).  CPU only."""
import numpy as np
import pytest

import oracle as O
from cpp1_b200 import workloads as W
from cpp1_b200.dsl import layout_functions as LF
from cpp1_b200.dsl.var import Var, evaluate


def test_gemm_restatement_bitexact(golden):
    assert np.array_equal(O.gemm_f32(golden["gemm_A"], golden["gemm_B"]), golden["gemm_C"])


def test_diag_restatement_bitexact(golden):
    assert np.array_equal(O.diag_rows_f32(golden["diag_d"], golden["diag_B"]), golden["diag_C"])


def test_upper_restatement_bitexact(golden):
    assert np.array_equal(O.upper_left_f32(golden["upper_U"], golden["upper_B"]), golden["upper_C"])


def test_sandwich_restatement_bitexact(golden):
    C = O.sandwich_f32(golden["sandwich_A"], golden["sandwich_S"], golden["sandwich_B"])
    assert np.array_equal(C, golden["sandwich_C"])


def test_toeplitz_restatement_bitexact(golden):
    assert np.array_equal(O.toeplitz_left_f32(golden["toeplitz_g"], golden["toeplitz_B"]), golden["toeplitz_C"])


@pytest.mark.parametrize("op", ["gemm", "upper", "sandwich", "toeplitz"])
def test_reference_outputs_meet_fp32_bound(golden, op):
    """The reference's own results are within the 1e-5 normwise bound of the
    fp64 recomputation (the bound the library's 3xTF32 mode is held to)."""
    if op == "gemm":
        R = O.gemm_rows_f64(golden["gemm_A"], golden["gemm_B"], np.arange(golden["gemm_A"].shape[0]))
    elif op == "upper":
        R = O.upper_left_rows_f64(golden["upper_U"], golden["upper_B"], np.arange(golden["upper_B"].shape[0]))
    elif op == "sandwich":
        R = O.sandwich_rows_f64(golden["sandwich_A"], golden["sandwich_S"], golden["sandwich_B"],
                                np.arange(golden["sandwich_A"].shape[0]))
    else:
        R = O.toeplitz_left_rows_f64(golden["toeplitz_g"], golden["toeplitz_B"],
                                     np.arange(golden["toeplitz_B"].shape[0]))
    assert O.relerr(golden[f"{op}_C"], R) <= 1e-5


def test_fp64_rows_match_dense_numpy():
    w = W.make_upper(37, 11, seed=5)
    R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(37))
    U = W.unpack_upper(w["U"], 37).astype(np.float64)
    assert np.allclose(R, U @ w["B"].astype(np.float64), rtol=0, atol=1e-12)
    t = W.make_toeplitz(29, 6, seed=2)
    R = O.toeplitz_left_rows_f64(t["g"], t["B"], np.arange(29))
    assert np.allclose(R, W.toeplitz_dense(t["g"], 29).astype(np.float64) @ t["B"], rtol=0, atol=1e-12)


def test_relerr_detects_planted_error(golden):
    """A single perturbed element in an oracle output is caught by the
    tolerance the GPU tests use (the mistake is planted on the CPU)."""
    A, B = golden["gemm_A"], golden["gemm_B"]
    R = O.gemm_rows_f64(A, B, np.arange(A.shape[0]))
    C = O.gemm_f32(A, B).copy()
    C[5, 7] += 0.05
    assert O.relerr(C, R) > 1e-5


# ---------------------------------------------------------------- layouts
def _index_of(expr):
    """Storage index an element expression selects, or -1 for a structural zero."""
    from cpp1_b200.dsl.var import ArithmeticExpression, Conditional
    if isinstance(expr, Conditional):
        return _index_of(expr.true_value if evaluate(expr.condition, {}) else expr.false_value)
    if isinstance(expr, int):
        return -1 if expr == 0 else expr
    assert isinstance(expr, ArithmeticExpression) and expr.op == "subscript", expr
    return evaluate(expr.right, {})


def _layout_map(fn, n):
    return np.array([[_index_of(fn(i, j, Var("X_data"), n)) for j in range(n)] for i in range(n)], np.int64)


@pytest.mark.parametrize("name", ["general", "upper_triangular", "lower_triangular", "diagonal", "toeplitz",
                                  "symmetric"])
def test_layouts_match_reference_dsl(golden_layouts, name):
    n = int(golden_layouts["layout_n"])
    mine = _layout_map(getattr(LF, f"{name}_layout"), n)
    assert np.array_equal(mine, golden_layouts[f"layout_{name}"])


def test_workload_packing_matches_reference_layouts(golden_layouts):
    n = int(golden_layouts["layout_n"])
    M = np.arange(n * n, dtype=np.float32).reshape(n, n)
    p = W.pack_upper(M)
    ref = golden_layouts["layout_upper_triangular"]
    for i in range(n):
        for j in range(n):
            if ref[i, j] >= 0:
                assert p[ref[i, j]] == M[i, j]
    g = np.arange(2 * n - 1, dtype=np.float32)
    T = W.toeplitz_dense(g, n)
    assert np.array_equal(T, g[golden_layouts["layout_toeplitz"]])
    S = W.unpack_symmetric(p, n)
    assert np.array_equal(S, p[golden_layouts["layout_symmetric"]])


# ---------------------------------------------------------------- elementwise / converters
_LAYOUT_OF = {"upper": "layout_upper_triangular", "lower": "layout_lower_triangular", "symm": "layout_symmetric",
              "diag": "layout_diagonal", "toeplitz": "layout_toeplitz"}


def _expand_by_map(storage, idx):
    """Dense matrix of `storage` under a reference layout map (-1 = zero)."""
    return np.where(idx >= 0, storage[np.maximum(idx, 0)], np.float32(0))


@pytest.mark.parametrize("fmt", sorted(_LAYOUT_OF))
def test_unpack_restatement_matches_reference_layouts(golden_layouts, fmt):
    n = int(golden_layouts["layout_n"])
    storage = np.arange(1, O.struct_numel(fmt, n) + 1, dtype=np.float32)
    assert np.array_equal(O.unpack_f32(storage, fmt, n), _expand_by_map(storage, golden_layouts[_LAYOUT_OF[fmt]]))


@pytest.mark.parametrize("fmt", ["upper", "lower", "symm"])
def test_pack_restatement_inverts_unpack(golden_layouts, fmt):
    n = int(golden_layouts["layout_n"])
    storage = np.arange(1, O.struct_numel(fmt, n) + 1, dtype=np.float32)
    assert np.array_equal(O.pack_f32(O.unpack_f32(storage, fmt, n), fmt), storage)


@pytest.mark.parametrize("fmt", sorted(_LAYOUT_OF))
def test_add_struct_restatement_is_one_add_per_element(golden_layouts, fmt):
    n = 9
    rng = np.random.default_rng(5)
    A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
    S = rng.uniform(-1, 1, O.struct_numel(fmt, n)).astype(np.float32)
    assert np.array_equal(O.add_struct_f32(A, S, fmt), A + O.unpack_f32(S, fmt, n))


def test_add_restatement():
    rng = np.random.default_rng(6)
    A, B = rng.standard_normal(1001).astype(np.float32), rng.standard_normal(1001).astype(np.float32)
    assert np.array_equal(O.add_f32(A, B), A + B)


def test_toeplitz_compact_restatement_matches_reference_builder(golden):
    assert np.array_equal(O.toeplitz_compact_f32(golden["tcompact_T"]), golden["tcompact_g"])


# ---------------------------------------------------------------- the reference's own orientation
@pytest.mark.parametrize("M,N", [(64, 128), (128, 64), (128, 128)])
def test_right_side_restatements_match_reference_kernels(M, N):
    """A·U and A·S (the reference drivers' orientation, upper_triag_matmul.cpp
    and symmetric_matmul.cpp run as built in oracle/_ref) against the C
    restatements the right-operand GPU tests rely on: bit for bit."""
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(M + N)
    X = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    P = rng.uniform(-1, 1, N * (N + 1) // 2).astype(np.float32)
    assert np.array_equal(O.upper_right_f32(X, P), O.ref_upper_right(X, P)[0])
    assert np.array_equal(O.symm_right_f32(X, P), O.ref_symm_right(X, P)[0])
    R = X.astype(np.float64) @ W.unpack_symmetric(P, N).astype(np.float64)
    assert np.abs(O.symm_right_rows_f64(X, P, np.arange(M)) - R).max() <= 1e-12
    assert O.relerr(O.symm_right_f32(X, P), R) <= 1e-5


def test_reference_right_kernels_reject_non_tile_shapes():
    """The reference's compiled kernels only take tile-multiple sizes; the
    wrapper turns their refusal into an error rather than a wrong result."""
    if not O.ref_available():
        pytest.skip("oracle/_ref not built")
    X = np.zeros((96, 192), np.float32)
    P = np.zeros(192 * 193 // 2, np.float32)
    with pytest.raises(ValueError, match="tile-multiple"):
        O.ref_upper_right(X, P)
