"""DSL surface (cpp1_b200.dsl, mirroring the reference's src/dsl): types,
shape inference, graph utilities, and the runner's lowering of each
(left type, right type) pair to one C-ABI entry point.  CPU only: the
library calls are replaced by recorders."""
import numpy as np
import pytest
import torch

from cpp1_b200.dsl import runner_cuda as RC
from cpp1_b200.dsl.matrix import (DiagonalMatrix, GeneralMatrix, LowerTriangularMatrix, SymmetricMatrix,
                                  ToeplitzMatrix, UpperTriangularMatrix, Vector)
from cpp1_b200.dsl.operations import Operation
from cpp1_b200.dsl.utils import get_graph_io, topological_sort_operations, var_names
from cpp1_b200.dsl.var import Var


def test_structured_types_require_square():
    n, m = Var("n"), Var("m")
    for cls in (DiagonalMatrix, UpperTriangularMatrix, LowerTriangularMatrix, ToeplitzMatrix, SymmetricMatrix):
        cls((n, n), "X")
        cls((4, 4), "X")
        with pytest.raises(ValueError):
            cls((4, 5), "X")
        with pytest.raises(ValueError):
            cls((n, m), "X")
    Vector((4, 1), "v")
    with pytest.raises(ValueError):
        Vector((4, 3), "v")


def test_shape_inference_and_auto_names():
    n, k = Var("n"), Var("k")
    A = GeneralMatrix((n, k), "A")
    B = GeneralMatrix((k, n), "B")
    C = A @ B
    assert isinstance(C, Operation) and C.operator == "matmul"
    assert C.shape == (n, n)
    assert C.name.startswith("intermediate_matmul_")
    assert (A.T).shape == (k, n)
    with pytest.raises(ValueError):
        GeneralMatrix((3, 4), "X") @ GeneralMatrix((5, 3), "Y")
    with pytest.raises(ValueError):
        GeneralMatrix((3, 4), "X") + GeneralMatrix((4, 3), "Y")


def test_graph_io_and_topological_order():
    n = Var("n")
    A, S, B = GeneralMatrix((n, n), "A"), SymmetricMatrix((n, n), "S"), GeneralMatrix((n, n), "B")
    inner = A @ S
    outer = inner @ B
    mats, dims = get_graph_io([outer])
    assert [m.name for m in mats] == ["A", "B", "S"]
    assert [d.name for d in dims] == ["n"]
    order = topological_sort_operations([outer])
    assert order.index(inner) < order.index(outer)


def test_var_names_fills_unnamed():
    X = GeneralMatrix((2, 2))
    var_names(None, {"X": X})
    assert X.name == "X"


def test_get_shape_lookup():
    n = Var("n")
    assert RC.get_shape((n, 5), {"n": 7}) == (7, 5)
    assert RC.get_shape((Var("N"), 3), {"n": 2}) == (2, 3)  # lower-case lookup first, as the reference
    with pytest.raises(KeyError):
        RC.get_shape((Var("q"),), {})


@pytest.mark.parametrize("cls,size", [(GeneralMatrix, 12), (SymmetricMatrix, 6), (UpperTriangularMatrix, 6),
                                      (LowerTriangularMatrix, 6), (DiagonalMatrix, 3), (ToeplitzMatrix, 5)])
def test_storage_sizes(cls, size):
    shape = (3, 4) if cls is GeneralMatrix else (3, 3)
    assert RC._storage_size(cls(shape, "X"), shape) == size


class _Recorder:
    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def f(*args, **kw):
            self.calls.append((name, [tuple(a.shape) if torch.is_tensor(a) else a for a in args], kw))
            return kw.get("out")
        return f


@pytest.fixture
def recorder(monkeypatch):
    rec = _Recorder()
    monkeypatch.setattr(RC, "ops", rec)
    monkeypatch.setattr(RC, "_device_tensor", lambda v: torch.as_tensor(np.asarray(v, np.float32)).reshape(-1))
    monkeypatch.setattr(RC, "_timed", lambda fn: (fn(), 1.0))
    return rec


@pytest.mark.parametrize("lhs,rhs,entry", [
    (GeneralMatrix, GeneralMatrix, "gemm"),
    (DiagonalMatrix, GeneralMatrix, "diag_rows"),
    (GeneralMatrix, DiagonalMatrix, "diag_cols"),
    (UpperTriangularMatrix, GeneralMatrix, "upper_left"),
    (ToeplitzMatrix, GeneralMatrix, "toeplitz_left"),
    (SymmetricMatrix, GeneralMatrix, "symm_left"),
    (GeneralMatrix, SymmetricMatrix, "gen_x_symm"),
    (GeneralMatrix, UpperTriangularMatrix, "gen_x_upper"),
    (SymmetricMatrix, SymmetricMatrix, "symm_x_symm"),
    (GeneralMatrix, LowerTriangularMatrix, "gen_x_lower"),
    (LowerTriangularMatrix, GeneralMatrix, "lower_left"),
    (LowerTriangularMatrix, LowerTriangularMatrix, "lower_x_lower"),
    (GeneralMatrix, ToeplitzMatrix, "gen_x_toeplitz"),
])
def test_lowering_table(recorder, lhs, rhs, entry):
    n = Var("n")
    nv = 4
    L, R = lhs((n, n), "A"), rhs((n, n), "B")
    sizes = {GeneralMatrix: nv * nv, DiagonalMatrix: nv, UpperTriangularMatrix: nv * (nv + 1) // 2,
             SymmetricMatrix: nv * (nv + 1) // 2, ToeplitzMatrix: 2 * nv - 1,
             LowerTriangularMatrix: nv * (nv + 1) // 2}
    inputs = {"n": nv, "A": np.ones(sizes[lhs], np.float32), "B": np.ones(sizes[rhs], np.float32)}
    out, ms, gflops = RC.run([L @ R], inputs, "cuda", GeneralMatrix((n, n), "C"))
    assert list(out) == ["C"] and out["C"].numel() == nv * nv
    assert [c[0] for c in recorder.calls] == [entry]
    assert ms == 1.0
    flops = nv * nv if "diag" in entry else 2 * nv ** 3
    assert gflops == pytest.approx(flops * 1e-9 / 1e-3)


def test_unsupported_pair_raises(recorder):
    n = Var("n")
    with pytest.raises(NotImplementedError):
        RC.run([ToeplitzMatrix((n, n), "A") @ ToeplitzMatrix((n, n), "B")],
               {"n": 2, "A": np.ones(3, np.float32), "B": np.ones(3, np.float32)})


def test_non_cuda_backend_rejected(recorder):
    n = Var("n")
    with pytest.raises(ValueError):
        RC.run([GeneralMatrix((n, n), "A") @ GeneralMatrix((n, n), "B")], {"n": 2, "A": np.ones(4), "B": np.ones(4)},
               backend="numpy")


def test_run_graph_sandwich_returns_every_operation(recorder):
    """A @ S @ B runs as the library's structured products in the
    expression's association and returns the intermediate under its name too,
    as the reference's run_graph does (src/dsl/runner_cuda.py:147-197)."""
    n = Var("n")
    A, S, B = GeneralMatrix((n, n), "A"), SymmetricMatrix((n, n), "S"), GeneralMatrix((n, n), "B")
    inputs = {"n": 4, "A": np.ones(16, np.float32), "S": np.ones(10, np.float32), "B": np.ones(16, np.float32)}
    inner = A @ S
    expr = inner @ B
    res, ms, _ = RC.run_graph([expr], inputs, "cuda")
    assert [c[0] for c in recorder.calls] == ["gen_x_symm", "gemm"]
    assert list(res) == [inner.name, expr.name]
    recorder.calls.clear()
    inner = S @ B
    expr = A @ inner
    res, ms, _ = RC.run_graph([expr], inputs, "cuda")
    assert [c[0] for c in recorder.calls] == ["symm_left", "gemm"]
    assert list(res) == [inner.name, expr.name]


def test_run_graph_chains_in_post_order(recorder):
    n = Var("n")
    A, B, C = (GeneralMatrix((n, n), x) for x in "ABC")
    inner = A @ B
    expr = inner @ C
    inputs = {"n": 3, "A": np.ones(9, np.float32), "B": np.ones(9, np.float32), "C": np.ones(9, np.float32)}
    res, ms, _ = RC.run_graph([expr], inputs, "cuda")
    assert [c[0] for c in recorder.calls] == ["gemm", "gemm"]
    assert list(res) == [inner.name, expr.name]
    assert ms == 2.0
    # the operands were restored after the placeholder substitution
    assert expr.operands[0] is inner


@pytest.mark.parametrize("lhs,rhs,entry,out_cls,size", [
    (GeneralMatrix, GeneralMatrix, "add", GeneralMatrix, 16),
    (SymmetricMatrix, SymmetricMatrix, "add", SymmetricMatrix, 10),
    (UpperTriangularMatrix, UpperTriangularMatrix, "add", UpperTriangularMatrix, 10),
    (DiagonalMatrix, DiagonalMatrix, "add", DiagonalMatrix, 4),
    (GeneralMatrix, SymmetricMatrix, "add_struct", GeneralMatrix, 16),
    (SymmetricMatrix, GeneralMatrix, "add_struct", GeneralMatrix, 16),
    (GeneralMatrix, UpperTriangularMatrix, "add_struct", GeneralMatrix, 16),
    (LowerTriangularMatrix, GeneralMatrix, "add_struct", GeneralMatrix, 16),
    (GeneralMatrix, DiagonalMatrix, "add_struct", GeneralMatrix, 16),
    (ToeplitzMatrix, GeneralMatrix, "add_struct", GeneralMatrix, 16),
])
def test_add_lowering(recorder, lhs, rhs, entry, out_cls, size):
    n = Var("n")
    nv = 4
    sizes = {GeneralMatrix: nv * nv, DiagonalMatrix: nv, UpperTriangularMatrix: nv * (nv + 1) // 2,
             LowerTriangularMatrix: nv * (nv + 1) // 2, SymmetricMatrix: nv * (nv + 1) // 2,
             ToeplitzMatrix: 2 * nv - 1}
    L, R = lhs((n, n), "A"), rhs((n, n), "B")
    inputs = {"n": nv, "A": np.ones(sizes[lhs], np.float32), "B": np.ones(sizes[rhs], np.float32)}
    out, ms, gflops = RC.run([L + R], inputs, "cuda", out_cls((n, n), "C"))
    assert list(out) == ["C"] and out["C"].numel() == size
    assert [c[0] for c in recorder.calls] == [entry]
    if entry == "add_struct":
        fmt = recorder.calls[0][1][2]
        assert fmt == {UpperTriangularMatrix: "upper", LowerTriangularMatrix: "lower", SymmetricMatrix: "symm",
                       DiagonalMatrix: "diag", ToeplitzMatrix: "toeplitz"}[rhs if lhs is GeneralMatrix else lhs]
    assert gflops == pytest.approx(size * 1e-9 / 1e-3)


def test_add_of_unrelated_structures_raises(recorder):
    n = Var("n")
    with pytest.raises(NotImplementedError):
        RC.run([SymmetricMatrix((n, n), "A") + UpperTriangularMatrix((n, n), "B")],
               {"n": 2, "A": np.ones(3, np.float32), "B": np.ones(3, np.float32)}, "cuda",
               GeneralMatrix((n, n), "C"))
