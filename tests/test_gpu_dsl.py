"""GPU: the right-side structured products and the DSL drop-in, driven the
way the reference's driver drives its CUDA runner (src/main2.py:38-132):
symbolic types, ``run([A @ B], {...}, "cuda", out)`` and ``.view(n, n)`` of
the flat output.  Checked against fp64 (normwise, 1e-5 for 3xTF32)."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import ops
from cpp1_b200 import workloads as W
from cpp1_b200.dsl.matrix import (DiagonalMatrix, GeneralMatrix, SymmetricMatrix, ToeplitzMatrix,
                                  UpperTriangularMatrix)
from cpp1_b200.dsl.runner_cuda import run, run_graph
from cpp1_b200.dsl.var import Var

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def relerr64(C, R):
    return O.relerr(np.ascontiguousarray(C, np.float32), np.asarray(R, np.float64))


@pytest.fixture(params=["1", "0"], ids=["expanded", "on_chip"])
def expand(request, monkeypatch):
    """Packed right operands expanded into a dense copy read by TMA (the
    default with a full workspace) or built on chip by the transform warps."""
    monkeypatch.setenv("SMM_EXPAND", request.param)
    return request.param


@pytest.mark.parametrize("mode,tol", [("3xtf32", 1e-5), ("bf16", 1e-2)])
@pytest.mark.parametrize("mn", [(1, 1), (7, 9), (128, 128), (200, 130), (512, 384), (300, 1000)])
def test_gen_x_upper(cuda, expand, mn, mode, tol):
    M, N = mn
    A = W.make_gemm(M, 1, N, seed=M)["A"]  # M x N
    Up = W.make_upper(N, 1, seed=N)["U"]
    C = ops.gen_x_upper(dev(A), dev(Up), mode=mode).cpu().numpy()
    R = A.astype(np.float64) @ W.unpack_upper(Up, N).astype(np.float64)
    assert relerr64(C, R) <= tol


@pytest.mark.parametrize("mode,tol", [("3xtf32", 1e-5), ("bf16", 1e-2)])
@pytest.mark.parametrize("mn", [(1, 1), (5, 6), (128, 256), (300, 257), (700, 600)])
def test_gen_x_symm(cuda, expand, mn, mode, tol):
    M, N = mn
    A = W.make_gemm(M, 1, N, seed=M + 1)["A"]  # M x N
    Sp = W.make_sandwich(N, seed=N)["S"]
    C = ops.gen_x_symm(dev(A), dev(Sp), mode=mode).cpu().numpy()
    R = A.astype(np.float64) @ W.unpack_symmetric(Sp, N).astype(np.float64)
    assert relerr64(C, R) <= tol


@pytest.mark.parametrize("mode,tol", [("3xtf32", 1e-5), ("bf16", 1e-2)])
@pytest.mark.parametrize("N", [1, 3, 128, 257, 700])
def test_symm_x_symm(cuda, expand, N, mode, tol):
    S1 = W.make_sandwich(N, seed=N)["S"]
    S2 = W.make_sandwich(N, seed=N + 9)["S"]
    C = ops.symm_x_symm(dev(S1), dev(S2), mode=mode).cpu().numpy()
    R = W.unpack_symmetric(S1, N).astype(np.float64) @ W.unpack_symmetric(S2, N).astype(np.float64)
    assert relerr64(C, R) <= tol


# ---------------------------------------------------------------- DSL drop-in
N_DSL = 512


def _tri_pack(full):
    idx = torch.triu_indices(full.shape[0], full.shape[0], device=full.device)
    return full[idx[0], idx[1]].contiguous()


def test_dsl_gen_x_symm_like_main2(cuda):
    """src/main2.py:110-132 test_gen_x_symm, at a smaller n."""
    n = Var("n")
    g = torch.Generator(device="cuda").manual_seed(0)
    A = torch.rand(N_DSL, N_DSL, device="cuda", generator=g)
    Bt = torch.rand(N_DSL, N_DSL, device="cuda", generator=g)
    B_full = (Bt + Bt.t()) * 0.5
    B_pack = _tri_pack(B_full)
    Am, Bm, out = GeneralMatrix((n, n), "A"), SymmetricMatrix((n, n), "B"), GeneralMatrix((n, n), "C")
    res, ms, gflops = run([Am @ Bm], {"n": N_DSL, "A": A, "B": B_pack}, "cuda", out)
    C = res["C"].view(N_DSL, N_DSL)
    exp = A.double() @ B_full.double()
    assert relerr64(C.cpu().numpy(), exp.cpu().numpy()) <= 1e-5
    assert ms > 0 and gflops > 0


def test_dsl_symm_x_gen_diag_x_gen_symm_x_symm(cuda):
    """src/main2.py:38-107: symm x gen, diag x gen, symm x symm."""
    n = Var("n")
    g = torch.Generator(device="cuda").manual_seed(1)
    At = torch.rand(N_DSL, N_DSL, device="cuda", generator=g)
    S_full = (At + At.t()) * 0.5
    S_pack = _tri_pack(S_full)
    B = torch.rand(N_DSL, N_DSL, device="cuda", generator=g)
    out = GeneralMatrix((n, n), "C")

    res, _, _ = run([SymmetricMatrix((n, n), "A") @ GeneralMatrix((n, n), "B")],
                    {"n": N_DSL, "A": S_pack, "B": B}, "cuda", out)
    exp = S_full.double() @ B.double()
    assert relerr64(res["C"].view(N_DSL, N_DSL).cpu().numpy(), exp.cpu().numpy()) <= 1e-5

    d = torch.rand(N_DSL, device="cuda", generator=g)
    res, _, gflops = run([DiagonalMatrix((n, n), "A") @ GeneralMatrix((n, n), "B")],
                         {"n": N_DSL, "A": d, "B": B}, "cuda", out)
    assert torch.equal(res["C"].view(N_DSL, N_DSL), d[:, None] * B)

    Bt = torch.rand(N_DSL, N_DSL, device="cuda", generator=g)
    B2 = (Bt + Bt.t()) * 0.5
    res, _, _ = run([SymmetricMatrix((n, n), "A") @ SymmetricMatrix((n, n), "B")],
                    {"n": N_DSL, "A": S_pack, "B": _tri_pack(B2)}, "cuda", out)
    exp = S_full.double() @ B2.double()
    assert relerr64(res["C"].view(N_DSL, N_DSL).cpu().numpy(), exp.cpu().numpy()) <= 1e-5


def test_dsl_upper_and_toeplitz_left(cuda):
    n = Var("n")
    u = W.make_upper(N_DSL, seed=3)
    res, _, _ = run([UpperTriangularMatrix((n, n), "U") @ GeneralMatrix((n, n), "B")],
                    {"n": N_DSL, "U": dev(u["U"]), "B": dev(u["B"])}, "cuda", GeneralMatrix((n, n), "C"))
    R = O.upper_left_rows_f64(u["U"], u["B"], np.arange(N_DSL))
    assert relerr64(res["C"].view(N_DSL, N_DSL).cpu().numpy(), R) <= 1e-5
    t = W.make_toeplitz(N_DSL, seed=4)
    res, _, _ = run([ToeplitzMatrix((n, n), "T") @ GeneralMatrix((n, n), "B")],
                    {"n": N_DSL, "T": dev(t["g"]), "B": dev(t["B"])}, "cuda", GeneralMatrix((n, n), "C"))
    R = O.toeplitz_left_rows_f64(t["g"], t["B"], np.arange(N_DSL))
    assert relerr64(res["C"].view(N_DSL, N_DSL).cpu().numpy(), R) <= 1e-5


def test_dsl_run_graph_sandwich_and_chain(cuda):
    n = Var("n")
    s = W.make_sandwich(256, seed=8)
    A, S, B = GeneralMatrix((n, n), "A"), SymmetricMatrix((n, n), "S"), GeneralMatrix((n, n), "B")
    inputs = {"n": 256, "A": dev(s["A"]), "S": dev(s["S"]), "B": dev(s["B"])}
    inner = A @ S
    expr = inner @ B
    res, ms, _ = run_graph([expr], inputs, "cuda")
    R = O.sandwich_rows_f64(s["A"], s["S"], s["B"], np.arange(256))
    assert relerr64(res[expr.name].view(256, 256).cpu().numpy(), R) <= 1e-5
    # the intermediate A @ S is returned under its own name
    Rm = O.symm_right_rows_f64(s["A"], s["S"], np.arange(256))
    assert relerr64(res[inner.name].view(256, 256).cpu().numpy(), Rm) <= 1e-5
    # a plain chain runs op by op
    G1, G2, G3 = (GeneralMatrix((n, n), x) for x in ("G1", "G2", "G3"))
    w = [W.make_gemm(256, 256, 256, seed=k)["A"] for k in range(3)]
    chain = (G1 @ G2) @ G3
    res, ms, _ = run_graph([chain], {"n": 256, "G1": dev(w[0]), "G2": dev(w[1]), "G3": dev(w[2])}, "cuda")
    exp = w[0].astype(np.float64) @ w[1] @ w[2]
    assert relerr64(res[chain.name].view(256, 256).cpu().numpy(), exp) <= 1e-5


def test_dsl_add_gen_symm_and_same_class(cuda):
    """The DSL's `+` (codegen_cuda.py:1643-1827): general + symmetric expands
    the packed operand; same-class operands add over their storage.  Exact
    against the oracle."""
    n = Var("n")
    rng = np.random.default_rng(9)
    nv = 300
    A = rng.uniform(-1, 1, (nv, nv)).astype(np.float32)
    Sp = rng.uniform(-1, 1, nv * (nv + 1) // 2).astype(np.float32)
    res, ms, gflops = run([GeneralMatrix((n, n), "A") + SymmetricMatrix((n, n), "S")],
                          {"n": nv, "A": dev(A), "S": dev(Sp)}, "cuda", GeneralMatrix((n, n), "C"))
    assert np.array_equal(res["C"].view(nv, nv).cpu().numpy(), O.add_struct_f32(A, Sp, "symm"))
    assert ms > 0 and gflops > 0
    Sq = rng.uniform(-1, 1, Sp.size).astype(np.float32)
    res, _, _ = run([SymmetricMatrix((n, n), "P") + SymmetricMatrix((n, n), "Q")],
                    {"n": nv, "P": dev(Sp), "Q": dev(Sq)}, "cuda", SymmetricMatrix((n, n), "R"))
    assert res["R"].numel() == Sp.size
    assert np.array_equal(res["R"].cpu().numpy(), O.add_f32(Sp, Sq))
