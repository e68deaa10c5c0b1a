"""Lower-triangular operands (packed lower, idx(i,j) = i(i+1)/2 + j, the
reference DSL's lower_triangular_layout, layout_functions.py:25-36) on the
GPU through the C ABI: L @ B, A @ L (the reference's Gen @ Lower,
codegen_multiply_avx.py:546) and L1 @ L2 (:644), in single-CTA and CTA-pair
tiles, against fp64 (normwise; 1e-5 for 3xTF32, 5e-3 TF32, 1e-2 bf16).  The
product of two lower matrices must be exactly zero above the diagonal."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import ops
from cpp1_b200.dsl.matrix import GeneralMatrix, LowerTriangularMatrix
from cpp1_b200.dsl.runner_cuda import run
from cpp1_b200.dsl.var import Var

pytestmark = pytest.mark.gpu

MODES = [("3xtf32", 1e-5), ("tf32", 5e-3), ("bf16", 1e-2)]


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def lower_packed(n, seed):
    return np.random.default_rng(seed).uniform(-1, 1, n * (n + 1) // 2).astype(np.float32)


def relerr(C, R):
    return O.relerr(np.ascontiguousarray(C, np.float32), np.asarray(R, np.float64))


@pytest.fixture(params=["0", "1"], ids=["single", "pair"])
def tiles(request, monkeypatch):
    monkeypatch.setenv("SMM_PAIR", request.param)
    return request.param


@pytest.mark.parametrize("mode,tol", MODES)
@pytest.mark.parametrize("n,ncols", [(1, 1), (7, 9), (128, 128), (300, 200), (1000, 512)])
@pytest.mark.parametrize("expand", ["1", "0"])
def test_lower_left(cuda, tiles, mode, tol, n, ncols, expand, monkeypatch):
    monkeypatch.setenv("SMM_EXPAND", expand)
    Lp = lower_packed(n, n)
    B = np.random.default_rng(n + 1).uniform(-1, 1, (n, ncols)).astype(np.float32)
    C = ops.lower_left(dev(Lp), dev(B), mode=mode).cpu().numpy()
    ref = O.unpack_f32(Lp, "lower", n).astype(np.float64) @ B.astype(np.float64)
    assert relerr(C, ref) <= tol


@pytest.mark.parametrize("mode,tol", MODES)
@pytest.mark.parametrize("m,n", [(1, 1), (9, 7), (128, 128), (200, 300), (512, 1000)])
@pytest.mark.parametrize("expand", ["1", "0"])
def test_gen_x_lower(cuda, tiles, mode, tol, m, n, expand, monkeypatch):
    monkeypatch.setenv("SMM_EXPAND", expand)
    A = np.random.default_rng(m).uniform(-1, 1, (m, n)).astype(np.float32)
    Lp = lower_packed(n, n + 3)
    C = ops.gen_x_lower(dev(A), dev(Lp), mode=mode).cpu().numpy()
    ref = A.astype(np.float64) @ O.unpack_f32(Lp, "lower", n).astype(np.float64)
    assert relerr(C, ref) <= tol


@pytest.mark.parametrize("mode,tol", MODES)
@pytest.mark.parametrize("n", [1, 7, 128, 300, 1000])
@pytest.mark.parametrize("expand", ["1", "0"])
def test_lower_x_lower(cuda, tiles, mode, tol, n, expand, monkeypatch):
    monkeypatch.setenv("SMM_EXPAND", expand)
    L1, L2 = lower_packed(n, 2 * n), lower_packed(n, 2 * n + 1)
    C = ops.lower_x_lower(dev(L1), dev(L2), mode=mode).cpu().numpy()
    D1, D2 = O.unpack_f32(L1, "lower", n), O.unpack_f32(L2, "lower", n)
    ref = D1.astype(np.float64) @ D2.astype(np.float64)
    assert relerr(C, ref) <= tol
    assert not np.triu(C, 1).any()


def test_dsl_lower_products(cuda):
    n = Var("n")
    nv = 384
    Lp = lower_packed(nv, 5)
    B = np.random.default_rng(6).uniform(-1, 1, (nv, nv)).astype(np.float32)
    D = O.unpack_f32(Lp, "lower", nv).astype(np.float64)
    out = GeneralMatrix((n, n), "C")
    res, _, _ = run([LowerTriangularMatrix((n, n), "L") @ GeneralMatrix((n, n), "B")],
                    {"n": nv, "L": dev(Lp), "B": dev(B)}, "cuda", out)
    assert relerr(res["C"].view(nv, nv).cpu().numpy(), D @ B) <= 1e-5
    res, _, _ = run([GeneralMatrix((n, n), "B") @ LowerTriangularMatrix((n, n), "L")],
                    {"n": nv, "L": dev(Lp), "B": dev(B)}, "cuda", out)
    assert relerr(res["C"].view(nv, nv).cpu().numpy(), B.astype(np.float64) @ D) <= 1e-5
    res, _, _ = run([LowerTriangularMatrix((n, n), "L") @ LowerTriangularMatrix((n, n), "M")],
                    {"n": nv, "L": dev(Lp), "M": dev(Lp)}, "cuda", out)
    assert relerr(res["C"].view(nv, nv).cpu().numpy(), D @ D) <= 1e-5
