"""GPU parity of every operation against the oracle (the reference's own CPU
kernels' outputs in tests/golden, and the fp64 recomputation of oracle.c).

Tolerances (normwise relative error against fp64):
  3xtf32  <= 1e-5   (fp32 semantics)
  tf32    <= 5e-3   (one TF32 pass)
  bf16    <= 1e-2
The diagonal scale is bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}


@pytest.fixture(params=["1", "0"], ids=["expanded", "on_chip"])
def expand(request, monkeypatch):
    """Packed left operands expanded into a dense copy (the default with a
    full workspace) or built on chip from their packed rows."""
    monkeypatch.setenv("SMM_EXPAND", request.param)
    return request.param


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ---------------------------------------------------------------- diagonal
def test_diag_rows_golden_bitexact(cuda, golden):
    C = host(ops.diag_rows(dev(golden["diag_d"]), dev(golden["diag_B"])))
    assert np.array_equal(C, golden["diag_C"])


@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (7, 129), (64, 4100), (129, 257), (8192, 8192)])
def test_diag_rows_bitexact(cuda, shape):
    M, N = shape
    w = W.make_diag(M, N, seed=M * 31 + N)
    C = host(ops.diag_rows(dev(w["d"]), dev(w["B"])))
    assert np.array_equal(C, O.diag_rows_f32(w["d"], w["B"]))


@pytest.mark.parametrize("shape", [(5, 3), (128, 256), (77, 1030)])
def test_diag_cols_bitexact(cuda, shape):
    M, N = shape
    rng = np.random.default_rng(7)
    A = rng.uniform(-1, 1, (M, N)).astype(np.float32)
    b = rng.uniform(0.5, 1.5, N).astype(np.float32)
    C = host(ops.diag_cols(dev(A), dev(b)))
    assert np.array_equal(C, O.diag_cols_f32(A, b))


def test_diag_rows_unaligned_views(cuda):
    # Offset views (not 16-byte aligned) take the scalar path.
    w = W.make_diag(33, 67, seed=3)
    Bbig = dev(np.concatenate([np.zeros(1, np.float32), w["B"].ravel()]))
    B = Bbig[1:].view(33, 67)
    out = torch.empty(33 * 67 + 1, device="cuda")[1:].view(33, 67)
    C = host(ops.diag_rows(dev(w["d"]), B, out=out))
    assert np.array_equal(C, O.diag_rows_f32(w["d"], w["B"]))


# ---------------------------------------------------------------- contractions
def _relerr_full(C, R):
    return O.relerr(C, R)


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
def test_gemm_golden(cuda, golden, mode):
    A, B = golden["gemm_A"], golden["gemm_B"]
    C = host(ops.gemm(dev(A), dev(B), mode=mode))
    R = O.gemm_rows_f64(A, B, np.arange(A.shape[0]))
    assert _relerr_full(C, R) <= TOL[mode]
    # The reference's own kernel meets the same bound on the same inputs.
    assert O.relerr(golden["gemm_C"], R) <= 1e-5


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
@pytest.mark.parametrize("mnk", [(128, 256, 64), (256, 512, 1024), (1, 1, 1), (7, 5, 3), (129, 257, 127),
                                 (300, 200, 100), (1024, 1024, 1024)])
def test_gemm_shapes(cuda, mode, mnk):
    M, N, K = mnk
    w = W.make_gemm(M, N, K, seed=M + 7 * N + 13 * K)
    C = host(ops.gemm(dev(w["A"]), dev(w["B"]), mode=mode))
    R = O.gemm_rows_f64(w["A"], w["B"], np.arange(M))
    assert _relerr_full(C, R) <= TOL[mode], (mnk, _relerr_full(C, R))


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
@pytest.mark.parametrize("mnk", [(1, 1, 1), (128, 128, 32), (7, 129, 257), (300, 200, 1000), (1024, 1024, 1024),
                                 (1000, 1000, 4100)])
def test_gemm_split_k_clusters(cuda, monkeypatch, mode, mnk):
    """Each 128 x 128 tile split along K over a cluster of two CTAs (the
    small-product form; SMM_SPLITK=2 forces it): ranges of whole stages, an
    empty second half for short K, ragged M, N and K.  Same bound as the
    unsplit product, and the same result on a second run."""
    monkeypatch.setenv("SMM_SPLITK", "2")
    M, N, K = mnk
    w = W.make_gemm(M, N, K, seed=M + 3 * N + 5 * K)
    A, B = dev(w["A"]), dev(w["B"])
    C = host(ops.gemm(A, B, mode=mode))
    rows = np.unique(np.linspace(0, M - 1, min(M, 64)).astype(np.int32))
    R = O.gemm_rows_f64(w["A"], w["B"], rows)
    assert _relerr_full(C[rows], R) <= TOL[mode], (mnk, _relerr_full(C[rows], R))
    assert np.array_equal(host(ops.gemm(A, B, mode=mode)), C)


def test_tf32_operand_reading_truncates(cuda):
    """kind::tf32 must ignore the 13 low mantissa bits of an fp32 operand
    (truncation): the 3xTF32 split relies on hi = raw bits & 0xffffe000.
    x = 1 + 3*2^-12 truncates to 1 and rounds to 1 + 2^-10."""
    x = np.float32(1.0 + 3.0 * 2.0 ** -12)
    A = np.full((128, 8), x, np.float32)
    B = np.zeros((8, 64), np.float32)
    B[0, :] = 1.0
    C = host(ops.gemm(dev(A), dev(B), mode="tf32"))
    assert np.all(C == 1.0), np.unique(C)


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
def test_upper_packed_golden(cuda, golden, mode):
    Up, B = golden["upper_U"], golden["upper_B"]
    C = host(ops.upper_left(dev(Up), dev(B), packed=True, mode=mode))
    R = O.upper_left_rows_f64(Up, B, np.arange(B.shape[0]))
    assert _relerr_full(C, R) <= TOL[mode]
    assert O.relerr(golden["upper_C"], R) <= 1e-5


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
@pytest.mark.parametrize("packed", [True, False])
@pytest.mark.parametrize("n_cols", [(1, 1), (5, 9), (128, 64), (129, 200), (300, 260), (1024, 1024)])
def test_upper_shapes(cuda, expand, packed, n_cols, mode):
    N, ncols = n_cols
    w = W.make_upper(N, ncols, seed=N + ncols)
    U = w["U"] if packed else W.unpack_upper(w["U"], N)
    C = host(ops.upper_left(dev(U), dev(w["B"]), packed=packed, mode=mode))
    R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(N))
    assert _relerr_full(C, R) <= TOL[mode], (n_cols, _relerr_full(C, R))


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
@pytest.mark.parametrize("n_cols", [(1, 1), (130, 70), (300, 260), (1024, 1024), (1100, 257)])
def test_upper_split_k_clusters(cuda, monkeypatch, n_cols, mode):
    """U B (U expanded, zeros skipped per row tile) with each 128 x 128 tile
    split along K over a two-CTA cluster (SMM_SPLITK=2 forces it): row tiles
    near the bottom leave the second CTA an empty K range.  Whole products
    and row slabs off the tile grid, against fp64; a second run is identical."""
    from cpp1_b200 import _lib
    monkeypatch.setenv("SMM_SPLITK", "2")
    N, ncols = n_cols
    w = W.make_upper(N, ncols, seed=N + 2 * ncols)
    U, B = dev(w["U"]), dev(w["B"])
    C = host(ops.upper_left(U, B, packed=True, mode=mode))
    R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(N))
    assert _relerr_full(C, R) <= TOL[mode], (n_cols, _relerr_full(C, R))
    assert np.array_equal(host(ops.upper_left(U, B, packed=True, mode=mode)), C)
    L = _lib.load()
    m = ops._mode(mode)
    ws = ops.workspace(L.smm_upper_left_workspace_size(N, ncols, _lib.FMT_PACKED, m), torch.device("cuda"))
    r0 = N // 3
    nrows = N - r0
    Cs = torch.full((nrows, ncols), float("nan"), device="cuda")
    _slab_call("smm_upper_left_rows", L, U, B, Cs, N, ncols, r0, nrows, m, ws.data_ptr(), ws.numel())
    assert _relerr_full(host(Cs), R[r0:]) <= TOL[mode]


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
def test_toeplitz_golden(cuda, golden, mode):
    g, B = golden["toeplitz_g"], golden["toeplitz_B"]
    C = host(ops.toeplitz_left(dev(g), dev(B), mode=mode))
    R = O.toeplitz_left_rows_f64(g, B, np.arange(B.shape[0]))
    assert _relerr_full(C, R) <= TOL[mode]
    assert O.relerr(golden["toeplitz_C"], R) <= 1e-5


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
@pytest.mark.parametrize("n_cols", [(1, 1), (3, 8), (128, 64), (130, 70), (512, 1024)])
def test_toeplitz_shapes(cuda, n_cols, mode):
    N, ncols = n_cols
    w = W.make_toeplitz(N, ncols, seed=N * 3 + ncols)
    C = host(ops.toeplitz_left(dev(w["g"]), dev(w["B"]), mode=mode))
    R = O.toeplitz_left_rows_f64(w["g"], w["B"], np.arange(N))
    assert _relerr_full(C, R) <= TOL[mode], (n_cols, _relerr_full(C, R))


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
@pytest.mark.parametrize("n_cols", [(1, 1), (6, 10), (128, 128), (257, 130), (700, 300)])
def test_symm_left_shapes(cuda, expand, n_cols, mode):
    N, ncols = n_cols
    s = W.make_sandwich(N, seed=N)
    B = W.make_gemm(N, 1, ncols, seed=ncols)["A"]  # N x ncols
    C = host(ops.symm_left(dev(s["S"]), dev(B), mode=mode))
    assert B.shape == (N, ncols)
    S = W.unpack_symmetric(s["S"], N).astype(np.float64)
    R = S @ B.astype(np.float64)
    assert _relerr_full(C, R) <= TOL[mode]


# ---------------------------------------------------------------- row slabs
def _slab_call(entry, L, first, B, C, N, ncols, r0, nrows, m, ws, wsb):
    from cpp1_b200 import _lib
    args = [first.data_ptr()] + ([_lib.FMT_PACKED] if entry == "smm_upper_left_rows" else [])
    rc = getattr(L, entry)(*args, B.data_ptr(), C.data_ptr(), N, ncols, r0, nrows, m, ws, wsb, None)
    assert rc == _lib.SMM_OK, _lib.last_error()


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
@pytest.mark.parametrize("kind", ["upper", "symm", "toeplitz"])
def test_row_slab_entries(cuda, expand, kind, mode):
    """The multi-GPU row-slab entries (rows [r0, r0 + nrows) of the product)
    against fp64, slabs starting off the 128- and 256-row tile grid."""
    from cpp1_b200 import _lib
    N, ncols = 1000, 384
    L = _lib.load()
    m = ops._mode(mode)
    if kind == "upper":
        w = W.make_upper(N, ncols, seed=5)
        first, Bn, entry = w["U"], w["B"], "smm_upper_left_rows"
        R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(N))
        need = L.smm_upper_left_workspace_size(N, ncols, _lib.FMT_PACKED, m)
    elif kind == "symm":
        s = W.make_sandwich(N, seed=6)
        Bn = W.make_gemm(N, 1, ncols, seed=7)["A"]
        first, entry = s["S"], "smm_symm_left_rows"
        R = W.unpack_symmetric(s["S"], N).astype(np.float64) @ Bn.astype(np.float64)
        need = L.smm_symm_left_workspace_size(N, ncols, m)
    else:
        w = W.make_toeplitz(N, ncols, seed=8)
        first, Bn, entry = w["g"], w["B"], "smm_toeplitz_left_rows"
        R = O.toeplitz_left_rows_f64(w["g"], w["B"], np.arange(N))
        need = L.smm_toeplitz_left_workspace_size(N, ncols, m)
    ws = ops.workspace(need, torch.device("cuda"))
    first_d, B = dev(first), dev(Bn)
    for r0, nrows in ((0, 300), (300, 333), (633, 367), (999, 1)):
        C = torch.full((nrows, ncols), float("nan"), device="cuda")
        _slab_call(entry, L, first_d, B, C, N, ncols, r0, nrows, m, ws.data_ptr(), ws.numel())
        assert _relerr_full(host(C), R[r0:r0 + nrows]) <= TOL[mode], (r0, nrows)


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
def test_sandwich_golden(cuda, golden, mode):
    A, S, B = golden["sandwich_A"], golden["sandwich_S"], golden["sandwich_B"]
    C = host(ops.symm_sandwich(dev(A), dev(S), dev(B), mode=mode))
    R = O.sandwich_rows_f64(A, S, B, np.arange(A.shape[0]))
    assert _relerr_full(C, R) <= TOL[mode]
    assert O.relerr(golden["sandwich_C"], R) <= 1e-5


@pytest.mark.parametrize("mode", ["3xtf32", "bf16"])
@pytest.mark.parametrize("N", [1, 7, 130, 512])
def test_sandwich_shapes(cuda, expand, N, mode):
    s = W.make_sandwich(N, seed=N + 1)
    C = host(ops.symm_sandwich(dev(s["A"]), dev(s["S"]), dev(s["B"]), mode=mode))
    R = O.sandwich_rows_f64(s["A"], s["S"], s["B"], np.arange(N))
    assert _relerr_full(C, R) <= TOL[mode]


@pytest.mark.parametrize("mode", ["3xtf32", "tf32", "bf16"])
def test_packed_left_without_room_for_expansion(cuda, mode):
    """A workspace with no room for the dense copy of the packed operand (none
    at all when B needs no staging) still computes the product, on chip."""
    from cpp1_b200 import _lib
    L = _lib.load()
    m = ops._mode(mode)
    N, ncols = 520, 256
    w = W.make_upper(N, ncols, seed=11)
    U, B = dev(w["U"]), dev(w["B"])
    full = L.smm_upper_left_workspace_size(N, ncols, _lib.FMT_PACKED, m)
    small = full - (N * ((N + 7) // 8 * 8) * 2 if mode == "bf16" else N * ((N + 3) // 4 * 4) * 4)
    small = small // 256 * 256
    ws = ops.workspace(max(small, 1), torch.device("cuda"))
    C = torch.full((N, ncols), float("nan"), device="cuda")
    rc = L.smm_upper_left(U.data_ptr(), _lib.FMT_PACKED, B.data_ptr(), C.data_ptr(), N, ncols, m,
                          ws.data_ptr() if small > 0 else None, small, None)
    assert rc == _lib.SMM_OK, _lib.last_error()
    R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(N))
    assert _relerr_full(host(C), R) <= TOL[mode]


# ---------------------------------------------------------------- failure detection
def test_timeout_probe_returns_status_and_context_survives(cuda):
    from cpp1_b200 import _lib
    L = _lib.load()
    rc = L.smm_debug_timeout_probe(50_000_000, None)  # 50 ms
    assert rc == _lib.SMM_ERR_DEVICE_TIMEOUT, _lib.last_error()
    # The status word was consumed; the context still works.
    ops.device_status()
    w = W.make_gemm(128, 128, 32, seed=1)
    C = host(ops.gemm(dev(w["A"]), dev(w["B"])))
    R = O.gemm_rows_f64(w["A"], w["B"], np.arange(128))
    assert O.relerr(C, R) <= 1e-5
    ops.device_status()


@pytest.mark.parametrize("mode", ["tf32", "bf16"])
@pytest.mark.parametrize("mnk", [(2048, 2048, 2048), (2300, 2100, 1000), (4096, 2048, 3000), (1536, 7936, 520)])
def test_persistent_pair_kernel_matches_per_tile_kernel(cuda, monkeypatch, mode, mnk):
    """One-pass modes on 256 x 256 pair tiles run the persistent kernel (one
    CTA pair per SM pair, double-buffered accumulator).  Each tile's MMA
    sequence is the per-tile kernel's, so the results are bit-identical
    (SMM_PERSIST=0 selects the per-tile kernel); ragged M, N and K."""
    M, N, K = mnk
    w = W.make_gemm(M, N, K, seed=M + N + K)
    A, B = dev(w["A"]), dev(w["B"])
    C_p = host(ops.gemm(A, B, mode=mode))
    monkeypatch.setenv("SMM_PERSIST", "0")
    C_t = host(ops.gemm(A, B, mode=mode))
    assert np.array_equal(C_p, C_t)
    rows = np.unique(np.linspace(0, M - 1, 48).astype(np.int32))
    assert _relerr_full(C_p[rows], O.gemm_rows_f64(w["A"], w["B"], rows)) <= TOL[mode]


@pytest.mark.parametrize("mode", ["tf32", "bf16"])
def test_persistent_upper_matches_per_tile_kernel(cuda, monkeypatch, mode):
    n = 3000
    w = W.make_upper(n, 2560, seed=41)
    U, B = dev(w["U"]), dev(w["B"])
    C_p = host(ops.upper_left(U, B, mode=mode))
    monkeypatch.setenv("SMM_PERSIST", "0")
    C_t = host(ops.upper_left(U, B, mode=mode))
    assert np.array_equal(C_p, C_t)
