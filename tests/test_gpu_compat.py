"""The reference-compatible wrappers (smm_compat_*: the generated
<Out>_computation calling convention of the DSL's CUDA runner) through the C
ABI: bit-identical to the primary entry points they wrap (same kernels, fp32
3xTF32 mode), synchronous, with the time and the gflops the generated
wrappers report (2 n^3 per product, n^2 for a diagonal scale or a sum)."""
import ctypes

import numpy as np
import pytest
import torch

from cpp1_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def rnd(shape, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.rand(shape, device="cuda", generator=g) * 2 - 1


def call(name, *tensors, n):
    gf, ms = ctypes.c_float(-1.0), ctypes.c_float(-1.0)
    L = _lib.load()
    ptrs = [t.data_ptr() for t in tensors]
    rc = getattr(L, name)(*ptrs, ctypes.addressof(gf), n, ctypes.addressof(ms))
    assert rc == _lib.SMM_OK, _lib.last_error()
    return gf.value, ms.value


@pytest.mark.parametrize("n", [300, 512])
def test_compat_products_match_primary_entries(cuda, n):
    p = n * (n + 1) // 2
    A, B = rnd((n, n), 1), rnd((n, n), 2)
    S, U, Lw = rnd(p, 3), rnd(p, 4), rnd(p, 5)
    d, g = rnd(n, 6), rnd(2 * n - 1, 7)
    cases = [
        ("smm_compat_gen_x_gen", (A, B), lambda: ops.gemm(A, B), 2 * n ** 3),
        ("smm_compat_diag_x_gen", (d, B), lambda: ops.diag_rows(d, B), n * n),
        ("smm_compat_gen_x_diag", (A, d), lambda: ops.diag_cols(A, d), n * n),
        ("smm_compat_upper_x_gen", (U, B), lambda: ops.upper_left(U, B), 2 * n ** 3),
        ("smm_compat_toeplitz_x_gen", (g, B), lambda: ops.toeplitz_left(g, B), 2 * n ** 3),
        ("smm_compat_symm_x_gen", (S, B), lambda: ops.symm_left(S, B), 2 * n ** 3),
        ("smm_compat_gen_x_symm", (A, S), lambda: ops.gen_x_symm(A, S), 2 * n ** 3),
        ("smm_compat_gen_x_upper", (A, U), lambda: ops.gen_x_upper(A, U), 2 * n ** 3),
        ("smm_compat_symm_x_symm", (S, U), lambda: ops.symm_x_symm(S, U), 2 * n ** 3),
        ("smm_compat_gen_x_lower", (A, Lw), lambda: ops.gen_x_lower(A, Lw), 2 * n ** 3),
        ("smm_compat_lower_x_gen", (Lw, B), lambda: ops.lower_left(Lw, B), 2 * n ** 3),
        ("smm_compat_lower_x_lower", (Lw, S), lambda: ops.lower_x_lower(Lw, S), 2 * n ** 3),
        ("smm_compat_add_gen_symm", (A, S), lambda: ops.add_struct(A, S, "symm"), n * n),
    ]
    for name, ins, ref, flops in cases:
        C = torch.full((n, n), float("nan"), device="cuda")
        gflops, ms = call(name, *ins, C, n=n)
        expect = ref()
        torch.cuda.synchronize()
        assert torch.equal(C, expect), name
        assert ms > 0 and gflops > 0, name
        assert gflops == pytest.approx(flops * 1e-9 / (ms * 1e-3), rel=1e-3), name


def test_compat_sandwich_matches_primary_entry(cuda):
    n = 384
    A, B, S = rnd((n, n), 11), rnd((n, n), 12), rnd(n * (n + 1) // 2, 13)
    C = torch.empty((n, n), device="cuda")
    gf, ms = ctypes.c_float(), ctypes.c_float()
    rc = _lib.load().smm_compat_symm_sandwich(A.data_ptr(), S.data_ptr(), B.data_ptr(), C.data_ptr(),
                                              ctypes.addressof(gf), n, ctypes.addressof(ms))
    assert rc == _lib.SMM_OK, _lib.last_error()
    assert torch.equal(C, ops.symm_sandwich(A, S, B))
    assert gf.value == pytest.approx(4 * n ** 3 * 1e-9 / (ms.value * 1e-3), rel=1e-3)


def test_compat_reports_invalid_arguments(cuda):
    gf, ms = ctypes.c_float(), ctypes.c_float()
    rc = _lib.load().smm_compat_gen_x_gen(None, None, None, ctypes.addressof(gf), 64, ctypes.addressof(ms))
    assert rc == _lib.SMM_ERR_INVALID


def test_generated_wrapper_order_of_the_reference_runner(cuda):
    """cpp1_b200.compat.generated_wrapper takes the arguments the way the
    reference's runner passes them (sorted names: C = U @ B gives B_data,
    C_data, U_data, gflops_out, n, time_ms_out) and matches the primary
    entry point bit for bit."""
    from cpp1_b200 import compat
    n = 320
    U, B = rnd(n * (n + 1) // 2, 21), rnd((n, n), 22)
    C = torch.full((n, n), float("nan"), device="cuda")
    arg_names = sorted(["U_data", "B_data", "C_data", "n", "gflops_out", "time_ms_out"])
    fn = compat.generated_wrapper(arg_names, "U", "B", "C", "upper", "gen")
    gf, ms = ctypes.c_float(), ctypes.c_float()
    by_name = {"U_data": ctypes.c_void_p(U.data_ptr()), "B_data": ctypes.c_void_p(B.data_ptr()),
               "C_data": ctypes.c_void_p(C.data_ptr()), "n": ctypes.c_int(n), "gflops_out": ctypes.byref(gf),
               "time_ms_out": ctypes.byref(ms)}
    fn(*[by_name[a] for a in arg_names])
    assert torch.equal(C, ops.upper_left(U, B))
    assert ms.value > 0 and gf.value > 0
