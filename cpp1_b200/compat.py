"""Reference-compatible call convention for the generated wrappers.

The reference's runner (src/dsl/runner_cuda.py:29-127) compiles
`<Out>_computation` for every expression and calls it with its arguments in
the order `generate_cuda_code` returns them: Python's `sorted()` of the
argument names (src/dsl/codegen_cuda.py:41-42) -- every `<Name>_data` pointer,
every dimension by its lower-case name, `gflops_out` and `time_ms_out`.  The
pointer order therefore depends on the matrices' names (`C = U @ B` gives
`B_data, C_data, U_data, gflops_out, n, time_ms_out`).

`generated_wrapper` returns a callable with exactly that signature that
routes to libsmm's prebuilt compatibility entry of the operand pair
(`smm_compat_<lhs>_x_<rhs>`, which takes lhs, rhs, out, gflops_out, n,
time_ms_out).  A maintainer who keeps the reference's runner replaces its
generate-compile-load block with

    kernel_func = generated_wrapper(arg_names, lhs.name, rhs.name, out.name,
                                    lhs_kind, rhs_kind)

and its `kernel_func(*c_args)` call stays as it is.
"""
from __future__ import annotations

from typing import Callable, Sequence

from . import _lib

# (lhs kind, rhs kind) -> compatibility entry point
ENTRIES = {
    ("gen", "gen"): "smm_compat_gen_x_gen", ("diag", "gen"): "smm_compat_diag_x_gen",
    ("gen", "diag"): "smm_compat_gen_x_diag", ("upper", "gen"): "smm_compat_upper_x_gen",
    ("toeplitz", "gen"): "smm_compat_toeplitz_x_gen", ("symm", "gen"): "smm_compat_symm_x_gen",
    ("gen", "symm"): "smm_compat_gen_x_symm", ("gen", "upper"): "smm_compat_gen_x_upper",
    ("symm", "symm"): "smm_compat_symm_x_symm", ("gen", "lower"): "smm_compat_gen_x_lower",
    ("lower", "gen"): "smm_compat_lower_x_gen", ("lower", "lower"): "smm_compat_lower_x_lower",
    ("gen", "symm", "add"): "smm_compat_add_gen_symm",
}


def generated_wrapper(arg_names: Sequence[str], lhs_name: str, rhs_name: str, out_name: str, lhs_kind: str,
                      rhs_kind: str, operator: str = "matmul") -> Callable[..., int]:
    """A callable taking the generated wrapper's arguments in `arg_names`
    order (ctypes objects, as the reference's runner builds them) and calling
    the compatibility entry point of the operand pair.  Raises SmmError on a
    non-OK status (the generated wrappers ignore errors; this one does not)."""
    key = (lhs_kind, rhs_kind) if operator == "matmul" else (lhs_kind, rhs_kind, "add")
    if operator == "add" and key not in ENTRIES and (rhs_kind, lhs_kind, "add") in ENTRIES:
        key = (rhs_kind, lhs_kind, "add")  # General + Symmetric in either order
        lhs_name, rhs_name = rhs_name, lhs_name
    if key not in ENTRIES:
        raise NotImplementedError(f"no compatibility entry for {lhs_kind} {operator} {rhs_kind}")
    names = list(arg_names)
    if names != sorted(names):
        raise ValueError("arg_names must be in the generated wrapper's (sorted) order")
    pos = {n: i for i, n in enumerate(names)}
    try:
        li, ri, oi = pos[f"{lhs_name}_data"], pos[f"{rhs_name}_data"], pos[f"{out_name}_data"]
        gi, ti = pos["gflops_out"], pos["time_ms_out"]
    except KeyError as e:
        raise ValueError(f"argument {e} missing from {names}") from None
    dims = [i for n, i in pos.items() if not n.endswith("_data") and n not in ("gflops_out", "time_ms_out")]
    if not dims:
        raise ValueError("no dimension argument")
    fn = getattr(_lib.load(), ENTRIES[key])
    entry = ENTRIES[key]

    def call(*args):
        if len(args) != len(names):
            raise TypeError(f"expected {len(names)} arguments, got {len(args)}")
        n = args[dims[0]]
        n = n.value if hasattr(n, "value") else int(n)
        rc = fn(args[li], args[ri], args[oi], args[gi], n, args[ti])
        _lib.check(rc, entry)
        return rc

    return call


__all__ = ["ENTRIES", "generated_wrapper"]
