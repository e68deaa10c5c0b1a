"""Generate the golden fixtures in tests/golden/ (run in a checkout that has
the reference next to it; the fixtures themselves are committed).

Two kinds of fixture:

1. ``golden_outputs.npz`` — seeded small inputs (``cpp1_b200.workloads``) and
   the outputs of the reference's OWN CPU kernels, compiled from the reference
   sources into ``oracle/_ref`` by ``oracle/Makefile``:

   ===========  =====================================================  ==============
   key prefix   reference kernel                                       shape
   ===========  =====================================================  ==============
   gemm_        gemm_benchmark.cpp:40-156                              M,N,K=128,128,64
   diag_        diag_matmul.cpp:45-111 (on B^T)                        64 x 128
   upper_       upper_triag_matmul.cpp:41-137 (via (UB)^T=(B^TJ)(JU^TJ)J)  N=64, 128 cols
   sandwich_    symmetric_matmul.cpp:84-211, then gemm_benchmark.cpp   N=64
   toeplitz_    toeplitz_matmul2.cpp:44-144 (via (TB)^T = B^T T^T)    N=128, 64 cols
   tcompact_    toeplitz_matmul2.cpp:34-41 build_toeplitz_compact      T 37 x 53
   ===========  =====================================================  ==============

2. ``golden_layouts.npz`` — the reference DSL's storage conventions, obtained
   by evaluating its own symbolic layout functions
   (``src/dsl/layout_functions.py``) on concrete indices for n = 7: for each
   (i, j) the element index into the storage array, or -1 for a structural
   zero.  This pins the packed-upper, packed-lower, symmetric, diagonal and
   Toeplitz formats the library's C ABI accepts.

Usage:  python tests/golden/make_golden.py [--reference /root/reference]
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from cpp1_b200 import workloads as W  # noqa: E402
import oracle as O  # noqa: E402

LAYOUT_N = 7


def _eval_index(expr, dsl_var):
    """Evaluate one of the reference DSL's index expressions built on
    concrete integers.  Returns the subscript into the data array, or -1 when
    the expression selects a structural zero."""
    var_mod = dsl_var
    if isinstance(expr, (int, np.integer)):
        return ("const", int(expr))
    if isinstance(expr, var_mod.Conditional):
        c = expr.condition
        lhs = _num(c.left, var_mod)
        rhs = _num(c.right, var_mod)
        ok = {"<=": lhs <= rhs, ">=": lhs >= rhs, "==": lhs == rhs, "<": lhs < rhs, ">": lhs > rhs}[c.op]
        return _eval_index(expr.true_value if ok else expr.false_value, var_mod)
    if isinstance(expr, var_mod.ArithmeticExpression) and expr.op == "subscript":
        return ("index", _num(expr.right, var_mod))
    raise TypeError(f"unexpected layout expression {expr!r}")


def _num(e, var_mod):
    if isinstance(e, (int, np.integer)):
        return int(e)
    if isinstance(e, var_mod.ArithmeticExpression):
        a = _num(e.left, var_mod)
        b = _num(e.right, var_mod)
        if e.op == "+":
            return a + b
        if e.op == "-":
            return a - b
        if e.op == "*":
            return a * b
        if e.op == "/":
            # the generated C divides integers; i*(i-1) and i*(i+1) are even
            return a // b
    raise TypeError(f"unexpected arithmetic {e!r}")


def layout_maps(reference: str) -> dict:
    sys.path.insert(0, os.path.join(reference, "src"))
    from dsl import layout_functions as LF  # reference DSL module
    from dsl import var as V

    n = LAYOUT_N
    data = V.Var("X_data")
    out = {}
    for name in ("general", "upper_triangular", "lower_triangular", "diagonal", "toeplitz", "symmetric"):
        fn = getattr(LF, f"{name}_layout")
        m = np.full((n, n), -1, np.int64)
        for i in range(n):
            for j in range(n):
                kind, val = _eval_index(fn(i, j, data, n), V)
                m[i, j] = val if kind == "index" else -1
        out[f"layout_{name}"] = m
    out["layout_n"] = np.array(n)
    return out


def outputs() -> dict:
    out = {}
    g = W.make_gemm(128, 128, 64, seed=11)
    out.update(gemm_A=g["A"], gemm_B=g["B"], gemm_C=O.ref_gemm(g["A"], g["B"])[0])
    d = W.make_diag(64, 128, seed=12)
    out.update(diag_d=d["d"], diag_B=d["B"], diag_C=O.ref_diag_rows(d["d"], d["B"])[0])
    u = W.make_upper(64, 128, seed=13)
    out.update(upper_U=u["U"], upper_B=u["B"], upper_C=O.ref_upper_left(u["U"], u["B"])[0])
    s = W.make_sandwich(64, seed=14)
    out.update(sandwich_A=s["A"], sandwich_S=s["S"], sandwich_B=s["B"],
               sandwich_C=O.ref_sandwich(s["A"], s["S"], s["B"])[0])
    t = W.make_toeplitz(128, 64, seed=15)
    out.update(toeplitz_g=t["g"], toeplitz_B=t["B"], toeplitz_C=O.ref_toeplitz_left(t["g"], t["B"])[0])
    # generator of a rectangular Toeplitz matrix, by the driver's own
    # build_toeplitz_compact (toeplitz_matmul2.cpp:34-41)
    rng = np.random.default_rng(16)
    tc = np.ascontiguousarray(rng.uniform(-1, 1, (37, 53)).astype(np.float32))
    out.update(tcompact_T=tc, tcompact_g=O.ref_toeplitz_compact(tc))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CPP1_REFERENCE", "/root/reference"),
                    help="reference checkout (default: $CPP1_REFERENCE, else this container's mount point)")
    args = ap.parse_args()
    O.build(with_reference=True)
    if not O.ref_available():
        raise SystemExit("reference kernels not built (is the reference checkout present?)")
    np.savez_compressed(os.path.join(HERE, "golden_outputs.npz"), **outputs())
    np.savez_compressed(os.path.join(HERE, "golden_layouts.npz"), **layout_maps(args.reference))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
