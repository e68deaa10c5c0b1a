"""cpp1_b200.compat.generated_wrapper on CPU: the reference runner's sorted
argument order (src/dsl/codegen_cuda.py:41-42) is mapped onto the
compatibility entry's (lhs, rhs, out, gflops_out, n, time_ms_out), whatever
the matrices are named.  The library is replaced by a recorder."""
import pytest

from cpp1_b200 import _lib, compat


class _Rec:
    def __init__(self):
        self.calls = []

    def __getattr__(self, name):
        def f(*args):
            self.calls.append((name, args))
            return 0
        return f


@pytest.fixture
def rec(monkeypatch):
    r = _Rec()
    monkeypatch.setattr(_lib, "load", lambda: r)
    return r


@pytest.mark.parametrize("names,lk,rk,entry", [
    (("A", "B", "C"), "gen", "gen", "smm_compat_gen_x_gen"),
    (("U", "B", "C"), "upper", "gen", "smm_compat_upper_x_gen"),
    (("X", "S", "Out"), "gen", "symm", "smm_compat_gen_x_symm"),
    (("d", "M", "R"), "diag", "gen", "smm_compat_diag_x_gen"),
])
def test_sorted_arguments_reach_the_entry_in_lhs_rhs_out_order(rec, names, lk, rk, entry):
    lhs, rhs, out = names
    arg_names = sorted([f"{lhs}_data", f"{rhs}_data", f"{out}_data", "n", "gflops_out", "time_ms_out"])
    fn = compat.generated_wrapper(arg_names, lhs, rhs, out, lk, rk)
    values = {f"{lhs}_data": "LHS", f"{rhs}_data": "RHS", f"{out}_data": "OUT", "n": 77, "gflops_out": "GF",
              "time_ms_out": "MS"}
    fn(*[values[a] for a in arg_names])
    assert rec.calls == [(entry, ("LHS", "RHS", "OUT", "GF", 77, "MS"))]


def test_add_either_order_and_errors(rec):
    arg_names = sorted(["S_data", "A_data", "C_data", "n", "gflops_out", "time_ms_out"])
    fn = compat.generated_wrapper(arg_names, "S", "A", "C", "symm", "gen", operator="add")
    vals = {"S_data": "S", "A_data": "A", "C_data": "C", "n": 5, "gflops_out": "G", "time_ms_out": "T"}
    fn(*[vals[a] for a in arg_names])
    assert rec.calls == [("smm_compat_add_gen_symm", ("A", "S", "C", "G", 5, "T"))]
    with pytest.raises(NotImplementedError):
        compat.generated_wrapper(arg_names, "S", "A", "C", "toeplitz", "toeplitz")
    with pytest.raises(ValueError):
        compat.generated_wrapper(list(reversed(arg_names)), "S", "A", "C", "symm", "gen", operator="add")
