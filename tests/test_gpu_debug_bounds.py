"""The bounds-checked build (libsmm_debug.so) on small odd shapes.

Every structured-operand read of the on-chip fills (packed upper, lower and
symmetric triangles, Toeplitz generators, on the left -- U B, L B, S B, T B --
and on the right -- A U, A L, A S, A T) and of the expansion kernels is
range-checked on the device in that build; a
read outside the operand would be skipped and reported as SMM_ERR_BOUNDS.
The products run in a child process that loads the debug library
(SMM_LIB=debug), on orders 1, 7, 127, 129 and 257 in every mode, with the
on-chip path (SMM_EXPAND=0) and the expanded one, against the oracle's fp64
rows; the device status word must stay clean."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, os, sys
import numpy as np
import torch
sys.path.insert(0, os.getcwd())
from cpp1_b200 import _lib, ops
from cpp1_b200 import workloads as W
import oracle as O
assert _lib.LIB_PATH.endswith("libsmm_debug.so"), _lib.LIB_PATH
TOL = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}
dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
def rel(C, R):
    return float(np.linalg.norm(C.astype(np.float64) - R) / max(np.linalg.norm(R), 1e-300))
worst = {}
for n in (1, 7, 127, 129, 257):
    nc = max(1, (n * 3) // 2)
    for mode in ("3xtf32", "tf32", "bf16"):
        w = W.make_upper(n, nc, seed=n)
        R = O.upper_left_rows_f64(w["U"], w["B"], np.arange(n))
        worst[f"upper{n}_{mode}"] = rel(ops.upper_left(dev(w["U"]), dev(w["B"]), packed=True, mode=mode).cpu().numpy(), R)
        t = W.make_toeplitz(n, nc, seed=n)
        R = O.toeplitz_left_rows_f64(t["g"], t["B"], np.arange(n))
        worst[f"toeplitz{n}_{mode}"] = rel(ops.toeplitz_left(dev(t["g"]), dev(t["B"]), mode=mode).cpu().numpy(), R)
        s = W.make_sandwich(n, seed=n)
        Sd = W.unpack_symmetric(s["S"], n).astype(np.float64)
        worst[f"symm{n}_{mode}"] = rel(ops.symm_left(dev(s["S"]), dev(s["B"]), mode=mode).cpu().numpy(), Sd @ s["B"].astype(np.float64))
        worst[f"gen_x_symm{n}_{mode}"] = rel(ops.gen_x_symm(dev(s["A"]), dev(s["S"]), mode=mode).cpu().numpy(), s["A"].astype(np.float64) @ Sd)
        Ud = W.unpack_upper(w["U"], n).astype(np.float64)
        A = W.make_gemm(nc, 1, n, seed=n)["A"]
        worst[f"gen_x_upper{n}_{mode}"] = rel(ops.gen_x_upper(dev(A), dev(w["U"]), mode=mode).cpu().numpy(), A.astype(np.float64) @ Ud)
        Td = W.toeplitz_dense(t["g"], n).astype(np.float64)
        worst[f"gen_x_toeplitz{n}_{mode}"] = rel(ops.gen_x_toeplitz(dev(A), dev(t["g"]), mode=mode).cpu().numpy(), A.astype(np.float64) @ Td)
        Ld = np.tril(Ud.T)  # lower triangular
        Lp = np.concatenate([Ld[i, :i + 1] for i in range(n)]).astype(np.float32)
        worst[f"lower{n}_{mode}"] = rel(ops.lower_left(dev(Lp), dev(w["B"]), mode=mode).cpu().numpy(), Ld @ w["B"].astype(np.float64))
        worst[f"gen_x_lower{n}_{mode}"] = rel(ops.gen_x_lower(dev(A), dev(Lp), mode=mode).cpu().numpy(), A.astype(np.float64) @ Ld)
        ops.device_status()   # raises SmmError(SMM_ERR_BOUNDS) if any check fired
print(json.dumps(worst))
"""


@pytest.mark.parametrize("expand", ["1", "0"])
def test_debug_bounds_build_small_odd_shapes(cuda, expand):
    lib = os.path.join(ROOT, "cpp1_b200", "libsmm_debug.so")
    assert os.path.exists(lib), "build it with python -m cpp1_b200.build --debug-bounds"
    env = dict(os.environ, SMM_LIB="debug", SMM_EXPAND=expand)
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    worst = json.loads(r.stdout.strip().splitlines()[-1])
    tol = {"3xtf32": 1e-5, "tf32": 5e-3, "bf16": 1e-2}
    bad = {k: v for k, v in worst.items() if v > tol[k.rsplit("_", 1)[1]]}
    assert not bad, bad
