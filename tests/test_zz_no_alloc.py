"""The allocation-free sandwich entry point, smm_symm_sandwich_noalloc, for
callers that cannot allocate device memory (a host framework that owns all
device memory through its own pool, or a latency-critical path that must not
pay cudaMalloc's implicit synchronisation).  Its scratch is a static 16 MiB
device array inside the library instead of a caller workspace.

Called through the C ABI twice in a row per case (the second call finds the
first one's data left in the shared scratch), it must meet the oracle's fp64
result within the mode's tolerance and agree with the allocating entry point
smm_symm_sandwich, at the limits of the scratch: S expanded into a dense copy
(N = 1000), padded operand copies (N = 601), the whole scratch with S mirrored
on chip (N = 2048, the fp32 maximum) and bf16 mode at its maximum (N = 1294).
Sizes beyond the scratch are rejected with a clear error.  This file is
collected last so that a run stopping at the first failure has already run
every other test; it also passes on its own in a fresh process."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import _lib, ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = {"3xtf32": 1e-5, "bf16": 1e-2}


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("N,mode,seed", [(1000, "3xtf32", 21), (601, "3xtf32", 22), (2048, "3xtf32", 23),
                                         (1294, "bf16", 24)],
                         ids=["expanded_S", "padded_copies", "mirror_full_scratch", "bf16_max"])
def test_noalloc_sandwich_two_calls_vs_oracle(cuda, N, mode, seed):
    L = _lib.load()
    m = _lib.MODES[mode]
    w = W.make_sandwich(N, seed=seed)
    A, S, B = dev(w["A"]), dev(w["S"]), dev(w["B"])
    rng = np.random.default_rng(seed)
    rows = np.sort(np.concatenate([[0, N - 1], rng.choice(N, 62, replace=False)])).astype(np.int32)
    truth = O.sandwich_rows_f64(w["A"], w["S"], w["B"], rows)
    outs = []
    for _ in range(2):
        C = torch.full((N, N), float("nan"), device="cuda")
        rc = L.smm_symm_sandwich_noalloc(A.data_ptr(), S.data_ptr(), B.data_ptr(), C.data_ptr(), N, m, None)
        assert rc == _lib.SMM_OK, _lib.last_error()
        torch.cuda.synchronize()
        ops.device_status()
        got = C.cpu().numpy()
        assert np.isfinite(got).all()
        assert O.relerr(got[rows], truth) <= TOL[mode]
        outs.append(got)
    assert np.array_equal(outs[0], outs[1])
    C_alloc = ops.symm_sandwich(A, S, B, mode=mode).cpu().numpy()
    assert O.relerr(outs[0], C_alloc.astype(np.float64)) <= TOL[mode]


@pytest.mark.parametrize("N,mode", [(4096, 0), (2052, 0), (1295, 2)])
def test_noalloc_sandwich_rejects_sizes_beyond_scratch(cuda, N, mode):
    L = _lib.load()
    small = torch.zeros(16, device="cuda")
    p = small.data_ptr()
    rc = L.smm_symm_sandwich_noalloc(p, p, p, p, N, mode, None)
    assert rc == _lib.SMM_ERR_WORKSPACE
    assert "static scratch" in _lib.last_error()
