"""The allocation-free sandwich entry point, smm_symm_sandwich_noalloc, for
callers that cannot allocate device memory (a host framework that owns all
device memory through its own pool, or a latency-critical path that must not
pay cudaMalloc's implicit synchronisation).  Its scratch is a static 16 MiB
device array inside the library instead of a caller workspace.

Called through the C ABI, it must give the same result as the allocating
entry point smm_symm_sandwich (same tolerance as the other 3xTF32 tests), on
two calls in a row — the second one finds the first one's data left in the
shared scratch — and reject sizes beyond the scratch with a clear error.
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import _lib, ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-5


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def test_noalloc_sandwich_matches_allocating_entry_two_calls(cuda):
    L = _lib.load()
    # N = 1000: aligned rows (intermediate + lo planes fill 16 MB of scratch).
    # N = 601: padded copies of A and B share the scratch too.
    for N, seed in ((1000, 21), (601, 22)):
        w = W.make_sandwich(N, seed=seed)
        A, S, B = dev(w["A"]), dev(w["S"]), dev(w["B"])
        C_ref = ops.symm_sandwich(A, S, B)
        C = torch.full((N, N), float("nan"), device="cuda")
        rc = L.smm_symm_sandwich_noalloc(A.data_ptr(), S.data_ptr(), B.data_ptr(), C.data_ptr(), N, 0, None)
        assert rc == _lib.SMM_OK, _lib.last_error()
        torch.cuda.synchronize()
        ops.device_status()
        got = C.cpu().numpy()
        ref = C_ref.cpu().numpy()
        assert np.isfinite(got).all()
        assert O.relerr(got, ref.astype(np.float64)) <= TOL


def test_noalloc_sandwich_rejects_sizes_beyond_scratch(cuda):
    L = _lib.load()
    N = 4096
    small = torch.zeros(16, device="cuda")
    p = small.data_ptr()
    rc = L.smm_symm_sandwich_noalloc(p, p, p, p, N, 0, None)
    assert rc == _lib.SMM_ERR_WORKSPACE
    assert "static scratch" in _lib.last_error()
