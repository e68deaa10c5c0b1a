"""Failure detection in the contraction kernel itself, without a GPU fault.

A 2048^3 3xTF32 GEMM (CTA pairs, 256-wide tiles) is launched with a pipeline
wait limit of one microsecond (smm_debug_wait_limit_next): some wait of every
CTA runs out long before its operands or accumulator are ready.  The kernel
must record the expiry in the device status word, stop every role, drain the
copies and MMAs it already issued (teardown waits keep a one-second floor),
free tensor memory and exit.  The host then reads SMM_ERR_DEVICE_TIMEOUT once
(the status word is consumed), and the next product on the same context is
correct.  Nothing here faults, traps or hangs: every wait is bounded and the
expiry is the designed outcome.

Also: the measurement hook smm_debug_time_next brackets exactly the
contraction kernel of one call with the caller's CUDA events."""
import numpy as np
import pytest
import torch

import oracle as O
from cpp1_b200 import _lib, ops
from cpp1_b200 import workloads as W

pytestmark = pytest.mark.gpu


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def test_contraction_wait_expiry_reports_timeout_then_recovers(cuda):
    L = _lib.load()
    n = 2048
    w = W.make_gemm(n, n, n, seed=9)
    A, B = dev(w["A"]), dev(w["B"])
    ops.device_status()  # start from a clean status word
    C = torch.full((n, n), float("nan"), device="cuda")
    assert L.smm_debug_wait_limit_next(1000) == _lib.SMM_OK  # 1 us for the next launch
    ops.gemm(A, B, out=C)
    torch.cuda.synchronize()
    rc = L.smm_device_status(None)
    assert rc == _lib.SMM_ERR_DEVICE_TIMEOUT, (rc, _lib.last_error())
    assert "bounded wait expired" in _lib.last_error()
    assert L.smm_device_status(None) == _lib.SMM_OK  # consumed
    # the context is intact: the same product with the default limit is right
    C2 = ops.gemm(A, B)
    torch.cuda.synchronize()
    ops.device_status()
    r = np.array([0, 1, 777, n - 1], np.int32)
    assert O.relerr(C2.cpu().numpy()[r], O.gemm_rows_f64(w["A"], w["B"], r)) <= 1e-5


def test_wait_limit_hook_rejects_out_of_range(cuda):
    L = _lib.load()
    assert L.smm_debug_wait_limit_next(11 * 10 ** 9) == _lib.SMM_ERR_INVALID
    assert L.smm_debug_wait_limit_next(0) == _lib.SMM_OK


def test_time_next_brackets_the_contraction_kernel(cuda):
    L = _lib.load()
    n = 4096
    w = W.make_upper(n, seed=2)
    U, B = dev(w["U"]), dev(w["B"])
    ops.upper_left(U, B)  # warm
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    e1.record(st)
    torch.cuda.synchronize()
    c0.record(st)
    assert L.smm_debug_time_next(e0.cuda_event, e1.cuda_event) == _lib.SMM_OK
    ops.upper_left(U, B)  # packed U: expansion kernel, then the contraction
    c1.record(st)
    torch.cuda.synchronize()
    kernel_ms, call_ms = e0.elapsed_time(e1), c0.elapsed_time(c1)
    assert 0.0 < kernel_ms < call_ms
