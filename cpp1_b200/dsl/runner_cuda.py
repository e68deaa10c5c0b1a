"""CUDA backend of the DSL: same entry points and return values as the
reference's src/dsl/runner_cuda.py —

    run(outs, inputs, backend="cuda", out_matrix_obj=None,
        bm=None, bn=None, bk=None, pipeline=None, swizzle_n=None, num_threads=None)
        -> ({out_name: flat output tensor}, time_ms, gflops)
    run_graph(outs, inputs, backend="cuda", **kwargs)
        -> ({op_name: tensor for every operation}, total time_ms, 0.0)

— but instead of generating CUDA source, compiling it with nvcc and loading
the result (src/dsl/runner_cuda.py:47-74, once per call), each matmul is
lowered by the (left type, right type) pair to one call of the prebuilt
libsmm C ABI.  The tiling knobs (bm ... num_threads) are accepted and
ignored: tile shapes are chosen by the library per structure and size.  One
extra keyword, ``mode`` ("3xtf32" default, "tf32", "bf16"), selects the
arithmetic of the tensor-core contractions.

Conventions kept from the reference:
* inputs are torch tensors (moved to the GPU and flattened like the
  reference does; numpy arrays are accepted too) keyed by matrix name, and
  symbolic dimensions by the Var's name (lower-case lookup first);
* the output is allocated as a flat float32 tensor of the packed size of its
  class (n(n+1)/2 symmetric/triangular, n diagonal, rows*cols otherwise);
* time_ms is the device time of the call (CUDA events), gflops counts 2*M*N*K
  (M*N for a diagonal scale), as the reference wrappers report.

A graph of the form A @ S @ B (S symmetric) is executed by the sandwich
entry point in one call instead of two.  `+` of two operands lowers to
smm_add (same class, over the storage) or smm_add_struct (general plus a
structured operand, expanded on the fly).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from .matrix import (DiagonalMatrix, GeneralMatrix, LowerTriangularMatrix, Matrix, SymmetricMatrix, ToeplitzMatrix,
                     UpperTriangularMatrix)
from .operations import Operation
from .utils import get_graph_io
from .var import Var


def get_shape(shape_tuple, inputs):
    """Concrete shape: Vars are looked up in ``inputs`` by lower-case name, then exact name."""
    real = []
    for dim in shape_tuple:
        if isinstance(dim, Var):
            val = inputs.get(str(dim.name).lower(), inputs.get(dim.name))
            if val is None:
                raise KeyError(f"no value for dimension {dim.name!r} in inputs")
            real.append(int(val))
        elif isinstance(dim, int):
            real.append(dim)
    return tuple(real)


def _storage_size(obj, shape) -> int:
    if isinstance(obj, (SymmetricMatrix, UpperTriangularMatrix, LowerTriangularMatrix)):
        return shape[0] * (shape[0] + 1) // 2
    if isinstance(obj, DiagonalMatrix):
        return shape[0]
    if isinstance(obj, ToeplitzMatrix):
        return 2 * shape[0] - 1
    return int(np.prod(shape))


def _device_tensor(val) -> torch.Tensor:
    if isinstance(val, np.ndarray):
        val = torch.from_numpy(np.ascontiguousarray(val, dtype=np.float32))
    if not torch.is_tensor(val):
        raise TypeError(f"inputs must be torch tensors or numpy arrays, got {type(val).__name__}")
    if not val.is_cuda:
        val = val.cuda()
    if val.dtype != torch.float32:
        val = val.float()
    return val.contiguous().view(-1)


def _kind(m: Matrix) -> str:
    # Exact class, as the reference codegen dispatches on type(lhs), type(rhs).
    for cls, k in ((GeneralMatrix, "gen"), (DiagonalMatrix, "diag"), (UpperTriangularMatrix, "upper"),
                   (SymmetricMatrix, "symm"), (ToeplitzMatrix, "toeplitz"), (LowerTriangularMatrix, "lower")):
        if type(m) is cls:
            return k
    if isinstance(m, Operation):
        return "gen"
    return type(m).__name__


# (left kind, right kind) -> callable(lhs, rhs, M, N, K, mode, out) and the
# reference's flop convention for gflops_out.
def _lower(lk: str, rk: str):
    if (lk, rk) == ("gen", "gen"):
        return (lambda a, b, M, N, K, mode, out: ops.gemm(a.view(M, K), b.view(K, N), mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("diag", "gen"):
        return (lambda d, b, M, N, K, mode, out: ops.diag_rows(d, b.view(K, N), out=out),
                lambda M, N, K: 1.0 * M * N)
    if (lk, rk) == ("gen", "diag"):
        return (lambda a, d, M, N, K, mode, out: ops.diag_cols(a.view(M, K), d, out=out),
                lambda M, N, K: 1.0 * M * N)
    if (lk, rk) == ("upper", "gen"):
        return (lambda u, b, M, N, K, mode, out: ops.upper_left(u, b.view(K, N), packed=True, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("toeplitz", "gen"):
        return (lambda g, b, M, N, K, mode, out: ops.toeplitz_left(g, b.view(K, N), mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("symm", "gen"):
        return (lambda s, b, M, N, K, mode, out: ops.symm_left(s, b.view(K, N), mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("gen", "symm"):
        return (lambda a, s, M, N, K, mode, out: ops.gen_x_symm(a.view(M, K), s, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("gen", "upper"):
        return (lambda a, u, M, N, K, mode, out: ops.gen_x_upper(a.view(M, K), u, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("gen", "toeplitz"):
        # the reference's own Toeplitz orientation (Cuda kernels/toeplitz.cu:76-253),
        # which its DSL CUDA backend does not lower (codegen_cuda.py:1681-1682)
        return (lambda a, g, M, N, K, mode, out: ops.gen_x_toeplitz(a.view(M, K), g, N, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("symm", "symm"):
        return (lambda s1, s2, M, N, K, mode, out: ops.symm_x_symm(s1, s2, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    # Lower-triangular operands: the reference implements Gen @ Lower and
    # Lower @ Lower in its CPU AVX backend only (codegen_multiply_avx.py:546,
    # 644); Lower @ Gen is the left-side counterpart of Upper @ Gen.
    if (lk, rk) == ("gen", "lower"):
        return (lambda a, l, M, N, K, mode, out: ops.gen_x_lower(a.view(M, K), l, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("lower", "gen"):
        return (lambda l, b, M, N, K, mode, out: ops.lower_left(l, b.view(K, N), mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    if (lk, rk) == ("lower", "lower"):
        return (lambda l1, l2, M, N, K, mode, out: ops.lower_x_lower(l1, l2, mode=mode, out=out),
                lambda M, N, K: 2.0 * M * N * K)
    raise NotImplementedError(f"Matmul for {lk} @ {rk} not implemented in the CUDA backend")


def _timed(fn):
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    res = fn()
    end.record()
    end.synchronize()
    ops.device_status()
    return res, start.elapsed_time(end)


def run(outs, inputs, backend="cuda", out_matrix_obj=None, bm=None, bn=None, bk=None, pipeline=None,
        swizzle_n=None, num_threads=None, mode="3xtf32"):
    if not outs:
        return ({}, 0.0, 0.0)
    if backend != "cuda":
        raise ValueError(f"runner_cuda only supports backend='cuda', got {backend!r}")
    node = outs[0]
    target = out_matrix_obj if out_matrix_obj is not None else node
    if isinstance(node, Operation) and node.operator == "add":
        return _run_add(node, target, inputs)
    if not isinstance(node, Operation) or node.operator != "matmul":
        op_name = getattr(node, "operator", type(node).__name__)
        raise NotImplementedError(f"CUDA backend supports matmul and add expressions, got {op_name!r}")
    lhs, rhs = node.operands
    M, K = get_shape(lhs.shape, inputs)
    K2, N = get_shape(rhs.shape, inputs)
    if K != K2:
        raise ValueError(f"Inner dimensions for matrix multiplication must match: {K} vs {K2}.")
    for m in (lhs, rhs):
        if m.name not in inputs:
            raise KeyError(f"input {m.name!r} missing")
    a = _device_tensor(inputs[lhs.name])
    b = _device_tensor(inputs[rhs.name])
    call, flops = _lower(_kind(lhs), _kind(rhs))
    out_shape = get_shape(target.shape, inputs)
    out = torch.zeros(_storage_size(target, out_shape), dtype=torch.float32, device=a.device)
    if _storage_size(target, out_shape) != M * N:
        raise NotImplementedError(f"output class {type(target).__name__} of a matmul must be general (M x N)")
    _, ms = _timed(lambda: call(a, b, M, N, K, mode, out.view(M, N)))
    gflops = flops(M, N, K) * 1e-9 / (ms * 1e-3) if ms > 0 else 0.0
    return {target.name: out}, ms, gflops


_STRUCT_FMT = {"upper": "upper", "lower": "lower", "symm": "symm", "diag": "diag", "toeplitz": "toeplitz"}


def _run_add(node, target, inputs):
    """The DSL's `+` (src/dsl/codegen_cuda.py:1643-1827).  Operands of the
    same class are added over their storage (kernel_add_1d_vec4's role); a
    general operand plus a structured one gives a general result with the
    structured operand expanded on the fly (kernel_add_gen_symm's role, here
    for every structured class and either operand order).  gflops counts one
    operation per stored output element, as the reference wrappers do."""
    lhs, rhs = node.operands
    shape = get_shape(lhs.shape, inputs)
    if get_shape(rhs.shape, inputs) != shape:
        raise ValueError(f"Shapes must match for add operation: {lhs.shape} vs {rhs.shape}")
    for m in (lhs, rhs):
        if m.name not in inputs:
            raise KeyError(f"input {m.name!r} missing")
    a = _device_tensor(inputs[lhs.name])
    b = _device_tensor(inputs[rhs.name])
    lk, rk = _kind(lhs), _kind(rhs)
    out_shape = get_shape(target.shape, inputs)
    out_size = _storage_size(target, out_shape)
    out = torch.zeros(out_size, dtype=torch.float32, device=a.device)
    if lk == rk:
        size = _storage_size(lhs, shape)
        if out_size != size:
            raise NotImplementedError(f"add of two {lk} operands into a {type(target).__name__} output")
        if a.numel() < size or b.numel() < size:
            raise ValueError(f"add operands hold {a.numel()} and {b.numel()} elements, need {size}")
        _, ms = _timed(lambda: ops.add(a[:size], b[:size], out=out))
        work = size
    elif (lk == "gen") != (rk == "gen") and (lk in _STRUCT_FMT or rk in _STRUCT_FMT):
        n = shape[0]
        if shape[1] != n:
            raise ValueError("a structured operand must be square")
        if out_size != n * n:
            raise NotImplementedError(f"general + {lk if lk != 'gen' else rk} gives a general output")
        gen, st, st_obj = (a, b, rhs) if lk == "gen" else (b, a, lhs)
        fmt = _STRUCT_FMT[_kind(st_obj)]
        st_size = _storage_size(st_obj, shape)
        _, ms = _timed(lambda: ops.add_struct(gen[:n * n].view(n, n), st[:st_size], fmt, out=out.view(n, n)))
        work = n * n
    else:
        raise NotImplementedError(f"Addition for {lk} + {rk} is not implemented in the CUDA backend")
    gflops = work * 1e-9 / (ms * 1e-3) if ms > 0 else 0.0
    return {target.name: out}, ms, gflops


def _build_compute_schedule(node, visited, schedule):
    """Post-order list of the Operations under ``node`` (operands first)."""
    if id(node) in visited:
        return
    visited.add(id(node))
    if isinstance(node, Operation):
        for child in node.operands:
            _build_compute_schedule(child, visited, schedule)
        schedule.append(node)


def _sandwich_parts(node):
    """(A, S, B) if node is (A @ S) @ B or A @ (S @ B) with S symmetric and
    A, B general leaves; else None."""
    if not (isinstance(node, Operation) and node.operator == "matmul"):
        return None
    l, r = node.operands
    if isinstance(l, Operation) and l.operator == "matmul" and not isinstance(r, Operation):
        a, s = l.operands
        b = r
    elif isinstance(r, Operation) and r.operator == "matmul" and not isinstance(l, Operation):
        a = l
        s, b = r.operands
    else:
        return None
    if _kind(a) == "gen" and _kind(s) == "symm" and _kind(b) == "gen" and not any(
            isinstance(x, Operation) for x in (a, s, b)):
        return a, s, b
    return None


def run_graph(outs, inputs, backend="cuda", **kwargs):
    """Execute a multi-operation expression, returning every operation's
    tensor under its name, like the reference (src/dsl/runner_cuda.py:147-197).
    A @ S @ B (S symmetric, A and B general) runs as the library's two
    structured products in the expression's own association: (A @ S) @ B as
    Gen@Symm then a GEMM, A @ (S @ B) as Symm@Gen then a GEMM, the symmetric
    operand expanded from its packed storage on the device, the intermediate
    returned under its name too.  Anything else runs operation by operation
    in post-order, each intermediate stored in ``inputs`` under its name."""
    mode = kwargs.get("mode", "3xtf32")
    if len(outs) == 1:
        parts = _sandwich_parts(outs[0])
        if parts is not None:
            a, s, b = parts
            n = get_shape(a.shape, inputs)[0]
            if get_shape(s.shape, inputs) == (n, n) and get_shape(b.shape, inputs) == (n, n):
                A = _device_tensor(inputs[a.name]).view(n, n)
                S = _device_tensor(inputs[s.name])
                B = _device_tensor(inputs[b.name]).view(n, n)
                root = outs[0]
                inner = root.operands[0] if isinstance(root.operands[0], Operation) else root.operands[1]
                mid = torch.zeros(n * n, dtype=torch.float32, device=A.device)
                out = torch.zeros(n * n, dtype=torch.float32, device=A.device)

                def both():
                    if inner is root.operands[0]:  # (A @ S) @ B
                        ops.gen_x_symm(A, S, mode=mode, out=mid.view(n, n))
                        ops.gemm(mid.view(n, n), B, mode=mode, out=out.view(n, n))
                    else:  # A @ (S @ B)
                        ops.symm_left(S, B, mode=mode, out=mid.view(n, n))
                        ops.gemm(A, mid.view(n, n), mode=mode, out=out.view(n, n))
                _, ms = _timed(both)
                return {inner.name: mid, root.name: out}, ms, 0.0

    schedule, visited = [], set()
    for o in outs:
        _build_compute_schedule(o, visited, schedule)
    if not schedule:
        schedule = list(outs)
    current = dict(inputs)
    total_ms, results = 0.0, {}
    for op in schedule:
        saved = list(op.operands)
        op.operands = [GeneralMatrix(c.shape, c.name) if isinstance(c, Operation) else c for c in saved]
        try:
            res, ms, _ = run([op], current, backend=backend, out_matrix_obj=op, **kwargs)
        finally:
            op.operands = saved
        current[op.name] = res[op.name]
        results[op.name] = res[op.name]
        total_ms += ms
    return results, total_ms, 0.0


__all__ = ["get_shape", "run", "run_graph", "get_graph_io"]
