"""Tensor-level API over libsmm: each function takes torch CUDA tensors
(row-major fp32, contiguous), calls one C ABI entry point on the current
stream, and returns the output tensor.

Storage conventions follow the reference DSL (src/dsl/layout_functions.py):
packed upper / symmetric operands are the row-major upper triangle
(``torch.triu_indices`` order), diagonals are length-N vectors and Toeplitz
matrices are their 2N-1 generator with ``T[i][j] = g[(N-1) + (j-i)]``.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_ws_cache = {}


def _stream_ptr(stream: Optional[torch.cuda.Stream]) -> Optional[int]:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _check_f32(name: str, t: torch.Tensor, numel: Optional[int] = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_contiguous():
        t = t.contiguous()
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name} has {t.numel()} elements, expected {numel}")
    return t


def _mode(mode: str) -> int:
    try:
        return _lib.MODES[mode]
    except KeyError:
        raise ValueError(f"unknown mode {mode!r}; expected one of {sorted(_lib.MODES)}") from None


def workspace(nbytes: int, device: torch.device) -> Optional[torch.Tensor]:
    """A cached device buffer of at least nbytes (grown on demand)."""
    if nbytes <= 0:
        return None
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def _ws_args(nbytes: int, device: torch.device):
    buf = workspace(nbytes, device)
    return (buf.data_ptr(), buf.numel()) if buf is not None else (None, 0)


def _out(out: Optional[torch.Tensor], shape, like: torch.Tensor) -> torch.Tensor:
    if out is None:
        return torch.empty(shape, dtype=torch.float32, device=like.device)
    out = _check_f32("out", out)
    if tuple(out.shape) != tuple(shape) and out.numel() != int(torch.tensor(shape).prod()):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {tuple(shape)}")
    return out


def diag_rows(d: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """C = diag(d) @ B (row scale), bit-exact single fp32 multiply."""
    B = _check_f32("B", B)
    M, N = B.shape
    d = _check_f32("d", d, M)
    C = _out(out, (M, N), B)
    _lib.check(_lib.load().smm_diag_rows(_ptr(d), _ptr(B), _ptr(C), M, N, _stream_ptr(stream)), "smm_diag_rows")
    return C


def diag_cols(A: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """C = A @ diag(b) (column scale)."""
    A = _check_f32("A", A)
    M, N = A.shape
    b = _check_f32("b", b, N)
    C = _out(out, (M, N), A)
    _lib.check(_lib.load().smm_diag_cols(_ptr(A), _ptr(b), _ptr(C), M, N, _stream_ptr(stream)), "smm_diag_cols")
    return C


def gemm(A: torch.Tensor, B: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
         stream=None) -> torch.Tensor:
    """C = A @ B."""
    A = _check_f32("A", A)
    B = _check_f32("B", B)
    M, K = A.shape
    K2, N = B.shape
    if K != K2:
        raise ValueError(f"inner dimensions differ: {K} vs {K2}")
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_gemm_workspace_size(M, N, K, m), A.device)
    C = _out(out, (M, N), A)
    _lib.check(L.smm_gemm(_ptr(A), _ptr(B), _ptr(C), M, N, K, m, ws, wsb, _stream_ptr(stream)), "smm_gemm")
    return C


def upper_left(U: torch.Tensor, B: torch.Tensor, packed: bool = True, mode: str = "3xtf32",
               out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """C = U @ B with U upper triangular, packed (N(N+1)/2) or dense N x N
    with exact zeros below the diagonal."""
    B = _check_f32("B", B)
    N, ncols = B.shape
    U = _check_f32("U", U, N * (N + 1) // 2 if packed else N * N)
    fmt = _lib.FMT_PACKED if packed else _lib.FMT_DENSE
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_upper_left_workspace_size(N, ncols, fmt, m), B.device)
    C = _out(out, (N, ncols), B)
    _lib.check(L.smm_upper_left(_ptr(U), fmt, _ptr(B), _ptr(C), N, ncols, m, ws, wsb, _stream_ptr(stream)),
               "smm_upper_left")
    return C


def toeplitz_left(g: torch.Tensor, B: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
                  stream=None) -> torch.Tensor:
    """C = T @ B, T the Toeplitz matrix of generator g (2N-1)."""
    B = _check_f32("B", B)
    N, ncols = B.shape
    g = _check_f32("g", g, 2 * N - 1)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_toeplitz_left_workspace_size(N, ncols, m), B.device)
    C = _out(out, (N, ncols), B)
    _lib.check(L.smm_toeplitz_left(_ptr(g), _ptr(B), _ptr(C), N, ncols, m, ws, wsb, _stream_ptr(stream)),
               "smm_toeplitz_left")
    return C


def symm_left(S: torch.Tensor, B: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
              stream=None) -> torch.Tensor:
    """C = S @ B, S symmetric given packed upper."""
    B = _check_f32("B", B)
    N, ncols = B.shape
    S = _check_f32("S", S, N * (N + 1) // 2)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_symm_left_workspace_size(N, ncols, m), B.device)
    C = _out(out, (N, ncols), B)
    _lib.check(L.smm_symm_left(_ptr(S), _ptr(B), _ptr(C), N, ncols, m, ws, wsb, _stream_ptr(stream)),
               "smm_symm_left")
    return C


def symm_sandwich(A: torch.Tensor, S: torch.Tensor, B: torch.Tensor, mode: str = "3xtf32",
                  out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """C = A @ S @ B, S symmetric given packed upper, all N x N."""
    A = _check_f32("A", A)
    N = A.shape[0]
    if tuple(A.shape) != (N, N):
        raise ValueError("A must be square")
    B = _check_f32("B", B, N * N)
    S = _check_f32("S", S, N * (N + 1) // 2)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_symm_sandwich_workspace_size(N, m), A.device)
    C = _out(out, (N, N), A)
    _lib.check(L.smm_symm_sandwich(_ptr(A), _ptr(S), _ptr(B), _ptr(C), N, m, ws, wsb, _stream_ptr(stream)),
               "smm_symm_sandwich")
    return C


def _gen_x_struct(entry: str, A: torch.Tensor, X: torch.Tensor, mode: str, out, stream) -> torch.Tensor:
    A = _check_f32("A", A)
    M, N = A.shape
    X = _check_f32("packed operand", X, N * (N + 1) // 2)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_gen_x_struct_workspace_size(M, N, m), A.device)
    C = _out(out, (M, N), A)
    _lib.check(getattr(L, entry)(_ptr(A), _ptr(X), _ptr(C), M, N, m, ws, wsb, _stream_ptr(stream)), entry)
    return C


def gen_x_upper(A: torch.Tensor, U: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
                stream=None) -> torch.Tensor:
    """C = A @ U, U upper triangular given packed (right side)."""
    return _gen_x_struct("smm_gen_x_upper", A, U, mode, out, stream)


def gen_x_symm(A: torch.Tensor, S: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
               stream=None) -> torch.Tensor:
    """C = A @ S, S symmetric given packed upper (right side)."""
    return _gen_x_struct("smm_gen_x_symm", A, S, mode, out, stream)


def gen_x_lower(A: torch.Tensor, Lp: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
                stream=None) -> torch.Tensor:
    """C = A @ L with L lower triangular given packed lower (i(i+1)/2 + j)."""
    return _gen_x_struct("smm_gen_x_lower", A, Lp, mode, out, stream)


def gen_x_toeplitz(A: torch.Tensor, g: torch.Tensor, N: Optional[int] = None, mode: str = "3xtf32",
                   out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """C = A @ T with T (K x N) the Toeplitz matrix of generator g (K + N - 1),
    T[k][n] = g[(K-1) + (n-k)]; N defaults to K (square T, 2K - 1 generator)."""
    A = _check_f32("A", A)
    M, K = A.shape
    N = K if N is None else N
    g = _check_f32("g", g, K + N - 1)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_gen_x_toeplitz_workspace_size(M, N, K, m), A.device)
    C = _out(out, (M, N), A)
    _lib.check(L.smm_gen_x_toeplitz(_ptr(A), _ptr(g), _ptr(C), M, N, K, m, ws, wsb, _stream_ptr(stream)),
               "smm_gen_x_toeplitz")
    return C


def _packed_order(name: str, t: torch.Tensor) -> int:
    p = t.numel()
    N = int((-1 + (1 + 8 * p) ** 0.5) // 2)
    if N * (N + 1) // 2 != p:
        raise ValueError(f"{name} has {p} elements, not a packed triangle")
    return N


def lower_left(Lp: torch.Tensor, B: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
               stream=None) -> torch.Tensor:
    """C = L @ B with L lower triangular given packed lower."""
    B = _check_f32("B", B)
    N, ncols = B.shape
    Lp = _check_f32("L", Lp, N * (N + 1) // 2)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_lower_left_workspace_size(N, ncols, m), B.device)
    C = _out(out, (N, ncols), B)
    _lib.check(L.smm_lower_left(_ptr(Lp), _ptr(B), _ptr(C), N, ncols, m, ws, wsb, _stream_ptr(stream)),
               "smm_lower_left")
    return C


def lower_x_lower(L1: torch.Tensor, L2: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
                  stream=None) -> torch.Tensor:
    """C = L1 @ L2, both lower triangular given packed lower."""
    L1 = _check_f32("L1", L1)
    N = _packed_order("L1", L1)
    L2 = _check_f32("L2", L2, L1.numel())
    C = _out(out, (N, N), L1)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_lower_x_lower_workspace_size(N, m), L1.device)
    _lib.check(L.smm_lower_x_lower_ws(_ptr(L1), _ptr(L2), _ptr(C), N, m, ws, wsb, _stream_ptr(stream)),
               "smm_lower_x_lower")
    return C


def symm_x_symm(S1: torch.Tensor, S2: torch.Tensor, mode: str = "3xtf32", out: Optional[torch.Tensor] = None,
                stream=None) -> torch.Tensor:
    """C = S1 @ S2, both symmetric given packed upper."""
    S1 = _check_f32("S1", S1)
    p = S1.numel()
    N = int((-1 + (1 + 8 * p) ** 0.5) // 2)
    if N * (N + 1) // 2 != p:
        raise ValueError(f"S1 has {p} elements, not a packed triangle")
    S2 = _check_f32("S2", S2, p)
    C = _out(out, (N, N), S1)
    m = _mode(mode)
    L = _lib.load()
    ws, wsb = _ws_args(L.smm_symm_x_symm_workspace_size(N, m), S1.device)
    _lib.check(L.smm_symm_x_symm_ws(_ptr(S1), _ptr(S2), _ptr(C), N, m, ws, wsb, _stream_ptr(stream)),
               "smm_symm_x_symm")
    return C


# ---------------------------------------------------------------- elementwise / converters
def _struct(fmt: str) -> int:
    try:
        return _lib.STRUCTS[fmt]
    except KeyError:
        raise ValueError(f"unknown structure {fmt!r}; expected one of {sorted(_lib.STRUCTS)}") from None


def struct_numel(fmt: str, N: int) -> int:
    """Storage size of an order-N structured matrix."""
    _struct(fmt)
    return {"upper": N * (N + 1) // 2, "lower": N * (N + 1) // 2, "symm": N * (N + 1) // 2, "diag": N,
            "toeplitz": max(2 * N - 1, 0)}[fmt]


def add(A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """C = A + B elementwise over the storage of two operands of the same
    structure (flat, any shape with equal element counts)."""
    A = _check_f32("A", A)
    B = _check_f32("B", B, A.numel())
    C = _out(out, tuple(A.shape), A)
    _lib.check(_lib.load().smm_add(_ptr(A), _ptr(B), _ptr(C), A.numel(), _stream_ptr(stream)), "smm_add")
    return C


def add_struct(A: torch.Tensor, S: torch.Tensor, fmt: str, out: Optional[torch.Tensor] = None,
               stream=None) -> torch.Tensor:
    """C = A + S with A dense N x N and S structured (fmt: upper, lower, symm,
    diag, toeplitz) in its packed storage."""
    A = _check_f32("A", A)
    N = int(round(A.numel() ** 0.5))
    if N * N != A.numel():
        raise ValueError(f"A has {A.numel()} elements, not a square matrix")
    S = _check_f32("S", S, struct_numel(fmt, N))
    C = _out(out, (N, N), A)
    _lib.check(_lib.load().smm_add_struct(_ptr(A), _ptr(S), _struct(fmt), _ptr(C), N, _stream_ptr(stream)),
               "smm_add_struct")
    return C


def unpack(S: torch.Tensor, fmt: str, N: int, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Dense N x N matrix of the structured storage S."""
    S = _check_f32("S", S, struct_numel(fmt, N))
    D = _out(out, (N, N), S)
    _lib.check(_lib.load().smm_unpack(_ptr(S), _struct(fmt), _ptr(D), N, _stream_ptr(stream)), "smm_unpack")
    return D


def pack(D: torch.Tensor, fmt: str, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Packed upper (fmt upper or symm) or lower triangle of the dense square D."""
    D = _check_f32("D", D)
    N = int(round(D.numel() ** 0.5))
    if N * N != D.numel():
        raise ValueError(f"D has {D.numel()} elements, not a square matrix")
    P = _out(out, (N * (N + 1) // 2,), D)
    _lib.check(_lib.load().smm_pack(_ptr(D), _struct(fmt), _ptr(P), N, _stream_ptr(stream)), "smm_pack")
    return P


def toeplitz_compact(T: torch.Tensor, out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Generator (rows + cols - 1) of the Toeplitz matrix T (2-D)."""
    if T.dim() != 2:
        raise ValueError("T must be 2-D")
    T = _check_f32("T", T)
    rows, cols = T.shape
    g = _out(out, (max(rows + cols - 1, 0),), T)
    _lib.check(_lib.load().smm_toeplitz_compact(_ptr(T), _ptr(g), rows, cols, _stream_ptr(stream)),
               "smm_toeplitz_compact")
    return g


def device_status(stream=None) -> None:
    """Raise SmmError(SMM_ERR_DEVICE_TIMEOUT) if a kernel gave up a bounded wait."""
    _lib.check(_lib.load().smm_device_status(_stream_ptr(stream)), "smm_device_status")


def launch_count() -> int:
    return int(_lib.load().smm_launch_count())


# ---------------------------------------------------------------- host buffers
def _check_host(name: str, t: torch.Tensor, numel: Optional[int] = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.is_cuda:
        raise ValueError(f"{name} must be a host (CPU) tensor")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_contiguous():
        t = t.contiguous()
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name} has {t.numel()} elements, expected {numel}")
    return t


def host_product(op: str, *inputs: torch.Tensor, mode: str = "3xtf32",
                 out: Optional[torch.Tensor] = None, toeplitz_cols: Optional[int] = None) -> torch.Tensor:
    """C = the product ``op`` of HOST tensors through the smm_*_host entry
    points: the left operand(s) cross PCIe once, B streams through in column
    chunks whose copies overlap the products (pinned tensors overlap; pageable
    ones work synchronously).  Synchronous; C is a host tensor (pinned unless
    ``out`` is given).

    op: "gemm" (A, B), "upper" (U_packed, B), "symm" (S_packed, B),
    "toeplitz" (g, B), "sandwich" (A, S_packed, B); the right-side
    orientation of the reference's CPU drivers: "gen_x_upper" (A, U_packed),
    "gen_x_symm" (A, S_packed), "gen_x_toeplitz" (A, g; T square unless
    ``toeplitz_cols`` is given), "diag_cols" (A, b)."""
    arity = {"gemm": 2, "upper": 2, "symm": 2, "toeplitz": 2, "sandwich": 3, "gen_x_upper": 2, "gen_x_symm": 2,
             "gen_x_toeplitz": 2, "diag_cols": 2}
    if op not in arity:
        raise ValueError(f"unknown host product {op!r}; expected one of {sorted(arity)}")
    if len(inputs) != arity[op]:
        raise ValueError(f"host product {op!r} takes {arity[op]} inputs, got {len(inputs)}")
    m = _mode(mode)
    L = _lib.load()
    if op == "gemm":
        A, B = _check_host("A", inputs[0]), _check_host("B", inputs[1])
        (M, K), (K2, N) = A.shape, B.shape
        if K != K2:
            raise ValueError(f"inner dimensions differ: {K} vs {K2}")
        shape = (M, N)
        size = L.smm_gemm_host_workspace_size(M, N, K, m)
        call = lambda C, ws, wsb: L.smm_gemm_host(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, m, ws, wsb)
    elif op in ("upper", "symm", "toeplitz"):
        B = _check_host("B", inputs[1])
        N, ncols = B.shape
        X = _check_host("left operand", inputs[0], 2 * N - 1 if op == "toeplitz" else N * (N + 1) // 2)
        shape = (N, ncols)
        size = getattr(L, f"smm_{op}_left_host_workspace_size")(N, ncols, m)
        fn = getattr(L, f"smm_{op}_left_host")
        call = lambda C, ws, wsb: fn(X.data_ptr(), B.data_ptr(), C.data_ptr(), N, ncols, m, ws, wsb)
    elif op == "sandwich":
        A = _check_host("A", inputs[0])
        N = A.shape[0]
        if tuple(A.shape) != (N, N):
            raise ValueError("A must be square")
        S = _check_host("S", inputs[1], N * (N + 1) // 2)
        B = _check_host("B", inputs[2], N * N)
        shape = (N, N)
        size = L.smm_symm_sandwich_host_workspace_size(N, m)
        call = lambda C, ws, wsb: L.smm_symm_sandwich_host(A.data_ptr(), S.data_ptr(), B.data_ptr(), C.data_ptr(),
                                                           N, m, ws, wsb)
    elif op in ("gen_x_upper", "gen_x_symm"):
        A = _check_host("A", inputs[0])
        M, N = A.shape
        X = _check_host("right operand", inputs[1], N * (N + 1) // 2)
        shape = (M, N)
        size = getattr(L, f"smm_{op}_host_workspace_size")(M, N, m)
        fn = getattr(L, f"smm_{op}_host")
        call = lambda C, ws, wsb: fn(A.data_ptr(), X.data_ptr(), C.data_ptr(), M, N, m, ws, wsb)
    elif op == "gen_x_toeplitz":
        A = _check_host("A", inputs[0])
        M, K = A.shape
        N = K if toeplitz_cols is None else toeplitz_cols
        g = _check_host("g", inputs[1], K + N - 1)
        shape = (M, N)
        size = L.smm_gen_x_toeplitz_host_workspace_size(M, N, K, m)
        call = lambda C, ws, wsb: L.smm_gen_x_toeplitz_host(A.data_ptr(), g.data_ptr(), C.data_ptr(), M, N, K, m,
                                                            ws, wsb)
    elif op == "diag_cols":
        A = _check_host("A", inputs[0])
        M, N = A.shape
        b = _check_host("b", inputs[1], N)
        shape = (M, N)
        size = L.smm_diag_cols_host_workspace_size(M, N)
        call = lambda C, ws, wsb: L.smm_diag_cols_host(A.data_ptr(), b.data_ptr(), C.data_ptr(), M, N, ws, wsb)
    if out is None:
        C = torch.empty(shape, dtype=torch.float32, pin_memory=True)
    else:
        C = _check_host("out", out, shape[0] * shape[1])
    ws, wsb = _ws_args(size, torch.device("cuda", torch.cuda.current_device()))
    # the entry points run on internal streams: finish work that may still
    # use the shared workspace
    torch.cuda.current_stream().synchronize()
    _lib.check(call(C, ws, wsb), f"host product {op}")
    return C
