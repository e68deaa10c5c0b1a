"""ctypes binding of libsmm.so (declared in include/smm.h).

There is no fallback: if the library is missing or fails to load, every
operation raises.  The CUDA path is the only path.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# SMM_LIB=debug selects the bounds-checked build (libsmm_debug.so: every
# computed offset into a structured operand is range-checked on the device;
# a violation is skipped and reported as SMM_ERR_BOUNDS by smm_device_status).
LIB_PATH = os.path.join(_HERE, "libsmm_debug.so" if os.environ.get("SMM_LIB") == "debug" else "libsmm.so")

SMM_OK = 0
SMM_ERR_INVALID = 1
SMM_ERR_CUDA = 2
SMM_ERR_NCCL = 3
SMM_ERR_DEVICE_TIMEOUT = 4
SMM_ERR_WORKSPACE = 5
SMM_ERR_UNSUPPORTED = 6
SMM_ERR_BOUNDS = 7

STATUS_NAMES = {
    SMM_OK: "SMM_OK",
    SMM_ERR_INVALID: "SMM_ERR_INVALID",
    SMM_ERR_CUDA: "SMM_ERR_CUDA",
    SMM_ERR_NCCL: "SMM_ERR_NCCL",
    SMM_ERR_DEVICE_TIMEOUT: "SMM_ERR_DEVICE_TIMEOUT",
    SMM_ERR_WORKSPACE: "SMM_ERR_WORKSPACE",
    SMM_ERR_UNSUPPORTED: "SMM_ERR_UNSUPPORTED",
    SMM_ERR_BOUNDS: "SMM_ERR_BOUNDS",
}

MODES = {"3xtf32": 0, "tf32": 1, "bf16": 2}
FMT_PACKED = 0
FMT_DENSE = 1
STRUCTS = {"upper": 0, "lower": 1, "symm": 2, "diag": 3, "toeplitz": 4}


class SmmError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        self.status = status
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}: {message}")


_vp = ctypes.c_void_p
_i = ctypes.c_int
_sz = ctypes.c_size_t
_ull = ctypes.c_ulonglong
_ll = ctypes.c_longlong

# (name, restype, argtypes) for every entry point of include/smm.h.
SIGNATURES = [
    ("smm_last_error", ctypes.c_char_p, []),
    ("smm_version", _i, []),
    ("smm_launch_count", _ull, []),
    ("smm_device_status", _i, [_vp]),
    ("smm_diag_rows", _i, [_vp, _vp, _vp, _i, _i, _vp]),
    ("smm_diag_cols", _i, [_vp, _vp, _vp, _i, _i, _vp]),
    ("smm_diag_rows_host_workspace_size", _sz, [_i, _i]),
    ("smm_diag_rows_host", _i, [_vp, _vp, _vp, _i, _i, _vp, _sz]),
    ("smm_gemm_host_workspace_size", _sz, [_i, _i, _i, _i]),
    ("smm_gemm_host", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz]),
    ("smm_upper_left_host_workspace_size", _sz, [_i, _i, _i]),
    ("smm_upper_left_host", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz]),
    ("smm_symm_left_host_workspace_size", _sz, [_i, _i, _i]),
    ("smm_symm_left_host", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz]),
    ("smm_toeplitz_left_host_workspace_size", _sz, [_i, _i, _i]),
    ("smm_toeplitz_left_host", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz]),
    ("smm_symm_sandwich_host_workspace_size", _sz, [_i, _i]),
    ("smm_symm_sandwich_host", _i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _sz]),
    ("smm_gemm_workspace_size", _sz, [_i, _i, _i, _i]),
    ("smm_upper_left_workspace_size", _sz, [_i, _i, _i, _i]),
    ("smm_toeplitz_left_workspace_size", _sz, [_i, _i, _i]),
    ("smm_symm_sandwich_workspace_size", _sz, [_i, _i]),
    ("smm_symm_left_workspace_size", _sz, [_i, _i, _i]),
    ("smm_gemm", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_upper_left", _i, [_vp, _i, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_toeplitz_left", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_symm_left", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_symm_sandwich", _i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    ("smm_upper_left_rows", _i, [_vp, _i, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_toeplitz_left_rows", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_symm_left_rows", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_gen_x_struct_workspace_size", _sz, [_i, _i, _i]),
    ("smm_gen_x_upper", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_gen_x_symm", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_symm_x_symm", _i, [_vp, _vp, _vp, _i, _i, _vp]),
    ("smm_symm_x_symm_workspace_size", _sz, [_i, _i]),
    ("smm_symm_x_symm_ws", _i, [_vp, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    ("smm_symm_sandwich_noalloc", _i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    ("smm_gen_x_lower", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_lower_left_workspace_size", _sz, [_i, _i, _i]),
    ("smm_lower_left", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_lower_x_lower", _i, [_vp, _vp, _vp, _i, _i, _vp]),
    ("smm_lower_x_lower_workspace_size", _sz, [_i, _i]),
    ("smm_lower_x_lower_ws", _i, [_vp, _vp, _vp, _i, _i, _vp, _sz, _vp]),
    ("smm_add", _i, [_vp, _vp, _vp, _ll, _vp]),
    ("smm_add_struct", _i, [_vp, _vp, _i, _vp, _i, _vp]),
    ("smm_unpack", _i, [_vp, _i, _vp, _i, _vp]),
    ("smm_pack", _i, [_vp, _i, _vp, _i, _vp]),
    ("smm_toeplitz_compact", _i, [_vp, _vp, _i, _i, _vp]),
    ("smm_compat_gen_x_gen", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_diag_x_gen", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_gen_x_diag", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_upper_x_gen", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_toeplitz_x_gen", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_symm_x_gen", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_gen_x_symm", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_gen_x_upper", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_symm_x_symm", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_gen_x_lower", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_lower_x_gen", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_lower_x_lower", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_add_gen_symm", _i, [_vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_compat_symm_sandwich", _i, [_vp, _vp, _vp, _vp, _vp, _i, _vp]),
    ("smm_debug_timeout_probe", _i, [_ull, _vp]),
    ("smm_debug_trace_next", _i, [_vp]),
    ("smm_debug_time_next", _i, [_vp, _vp]),
    ("smm_mg_unique_id", _i, [_vp]),
    ("smm_mg_comm_init", _i, [_vp, _i, _i, _vp]),
    ("smm_mg_comm_destroy", _i, [_vp]),
    ("smm_mg_comm_abort", _i, [_vp]),
    ("smm_mg_comm_status", _i, [_vp]),
    ("smm_mg_row_slabs", _i, [_i, _i, _i, _vp]),
    ("smm_mg_chunks", _i, [_i, _i, _vp]),
    ("smm_mg_gather_chunks", _i, [_i, _i, _vp]),
    ("smm_mg_share_rows", _i, [_i, _i]),
    ("smm_mg_plane_bytes", _sz, [_vp, _i, _i, _i]),
    ("smm_mg_enable_copy_engines", _i, [_vp, _sz]),
    ("smm_mg_copy_engines_enabled", _i, [_vp]),
    ("smm_mg_gemm_workspace_size", _sz, [_vp, _i, _i, _i, _i]),
    ("smm_mg_gemm", _i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_mg_upper_left_workspace_size", _sz, [_vp, _i, _i, _i, _i]),
    ("smm_mg_upper_left", _i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_mg_upper_row_tiles", _i, [_i, _i, _i, _vp, _i, _vp]),
    ("smm_mg_upper_left_tiles_workspace_size", _sz, [_vp, _i, _i, _i, _i]),
    ("smm_mg_upper_left_tiles", _i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_mg_toeplitz_left_workspace_size", _sz, [_vp, _i, _i, _i]),
    ("smm_mg_toeplitz_left", _i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_mg_symm_sandwich_workspace_size", _sz, [_vp, _i, _i, _i]),
    ("smm_mg_symm_sandwich", _i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_debug_wait_limit_next", _i, [_ull]),
    ("smm_gen_x_toeplitz_workspace_size", _sz, [_i, _i, _i, _i]),
    ("smm_gen_x_toeplitz", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz, _vp]),
    ("smm_gen_x_upper_host_workspace_size", _sz, [_i, _i, _i]),
    ("smm_gen_x_upper_host", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz]),
    ("smm_gen_x_symm_host_workspace_size", _sz, [_i, _i, _i]),
    ("smm_gen_x_symm_host", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _sz]),
    ("smm_gen_x_toeplitz_host_workspace_size", _sz, [_i, _i, _i, _i]),
    ("smm_gen_x_toeplitz_host", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _sz]),
    ("smm_diag_cols_host_workspace_size", _sz, [_i, _i]),
    ("smm_diag_cols_host", _i, [_vp, _vp, _vp, _i, _i, _vp, _sz]),
]

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libsmm.so (building nothing); raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m cpp1_b200.build` "
                    "(there is no CPU fallback)")
            try:  # share the CUDA runtime PyTorch already loaded, if any
                import torch  # noqa: F401
            except Exception:
                pass
            L = ctypes.CDLL(LIB_PATH)
            for name, res, args in SIGNATURES:
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    msg = load().smm_last_error()
    return msg.decode() if msg else ""


def check(status: int, where: str) -> None:
    if status != SMM_OK:
        raise SmmError(status, where, last_error())
