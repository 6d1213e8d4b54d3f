"""ctypes binding of the C ABI declared in include/b2g.h (the library `cs464_b200/libb2g.so`).

There is no fallback: if the library is missing or fails to load, every GEMM entry point raises. The reference reaches
its vendor comparator the same way (ctypes into libcublasLt, baselines/cublaslt.py:44-55).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from cs464_b200.build import LIB_PATH

B2G_OK = 0
B2G_ERR_INVALID_ARG = -1
B2G_ERR_UNSUPPORTED = -2
B2G_ERR_WORKSPACE = -3
B2G_ERR_CUDA = -4

DTYPE_F16 = 0
DTYPE_BF16 = 1

SCHED_PERSISTENT = 0
SCHED_TILE = 1
SCHED_STREAMK = 2

# every symbol include/b2g.h declares (checked by the CPU tests against the built library)
EXPORTS = (
    "b2g_abi_version", "b2g_version", "b2g_source_hash", "b2g_last_error", "b2g_error_string", "b2g_status_string",
    "b2g_check", "b2g_workspace_size", "b2g_smem_bytes", "b2g_plan_create", "b2g_plan_launch",
    "b2g_plan_num_kernels", "b2g_plan_grid", "b2g_plan_destroy", "b2g_gemm", "b2g_splitk_reduce",
    "b2g_gemm_noalloc", "b2g_host_flag_create", "b2g_host_flag_set", "b2g_host_flag_destroy", "b2g_hold",
    "b2g_forest_predict", "b2g_plan_rebind",
)


class Config(ctypes.Structure):
    _fields_ = [("block_m", ctypes.c_int32), ("block_n", ctypes.c_int32), ("block_k", ctypes.c_int32),
                ("num_warps", ctypes.c_int32), ("num_stages", ctypes.c_int32), ("group_m", ctypes.c_int32),
                ("split_k", ctypes.c_int32), ("schedule", ctypes.c_int32), ("cluster", ctypes.c_int32),
                ("wait_limit_us", ctypes.c_int32), ("reserved", ctypes.c_int32 * 6)]


class Problem(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("stride_am", ctypes.c_int64), ("stride_ak", ctypes.c_int64),
                ("stride_bk", ctypes.c_int64), ("stride_bn", ctypes.c_int64),
                ("stride_cm", ctypes.c_int64), ("stride_cn", ctypes.c_int64),
                ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class B2GError(RuntimeError):
    """A non-OK return from the C ABI. `code` is the B2G_ERR_* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


class Unsupported(B2GError):
    """The config cannot run this shape/layout (B2G_ERR_UNSUPPORTED). Not a CUDA fault: the context is fine."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def _declare(lib: ctypes.CDLL) -> None:
    c_int32, c_size_t, c_void_p, c_char_p = ctypes.c_int32, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p
    P = ctypes.POINTER
    sig = {
        "b2g_abi_version": (c_int32, []),
        "b2g_version": (c_char_p, []),
        "b2g_source_hash": (c_char_p, []),
        "b2g_last_error": (c_char_p, []),
        "b2g_error_string": (c_char_p, [c_int32]),
        "b2g_status_string": (c_char_p, [c_int32]),
        "b2g_check": (c_int32, [P(Config), P(Problem), c_char_p, c_size_t]),
        "b2g_workspace_size": (c_int32, [P(Config), P(Problem), c_void_p, c_void_p, P(c_size_t)]),
        "b2g_smem_bytes": (c_int32, [P(Config), P(Problem), P(c_size_t)]),
        "b2g_plan_create": (c_int32, [P(Config), P(Problem), c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                      c_void_p, P(c_void_p)]),
        "b2g_plan_launch": (c_int32, [c_void_p, c_void_p]),
        "b2g_plan_rebind": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p]),
        "b2g_plan_num_kernels": (c_int32, [c_void_p]),
        "b2g_plan_grid": (c_int32, [c_void_p]),
        "b2g_plan_destroy": (c_int32, [c_void_p]),
        "b2g_gemm": (c_int32, [P(Config), P(Problem), c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p,
                               c_void_p]),
        "b2g_splitk_reduce": (c_int32, [c_void_p, c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, c_int32, c_int32, c_void_p]),
        "b2g_gemm_noalloc": (c_int32, [P(Config), P(Problem), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
        "b2g_host_flag_create": (c_int32, [P(c_void_p), P(c_void_p)]),
        "b2g_host_flag_set": (c_int32, [c_void_p, c_int32]),
        "b2g_host_flag_destroy": (c_int32, [c_void_p]),
        "b2g_hold": (c_int32, [c_void_p, c_int32, ctypes.c_uint64, c_void_p, c_void_p]),
        "b2g_forest_predict": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_int32, ctypes.c_double, c_void_p, ctypes.c_int64, c_int32, c_void_p,
                                         c_int32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """The loaded library (built on first use if this machine has nvcc and the library is missing or stale)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = LIB_PATH
            if not path.exists():
                from cs464_b200.build import build
                build()
            lib = ctypes.CDLL(str(path))
            _declare(lib)
            if lib.b2g_abi_version() != 1:
                raise RuntimeError(f"{path}: ABI version {lib.b2g_abi_version()} != 1")
            _lib = lib
    return _lib


def last_error() -> str:
    return load().b2g_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == B2G_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == B2G_ERR_UNSUPPORTED:
        raise Unsupported(rc, f"unsupported: {last_error()}")
    raise B2GError(rc, msg)


def status_string(code: int) -> str:
    return load().b2g_status_string(int(code)).decode()


def source_hash() -> str:
    return load().b2g_source_hash().decode()
