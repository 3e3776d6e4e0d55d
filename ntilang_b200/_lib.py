"""ctypes binding of libntl_kernels.so (the C ABI in ``include/ntl_kernels.h``).

The library is loaded once per process.  There is no fallback: if the shared library is
missing or fails to load, every launch raises ``RuntimeError`` naming the problem.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB

_lock = threading.Lock()
_handle = None

c_f32p = ctypes.c_void_p
c_i64 = ctypes.c_int64

# name -> (restype, argtypes); must match include/ntl_kernels.h
SIGNATURES = {
    "ntl_version": (ctypes.c_int, []),
    "ntl_last_error": (ctypes.c_char_p, []),
    "ntl_vadd_f32": (ctypes.c_int, [c_f32p, c_f32p, c_f32p, c_i64, ctypes.c_void_p]),
    "ntl_binary_f32": (ctypes.c_int, [ctypes.c_int, c_f32p, c_f32p, c_f32p, c_i64, ctypes.c_void_p]),
    "ntl_cumsum_f32": (ctypes.c_int, [c_f32p, c_f32p, c_i64, c_i64, ctypes.c_int, ctypes.c_void_p]),
    "ntl_cummax_f32": (ctypes.c_int, [c_f32p, c_f32p, c_i64, c_i64, ctypes.c_int, ctypes.c_void_p]),
    "ntl_softmax_f32": (ctypes.c_int, [c_f32p, c_f32p, c_i64, c_i64, ctypes.c_void_p]),
    "ntl_rmsnorm_f32": (ctypes.c_int, [c_f32p, c_f32p, c_f32p, c_i64, c_i64, ctypes.c_float, ctypes.c_float,
                                       ctypes.c_void_p]),
    "ntl_layernorm_f32": (ctypes.c_int, [c_f32p, c_f32p, c_f32p, c_f32p, c_i64, c_i64, ctypes.c_float,
                                         ctypes.c_float, ctypes.c_void_p]),
    "ntl_transpose_f32": (ctypes.c_int, [c_f32p, c_f32p, c_i64, c_i64, ctypes.c_void_p]),
    "ntl_gemm_f16_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, c_f32p, c_f32p, ctypes.c_int,
                                        ctypes.c_float, ctypes.c_int, c_i64, c_i64, c_i64, ctypes.c_int,
                                        ctypes.c_void_p]),
    "ntl_gemm_workspace_size": (ctypes.c_int, [c_i64, c_i64, c_i64, ctypes.c_int, ctypes.POINTER(ctypes.c_uint64)]),
    "ntl_gemm_f16_f32_ws": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, c_f32p, c_f32p, ctypes.c_int,
                                           ctypes.c_float, ctypes.c_int, c_i64, c_i64, c_i64, ctypes.c_int,
                                           ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]),
    "ntl_gemm_f16_f32_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, c_f32p, c_f32p, ctypes.c_int,
                                                ctypes.c_float, ctypes.c_int, c_i64, c_i64, c_i64, ctypes.c_int,
                                                ctypes.c_void_p]),
    "ntl_fa2_fwd_f16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, c_i64,
                                       c_i64, c_i64, c_i64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]),
    "ntl_rtc_build": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
    "ntl_rtc_launch": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint32,
                                      ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "ntl_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "ntl_clear_device_status": (ctypes.c_int, []),
    "ntl_set_wait_limit": (ctypes.c_int, [c_i64]),
    "ntl_fa2_set_causal_grid": (ctypes.c_int, [ctypes.c_int]),
    "ntl_launch_count": (ctypes.c_int64, []),
}


def library_path() -> Path:
    return LIB


def lib():
    """The loaded library (loads it on first use)."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            if not LIB.exists():
                raise RuntimeError(
                    f"{LIB} is missing: build it with `python -m ntilang_b200.build` "
                    "(the sm_100a kernels have no CPU fallback)"
                )
            handle = ctypes.CDLL(str(LIB))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _handle = handle
    return _handle


class KernelError(RuntimeError):
    def __init__(self, name, code, message):
        self.code = code
        super().__init__(f"{name} failed with code {code}: {message}")


def call(name, *args):
    """Call a C-ABI entry point; a non-zero return raises ``KernelError``."""
    handle = lib()
    rc = getattr(handle, name)(*args)
    if rc != 0:
        msg = handle.ntl_last_error()
        raise KernelError(name, rc, msg.decode() if msg else "")
    return rc


def device_status() -> int:
    value = ctypes.c_uint32(0)
    call("ntl_device_status", ctypes.byref(value))
    return int(value.value)


def clear_device_status() -> None:
    call("ntl_clear_device_status")


def set_wait_limit(polls: int) -> None:
    call("ntl_set_wait_limit", int(polls))


FA2_GRID_AUTO, FA2_GRID_PERSISTENT, FA2_GRID_PER_BLOCK = 0, 1, 2


def set_fa2_causal_grid(mode: int) -> None:
    """Grid of later causal attention launches: FA2_GRID_AUTO (default), _PERSISTENT or _PER_BLOCK."""
    call("ntl_fa2_set_causal_grid", int(mode))


def gemm_workspace_size(M, N, K, b_trans) -> int:
    out = ctypes.c_uint64(0)
    call("ntl_gemm_workspace_size", int(M), int(N), int(K), int(b_trans), ctypes.byref(out))
    return int(out.value)


def launch_count() -> int:
    return int(lib().ntl_launch_count())


__all__ = ["KernelError", "SIGNATURES", "call", "clear_device_status", "device_status", "gemm_workspace_size",
           "launch_count", "lib",
           "library_path", "set_wait_limit"]
