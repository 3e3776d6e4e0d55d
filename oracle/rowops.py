"""ctypes loader for oracle/_build/liboracle_rowops.so — TEST INFRASTRUCTURE ONLY.

``build()`` runs ``make -C oracle``.  Functions take and return NumPy float32 arrays.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle_rowops.so"
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = ctypes.CDLL(str(LIB))
        p, i64 = ctypes.c_void_p, ctypes.c_int64
        h.oracle_threads.restype = ctypes.c_int
        h.oracle_set_threads.argtypes = [ctypes.c_int]
        h.oracle_vadd_f32.argtypes = [p, p, p, i64]
        h.oracle_cumsum_f32.argtypes = [p, p, i64, i64, ctypes.c_int]
        h.oracle_softmax_f32.argtypes = [p, p, i64, i64]
        h.oracle_rmsnorm_f32.argtypes = [p, p, p, i64, i64, ctypes.c_float, ctypes.c_float]
        h.oracle_layernorm_f32.argtypes = [p, p, p, p, i64, i64, ctypes.c_float, ctypes.c_float]
        h.oracle_transpose_f32.argtypes = [p, p, i64, i64]
        _lib = h
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def threads() -> int:
    return int(lib().oracle_threads())


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def vadd(a, b):
    a, b = _f32(a), _f32(b)
    c = np.empty_like(a)
    lib().oracle_vadd_f32(a.ctypes.data, b.ctypes.data, c.ctypes.data, a.size)
    return c


def cumsum(x, reverse=False):
    x = _f32(x)
    y = np.empty_like(x)
    cols = x.shape[-1]
    lib().oracle_cumsum_f32(x.ctypes.data, y.ctypes.data, x.size // cols, cols, int(bool(reverse)))
    return y


def softmax(x):
    x = _f32(x)
    y = np.empty_like(x)
    cols = x.shape[-1]
    lib().oracle_softmax_f32(x.ctypes.data, y.ctypes.data, x.size // cols, cols)
    return y


def rmsnorm(x, w, eps, inv_n=None):
    x, w = _f32(x), _f32(w)
    y = np.empty_like(x)
    cols = x.shape[-1]
    inv_n = 1.0 / cols if inv_n is None else inv_n
    lib().oracle_rmsnorm_f32(x.ctypes.data, w.ctypes.data, y.ctypes.data, x.size // cols, cols, eps, inv_n)
    return y


def layernorm(x, w, b, eps, inv_n=None):
    x, w, b = _f32(x), _f32(w), _f32(b)
    y = np.empty_like(x)
    cols = x.shape[-1]
    inv_n = 1.0 / cols if inv_n is None else inv_n
    lib().oracle_layernorm_f32(x.ctypes.data, w.ctypes.data, b.ctypes.data, y.ctypes.data, x.size // cols, cols, eps,
                               inv_n)
    return y


def transpose(a):
    a = _f32(a)
    m, n = a.shape
    b = np.empty((n, m), dtype=np.float32)
    lib().oracle_transpose_f32(a.ctypes.data, b.ctypes.data, m, n)
    return b
