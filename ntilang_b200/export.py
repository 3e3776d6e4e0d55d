"""``CompiledKernel.save()`` / ``LoweredProgram.emit()``: a standalone launcher module.

The reference exports the generated CuTe DSL module, which runs wherever CuTe runs without
``ntilang`` (python/ntilang/compiler.py:44-49, tests/test_compiler.py:177-188).  Here the
device code is libntl_kernels.so (prebuilt sm_100a kernels plus the NVRTC path), so the
exported module is plain Python over ``ctypes``: it imports nothing from ``ntilang`` /
``ntilang_b200``, finds the library through ``$NTL_KERNELS_LIB`` or the path recorded when it
was saved, and its ``compile_kernel()`` returns a callable (``run(...)`` launches directly) taking the kernel's arguments in
prim_func order (objects with ``data_ptr()`` and ``shape``, e.g. torch CUDA tensors, for
tensors; Python numbers for scalars) plus ``stream=`` (a CUDA stream handle, default the
legacy stream).  It performs no argument checks: it is the launch, not the drop-in wrapper.
"""

from __future__ import annotations

from .launch import abi_calls, describe
from .pointwise import BLOCK_THREADS, POINTS_PER_THREAD

_RUNTIME = r'''
import ctypes
import os

_C = {"i32": ctypes.c_int, "i64": ctypes.c_int64, "f32": ctypes.c_float}


def _library():
    path = os.environ.get("NTL_KERNELS_LIB") or LIBRARY
    if not path or not os.path.exists(path):
        raise RuntimeError("libntl_kernels.so not found: set NTL_KERNELS_LIB")
    return ctypes.CDLL(path)


def _check(lib, rc, what):
    if rc != 0:
        lib.ntl_last_error.restype = ctypes.c_char_p
        raise RuntimeError(f"{what} failed with code {rc}: {lib.ntl_last_error().decode()}")
'''

_ABI_KERNEL = r'''

class _Kernel:
    has_gpu_module = True

    def __init__(self, lib):
        self.lib = lib
        self.calls = []
        for entry, recipe in CALLS:
            fn = getattr(lib, entry)
            fn.restype = ctypes.c_int
            self.calls.append((entry, fn, recipe))

    def __call__(self, *args, stream=0):
        for entry, fn, recipe in self.calls:
            _check(self.lib, fn(*self._values(recipe, args, stream)), entry)

    @staticmethod
    def _values(recipe, args, stream):
        values = []
        for item in recipe:
            kind = item[0]
            if kind == "ptr":
                a = args[item[1]]
                values.append(ctypes.c_void_p(a.data_ptr() if hasattr(a, "data_ptr") else int(a)))
            elif kind == "null":
                values.append(ctypes.c_void_p(0))
            elif kind in _C:
                values.append(_C[kind](item[1]))
            elif kind == "dim":
                values.append(ctypes.c_int64(int(args[item[1]].shape[item[2]])))
            elif kind == "rows":
                shape = tuple(args[item[1]].shape)
                rows = 1
                for d in shape[:-1]:
                    rows *= int(d)
                values.append(ctypes.c_int64(rows))
            else:  # stream
                values.append(ctypes.c_void_p(int(stream)))
        return values


def compile_kernel():
    """Load libntl_kernels.so and return the launch callable."""
    return _Kernel(_library())


_CACHED = []


def run(*args, stream=0):
    """Launch with the kernel's arguments (compile_kernel() on first use)."""
    if not _CACHED:
        _CACHED.append(compile_kernel())
    _CACHED[0](*args, stream=stream)
'''

_RTC_KERNEL = r'''

_SCALAR = {"bool": ctypes.c_bool, "int8": ctypes.c_int8, "int16": ctypes.c_int16, "int32": ctypes.c_int32,
           "int64": ctypes.c_int64, "uint8": ctypes.c_uint8, "uint16": ctypes.c_uint16, "uint32": ctypes.c_uint32,
           "uint64": ctypes.c_uint64, "float16": ctypes.c_float, "bfloat16": ctypes.c_float,
           "float32": ctypes.c_float, "float64": ctypes.c_double}


def _extent(e, sizes):
    if isinstance(e, int):
        return e
    if isinstance(e, str):
        return sizes[e]
    op, a, b = e
    a, b = _extent(a, sizes), _extent(b, sizes)
    return {"+": a + b, "-": a - b, "*": a * b, "//": a // b if b else 0, "%": a % b if b else 0}[op]


class _Kernel:
    has_gpu_module = True

    def __init__(self, lib):
        self.lib = lib
        handle = ctypes.c_uint64(0)
        lib.ntl_rtc_build.restype = ctypes.c_int
        _check(lib, lib.ntl_rtc_build(ctypes.c_char_p(CUDA_SOURCE.encode()), ctypes.c_char_p(KERNEL.encode()),
                                      ctypes.byref(handle)), "ntl_rtc_build")
        self.handle = handle.value
        lib.ntl_rtc_launch.restype = ctypes.c_int

    def __call__(self, *args, stream=0):
        sizes = {}
        for (kind, dtype, syms), a in zip(PARAMS, args):
            for d, s in enumerate(syms):
                if s is not None:
                    sizes[s] = int(a.shape[d])
        keep = []
        for (kind, dtype, syms), a in zip(PARAMS, args):
            if kind == "scalar":
                keep.append(_SCALAR[dtype](a))
            else:
                keep.append(ctypes.c_void_p(a.data_ptr() if hasattr(a, "data_ptr") else int(a)))
        keep += [ctypes.c_int64(sizes[s]) for s in SYMBOLS]
        extents = [_extent(g, sizes) for g in GRID]
        blocks = 1
        for e in extents:
            blocks *= max(e, 0)
        total = blocks * POINTS
        if total == 0:
            return
        keep += [ctypes.c_int64(extents[i]) for i in GRID_ARGS]
        keep.append(ctypes.c_int64(total))
        argv = (ctypes.c_void_p * len(keep))(*[ctypes.cast(ctypes.pointer(k), ctypes.c_void_p) for k in keep])
        grid = (total + BLOCK * UNROLL - 1) // (BLOCK * UNROLL)
        _check(self.lib, self.lib.ntl_rtc_launch(ctypes.c_uint64(self.handle), ctypes.c_uint64(grid),
                                                 ctypes.c_uint32(BLOCK), argv, ctypes.c_void_p(int(stream))),
               "ntl_rtc_launch")


def compile_kernel():
    """Load libntl_kernels.so, compile the CUDA source with NVRTC and return the launch callable."""
    return _Kernel(_library())


_CACHED = []


def run(*args, stream=0):
    """Launch with the kernel's arguments (compile_kernel() on first use)."""
    if not _CACHED:
        _CACHED.append(compile_kernel())
    _CACHED[0](*args, stream=stream)
'''


def _grid_literal(e):
    """A grid extent as a literal the exported module evaluates: int, symbol name or (op, a, b)."""
    from .frontend import Bin, Const, Var

    if isinstance(e, int):
        return e
    if isinstance(e, Const):
        return int(e.value)
    if isinstance(e, Var) and e.name.startswith("$sym:"):
        return e.name[5:]
    if isinstance(e, Bin) and e.op in ("+", "-", "*", "//", "%"):
        return (e.op, _grid_literal(e.a), _grid_literal(e.b))
    raise ValueError(f"grid extent {e!r} cannot be exported")


def standalone_module(spec, prog, name: str, target: str, library: str | None) -> str:
    """Python source of the standalone launcher for one compiled kernel."""
    from .ir import ScalarParameter, SymDim

    plan = describe(spec, name, target)
    head = [
        f'"""Standalone launcher for `{name}` exported by ntilang_b200 (no ntilang import).',
        "",
        "compile_kernel() returns a callable taking the kernel's arguments in prim_func order",
        "(tensors as objects with data_ptr() and shape, scalars as Python numbers) and stream=.",
        '"""',
        "",
        plan.rstrip("\n"),
    ]
    body = [_RUNTIME.strip("\n"), "", f"LIBRARY = {library!r}"]
    if spec.family == "pointwise":
        k = spec.params["kernel"]
        params = []
        for p in prog.params:
            if isinstance(p, ScalarParameter):
                params.append(("scalar", p.dtype, ()))
            else:
                params.append(("tensor", p.type.dtype,
                               tuple(d.name if isinstance(d, SymDim) else None for d in p.type.shape)))
        body += [
            f"KERNEL = {k.name!r}",
            f"PARAMS = {tuple(params)!r}",
            f"SYMBOLS = {tuple(k.sym_names)!r}",
            f"GRID = {tuple(_grid_literal(g) for g in k.grid)!r}",
            f"GRID_ARGS = {tuple(k.grid_args)!r}",
            f"POINTS = {k.points}",
            f"BLOCK = {BLOCK_THREADS}",
            f"UNROLL = {POINTS_PER_THREAD}",
            "CUDA_SOURCE = r'''",
            k.source.replace("'''", "' ' '"),
            "'''",
            _RTC_KERNEL.strip("\n"),
        ]
    else:
        calls = tuple((entry, tuple(tuple(r) for r in recipe)) for entry, recipe in abi_calls(spec))
        body += [f"CALLS = {calls!r}", _ABI_KERNEL.strip("\n")]
    return "\n".join(head + [""] + body) + "\n"


__all__ = ["standalone_module"]
