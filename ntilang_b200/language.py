"""The ``T.*`` surface TileLang programs are written against.

Kernel bodies are never executed: every ``T.<op>`` here is a marker that raises when
called from Python, and ``@T.prim_func`` only captures the function plus the caller's
locals its annotations and body refer to.  ``ntilang_b200.frontend`` reads the body's
AST.  The names and their argument meaning follow the reference's
``python/ntilang/language.py`` (markers :239-373, ``prim_func`` :191-217, ``Tensor``
:115-125, ``dynamic`` :101-104, ``jit`` :420-476) so that programs written for it (and
for upstream TileLang) parse unchanged.
"""

from __future__ import annotations

import ast
import builtins
import inspect
import textwrap
from dataclasses import dataclass
from functools import wraps
from typing import Callable

from . import layout as layout  # noqa: F401  (``T.layout`` is part of the surface)
from .ir import DTYPE_ALIASES, DTYPES, TensorType, canonical_dtype


class DType(str):
    """A dtype name; inside a kernel body ``T.float32(x)`` denotes a cast."""

    def __new__(cls, value):
        if value is builtins.bool:
            value = "bool"
        elif value is builtins.int:
            value = "int32"
        elif value is builtins.float:
            value = "float32"
        if not isinstance(value, str):
            raise TypeError("dtype requires a supported name or Python scalar type")
        return super().__new__(cls, canonical_dtype(value))

    @property
    def bits(self):
        return DTYPES[self] * 8

    @property
    def bytes(self):
        return DTYPES[self]

    itemsize = bytes

    @property
    def lanes(self):
        return 1

    def __call__(self, value):
        raise RuntimeError(f"T.{self}(value) is a scalar cast inside a @T.prim_func body")


for _alias in (*DTYPES, *DTYPE_ALIASES):
    globals()[_alias] = DType(_alias)
del _alias

dtype = DType


def get_tvm_dtype(value):
    return value if type(value) is DType else DType(value)


@dataclass(frozen=True)
class SymbolicDim:
    """A dimension created by ``T.dynamic(name)``; bound from tensor shapes per call."""

    name: str
    dtype: str = "int32"

    def __post_init__(self):
        if not isinstance(self.name, str) or not self.name:
            raise ValueError("T.dynamic requires a non-empty dimension name")
        object.__setattr__(self, "dtype", str(DType(self.dtype)))


@dataclass(frozen=True)
class SymbolicTensorSpec:
    """``T.Tensor`` annotation with at least one ``T.dynamic`` dimension."""

    shape: tuple
    dtype: str


class GemmWarpPolicy:
    """Accepted for compatibility; the sm_100a kernels choose their own warp roles."""

    Square = 0
    FullRow = 1
    FullCol = 2


def dynamic(name: str, dtype: str = "int32") -> SymbolicDim:
    return SymbolicDim(name, dtype)


def infinity(dtype: str = "float32") -> float:
    if str(DType(dtype)) not in ("float16", "bfloat16", "float32", "float64"):
        raise ValueError(f"T.infinity requires a floating-point dtype, got {dtype!r}")
    return builtins.float("inf")


def Tensor(shape, dtype="float32", data=None, scope=None):
    if data is not None or scope not in (None, "global"):
        raise ValueError("Only global tensor parameters are supported")
    dims = (shape,) if isinstance(shape, (builtins.int, SymbolicDim)) else tuple(shape)
    resolved = DType(dtype)
    if any(isinstance(d, SymbolicDim) for d in dims):
        for d in dims:
            if not isinstance(d, SymbolicDim) and (type(d) is not builtins.int or d <= 0):
                raise ValueError("Static dimensions alongside T.dynamic must be positive integers")
        return SymbolicTensorSpec(dims, str(resolved))
    return TensorType(dims, str(resolved))


Buffer = Tensor


def ceildiv(lhs, rhs, span=None):
    if type(lhs) is not builtins.int or type(rhs) is not builtins.int:
        raise TypeError("ceildiv specialization arguments must be integers")
    if rhs == 0:
        raise ValueError("ceildiv requires a nonzero divisor")
    return (lhs + rhs - 1) // rhs


cdiv = ceildiv


def align_up(x: int, y: int) -> int:
    return ceildiv(x, y) * y


@dataclass(frozen=True)
class PrimFunc:
    """A captured kernel function: the function plus the caller locals it names."""

    function: Callable
    annotation_locals: tuple = ()
    specializations: tuple = ()

    @property
    def __name__(self):
        return self.function.__name__

    def __call__(self, *args, **kwargs):
        raise TypeError("Compile a prim_func with ntilang.compile() before calling it")


@dataclass(frozen=True, eq=False)
class Macro:
    function: Callable
    annotation_locals: tuple = ()

    @property
    def __name__(self):
        return self.function.__name__

    def __call__(self, *args, **kwargs):
        raise TypeError("T.macro calls are expanded inside a compiled prim_func")


def _referenced_caller_locals(function, caller) -> tuple:
    """Caller locals named by the function's annotations or body.

    With ``from __future__ import annotations`` the annotations are strings that may
    name factory arguments the function body never closes over (e.g. ``batch``).
    """
    names = set()
    for annotation in function.__annotations__.values():
        if isinstance(annotation, str):
            try:
                names.update(n.id for n in ast.walk(ast.parse(annotation, mode="eval")) if isinstance(n, ast.Name))
            except SyntaxError:
                pass
    try:
        tree = ast.parse(textwrap.dedent(inspect.getsource(function)))
        names.update(n.id for n in ast.walk(tree) if isinstance(n, ast.Name))
    except (OSError, TypeError, SyntaxError):
        pass
    return tuple((name, caller[name]) for name in sorted(names) if name in caller)


def _caller_locals(depth: int = 2) -> dict:
    frame = inspect.currentframe()
    try:
        for _ in range(depth):
            frame = frame.f_back if frame is not None else None
        return dict(frame.f_locals) if frame is not None else {}
    finally:
        del frame


def prim_func(function: Callable) -> PrimFunc:
    return PrimFunc(function, _referenced_caller_locals(function, _caller_locals()))


def macro(func=None):
    caller = _caller_locals()

    def decorate(function):
        return Macro(function, _referenced_caller_locals(function, caller))

    return decorate(func) if func is not None else decorate


class Ref:
    """Macro parameter annotation for a mutable scalar or buffer region."""


def _marker(name):
    def operation(*args, **kwargs):
        raise RuntimeError(f"T.{name} is syntax inside a @T.prim_func body")

    operation.__name__ = name
    operation.__qualname__ = name
    return operation


# The kernel-body vocabulary (upstream TileLang names).  Markers only.
MARKERS = (
    "Kernel", "Parallel", "grid", "serial", "Serial", "Pipelined", "unroll", "Unroll",
    "alloc_shared", "alloc_fragment", "alloc_local", "alloc_var", "use_swizzle",
    "annotate_layout", "loop_break", "break_loop", "continue_loop", "print", "device_assert",
    "Assert", "likely", "copy", "transpose", "clamp", "clear", "fill", "atomic_add",
    "atomic_max", "gemm", "reduce", "reduce_sum", "reduce_abssum", "reduce_max",
    "reduce_absmax", "reduce_min", "reduce_bitand", "reduce_bitor", "reduce_bitxor",
    "cumsum", "cummax", "cumsum_fragment", "cummax_fragment", "exp", "exp2", "sqrt", "pow",
    "fmod", "atan2", "copysign", "hypot", "nextafter", "ldexp", "ieee_add", "ieee_sub",
    "ieee_mul", "ieee_fmaf", "ieee_frcp", "ieee_fsqrt", "ieee_frsqrt", "ieee_fdiv", "fma",
    "fmul", "__exp", "__exp10", "__log", "__log2", "__log10", "__sin", "__cos", "__tan",
    "fast_rcp", "exp10", "log", "log2", "log10", "log1p", "rsqrt", "erf", "sigmoid", "sin",
    "cos", "tan", "asin", "acos", "atan", "sinh", "cosh", "tanh", "asinh", "acosh", "atanh",
    "abs", "floor", "ceil", "trunc", "round", "nearbyint", "isnan", "isinf", "isfinite",
    "maximum", "minimum", "max", "min", "cast", "reinterpret", "popcount", "clz",
    "bitwise_and", "bitwise_or", "bitwise_xor", "bitwise_not", "shift_left", "shift_right",
    "floordiv", "floormod", "truncdiv", "truncmod", "Select", "if_then_else",
)
for _name in MARKERS:
    globals()[_name] = _marker(_name)
del _name


def _is_direct_kernel(function: Callable) -> bool:
    """True when ``function`` is itself a kernel (its last statement is ``with T.Kernel``)."""
    try:
        tree = ast.parse(textwrap.dedent(inspect.getsource(function)))
    except (OSError, TypeError, SyntaxError):
        return False
    if not tree.body or not isinstance(tree.body[0], ast.FunctionDef):
        return False
    body = [s for s in tree.body[0].body if not (isinstance(s, ast.Expr) and isinstance(s.value, ast.Constant))]
    if not body or not isinstance(body[-1], ast.With) or len(body[-1].items) != 1:
        return False
    ctx = body[-1].items[0].context_expr
    if not isinstance(ctx, ast.Call):
        return False
    f = ctx.func
    return (isinstance(f, ast.Attribute) and f.attr == "Kernel") or (isinstance(f, ast.Name) and f.id == "Kernel")


def has_symbolic_annotations(program: PrimFunc) -> bool:
    values = list(program.function.__annotations__.values()) + [v for _, v in program.annotation_locals]
    for cell in program.function.__closure__ or ():
        try:
            values.append(cell.cell_contents)
        except ValueError:
            pass
    return any(isinstance(v, (SymbolicDim, SymbolicTensorSpec)) for v in values)


def jit(
    function=None,
    *,
    out_idx=None,
    target="auto",
    target_host=None,
    execution_backend=None,
    verbose=False,
    pass_configs=None,
    compile_flags=None,
):
    """``@tilelang.jit``: compile a kernel, or wrap a kernel factory with a per-argument cache.

    Cache key = (args, sorted kwargs, resolved target, out_idx), as in the reference's
    ``language.py:447-472``.  ``target_host``, ``execution_backend``, ``verbose``,
    ``pass_configs`` and ``compile_flags`` are accepted and ignored.
    """
    from .compat import resolve_target
    from .compiler import DynamicJitKernel, compile

    del target_host, execution_backend, verbose, compile_flags
    caller = _caller_locals()

    def decorate(factory):
        if _is_direct_kernel(factory):
            program = PrimFunc(factory, _referenced_caller_locals(factory, caller))
            if has_symbolic_annotations(program):
                return DynamicJitKernel(program, target=target, out_idx=out_idx, pass_configs=pass_configs)
            return compile(program, target=resolve_target(target), out_idx=out_idx, pass_configs=pass_configs)

        cache = {}

        @wraps(factory)
        def wrapped(*args, **kwargs):
            resolved = resolve_target(target)
            key_out = out_idx if out_idx is None or isinstance(out_idx, builtins.int) else tuple(out_idx)
            key = (args, tuple(sorted(kwargs.items())), resolved, key_out)
            if key in cache:
                return cache[key]
            program = factory(*args, **kwargs)
            if isinstance(program, PrimFunc) and has_symbolic_annotations(program):
                kernel = DynamicJitKernel(program, target=resolved, out_idx=out_idx, pass_configs=pass_configs)
            else:
                kernel = compile(program, target=resolved, out_idx=out_idx, pass_configs=pass_configs)
            cache[key] = kernel
            return kernel

        wrapped.cache = cache
        return wrapped

    return decorate(function) if function is not None else decorate
