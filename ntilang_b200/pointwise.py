"""Generic elementwise programs -> one CUDA C kernel for sm_100a, compiled at run time.

The recognised op families (``recognize``) cover the hot kernels with hand-written tcgen05 /
row-reduction code.  Every other program whose work is independent per ``T.Parallel`` point
(the reference's examples/fragment_affine.py, piecewise.py, window_sum.py, scalar-parameter
and symbolic-size kernels, atomics) lowers here to CUDA C: one CUDA thread per
(block instance, parallel point), loads and stores in the reference's semantics, compiled by
NVRTC through ``ntl_rtc_build`` (csrc/rtc.cu) and launched by ``ntl_rtc_launch``.

Semantics (the reference's evaluator, python/ntilang/testing.py:133-143 and its lowering,
codegen.py:541-562, :590-623, :1494-1517):

* a global load outside the tensor reads 0 of the tensor's dtype; a global store outside the
  tensor is skipped;
* scalar types follow the reference's promotion (python/ntilang/scalar.py:60-78, 104-230):
  Python int literals are int32, float literals float32, mixed float widths widen, a float
  operand makes the result float; ``/`` on integers is an error; ``//`` and ``%`` floor
  like Python on signed integers;
* float16 / bfloat16 values are held in fp32 registers and rounded to their type after every
  operation (fp16/bf16 + - * of two such values is exact in fp32, so this equals rounding the
  exact result, as numpy's float16 arithmetic does); integer + - * wrap;
* every multiply and add rounds separately (NVRTC ``--fmad=false``), division and square
  root are IEEE, so float32 + - * / match numpy bit for bit; transcendental functions use
  CUDA's library functions (ulp-level differences from numpy's).

Fragments (``T.alloc_fragment`` / ``alloc_local`` / ``alloc_shared``) are kept per thread:
each must be read and written only at the coordinates of a ``T.Parallel`` loop of the same
shape, or copied / filled whole — the register-slot mapping the reference's lowering uses
(codegen.py:590-601), which makes the values a thread needs its own.  ``T.alloc_var`` scalars
are per thread too; one declared outside a ``T.Parallel`` loop may not be assigned inside it
(that would be a cross-point reduction, which the reference's GPU code does not compute either).
Reductions, scans and GEMMs belong to the recognised families and are rejected here.
"""

from __future__ import annotations

import ctypes
import math
import re
from dataclasses import dataclass, field

from . import _lib
from .frontend import (Alloc, Atomic, Bin, Break, Call, Cmp, Const, Continue, Copy, Fill, Gemm, Hint, If, Let, Load,
                       Loop, Parallel, Program, Reduce, Scan, Select, Store, Var, While)
from .ir import DTYPES, CompileError, ScalarParameter, SymDim, integer_limits

BLOCK_THREADS = 256
# Points per thread: a CTA covers POINTS_PER_THREAD consecutive runs of BLOCK_THREADS points
# (each run coalesced), and the unrolled loop lets one thread keep that many points' loads in
# flight (one point per thread left HBM at ~72% of a copy's bandwidth on B200).
POINTS_PER_THREAD = 4

FLOATS = ("float16", "bfloat16", "float32", "float64")
# C type of a value held in registers (float16 / bfloat16 live in fp32 registers).
CTYPE = {
    "bool": "bool", "int8": "signed char", "int16": "short", "int32": "int", "int64": "long long",
    "uint8": "unsigned char", "uint16": "unsigned short", "uint32": "unsigned", "uint64": "unsigned long long",
    "float16": "float", "bfloat16": "float", "float32": "float", "float64": "double",
}
# C type of an element in memory.
STORAGE = dict(CTYPE, float16="unsigned short", bfloat16="unsigned short")
# Vector type of four elements of a storage type, for the 4-point groups of a vectorised
# kernel (one 16-, 8- or 4-byte access instead of four scalar ones).
VEC4 = {"float": "float4", "int": "int4", "unsigned": "uint4", "unsigned short": "ushort4", "short": "short4",
        "signed char": "char4", "unsigned char": "uchar4"}
# Unsigned type of the same width, for wrapping + - *.
UNSIGNED = {"int8": "unsigned char", "int16": "unsigned short", "int32": "unsigned", "int64": "unsigned long long",
            "uint8": "unsigned", "uint16": "unsigned", "uint32": "unsigned", "uint64": "unsigned long long"}
_CTYPES_SCALAR = {
    "bool": ctypes.c_bool, "int8": ctypes.c_int8, "int16": ctypes.c_int16, "int32": ctypes.c_int32,
    "int64": ctypes.c_int64, "uint8": ctypes.c_uint8, "uint16": ctypes.c_uint16, "uint32": ctypes.c_uint32,
    "uint64": ctypes.c_uint64, "float16": ctypes.c_float, "bfloat16": ctypes.c_float, "float32": ctypes.c_float,
    "float64": ctypes.c_double,
}

_PRELUDE = r"""
__device__ __forceinline__ float ntl_h2f(unsigned short h) {
  float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ unsigned short ntl_f2h(float f) {
  unsigned short h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
__device__ __forceinline__ float ntl_r16(float f) { return ntl_h2f(ntl_f2h(f)); }
__device__ __forceinline__ float ntl_b2f(unsigned short b) { return __uint_as_float(((unsigned)b) << 16); }
__device__ __forceinline__ unsigned short ntl_f2b(float f) {
  unsigned short b; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(b) : "f"(f)); return b; }
__device__ __forceinline__ float ntl_rb16(float f) { return ntl_b2f(ntl_f2b(f)); }
template <class T> __device__ __forceinline__ T ntl_nan_or(T a, T b, T r) {
  return a != a ? a : (b != b ? b : r); }
template <class T> __device__ __forceinline__ T ntl_floordiv(T a, T b) {
  T q = a / b; return (q * b != a && ((a < 0) != (b < 0))) ? q - 1 : q; }
template <class T> __device__ __forceinline__ T ntl_floormod(T a, T b) {
  T r = a % b; return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r; }
"""


def promote(left: str, right: str) -> str:
    """Result dtype of a binary operation (the reference's rule, python/ntilang/scalar.py:60-78)."""
    if left == right:
        return left
    if left == "bool":
        return right
    if right == "bool":
        return left
    lf, rf = left in FLOATS, right in FLOATS
    if lf and rf:
        return f"float{max(DTYPES[left], DTYPES[right]) * 8}"
    if lf or rf:
        return left if lf else right
    lu, ru = left.startswith("uint"), right.startswith("uint")
    if lu != ru:
        uns, sig = (left, right) if lu else (right, left)
        return uns if DTYPES[uns] >= DTYPES[sig] else sig
    return left if DTYPES[left] >= DTYPES[right] else right


def _const_dtype(value) -> str:
    if isinstance(value, bool):
        return "bool"
    if isinstance(value, int):
        if -(2**31) <= value < 2**31:
            return "int32"
        if -(2**63) <= value < 2**63:
            return "int64"
        raise CompileError("Bare scalar integer constants must fit signed 64-bit arithmetic")
    return "float32"


def _c_literal(value, dtype: str) -> str:
    if dtype == "bool":
        return "true" if value else "false"
    if dtype in FLOATS:
        v = float(value)
        if math.isnan(v):
            return "__int_as_float(0x7fc00000)" if dtype != "float64" else "__longlong_as_double(0x7ff8000000000000LL)"
        if math.isinf(v):
            return ("-" if v < 0 else "") + ("__int_as_float(0x7f800000)" if dtype != "float64"
                                             else "__longlong_as_double(0x7ff0000000000000LL)")
        text = repr(v)
        if "e" not in text and "." not in text and "inf" not in text:
            text += ".0"
        return text + ("" if dtype == "float64" else "f")
    v = int(value)
    if dtype in ("int64",):
        return f"{v}LL" if v != -(2**63) else "(-9223372036854775807LL - 1)"
    if dtype in ("uint64",):
        return f"{v}ULL"
    if dtype.startswith("uint"):
        return f"{v}u"
    return str(v) if v != -(2**31) else "(-2147483647 - 1)"


@dataclass
class PointwiseKernel:
    """A lowered program: CUDA C source plus what the host needs to launch it."""

    name: str
    source: str
    program: Program
    sym_names: tuple  # symbolic dimension names, passed as int64 arguments in this order
    grid: tuple  # int or Expr per block dimension
    grid_args: tuple  # indices of grid dims passed as int64 arguments
    points: int  # CUDA threads per block instance (largest parallel domain)
    _handle: int = field(default=0, repr=False)
    _fast: object = field(default=None, repr=False)

    def build(self) -> int:
        """Compile with NVRTC (host only) and return the library's kernel handle."""
        if not self._handle:
            h = ctypes.c_uint64(0)
            _lib.call("ntl_rtc_build", self.source.encode(), self.name.encode(), ctypes.byref(h))
            self._handle = int(h.value)
        return self._handle

    def launch_geometry(self, bindings: dict):
        extents = [_eval_host(g, bindings) for g in self.grid]
        blocks = 1
        for e in extents:
            blocks *= max(int(e), 0)
        total = blocks * self.points
        return extents, total

    def launch(self, arguments, bindings: dict, stream: int) -> None:
        fast = self._fast
        if fast is None:
            fast = self._fast = self._prepare()
        fn, kinds, static = fast
        if static is not None:
            tail, grid_x = static
        else:
            extents, total = self.launch_geometry(bindings)
            if total == 0:
                return
            tail = [ctypes.c_int64(int(bindings[s])) for s in self.sym_names]
            tail += [ctypes.c_int64(int(extents[i])) for i in self.grid_args]
            tail.append(ctypes.c_int64(total))
            per_cta = BLOCK_THREADS * POINTS_PER_THREAD
            grid_x = (total + per_cta - 1) // per_cta
        if grid_x == 0:
            return
        keep = [ctypes.c_void_p(a.data_ptr()) if k is None else k(a) for k, a in zip(kinds, arguments)]
        keep += tail
        argv = (ctypes.c_void_p * len(keep))(*[ctypes.addressof(k) for k in keep])
        rc = fn(self._handle, grid_x, BLOCK_THREADS, argv, stream)
        if rc:
            msg = _lib.lib().ntl_last_error()
            raise _lib.KernelError("ntl_rtc_launch", rc, msg.decode() if msg else "")

    def _prepare(self):
        """Per-kernel launch state: the bound C entry, argument converters, and for programs
        without symbolic sizes the fixed trailing arguments and grid."""
        self.build()
        fn = _lib.lib().ntl_rtc_launch
        kinds = [(_CTYPES_SCALAR[p.dtype] if isinstance(p, ScalarParameter) else None) for p in self.program.params]
        static = None
        if not self.sym_names and not self.grid_args:
            _, total = self.launch_geometry({})
            per_cta = BLOCK_THREADS * POINTS_PER_THREAD
            static = ([ctypes.c_int64(total)], (total + per_cta - 1) // per_cta)
        return fn, kinds, static


def _eval_host(e, bindings):
    """A grid extent: an int, or an integer Expr over symbolic dimensions."""
    if isinstance(e, int):
        return e
    if isinstance(e, Const):
        return int(e.value)
    if isinstance(e, Var):
        if e.name.startswith("$sym:"):
            return int(bindings[e.name[5:]])
        raise CompileError(f"grid extent depends on kernel-time value {e.name!r}")
    if isinstance(e, Bin):
        a, b = _eval_host(e.a, bindings), _eval_host(e.b, bindings)
        return {"+": a + b, "-": a - b, "*": a * b, "//": a // b if b else 0, "%": a % b if b else 0}[e.op]
    if isinstance(e, Call) and e.fn in ("max", "min"):
        vals = [_eval_host(x, bindings) for x in e.args]
        return max(vals) if e.fn == "max" else min(vals)
    raise CompileError("grid extents must be integer expressions of symbolic sizes")


def _buffer_uses(prog: Program):
    """(loaded, stored) global buffer names of a program: read by a load, copy source or
    atomic; written by a store, copy destination or atomic."""
    loaded, stored = set(), set()

    def walk(x):
        if isinstance(x, (list, tuple)):
            for y in x:
                walk(y)
            return
        if not hasattr(x, "__dataclass_fields__"):
            return
        if isinstance(x, Load):
            loaded.add(x.buf)
        elif isinstance(x, Store):
            stored.add(x.buf)
        elif isinstance(x, Atomic):
            loaded.add(x.buf)
            stored.add(x.buf)
        elif isinstance(x, Copy):
            loaded.add(x.src.buf)
            stored.add(x.dst.buf)
        for f in x.__dataclass_fields__:
            walk(getattr(x, f))

    walk(prog.body)
    return loaded, stored


class _Lowering:
    def __init__(self, prog: Program, vec: bool = False):
        self.prog = prog
        # Vectorised form: thread t of a CTA takes the 4 consecutive points 4t .. 4t+3 of its
        # 1024, and a global access whose 4 points are contiguous (unit stride in the innermost
        # T.Parallel variable, index otherwise free of per-point values) becomes one vector
        # access when the group is in bounds and aligned (checked at run time, else per point).
        # Loads only from tensors the program never writes; stores only at the top level of a
        # T.Parallel body to tensors it never reads (they are issued after the 4 points ran).
        self.vec = vec
        self.vec_decls: list = []  # declared before the point loop
        self.vec_flush: list = []  # vector stores after the point loop
        self.vec_loads: dict = {}  # (buffer, index) -> slot of a vectorised load
        self.vec_count = 0
        self.guard_sizes: list = []  # every `pt < n` guard
        self.top_stmt = None  # the statement being lowered at the top level of a T.Parallel body
        self.loaded, self.stored = _buffer_uses(prog)
        self.lines: list = []
        self.depth = 1
        self.types: dict = {}  # kernel variable -> dtype
        self.ranges: dict = {}  # kernel variable -> (lo, hi) when static
        self.fragments: dict = {}  # fragment name -> shape
        self.mutable_scope: dict = {}  # alloc_var name -> parallel nesting level at declaration
        self.parallel_level = 0
        self.guards: list = []  # open `pt < n` guards (collective copies / fills)
        self.loops: list = []  # enclosing loops, innermost last: "serial" (a program loop) or "parallel"
        self.current_parallel = None  # the T.Parallel loop being lowered
        self.points = 1
        self.sym_names = tuple(s.name for s in prog.sym_dims)
        for p in prog.params:
            if isinstance(p, ScalarParameter):
                self.types[p.name] = p.dtype
        for s in self.sym_names:
            self.types[f"$sym:{s}"] = "int32"
        self.grid_args = []
        for i, (bv, g) in enumerate(zip(prog.block_vars, prog.grid)):
            self.types[bv] = "int32"
            if isinstance(g, int):
                self.ranges[bv] = (0, g - 1)
            elif isinstance(g, Const):
                self.ranges[bv] = (0, int(g.value) - 1)
            else:
                self.grid_args.append(i)

    # ------------------------------------------------------------------ helpers
    def fail(self, msg):
        raise CompileError(f"{self.prog.name}: {msg}")

    def emit(self, line):
        self.lines.append("  " * self.depth + line)

    def buf(self, name) -> Alloc:
        b = self.prog.buffers.get(name)
        if b is None:
            self.fail(f"unknown buffer {name!r}")
        return b

    def dim_code(self, d) -> str:
        if isinstance(d, SymDim):
            return f"s_{_ident(d.name)}"
        return f"{int(d)}LL"

    def conv(self, code: str, src: str, dst: str) -> str:
        if src == dst:
            return code
        if dst == "bool":
            return f"(({code}) != 0)"
        if dst == "float16":
            return f"ntl_r16((float)({code}))" if src != "bfloat16" else f"ntl_r16({code})"
        if dst == "bfloat16":
            return f"ntl_rb16((float)({code}))" if src != "float16" else f"ntl_rb16({code})"
        return f"(({CTYPE[dst]})({code}))"

    def round_to(self, code: str, dtype: str) -> str:
        if dtype == "float16":
            return f"ntl_r16({code})"
        if dtype == "bfloat16":
            return f"ntl_rb16({code})"
        return code

    # -------------------------------------------------------------- intervals
    def interval(self, e):
        if isinstance(e, Const) and isinstance(e.value, int) and not isinstance(e.value, bool):
            return (e.value, e.value)
        if isinstance(e, Var):
            return self.ranges.get(e.name)
        if isinstance(e, Bin) and e.op in ("+", "-", "*"):
            a, b = self.interval(e.a), self.interval(e.b)
            if a is None or b is None:
                return None
            if e.op == "+":
                return (a[0] + b[0], a[1] + b[1])
            if e.op == "-":
                return (a[0] - b[1], a[1] - b[0])
            prods = [x * y for x in a for y in b]
            return (min(prods), max(prods))
        return None

    # ---------------------------------------------------------- vector groups
    def _vec_deps(self, e):
        """Names an index expression depends on, or None when it holds anything but integer
        constants, kernel values and + - * // %."""
        if isinstance(e, Const):
            return set() if isinstance(e.value, int) and not isinstance(e.value, bool) else None
        if isinstance(e, Var):
            return {e.name}
        if isinstance(e, Bin) and e.op in ("+", "-", "*", "//", "%"):
            a, b = self._vec_deps(e.a), self._vec_deps(e.b)
            return None if a is None or b is None else a | b
        return None

    def _vec_group_ok(self, name, idx) -> bool:
        """The 4 points of a group access 4 contiguous elements of ``name``."""
        par = self.current_parallel
        b = self.buf(name)
        if not self.vec or par is None or b.scope != "global" or STORAGE[b.dtype] not in VEC4 or not idx:
            return False
        if par.extents[-1] % 4 or any(g % 4 for g in self.guards):
            return False
        inner = par.vars[-1]
        free = set(self.prog.block_vars) | set(par.vars) | {f"$sym:{n}" for n in self.sym_names}
        free |= {p.name for p in self.prog.params if isinstance(p, ScalarParameter)}
        for e in idx[:-1]:
            d = self._vec_deps(e)
            if d is None or not d <= free or inner in d:
                return False
        # the shape test first: it rejects indices holding loads, whose code generation would emit
        return self._unit_stride(idx[-1], inner, free) and self.dtype(idx[-1]) in ("int32", "int64", "uint32",
                                                                                   "uint64")

    def _unit_stride(self, e, inner, free) -> bool:
        """``e`` is ``inner`` plus / minus terms free of it, through + and - only.  Wrapping
        integer + and - are linear modulo 2^32 (2^64), so the index of point u of a group is
        the group's first index + u exactly whenever that sum stays below the type's maximum,
        which the run-time group check asserts."""
        if isinstance(e, Var) and e.name == inner:
            return True
        if not (isinstance(e, Bin) and e.op in ("+", "-")):
            return False
        da, db = self._vec_deps(e.a), self._vec_deps(e.b)
        if da is None or db is None:
            return False
        if inner in da and inner not in db and db <= free:
            return self._unit_stride(e.a, inner, free)
        if e.op == "+" and inner in db and inner not in da and da <= free:
            return self._unit_stride(e.b, inner, free)
        return False

    def _vec_group_check(self, name, idx, codes, off) -> str:
        """Run-time test that a group's 4 elements are in bounds and vector-aligned."""
        b = self.buf(name)
        clauses = []
        last = len(idx) - 1
        for n, (e, c, d) in enumerate(zip(idx, codes, b.shape)):
            if not isinstance(d, SymDim):
                iv = self.interval(e)
                if iv is not None and 0 <= iv[0] and iv[1] < d and iv[1] < 2**31 - 4:
                    continue  # every point's index is in range (and far from wrapping), so the group's is
            if n == last:  # the 4 indices c .. c+3 are in range and did not wrap
                clauses.append(f"(0 <= ({c}) && (long long)({c}) + 3LL < {self.dim_code(d)} && "
                               f"(long long)({c}) <= 2147483643LL)")
            else:
                clauses.append(f"(0 <= ({c}) && ({c}) < {self.dim_code(d)})")
        size = 4 * DTYPES[b.dtype]
        clauses.append(f"(((unsigned long long)(p_{_ident(name)} + ({off}))) & {size - 1}ULL) == 0ULL")
        return " && ".join(clauses)

    def vec_load(self, e: Load, codes):
        if not self._vec_group_ok(e.buf, e.idx):
            return None
        key = (e.buf, repr(e.idx))
        if key in self.vec_loads:
            return self.vec_loads[key]
        k = self.vec_count
        self.vec_count += 1
        self.vec_loads[key] = k
        st = STORAGE[self.buf(e.buf).dtype]
        vt = VEC4[st]
        off = self.offset(e.buf, codes)
        self.vec_decls += [f"bool vl{k}_ok = false;", f"{st} vl{k}_v[4];"]
        self.emit("if (unit == 0) {")
        self.emit(f"  const long long o_ = {off};")
        self.emit(f"  vl{k}_ok = {self._vec_group_check(e.buf, e.idx, codes, 'o_')};")
        self.emit(f"  if (vl{k}_ok) {{ const {vt} t_ = *reinterpret_cast<const {vt}*>(p_{_ident(e.buf)} + o_); "
                  f"vl{k}_v[0] = t_.x; vl{k}_v[1] = t_.y; vl{k}_v[2] = t_.z; vl{k}_v[3] = t_.w; }}")
        self.emit("}")
        return k

    def vec_store(self, name, idx, codes):
        if not self._vec_group_ok(name, idx):
            return None
        k = self.vec_count
        self.vec_count += 1
        st = STORAGE[self.buf(name).dtype]
        vt = VEC4[st]
        off = self.offset(name, codes)
        self.vec_decls += [f"bool vs{k}_ok = false;", f"long long vs{k}_o = 0;", f"{st} vs{k}_v[4];"]
        self.emit(f"if (unit == 0) {{ vs{k}_o = {off}; vs{k}_ok = {self._vec_group_check(name, idx, codes, f'vs{k}_o')}; }}")
        self.vec_flush.append(f"if (vs{k}_ok) *reinterpret_cast<{vt}*>(p_{_ident(name)} + vs{k}_o) = "
                              f"make_{vt}(vs{k}_v[0], vs{k}_v[1], vs{k}_v[2], vs{k}_v[3]);")
        return k

    def in_bounds(self, name, idx_exprs, idx_codes) -> str:
        shape = self.buf(name).shape
        if len(shape) != len(idx_codes):
            self.fail(f"{name} has rank {len(shape)}, indexed with {len(idx_codes)} subscripts")
        clauses = []
        for e, c, d in zip(idx_exprs, idx_codes, shape):
            if not isinstance(d, SymDim):
                iv = e if isinstance(e, tuple) else (self.interval(e) if e is not None else None)
                if iv is not None and 0 <= iv[0] and iv[1] < d:
                    continue
            clauses.append(f"(0 <= ({c}) && ({c}) < {self.dim_code(d)})")
        return " && ".join(clauses) if clauses else ""

    def offset(self, name, idx_codes) -> str:
        shape = self.buf(name).shape
        off = f"(long long)({idx_codes[0]})"
        for c, d in zip(idx_codes[1:], shape[1:]):
            off = f"({off} * {self.dim_code(d)} + (long long)({c}))"
        return off

    # ------------------------------------------------------------- expressions
    def dtype(self, e) -> str:
        return self.expr(e)[1]

    def expr(self, e):
        """(C code, dtype) of an expression."""
        if isinstance(e, Const):
            d = _const_dtype(e.value)
            return _c_literal(e.value, d), d
        if isinstance(e, Var):
            if e.name not in self.types:
                self.fail(f"unknown kernel value {e.name!r}")
            d = self.types[e.name]
            if e.name.startswith("$sym:"):
                return f"((int)s_{_ident(e.name[5:])})", d
            return f"v_{_ident(e.name)}", d
        if isinstance(e, Load):
            return self.load(e)
        if isinstance(e, Cmp):
            (a, da), (b, db) = self.expr(e.a), self.expr(e.b)
            d = promote(da, db)
            return f"({self.conv(a, da, d)} {e.op} {self.conv(b, db, d)})", "bool"
        if isinstance(e, Bin):
            return self.binary(e)
        if isinstance(e, Select):
            c, dc = self.expr(e.cond)
            if dc != "bool":
                self.fail("conditional expressions require a Boolean condition")
            (a, da), (b, db) = self.expr(e.a), self.expr(e.b)
            d = promote(da, db)
            return f"(({c}) ? {self.conv(a, da, d)} : {self.conv(b, db, d)})", d
        if isinstance(e, Call):
            return self.call(e)
        self.fail(f"unsupported expression {type(e).__name__}")

    def binary(self, e):
        (a, da), (b, db) = self.expr(e.a), self.expr(e.b)
        if e.op in ("&", "|", "^", "<<", ">>"):
            return self.bitwise(e.op, e.a, e.b, a, da, b, db)
        d = promote(da, db)
        if d == "bool":
            self.fail(f"arithmetic operator {e.op!r} on two Boolean operands")
        ca, cb = self.conv(a, da, d), self.conv(b, db, d)
        op = e.op
        if op == "/":
            if d not in FLOATS:
                self.fail("Integer '/' is ambiguous; use explicit integer division or cast to a floating dtype")
            return self.round_to(f"({ca} / {cb})", d), d
        if op in ("//", "%"):
            if d in FLOATS:
                self.fail("Integer division and remainder require integer operands")
            if d.startswith("uint"):
                return f"(({CTYPE[d]})({ca} {'/' if op == '//' else '%'} {cb}))", d
            fn = "ntl_floordiv" if op == "//" else "ntl_floormod"
            return f"{fn}<{CTYPE[d]}>({ca}, {cb})", d
        if op not in ("+", "-", "*"):
            self.fail(f"unsupported operator {op!r}")
        if d in FLOATS:
            return self.round_to(f"({ca} {op} {cb})", d), d
        u = UNSIGNED[d]
        return f"(({CTYPE[d]})(({u})({ca}) {op} ({u})({cb})))", d

    def bitwise(self, op, ea, eb, a, da, b, db):
        """& | ^ << >> on integers / Booleans; an int literal takes the other operand's integer
        dtype when it fits (python/ntilang/scalar.py:81-96)."""
        for d in (da, db):
            if d in FLOATS:
                self.fail("Bitwise operations require integer or Boolean operands")
        lit_a = isinstance(ea, Const) and type(ea.value) is int
        lit_b = isinstance(eb, Const) and type(eb.value) is int
        if lit_a != lit_b:
            lit, other = (ea, db) if lit_a else (eb, da)
            if other in CTYPE and other not in FLOATS:
                low, high = integer_limits(other)
                if not low <= lit.value <= high:
                    self.fail(f"Bitwise integer literal must fit the other operand's {other} dtype")
                if lit_a:
                    da = other
                else:
                    db = other
        d = promote(da, db)
        if op in ("<<", ">>"):
            if "bool" in (da, db):
                self.fail("Shift operations require integer operands, excluding Boolean")
            x, y = self.conv(a, da, d), self.conv(b, db, d)
            if op == "<<":
                return f"(({CTYPE[d]})(({UNSIGNED[d]})({x}) << (unsigned)({y})))", d
            return f"(({CTYPE[d]})(({x}) >> (unsigned)({y})))", d
        if d == "bool":
            return f"({a} {op} {b})", "bool"
        return f"(({CTYPE[d]})({self.conv(a, da, d)} {op} {self.conv(b, db, d)}))", d

    def call(self, e):
        fn = e.fn
        if fn == "invert":
            a, da = self.expr(e.args[0])
            if da in FLOATS:
                self.fail("Bitwise operations require integer or Boolean operands")
            if da == "bool":
                return f"(!{a})", "bool"
            return f"(({CTYPE[da]})(~({a})))", da
        if fn == "cast":
            (a, da) = self.expr(e.args[0])
            target = e.args[1].value if len(e.args) > 1 else "float32"
            return self.conv(a, da, target), target
        if fn in ("and", "or"):
            (a, da), (b, db) = self.expr(e.args[0]), self.expr(e.args[1])
            if da != "bool" or db != "bool":
                self.fail("Logical operations require Boolean operands")
            return f"({a} {'&&' if fn == 'and' else '||'} {b})", "bool"
        if fn == "not":
            a, da = self.expr(e.args[0])
            if da != "bool":
                self.fail("Logical operations require Boolean operands")
            return f"(!{a})", "bool"
        if fn == "neg":
            a, da = self.expr(e.args[0])
            if da in FLOATS:
                return f"(-{a})", da
            if da == "bool":
                return f"(-(int)({a}))", "int32"
            return f"(({CTYPE[da]})(({UNSIGNED[da]})0 - ({UNSIGNED[da]})({a})))", da
        if fn in ("max", "min", "maximum", "minimum"):
            # max / min ignore a NaN operand (np.fmax / PTX max), maximum / minimum propagate
            # it (np.maximum); both order +0 above -0 (python/ntilang/testing.py:121-124).
            (a, da), (b, db) = self.expr(e.args[0]), self.expr(e.args[1])
            d = promote(da, db)
            x, y = self.conv(a, da, d), self.conv(b, db, d)
            kind = "max" if fn in ("max", "maximum") else "min"
            if d in FLOATS:
                f = ("fmax" if kind == "max" else "fmin") + ("" if d == "float64" else "f")
                code = f"{f}({x}, {y})"
                if fn in ("maximum", "minimum"):
                    code = f"ntl_nan_or({x}, {y}, {code})"
                return code, d
            return f"(({x}) {'>' if kind == 'max' else '<'} ({y}) ? ({x}) : ({y}))", d
        if fn == "abs":
            a, da = self.expr(e.args[0])
            if da in FLOATS:
                return (f"fabs({a})" if da == "float64" else f"fabsf({a})"), da
            if da.startswith("uint") or da == "bool":
                return a, da
            return f"(({a}) < 0 ? ({CTYPE[da]})(({UNSIGNED[da]})0 - ({UNSIGNED[da]})({a})) : ({a}))", da
        if fn in ("isnan", "isinf", "isfinite"):
            a, da = self.expr(e.args[0])
            if da not in FLOATS:
                return ("false" if fn != "isfinite" else "true"), "bool"
            return f"{fn}({a})", "bool"
        if fn in ("pow", "fmod"):
            (a, da), (b, db) = self.expr(e.args[0]), self.expr(e.args[1])
            d = promote(da, db) if fn == "pow" else da
            if d not in FLOATS:
                self.fail(f"T.{fn} requires a floating result dtype")
            cf = fn if d == "float64" else fn + "f"
            return self.round_to(f"{cf}({self.conv(a, da, d)}, {self.conv(b, db, d)})", d), d
        unary = {
            "exp": "exp", "exp2": "exp2", "exp10": "exp10", "log": "log", "log2": "log2", "log10": "log10",
            "log1p": "log1p", "sqrt": "sqrt", "rsqrt": "rsqrt", "sin": "sin", "cos": "cos", "tan": "tan",
            "tanh": "tanh", "erf": "erf", "floor": "floor", "ceil": "ceil", "trunc": "trunc", "round": "rint",
            "nearbyint": "nearbyint",
        }
        if fn in unary or fn in ("sigmoid", "rcp"):
            a, da = self.expr(e.args[0])
            if da not in FLOATS:
                if fn == "exp":
                    a, da = self.conv(a, da, "float32"), "float32"
                else:
                    self.fail(f"T.{fn} requires floating inputs")
            suffix = "" if da == "float64" else "f"
            one = "1.0" if da == "float64" else "1.0f"
            if fn == "sigmoid":
                # 1 / (1 + exp(-x)), every step rounded to the value's type (testing.py:213-216)
                ex = self.round_to(f"exp{suffix}(-({a}))", da)
                code = f"({one} / {self.round_to(f'({one} + {ex})', da)})"
            elif fn == "rcp":
                code = f"({one} / ({a}))"
            else:
                code = f"{unary[fn]}{suffix}({a})"
            return self.round_to(code, da), da
        self.fail(f"unsupported function T.{fn}")

    def load(self, e: Load):
        b = self.buf(e.buf)
        if b.scope == "global":
            codes, dts = zip(*(self.expr(i) for i in e.idx)) if e.idx else ((), ())
            for dt in dts:
                if dt in FLOATS or dt == "bool":
                    self.fail(f"{e.buf}: indices must be integers")
            pred = self.in_bounds(e.buf, e.idx, codes)
            elem = f"p_{_ident(e.buf)}[{self.offset(e.buf, codes)}]"
            slot = self.vec_load(e, codes) if e.buf not in self.stored else None
            if slot is not None:
                elem = f"(vl{slot}_ok ? vl{slot}_v[unit] : {elem})"
            if b.dtype == "float16":
                elem = f"ntl_h2f({elem})"
            elif b.dtype == "bfloat16":
                elem = f"ntl_b2f({elem})"
            if pred:
                zero = self.conv("0", "int32", b.dtype)
                if slot is not None:
                    return f"(vl{slot}_ok || ({pred}) ? {elem} : {zero})", b.dtype
                return f"(({pred}) ? {elem} : {zero})", b.dtype
            return elem, b.dtype
        if b.scope == "var":
            return f"v_{_ident(e.buf)}", b.dtype
        self.check_slot_access(e.buf, e.idx)
        return f"f_{_ident(e.buf)}", b.dtype

    # ------------------------------------------------------------- fragments
    def check_slot_access(self, name, idx):
        shape = self.fragments.get(name)
        if shape is None:
            self.fail(f"{name} is not allocated before use")
        par = self.current_parallel
        ok = (par is not None and tuple(par.extents) == tuple(shape) and len(idx) == len(par.vars)
              and all(isinstance(i, Var) and i.name == v for i, v in zip(idx, par.vars)))
        if not ok:
            self.fail(f"fragment {name} must be accessed at the coordinates of a T.Parallel loop of its shape "
                      f"{tuple(shape)} (the per-thread slot mapping)")

    # ------------------------------------------------------------- statements
    def stmts(self, body):
        for s in body:
            self.stmt(s)

    def stmt(self, s):
        if isinstance(s, Alloc):
            if s.scope == "var":
                self.types[s.name] = s.dtype
                self.mutable_scope[s.name] = self.parallel_level
                self.emit(f"{CTYPE[s.dtype]} v_{_ident(s.name)} = 0;")
                return
            if s.scope in ("fragment", "shared"):
                if any(isinstance(d, SymDim) for d in s.shape):
                    self.fail(f"fragment {s.name} needs a static shape")
                self.fragments[s.name] = tuple(s.shape)
                self.points = max(self.points, math.prod(s.shape))
                self.emit(f"{CTYPE[s.dtype]} f_{_ident(s.name)} = 0;")
                return
            self.fail(f"unsupported allocation scope {s.scope!r}")
        if isinstance(s, Parallel):
            self.parallel(s)
            return
        if isinstance(s, Loop):
            (a, da), (b, db) = self.expr(s.start), self.expr(s.stop)
            step = s.step if s.step is not None else Const(1)
            c, dc = self.expr(step)
            if da in FLOATS or db in FLOATS or dc in FLOATS:
                self.fail("loop bounds must be integers")
            d = promote(promote(promote(da, db), dc), "int32")
            v = _ident(s.var)
            self.types[s.var] = d
            lo, hi = self.interval(s.start), self.interval(s.stop)
            if s.step is None and lo is not None and hi is not None:
                self.ranges[s.var] = (lo[0], hi[1] - 1)
            else:
                self.ranges.pop(s.var, None)
            # Bounds and step are evaluated once, before the first iteration (a Python range).
            init = f"{CTYPE[d]} v_{v} = {self.conv(a, da, d)}, e_{v} = {self.conv(b, db, d)}"
            if s.step is None:
                head = f"for ({init}; v_{v} < e_{v}; ++v_{v}) {{"
            elif isinstance(step, Const):
                cmp = "<" if step.value > 0 else ">"
                head = f"for ({init}; v_{v} {cmp} e_{v}; v_{v} += {self.conv(c, dc, d)}) {{"
            else:  # a runtime step: its sign picks the test; 0 runs no iteration
                head = (f"for ({init}, t_{v} = {self.conv(c, dc, d)}; (t_{v} > 0 && v_{v} < e_{v}) || "
                        f"(t_{v} < 0 && v_{v} > e_{v}); v_{v} += t_{v}) {{")
            self.emit(head)
            self.depth += 1
            self.loops.append("serial")
            self.stmts(s.body)
            self.loops.pop()
            self.depth -= 1
            self.emit("}")
            return
        if isinstance(s, While):
            c, dc = self.expr(s.cond)
            self.emit(f"while ({self.conv(c, dc, 'bool')}) {{")
            self.depth += 1
            self.loops.append("serial")
            self.stmts(s.body)
            self.loops.pop()
            self.depth -= 1
            self.emit("}")
            return
        if isinstance(s, (Break, Continue)):
            if not self.loops or self.loops[-1] != "serial":
                self.fail("break / continue must be inside a serial loop (T.serial, T.grid, range, while), "
                          "not directly in T.Parallel")
            self.emit("break;" if isinstance(s, Break) else "continue;")
            return
        if isinstance(s, If):
            c, dc = self.expr(s.cond)
            self.emit(f"if ({self.conv(c, dc, 'bool')}) {{")
            self.depth += 1
            self.stmts(s.then)
            self.depth -= 1
            if s.orelse:
                self.emit("} else {")
                self.depth += 1
                self.stmts(s.orelse)
                self.depth -= 1
            self.emit("}")
            return
        if isinstance(s, Let):
            if s.name not in self.mutable_scope:
                self.fail(f"{s.name!r} is reassigned; declare it with T.alloc_var")
            if self.mutable_scope[s.name] < self.parallel_level:
                self.fail(f"{s.name!r} is declared outside a T.Parallel loop and assigned inside it: a reduction "
                          "across parallel points (use T.reduce_*)")
            code, d = self.expr(s.value)
            self.emit(f"v_{_ident(s.name)} = {self.conv(code, d, self.types[s.name])};")
            return
        if isinstance(s, Store):
            self.store(s.buf, s.idx, s.value, top=s is self.top_stmt)
            return
        if isinstance(s, Atomic):
            self.atomic(s)
            return
        if isinstance(s, (Copy, Fill)) and self.current_parallel is not None:
            self.fail("Collective T.copy / T.fill / T.clear inside T.Parallel (each point would run it)")
        if isinstance(s, Copy):
            self.copy(s)
            return
        if isinstance(s, Fill):
            b = self.buf(s.buf)
            if b.scope == "var":
                self.emit(f"v_{_ident(s.buf)} = {self.conv(_c_literal(s.value, 'float32'), 'float32', b.dtype)};")
                return
            if b.scope == "global":
                self.fail("T.fill / T.clear of a global tensor")
            shape = self.fragments[s.buf]
            with self._points(math.prod(shape)):
                self.emit(f"f_{_ident(s.buf)} = {self.conv(_c_literal(s.value, 'float32'), 'float32', b.dtype)};")
            return
        if isinstance(s, Hint):
            return
        if isinstance(s, (Reduce, Scan, Gemm)):
            self.fail(f"T.{type(s).__name__.lower()} is not elementwise (no recognised op family matched)")
        self.fail(f"unsupported statement {type(s).__name__}")

    class _PointsGuard:
        """`if (pt < n) { ... }`: the statements run for the first n points of a block instance."""

        def __init__(self, low, n):
            self.low, self.n = low, n

        def __enter__(self):
            low = self.low
            low.points = max(low.points, self.n)
            low.guards.append(self.n)
            low.guard_sizes.append(self.n)
            low.emit(f"if (pt < {self.n}LL) {{")
            low.depth += 1

        def __exit__(self, *exc):
            self.low.depth -= 1
            self.low.emit("}")
            self.low.guards.pop()

    def _points(self, n):
        return self._PointsGuard(self, n)

    def parallel(self, s: Parallel):
        if self.current_parallel is not None:
            self.fail("nested T.Parallel loops")
        # Every global store of one T.Parallel loop to a tensor must use the same index (each
        # point owns its element), or two points could write one element.
        owners: dict = {}

        def own(stmts):
            for t in stmts:
                if isinstance(t, Store) and self.buf(t.buf).scope == "global":
                    if owners.setdefault(t.buf, t.idx) != t.idx:
                        self.fail(f"stores to {t.buf} in one T.Parallel loop need identical ownership "
                                  "(the same index expression)")
                for attr in ("body", "then", "orelse"):
                    own(getattr(t, attr, ()))

        own(s.body)
        n = math.prod(s.extents)
        saved = dict(self.ranges)
        with self._points(n):
            stride = n
            for v, ext in zip(s.vars, s.extents):
                stride //= ext
                self.types[v] = "int32"
                self.ranges[v] = (0, ext - 1)
                code = "(int)pt" if stride == 1 else f"(int)(pt / {stride}LL)"
                if stride * ext != n:
                    code = f"({code} % {ext})"
                self.emit(f"const int v_{_ident(v)} = {code};")
            self.current_parallel = s
            self.parallel_level += 1
            self.loops.append("parallel")
            for t in s.body:
                self.top_stmt = t
                self.stmt(t)
            self.top_stmt = None
            self.loops.pop()
            self.parallel_level -= 1
            self.current_parallel = None
        self.ranges = saved

    def store(self, name, idx, value, top=False):
        b = self.buf(name)
        code, d = self.expr(value)
        if b.scope == "var":
            self.emit(f"v_{_ident(name)} = {self.conv(code, d, b.dtype)};")
            return
        if b.scope != "global":
            self.check_slot_access(name, idx)
            self.emit(f"f_{_ident(name)} = {self.conv(code, d, b.dtype)};")
            return
        codes = [self.expr(i)[0] for i in idx]
        pred = self.in_bounds(name, idx, codes)
        val = self.conv(code, d, b.dtype)
        if b.dtype == "float16":
            val = f"ntl_f2h({val})"
        elif b.dtype == "bfloat16":
            val = f"ntl_f2b({val})"
        line = f"p_{_ident(name)}[{self.offset(name, codes)}] = {val};"
        guard = pred
        if self.current_parallel is None and not self.guards:
            guard = f"pt == 0" + (f" && {pred}" if pred else "")  # one writer per block instance
        slot = self.vec_store(name, idx, codes) if top and name not in self.loaded else None
        if slot is not None:
            self.emit(f"if (vs{slot}_ok) vs{slot}_v[unit] = {val};")
            self.emit(f"else if ({guard}) {line}" if guard else f"else {line}")
            return
        self.emit(f"if ({guard}) {line}" if guard else line)

    def atomic(self, s: Atomic):
        b = self.buf(s.buf)
        if b.scope != "global":
            self.fail("atomics need a global tensor")
        allowed = {"add": ("float32", "float64", "int32", "uint32", "uint64"),
                   "max": ("int32", "uint32", "int64", "uint64"), "min": ("int32", "uint32", "int64", "uint64")}
        if b.dtype not in allowed[s.op]:
            self.fail(f"T.atomic_{s.op} on {b.dtype} is not supported")
        code, d = self.expr(s.value)
        codes = [self.expr(i)[0] for i in s.idx]
        pred = self.in_bounds(s.buf, s.idx, codes)
        fn = {"add": "atomicAdd", "max": "atomicMax", "min": "atomicMin"}[s.op]
        line = f"{fn}(&p_{_ident(s.buf)}[{self.offset(s.buf, codes)}], {self.conv(code, d, b.dtype)});"
        guard = pred
        if self.current_parallel is None and not self.guards:
            guard = "pt == 0" + (f" && {pred}" if pred else "")
        self.emit(f"if ({guard}) {line}" if guard else line)

    def copy(self, s: Copy):
        src, dst = s.src, s.dst
        sb, db = self.buf(src.buf), self.buf(dst.buf)
        if sb.scope not in ("global", "fragment", "shared") or db.scope not in ("global", "fragment", "shared"):
            self.fail("T.copy between unsupported buffers")
        # The copy's shape: a fragment side's shape, else the non-point region's extents.
        if sb.scope != "global":
            shape = self.fragments[src.buf]
        elif db.scope != "global":
            shape = self.fragments[dst.buf]
        elif not src.point:
            shape = tuple(e for e in src.extents)
        elif not dst.point:
            shape = tuple(e for e in dst.extents)
        else:
            self.fail("T.copy between two tile origins needs an extent")
        for side in (src, dst):
            b = self.buf(side.buf)
            if b.scope != "global" and not side.point and tuple(side.extents) != tuple(shape):
                self.fail(f"T.copy must cover the whole fragment {side.buf}")
            if b.scope != "global" and side.point and any(not (isinstance(x, Const) and x.value == 0)
                                                            for x in side.starts):
                self.fail(f"T.copy into fragment {side.buf} at an offset")
        if any(isinstance(x, SymDim) or x is None for x in shape):
            self.fail("T.copy needs a static extent")
        n = math.prod(shape)
        with self._points(n):
            coords = []
            stride = n
            for ext in shape:
                stride //= ext
                c = "pt" if stride == 1 else f"(pt / {stride}LL)"
                if stride * ext != n:
                    c = f"({c} % {ext}LL)"
                coords.append(c)

            def global_index(region):
                """Per buffer dim: (Expr or None for the interval check, C index) of this point."""
                rank = len(self.buf(region.buf).shape)
                if region.point:
                    if len(shape) > rank:
                        self.fail(f"T.copy shape {tuple(shape)} has more dims than {region.buf}")
                    mapped = dict(zip(range(rank - len(shape), rank), zip(coords, shape)))  # trailing dims
                elif len(region.extents) == len(shape):
                    mapped = dict(zip(range(rank), zip(coords, shape)))
                else:
                    axes = [k for k, ext in enumerate(region.extents) if ext != 1]
                    squeezed = [(c, ext) for ext, c in zip(shape, coords) if ext != 1]
                    if len(axes) != len(squeezed):
                        self.fail(f"T.copy region of {region.buf} does not match the copy shape {tuple(shape)}")
                    mapped = dict(zip(axes, squeezed))
                out_e, out_c = [], []
                for k in range(rank):
                    start_code, start_dt = self.expr(region.starts[k])
                    if start_dt in FLOATS or start_dt == "bool":
                        self.fail(f"{region.buf}: indices must be integers")
                    if k in mapped:
                        c, ext = mapped[k]
                        out_c.append(f"((long long)({start_code}) + {c})")
                        iv = self.interval(region.starts[k])
                        out_e.append(None if iv is None else (iv[0], iv[1] + ext - 1))
                    else:
                        out_c.append(f"(long long)({start_code})")
                        out_e.append(region.starts[k])
                return out_e, out_c

            if sb.scope == "global":
                e_idx, c_idx = global_index(src)
                pred = self.in_bounds(src.buf, e_idx, c_idx)
                elem = f"p_{_ident(src.buf)}[{self.offset(src.buf, c_idx)}]"
                if sb.dtype == "float16":
                    elem = f"ntl_h2f({elem})"
                elif sb.dtype == "bfloat16":
                    elem = f"ntl_b2f({elem})"
                value = f"(({pred}) ? {elem} : {self.conv('0', 'int32', sb.dtype)})" if pred else elem
            else:
                value = f"f_{_ident(src.buf)}"
            if db.scope == "global":
                e_idx, c_idx = global_index(dst)
                pred = self.in_bounds(dst.buf, e_idx, c_idx)
                val = self.conv(value, sb.dtype, db.dtype)
                if db.dtype == "float16":
                    val = f"ntl_f2h({val})"
                elif db.dtype == "bfloat16":
                    val = f"ntl_f2b({val})"
                line = f"p_{_ident(dst.buf)}[{self.offset(dst.buf, c_idx)}] = {val};"
                self.emit(f"if ({pred}) {line}" if pred else line)
            else:
                self.emit(f"f_{_ident(dst.buf)} = {self.conv(value, sb.dtype, db.dtype)};")


def _ident(name: str) -> str:
    return re.sub(r"[^0-9A-Za-z_]", "_", name)


def _lower_body(prog: Program, vec: bool) -> _Lowering:
    low = _Lowering(prog, vec=vec)
    low.depth = 2
    low.stmts(prog.body)
    return low


def lower(prog: Program) -> PointwiseKernel:
    """Lower ``prog`` to CUDA C or raise ``CompileError`` when it is not elementwise."""
    low = _lower_body(prog, vec=False)
    if low.points % 4 == 0 and all(n % 4 == 0 for n in low.guard_sizes):
        vlow = _lower_body(prog, vec=True)
        if vlow.vec_count:
            low = vlow
    vec = low.vec
    body = low.lines
    name = f"ntl_pw_{_ident(prog.name)}"
    params = []
    stored = set()

    def scan(stmts):
        for s in stmts:
            if isinstance(s, (Store, Atomic)):
                stored.add(s.buf)
            elif isinstance(s, Copy):
                stored.add(s.dst.buf)
            for attr in ("body", "then", "orelse"):
                if hasattr(s, attr):
                    scan(getattr(s, attr))

    scan(prog.body)
    for p in prog.params:
        if isinstance(p, ScalarParameter):
            params.append(f"{CTYPE[p.dtype]} v_{_ident(p.name)}")
        else:
            const = "" if p.name in stored else "const "
            params.append(f"{const}{STORAGE[p.type.dtype]}* __restrict__ p_{_ident(p.name)}")
    params += [f"long long s_{_ident(s)}" for s in low.sym_names]
    params += [f"long long g_{i}" for i in low.grid_args]
    params.append("long long total")
    points = low.points
    head = [
        f"// {name}: lowered from `{prog.name}` by ntilang_b200.pointwise (one thread per",
        "// (block instance, T.Parallel point); loads outside a tensor read 0, stores outside it are skipped)",
        _PRELUDE.strip("\n"),
        "",
        f'extern "C" __global__ void __launch_bounds__({BLOCK_THREADS}) {name}(',
        "    " + ",\n    ".join(params) + ") {",
    ]
    if vec:  # thread t: points 4t .. 4t+3 of the CTA's run (a group never straddles a block instance)
        head += [f"  const long long gbase = (long long)blockIdx.x * {BLOCK_THREADS * POINTS_PER_THREAD} + "
                 f"(long long)threadIdx.x * {POINTS_PER_THREAD};"]
        head += [f"  {d}" for d in low.vec_decls]
    else:  # thread t: points t, t + 256, t + 512, t + 768 (each run coalesced)
        head += [f"  const long long gbase = (long long)blockIdx.x * {BLOCK_THREADS * POINTS_PER_THREAD} + threadIdx.x;"]
    head += [
        "#pragma unroll",
        f"  for (int unit = 0; unit < {POINTS_PER_THREAD}; ++unit) {{",
        f"  const long long gid = gbase + (long long)unit * {1 if vec else BLOCK_THREADS};",
        "  if (gid >= total) break;",
        f"  const long long pt = gid % {points}LL;",
        f"  long long blk = gid / {points}LL;",
    ]
    for i, (bv, g) in enumerate(zip(prog.block_vars, prog.grid)):
        ext = f"g_{i}" if i in low.grid_args else f"{int(g.value) if isinstance(g, Const) else int(g)}LL"
        last = i == len(prog.grid) - 1
        head.append(f"  const int v_{_ident(bv)} = (int)({'blk' if last else f'(blk % {ext})'});")
        if not last:
            head.append(f"  blk /= {ext};")
    head.append("  (void)pt; (void)blk;")
    head.append("  {")
    tail = ["  }", "  }"] + [f"  {f}" for f in low.vec_flush] + ["}", ""]
    source = "\n".join(head + body + tail)
    return PointwiseKernel(name=name, source=source, program=prog, sym_names=low.sym_names, grid=tuple(prog.grid),
                           grid_args=tuple(low.grid_args), points=points)


def validate_scalar(value, param: ScalarParameter):
    """Host check of a scalar argument (python/ntilang/runtime.py:29-46): bool needs a Python
    bool, integer dtypes an integer in range, floating dtypes a real number."""
    from numbers import Integral, Real

    name, dtype = param.name, param.dtype
    if dtype == "bool":
        if type(value) is not bool:
            raise TypeError(f"{name} requires a Python bool")
        return value
    if dtype.startswith(("int", "uint")):
        if not isinstance(value, Integral) or isinstance(value, bool):
            raise TypeError(f"{name} requires an integer scalar for {dtype}")
        value = int(value)
        low, high = integer_limits(dtype)
        if not low <= value <= high:
            raise ValueError(f"{name}: {value} is outside the {dtype} range [{low}, {high}]")
        return value
    if not isinstance(value, Real) or isinstance(value, bool):
        raise TypeError(f"{name} requires a real scalar for {dtype}")
    return float(value)


__all__ = ["PointwiseKernel", "lower", "promote", "validate_scalar"]
