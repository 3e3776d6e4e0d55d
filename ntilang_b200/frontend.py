"""Restricted-AST reader: ``@T.prim_func`` -> a small statement tree the recognizer matches.

The reference parses the full TileLang language into its tile IR
(``python/ntilang/frontend.py:2010-2186``) and lowers every statement.  This package
does not lower arbitrary programs; it only needs enough structure to recognise the op
families its sm_100a kernels implement (``ntilang_b200.recognize``).  So this reader:

* evaluates everything static (factory arguments, ``T.ceildiv``, ``math.*``, static
  ``if`` / conditional expressions) in the function's globals + captured caller locals +
  closure, like the reference's annotation/closure environment (``language.py:191-217``);
* keeps kernel-time expressions (block indices, loop / parallel variables, buffer loads)
  as a tiny expression tree;
* turns ``T.copy / T.gemm / T.reduce_* / T.cumsum / T.fill / T.clear`` calls, ``T.Parallel``
  / ``T.Pipelined`` / ``T.serial`` loops and element stores into statement nodes.
"""

from __future__ import annotations

import ast
import builtins
import inspect
import math
import textwrap
from dataclasses import dataclass, field

from .ir import CompileError, ScalarParameter, SourceLocation, SymDim, TensorParameter, TensorType, canonical_dtype
from .language import DType, PrimFunc, SymbolicDim, SymbolicTensorSpec

# ----------------------------------------------------------------------------- expressions


@dataclass(frozen=True)
class Const:
    value: object


@dataclass(frozen=True)
class Var:
    name: str


@dataclass(frozen=True)
class Load:
    buf: str
    idx: tuple


@dataclass(frozen=True)
class Bin:
    op: str  # + - * / // %
    a: object
    b: object


@dataclass(frozen=True)
class Cmp:
    op: str  # < <= > >= == !=
    a: object
    b: object


@dataclass(frozen=True)
class Call:
    fn: str  # exp exp2 rsqrt sqrt max min abs neg cast ...
    args: tuple


@dataclass(frozen=True)
class Select:
    cond: object
    a: object
    b: object


# ------------------------------------------------------------------------------ statements


@dataclass
class Region:
    buf: str
    starts: tuple  # Expr per dim
    extents: tuple  # int per dim, or None when the other copy side decides
    point: bool = False  # written as A[i, j] (a tile origin) rather than a slice/whole buffer


@dataclass
class Alloc:
    name: str
    scope: str
    shape: tuple
    dtype: str


@dataclass
class Copy:
    src: Region
    dst: Region


@dataclass
class Gemm:
    a: str
    b: str
    c: str
    transpose_a: bool
    transpose_b: bool
    clear_accum: bool


@dataclass
class Fill:
    buf: str
    value: float


@dataclass
class Reduce:
    kind: str
    src: str
    dst: str
    dim: int
    clear: bool


@dataclass
class Scan:
    kind: str
    src: Region
    dst: Region
    dim: int
    reverse: bool


@dataclass
class Parallel:
    vars: tuple
    extents: tuple
    body: list


@dataclass
class Loop:
    var: str
    start: object
    stop: object
    kind: str  # serial | pipelined | unroll
    stages: int
    body: list
    step: object = None  # None: 1


@dataclass
class Store:
    buf: str
    idx: tuple
    value: object


@dataclass
class Atomic:
    op: str  # add | max | min
    buf: str
    idx: tuple
    value: object


@dataclass
class Let:
    """Assignment to a mutable kernel scalar (``T.alloc_var``), or a loop-carried update."""

    name: str
    value: object


@dataclass
class If:
    cond: object
    then: list
    orelse: list


@dataclass
class While:
    cond: object
    body: list


@dataclass
class Break:
    pass


@dataclass
class Continue:
    pass


@dataclass
class Hint:
    kind: str
    args: dict = field(default_factory=dict)


@dataclass
class Program:
    name: str
    params: tuple  # TensorParameter | ScalarParameter
    grid: tuple  # int or Expr (symbolic)
    block_vars: tuple
    threads: int
    buffers: dict  # name -> Alloc (params included with scope "global")
    body: list
    source: str
    sym_dims: tuple = ()

    def param(self, name):
        for p in self.params:
            if p.name == name:
                return p
        return None


class NotStatic(Exception):
    pass


_LANGUAGE_MODULE = PrimFunc.__module__

_MATH_FUNCS = {
    "exp": "exp", "exp2": "exp2", "__exp": "exp", "log": "log", "log2": "log2", "sqrt": "sqrt",
    "rsqrt": "rsqrt", "abs": "abs", "maximum": "maximum", "max": "max", "minimum": "minimum", "min": "min",
    "tanh": "tanh", "sigmoid": "sigmoid", "fast_rcp": "rcp", "erf": "erf", "exp10": "exp10",
    "log10": "log10", "log1p": "log1p", "sin": "sin", "cos": "cos", "tan": "tan", "floor": "floor",
    "ceil": "ceil", "trunc": "trunc", "round": "round", "nearbyint": "nearbyint", "isnan": "isnan",
    "isinf": "isinf", "isfinite": "isfinite", "pow": "pow", "fmod": "fmod", "clamp": "clamp",
    "floordiv": "//", "floormod": "%", "truncdiv": "truncdiv", "truncmod": "truncmod",
    "bitwise_and": "&", "bitwise_or": "|", "bitwise_xor": "^", "shift_left": "<<", "shift_right": ">>",
    "bitwise_not": "invert",
}
_ATOMICS = {"atomic_add": "add", "atomic_max": "max", "atomic_min": "min"}

_COPY_LIKE = {"copy"}
_REDUCE_KINDS = {
    "reduce_sum": "sum", "reduce_max": "max", "reduce_min": "min", "reduce_abssum": "abssum",
    "reduce_absmax": "absmax",
}


class _Reader:
    def __init__(self, program: PrimFunc):
        self.program = program
        fn = program.function
        try:
            raw = inspect.getsource(fn)
        except (OSError, TypeError) as exc:
            raise CompileError(f"Kernel source for {fn.__name__} is unavailable") from exc
        self.source = textwrap.dedent(raw)
        self.filename = inspect.getsourcefile(fn) or "<kernel>"
        self.line_offset = (inspect.getsourcelines(fn)[1] - 1) if hasattr(fn, "__code__") else 0
        tree = ast.parse(self.source)
        defs = [n for n in tree.body if isinstance(n, (ast.FunctionDef, ast.AsyncFunctionDef))]
        if not defs:
            raise CompileError("prim_func source does not contain a function definition")
        self.fdef = defs[0]
        env = dict(fn.__globals__)
        env.update(dict(program.annotation_locals))
        try:
            env.update(inspect.getclosurevars(fn).nonlocals)
        except (TypeError, ValueError):
            pass
        for cell_name, cell in zip(fn.__code__.co_freevars, fn.__closure__ or ()):
            try:
                env[cell_name] = cell.cell_contents
            except ValueError:
                pass
        self.env = env
        # T.dynamic specialisation: symbolic name -> concrete value
        self.special = dict(program.specializations)
        self.kernel_names: set = set()  # names bound at kernel time (shadow env)
        self.lets: dict = {}  # kernel-scope name -> Expr (immutable binding, substituted at each use)
        self.let_paths: dict = {}  # name -> control-flow path of its binding
        self.path: list = []  # ids of the enclosing if-branches / loop bodies
        self._next_block = 0
        self.mutables: dict = {}  # T.alloc_var name -> dtype
        self.buffers: dict = {}
        self.sym_dims: dict = {}

    # -------------------------------------------------------------------- helpers
    def loc(self, node):
        return SourceLocation(self.filename, getattr(node, "lineno", 0) + self.line_offset, getattr(node, "col_offset", 0))

    def fail(self, node, msg):
        raise CompileError(msg, self.loc(node) if node is not None else None)

    def is_T(self, node, *names):
        """True when ``node`` is ``T.<name>`` / ``tilelang.language.<name>`` / a bare marker name."""
        if isinstance(node, ast.Attribute) and node.attr in names:
            return True
        if isinstance(node, ast.Name) and node.id in names and node.id not in self.kernel_names:
            value = self.env.get(node.id)
            return callable(value) and getattr(value, "__name__", None) == node.id
        return False

    def call_name(self, node):
        """The T.* (or builtin) name a call refers to.  A bare name bound in the environment to a
        marker or to ``range`` (``loop = T.serial``, ``stop = T.loop_break``) resolves to it."""
        if isinstance(node, ast.Call):
            f = node.func
            if isinstance(f, ast.Attribute):
                return f.attr
            if isinstance(f, ast.Name):
                if f.id not in self.kernel_names and f.id in self.env:
                    value = self.env[f.id]
                    if value is builtins.range:
                        return "range"
                    marker = getattr(value, "__qualname__", None)
                    if callable(value) and getattr(value, "__module__", "") == _LANGUAGE_MODULE and marker:
                        return marker
                return f.id
        return None

    # ------------------------------------------------------------- static values
    def static(self, node):
        if isinstance(node, ast.Constant):
            return node.value
        if isinstance(node, ast.Name):
            if node.id in self.kernel_names or node.id in self.lets:
                raise NotStatic(node.id)
            if node.id in self.special:
                return self.special[node.id]
            if node.id in self.env:
                value = self.env[node.id]
                if isinstance(value, SymbolicDim) and value.name in self.special:
                    return self.special[value.name]
                return value
            if hasattr(builtins, node.id):
                return getattr(builtins, node.id)
            raise NotStatic(node.id)
        if isinstance(node, ast.Attribute):
            base = self.static(node.value)
            try:
                return getattr(base, node.attr)
            except AttributeError as exc:
                raise NotStatic(node.attr) from exc
        if isinstance(node, ast.Tuple) or isinstance(node, ast.List):
            return tuple(self.static(e) for e in node.elts)
        if isinstance(node, ast.Dict):
            return {self.static(k): self.static(v) for k, v in zip(node.keys, node.values)}
        if isinstance(node, ast.UnaryOp):
            v = self.static(node.operand)
            if isinstance(node.op, ast.USub):
                return -v
            if isinstance(node.op, ast.UAdd):
                return +v
            if isinstance(node.op, ast.Not):
                return not v
            if isinstance(node.op, ast.Invert):
                return ~v
        if isinstance(node, ast.BinOp):
            a, b = self.static(node.left), self.static(node.right)
            if isinstance(a, SymbolicDim) or isinstance(b, SymbolicDim):
                raise NotStatic("symbolic")
            return _BINOPS[type(node.op)](a, b)
        if isinstance(node, ast.Compare) and len(node.ops) == 1:
            a, b = self.static(node.left), self.static(node.comparators[0])
            return _CMPOPS[type(node.ops[0])](a, b)
        if isinstance(node, ast.BoolOp):
            vals = [self.static(v) for v in node.values]
            return all(vals) if isinstance(node.op, ast.And) else any(vals)
        if isinstance(node, ast.IfExp):
            return self.static(node.body) if self.static(node.test) else self.static(node.orelse)
        if isinstance(node, ast.Subscript):
            base = self.static(node.value)
            return base[self.static(node.slice)]
        if isinstance(node, ast.Call):
            name = self.call_name(node)
            if name in ("ceildiv", "cdiv"):
                a, b = (self.static(x) for x in node.args[:2])
                if isinstance(a, SymbolicDim) or isinstance(b, SymbolicDim):
                    raise NotStatic("symbolic")
                return (a + b - 1) // b
            if name == "infinity":
                return float("inf")
            func = self.static(node.func)
            if func is None:
                raise NotStatic("call")
            module = getattr(func, "__module__", "") or ""
            allowed = (
                module in ("math", "builtins", "numpy")
                or func in (float, int, abs, min, max, round, len, bool, pow)
                or isinstance(func, type) and issubclass(func, DType)
                or module.endswith(".language") and name in ("Tensor", "dynamic", "ceildiv", "infinity", "align_up")
            )
            if not allowed:
                raise NotStatic(name or "call")
            args = [self.static(a) for a in node.args]
            kwargs = {k.arg: self.static(k.value) for k in node.keywords}
            return func(*args, **kwargs)
        raise NotStatic(type(node).__name__)

    def try_static(self, node):
        try:
            return True, self.static(node)
        except NotStatic:
            return False, None
        except (TypeError, ValueError, ZeroDivisionError, KeyError, IndexError, AttributeError):
            return False, None

    # --------------------------------------------------------------- expressions
    def expr(self, node):
        ok, value = self.try_static(node)
        if ok and isinstance(value, (int, float, bool)):
            return Const(value)
        if ok and isinstance(value, SymbolicDim):
            self.sym_dims[value.name] = SymDim(value.name)
            return Var(f"$sym:{value.name}")
        if isinstance(node, ast.Name):
            if node.id in self.mutables:
                return Var(node.id)
            if node.id in self.lets:
                bound = self.let_paths.get(node.id, ())
                if tuple(self.path[:len(bound)]) != bound:
                    self.fail(node, f"{node.id!r} is used outside its defining region (it is assigned inside a "
                                    "branch or loop body); declare it with T.alloc_var")
                return self.lets[node.id]
            if node.id in self.kernel_names:
                return Var(node.id)
            self.fail(node, f"Unknown name {node.id!r} in kernel expression")
        if isinstance(node, ast.BoolOp):
            fn = "and" if isinstance(node.op, ast.And) else "or"
            out = self.expr(node.values[0])
            for v in node.values[1:]:
                out = Call(fn, (out, self.expr(v)))
            return out
        if isinstance(node, ast.BinOp):
            op = _BINSYM.get(type(node.op))
            if op is None:
                self.fail(node, "Unsupported binary operator")
            return Bin(op, self.expr(node.left), self.expr(node.right))
        if isinstance(node, ast.UnaryOp):
            if isinstance(node.op, ast.USub):
                inner = self.expr(node.operand)
                if isinstance(inner, Const):
                    return Const(-inner.value)
                return Call("neg", (inner,))
            if isinstance(node.op, ast.UAdd):
                return self.expr(node.operand)
            if isinstance(node.op, ast.Not):
                return Call("not", (self.expr(node.operand),))
            if isinstance(node.op, ast.Invert):
                return Call("invert", (self.expr(node.operand),))
            self.fail(node, "Unsupported unary operator")
        if isinstance(node, ast.Compare) and len(node.ops) == 1:
            return Cmp(_CMPSYM[type(node.ops[0])], self.expr(node.left), self.expr(node.comparators[0]))
        if isinstance(node, ast.IfExp):
            ok, test = self.try_static(node.test)
            if ok:
                return self.expr(node.body) if test else self.expr(node.orelse)
            return Select(self.expr(node.test), self.expr(node.body), self.expr(node.orelse))
        if isinstance(node, ast.Subscript):
            buf = self.buffer_name(node.value)
            idx = self.index_list(node.slice)
            if any(isinstance(i, slice) for i in idx):
                self.fail(node, "Slices are only allowed in copy regions")
            return Load(buf, tuple(idx))
        if isinstance(node, ast.Call):
            name = self.call_name(node)
            if name == "cast":
                kw = {k.arg: k.value for k in node.keywords}
                target = node.args[1] if len(node.args) > 1 else kw.get("dtype")
                if target is None or not node.args:
                    self.fail(node, "T.cast needs a value and a dtype")
                return Call("cast", (self.expr(node.args[0]), Const(canonical_dtype(str(self.static(target))))))
            args = [self.expr(a) for a in node.args]
            if name in ("if_then_else", "Select"):
                return Select(*args)
            if name in ("ceildiv", "cdiv") and len(args) == 2:
                return Bin("//", Bin("+", args[0], Bin("-", args[1], Const(1))), args[1])
            if name == "clamp":  # min(max(value, low), high), as the reference reads it (frontend.py:1098-1102)
                kwe = {k.arg: self.expr(k.value) for k in node.keywords}
                names = ("dst", "min_val", "max_val")
                vals = list(args) + [kwe[n] for n in names[len(args):] if n in kwe]
                if len(vals) != 3:
                    self.fail(node, "T.clamp takes (value, min_val, max_val)")
                return Call("min", (Call("max", (vals[0], vals[1])), vals[2]))
            if name in _MATH_FUNCS:
                fn = _MATH_FUNCS[name]
                if fn in ("//", "%", "&", "|", "^", "<<", ">>"):
                    return Bin(fn, *args)
                return Call(fn, tuple(args))
            if name in _DTYPE_CALLS:
                return Call("cast", (args[0], Const(_DTYPE_CALLS[name])))
            if name == "likely":
                return args[0]
            self.fail(node, f"Unsupported call {name!r} in kernel expression")
        self.fail(node, f"Unsupported expression {type(node).__name__}")

    def buffer_name(self, node):
        if isinstance(node, ast.Name) and node.id in self.buffers:
            return node.id
        self.fail(node, "Expected a tensor parameter or allocated buffer")

    def index_list(self, node):
        elts = node.elts if isinstance(node, ast.Tuple) else [node]
        out = []
        for e in elts:
            if isinstance(e, ast.Slice):
                lo = self.expr(e.lower) if e.lower is not None else None
                hi = self.expr(e.upper) if e.upper is not None else None
                if e.step is not None:
                    self.fail(e, "Strided slices are not supported")
                out.append(slice(lo, hi))
            else:
                out.append(self.expr(e))
        return out

    def region(self, node):
        """A copy/scan operand: whole buffer, a slice region or a tile origin A[i, j]."""
        if isinstance(node, ast.Name):
            buf = self.buffer_name(node)
            shape = self.buffers[buf].shape
            return Region(buf, tuple(Const(0) for _ in shape), tuple(shape))
        if isinstance(node, ast.Subscript):
            buf = self.buffer_name(node.value)
            shape = self.buffers[buf].shape
            idx = self.index_list(node.slice)
            if len(idx) != len(shape):
                self.fail(node, f"{buf} has rank {len(shape)}, indexed with {len(idx)} subscripts")
            if not any(isinstance(i, slice) for i in idx):
                return Region(buf, tuple(idx), tuple(None for _ in idx), point=True)
            starts, extents = [], []
            for dim, i in enumerate(idx):
                if isinstance(i, slice):
                    lo = i.start if i.start is not None else Const(0)
                    if i.stop is None:
                        ext = shape[dim] if not isinstance(lo, Const) or lo.value == 0 else shape[dim] - lo.value
                    else:
                        diff = simplify(Bin("-", i.stop, lo))
                        if not isinstance(diff, Const):
                            self.fail(node, "Slice extents must be static")
                        ext = diff.value
                    starts.append(lo)
                    extents.append(ext)
                else:
                    starts.append(i)
                    extents.append(1)
            return Region(buf, tuple(starts), tuple(extents))
        self.fail(node, "Expected a buffer region")

    # ------------------------------------------------------------------ parameters
    def params(self):
        params = []
        for arg in self.fdef.args.args:
            ann = self.program.function.__annotations__.get(arg.arg)
            if isinstance(ann, str) and not isinstance(ann, DType):
                try:
                    ann = eval(ann, dict(self.env))  # noqa: S307 - annotation strings of the user's own kernel
                except Exception as exc:
                    raise CompileError(f"Cannot evaluate annotation of {arg.arg}: {exc}") from exc
            if ann is None and arg.annotation is not None:
                ann = self.static(arg.annotation)
            if isinstance(ann, SymbolicTensorSpec):
                shape = []
                for d in ann.shape:
                    if isinstance(d, SymbolicDim):
                        if d.name in self.special:
                            shape.append(int(self.special[d.name]))
                        else:
                            self.sym_dims[d.name] = SymDim(d.name)
                            shape.append(SymDim(d.name))
                    else:
                        shape.append(d)
                ttype = TensorType(tuple(shape), ann.dtype)
                params.append(TensorParameter(arg.arg, ttype))
            elif isinstance(ann, TensorType):
                params.append(TensorParameter(arg.arg, ann))
            elif isinstance(ann, (DType, str)) or ann in (builtins.int, builtins.float, builtins.bool):
                params.append(ScalarParameter(arg.arg, str(DType(ann))))
            else:
                raise CompileError(f"Parameter {arg.arg} needs a T.Tensor or scalar dtype annotation")
        for p in params:
            if isinstance(p, TensorParameter):
                self.buffers[p.name] = Alloc(p.name, "global", p.type.shape, p.type.dtype)
            else:
                self.kernel_names.add(p.name)
        return tuple(params)

    # ------------------------------------------------------------------ statements
    def read(self) -> Program:
        params = self.params()
        body = [s for s in self.fdef.body if not (isinstance(s, ast.Expr) and isinstance(s.value, ast.Constant))]
        kernel = None
        for stmt in body:
            if isinstance(stmt, ast.With):
                kernel = stmt
                break
            if isinstance(stmt, ast.Assign) and len(stmt.targets) == 1 and isinstance(stmt.targets[0], ast.Name):
                ok, value = self.try_static(stmt.value)
                if ok:
                    self.env[stmt.targets[0].id] = value
                    continue
            self.fail(stmt, "Only static assignments may precede T.Kernel")
        if kernel is None:
            raise CompileError("prim_func body must contain `with T.Kernel(...)`")
        item = kernel.items[0]
        call = item.context_expr
        if not (isinstance(call, ast.Call) and self.call_name(call) == "Kernel"):
            self.fail(kernel, "Expected `with T.Kernel(...)`")
        grid = []
        for g in call.args:
            ok, v = self.try_static(g)
            if ok and isinstance(v, int):
                grid.append(v)
            else:
                grid.append(simplify(self.expr(g)))
        kw = {k.arg: k for k in call.keywords}
        threads = 128
        if "threads" in kw:
            threads = self.static(kw["threads"].value)
            if isinstance(threads, (tuple, list)):
                threads = math.prod(threads)
        names = []
        if item.optional_vars is not None:
            target = item.optional_vars
            elts = target.elts if isinstance(target, ast.Tuple) else [target]
            for e in elts:
                if not isinstance(e, ast.Name):
                    self.fail(e, "Kernel block variables must be names")
                names.append(e.id)
        block_vars = tuple(names) + tuple(f"$b{i}" for i in range(len(names), len(grid)))
        self.kernel_names.update(block_vars)
        stmts = self.block(kernel.body)
        return Program(
            name=self.fdef.name,
            params=params,
            grid=tuple(grid),
            block_vars=block_vars,
            threads=int(threads),
            buffers=self.buffers,
            body=stmts,
            source=self.source,
            sym_dims=tuple(self.sym_dims.values()),
        )

    def block(self, stmts):
        out = []
        for s in stmts:
            out.extend(self.stmt(s))
        return out

    def nested(self, stmts):
        """A branch or loop body: bindings made inside it are not visible after it."""
        self._next_block += 1
        self.path.append(self._next_block)
        try:
            return self.block(stmts)
        finally:
            self.path.pop()

    def stmt(self, node):
        if isinstance(node, ast.Expr):
            if isinstance(node.value, ast.Constant):
                return []
            if isinstance(node.value, ast.Call):
                return self.call_stmt(node.value)
            self.fail(node, "Unsupported expression statement")
        if isinstance(node, ast.Assign):
            if len(node.targets) != 1:
                self.fail(node, "Chained assignment is not supported")
            target = node.targets[0]
            if isinstance(target, ast.Name):
                name = self.call_name(node.value)
                if name in ("alloc_shared", "alloc_fragment", "alloc_local"):
                    return [self.alloc(target.id, node.value, name)]
                if name == "alloc_var":
                    return self.alloc_var(target.id, node.value)
                if target.id in self.mutables:
                    return [Let(target.id, simplify(self.expr(node.value)))]
                ok, value = self.try_static(node.value)
                if ok and not isinstance(value, (SymbolicDim,)):
                    self.env[target.id] = value
                    return []
                # Kernel-time scalar binding: substituted at each use, valid inside the block
                # (and the blocks nested in it) where it was made.
                self.lets[target.id] = simplify(self.expr(node.value))
                self.let_paths[target.id] = tuple(self.path)
                return []
            if isinstance(target, ast.Subscript):
                buf = self.buffer_name(target.value)
                idx = tuple(self.index_list(target.slice))
                return [Store(buf, idx, simplify(self.expr(node.value)))]
            self.fail(node, "Unsupported assignment target")
        if isinstance(node, ast.AugAssign):
            op = _BINSYM.get(type(node.op))
            target = node.target
            if isinstance(target, ast.Subscript):
                buf = self.buffer_name(target.value)
                idx = tuple(self.index_list(target.slice))
                return [Store(buf, idx, simplify(Bin(op, Load(buf, idx), self.expr(node.value))))]
            if isinstance(target, ast.Name) and (target.id in self.kernel_names or target.id in self.mutables):
                value = Bin(op, Var(target.id), self.expr(node.value))
                return [Let(target.id, simplify(value))]
            self.fail(node, "Unsupported augmented assignment")
        if isinstance(node, ast.For):
            return self.for_stmt(node)
        if isinstance(node, ast.While):
            if node.orelse:
                self.fail(node, "while ... else is not supported")
            return [While(simplify(self.expr(node.test)), self.nested(node.body))]
        if isinstance(node, ast.Break):
            return [Break()]
        if isinstance(node, ast.Continue):
            return [Continue()]
        if isinstance(node, ast.If):
            ok, test = self.try_static(node.test)
            if ok:
                return self.block(node.body if test else node.orelse)
            cond = simplify(self.expr(node.test))
            return [If(cond, self.nested(node.body), self.nested(node.orelse))]
        if isinstance(node, ast.Pass):
            return []
        self.fail(node, f"Unsupported statement {type(node).__name__}")

    in_parallel = False

    def alloc(self, name, call, kind):
        shape = self.static(call.args[0]) if call.args else self.static(call.keywords[0].value)
        shape = (shape,) if isinstance(shape, int) else tuple(shape)
        dtype = "float32"
        if len(call.args) > 1:
            dtype = str(self.static(call.args[1]))
        for k in call.keywords:
            if k.arg == "dtype":
                dtype = str(self.static(k.value))
        scope = {"alloc_shared": "shared", "alloc_fragment": "fragment", "alloc_local": "fragment"}[kind]
        a = Alloc(name, scope, shape, canonical_dtype(dtype))
        self.buffers[name] = a
        return a

    def alloc_var(self, name, call):
        """``T.alloc_var(dtype, init=0)``: a mutable per-thread scalar (python/ntilang/frontend.py:916-965)."""
        kw = {k.arg: k.value for k in call.keywords}
        args = list(call.args)
        if args:
            dtype_node = args.pop(0)
        elif "dtype" in kw:
            dtype_node = kw["dtype"]
        else:
            self.fail(call, "alloc_var requires dtype")
        dtype = canonical_dtype(str(self.static(dtype_node)))
        init = kw.get("init", args[0] if args else None)
        if init is not None:
            ok, v = self.try_static(init)
            value = Const(v) if ok and v is None else self.expr(init)
            if isinstance(value, Const) and value.value is None:
                value = Const(0)
        else:
            value = Const(0)
        a = Alloc(name, "var", (1,), dtype)
        self.buffers[name] = a
        self.mutables[name] = dtype
        return [a, Let(name, Call("cast", (simplify(value), Const(dtype))))]

    def for_stmt(self, node):
        it = node.iter
        name = self.call_name(it) if isinstance(it, ast.Call) else None
        target = node.target
        tnames = [e.id for e in (target.elts if isinstance(target, ast.Tuple) else [target])]
        if name == "Parallel":
            extents = tuple(self.static(a) for a in it.args)
            saved = self.in_parallel
            self.in_parallel = True
            self.kernel_names.update(tnames)
            body = self.nested(node.body)
            self.in_parallel = saved
            return [Parallel(tuple(tnames), extents, body)]
        if name in ("Pipelined", "serial", "Serial", "unroll", "Unroll", "range", "grid"):
            kw = {k.arg: k.value for k in it.keywords}
            args = list(it.args)
            stages = 0
            if "num_stages" in kw:
                stages = int(self.static(kw["num_stages"]))
            if name == "grid":
                if len(tnames) != len(args):
                    self.fail(node, "T.grid target count must match its extents")
                self.kernel_names.update(tnames)
                stmts = self.nested(node.body)
                for var, ext in reversed(list(zip(tnames, args))):
                    stmts = [Loop(var, Const(0), simplify(self.expr(ext)), "serial", 0, stmts)]
                self.kernel_names.update(tnames)
                return stmts
            if len(tnames) != 1:
                self.fail(node, "Serial loops bind a single variable")
            if not args and "stop" in kw:
                args = ([kw["start"]] if "start" in kw else []) + [kw["stop"]]
            if not args or len(args) > 3:
                self.fail(node, "serial loops take (stop), (start, stop) or (start, stop, step)")
            start, stop = (Const(0), args[0]) if len(args) == 1 else (args[0], args[1])
            start = start if isinstance(start, Const) else simplify(self.expr(start))
            stop = simplify(self.expr(stop))
            step_node = args[2] if len(args) == 3 else kw.get("step")
            step = None
            if step_node is not None:
                step = simplify(self.expr(step_node))
                if isinstance(step, Const):
                    if step.value == 0:
                        self.fail(node, "loop step must not be zero")
                    if step.value == 1:
                        step = None
            self.kernel_names.add(tnames[0])
            body = self.nested(node.body)
            kind = "pipelined" if name == "Pipelined" else "serial"
            return [Loop(tnames[0], start, stop, kind, stages, body, step)]
        self.fail(node, "Loops must iterate T.Parallel, T.Pipelined, T.serial, T.grid or range")

    def call_stmt(self, call):
        name = self.call_name(call)
        args = call.args
        kw = {k.arg: k.value for k in call.keywords}

        def arg(i, key, default=None):
            if len(args) > i:
                return args[i]
            return kw.get(key, default)

        if name == "copy":
            return [Copy(self.region(arg(0, "src")), self.region(arg(1, "dst")))]
        if name == "gemm":
            a, b, c = (self.buffer_name(x) for x in (arg(0, "A"), arg(1, "B"), arg(2, "C")))
            ta = bool(self.static(arg(3, "transpose_A", ast.Constant(False))))
            tb = bool(self.static(arg(4, "transpose_B", ast.Constant(False))))
            clear = bool(self.static(kw.get("clear_accum", ast.Constant(False))))
            if "k_pack" in kw and self.static(kw["k_pack"]) != 1:
                self.fail(call, "T.gemm k_pack must be 1")
            return [Gemm(a, b, c, ta, tb, clear)]
        if name == "clear":
            return [Fill(self.buffer_name(args[0]), 0.0)]
        if name == "fill":
            buf = self.buffer_name(args[0])
            v = self.static(arg(1, "value"))
            return [Fill(buf, float(v))]
        if name in _REDUCE_KINDS or name == "reduce":
            kind = _REDUCE_KINDS.get(name) or str(self.static(arg(2, "reduce_type")))
            off = 1 if name == "reduce" else 0
            src = self.buffer_name(arg(0, "buffer"))
            dst = self.buffer_name(arg(1, "out"))
            dim = int(self.static(arg(2 + off, "dim", ast.Constant(-1))))
            clear = bool(self.static(arg(3 + off, "clear", ast.Constant(True))))
            rank = len(self.buffers[src].shape)
            return [Reduce(kind, src, dst, dim % rank, clear)]
        if name in ("cumsum", "cummax", "cumsum_fragment", "cummax_fragment"):
            src = self.region(arg(0, "src"))
            dst_node = arg(1, "dst")
            dst = self.region(dst_node) if dst_node is not None and not (
                isinstance(dst_node, ast.Constant) and dst_node.value is None) else src
            dim = int(self.static(arg(2, "dim", ast.Constant(0))))
            reverse = bool(self.static(arg(3, "reverse", ast.Constant(False))))
            rank = len(src.extents)
            if not -rank <= dim < rank:
                self.fail(call, "Scan dimension is outside the source rank")
            return [Scan("sum" if name.startswith("cumsum") else "max", src, dst, dim % rank, reverse)]
        if name in _ATOMICS:
            dst = arg(0, "dst")
            if not isinstance(dst, ast.Subscript):
                self.fail(call, f"T.{name} needs an element destination")
            buf = self.buffer_name(dst.value)
            idx = tuple(self.index_list(dst.slice))
            return [Atomic(_ATOMICS[name], buf, idx, simplify(self.expr(arg(1, "value"))))]
        if name in ("loop_break", "break_loop"):
            return [Break()]
        if name == "continue_loop":
            return [Continue()]
        if name in ("use_swizzle", "annotate_layout", "print", "device_assert", "Assert"):
            return [Hint(name)]
        self.fail(call, f"Unsupported kernel statement T.{name}")


_BINOPS = {
    ast.Add: lambda a, b: a + b, ast.Sub: lambda a, b: a - b, ast.Mult: lambda a, b: a * b,
    ast.Div: lambda a, b: a / b, ast.FloorDiv: lambda a, b: a // b, ast.Mod: lambda a, b: a % b,
    ast.Pow: lambda a, b: a**b, ast.LShift: lambda a, b: a << b, ast.RShift: lambda a, b: a >> b,
    ast.BitAnd: lambda a, b: a & b, ast.BitOr: lambda a, b: a | b, ast.BitXor: lambda a, b: a ^ b,
}
_BINSYM = {ast.Add: "+", ast.Sub: "-", ast.Mult: "*", ast.Div: "/", ast.FloorDiv: "//", ast.Mod: "%",
           ast.BitAnd: "&", ast.BitOr: "|", ast.BitXor: "^", ast.LShift: "<<", ast.RShift: ">>"}
_CMPOPS = {
    ast.Lt: lambda a, b: a < b, ast.LtE: lambda a, b: a <= b, ast.Gt: lambda a, b: a > b,
    ast.GtE: lambda a, b: a >= b, ast.Eq: lambda a, b: a == b, ast.NotEq: lambda a, b: a != b,
}
_CMPSYM = {ast.Lt: "<", ast.LtE: "<=", ast.Gt: ">", ast.GtE: ">=", ast.Eq: "==", ast.NotEq: "!="}
_DTYPE_CALLS = {n: n for n in ("float32", "float16", "bfloat16", "float64", "int8", "int16", "int32", "int64",
                                "uint8", "uint16", "uint32", "uint64", "bool")}
_DTYPE_CALLS.update({"half": "float16", "float": "float32", "double": "float64", "int": "int32", "long": "int64"})


# ------------------------------------------------------------------------ simplification


def simplify(e):
    """Constant folding plus a canonical affine form for index arithmetic."""
    if isinstance(e, Bin):
        a, b = simplify(e.a), simplify(e.b)
        if isinstance(a, Const) and isinstance(b, Const):
            try:
                return Const(_PYOP[e.op](a.value, b.value))
            except (ZeroDivisionError, TypeError, ValueError):
                return Bin(e.op, a, b)
        if e.op in ("+", "-", "*"):
            fa, fb = affine(a), affine(b)
            if fa is not None and fb is not None:
                if e.op == "*":
                    res = _affine_mul(fa, fb)
                else:
                    res = _affine_add(fa, fb, 1 if e.op == "+" else -1)
                if res is not None:
                    return from_affine(res)
        return Bin(e.op, a, b)
    if isinstance(e, Call):
        return Call(e.fn, tuple(simplify(x) for x in e.args))
    if isinstance(e, Select):
        return Select(simplify(e.cond), simplify(e.a), simplify(e.b))
    if isinstance(e, Cmp):
        return Cmp(e.op, simplify(e.a), simplify(e.b))
    if isinstance(e, Load):
        return Load(e.buf, tuple(simplify(i) for i in e.idx))
    return e


_PYOP = {"+": lambda a, b: a + b, "-": lambda a, b: a - b, "*": lambda a, b: a * b,
         "/": lambda a, b: a / b, "//": lambda a, b: a // b, "%": lambda a, b: a % b,
         "&": lambda a, b: a & b, "|": lambda a, b: a | b, "^": lambda a, b: a ^ b,
         "<<": lambda a, b: a << b, ">>": lambda a, b: a >> b}


def affine(e):
    """Expr -> {var_name or 1: int coeff} for integer affine expressions, else None."""
    if isinstance(e, Const):
        if isinstance(e.value, bool) or not isinstance(e.value, int):
            return None
        return {1: e.value}
    if isinstance(e, Var):
        return {e.name: 1}
    if isinstance(e, Bin) and e.op in ("+", "-", "*"):
        fa, fb = affine(e.a), affine(e.b)
        if fa is None or fb is None:
            return None
        if e.op == "*":
            return _affine_mul(fa, fb)
        return _affine_add(fa, fb, 1 if e.op == "+" else -1)
    return None


def _affine_add(fa, fb, sign):
    out = dict(fa)
    for k, v in fb.items():
        out[k] = out.get(k, 0) + sign * v
    return {k: v for k, v in out.items() if v != 0 or k == 1}


def _affine_mul(fa, fb):
    if set(fa) <= {1}:
        c = fa.get(1, 0)
        return {k: c * v for k, v in fb.items() if c * v != 0 or k == 1}
    if set(fb) <= {1}:
        c = fb.get(1, 0)
        return {k: c * v for k, v in fa.items() if c * v != 0 or k == 1}
    return None


def from_affine(f):
    terms = None
    for k in sorted((k for k in f if k != 1), key=str):
        v = f[k]
        t = Var(k) if v == 1 else Bin("*", Const(v), Var(k))
        terms = t if terms is None else Bin("+", terms, t)
    c = f.get(1, 0)
    if terms is None:
        return Const(c)
    return terms if c == 0 else Bin("+", terms, Const(c))


def read_program(program: PrimFunc) -> Program:
    if not isinstance(program, PrimFunc):
        raise TypeError("compile() expects a @T.prim_func")
    return _Reader(program).read()


__all__ = [
    "Alloc", "Atomic", "Bin", "Break", "Call", "Cmp", "Const", "Continue", "Copy", "Fill", "Gemm", "Hint", "If",
    "Let", "Load",
    "Loop", "Parallel", "Program", "Reduce", "Region", "Scan", "Select", "Store", "Var", "While", "affine",
    "read_program", "simplify",
]
