"""Serial CPU evaluator of generic elementwise programs — TEST INFRASTRUCTURE ONLY.

The checker for the NVRTC path (``ntilang_b200.pointwise``).  It restates the reference's
NumPy evaluator (python/ntilang/testing.py:34-400) for the statements that path accepts:
block instances in grid order, each ``T.Parallel`` loop point by point in row-major order,
fragments as arrays, and per operation the reference's typing (python/ntilang/scalar.py:60-230):
operands are cast to the promoted operand dtype, the operation runs in NumPy on that dtype and
the result is cast to the expression's dtype.  Loads outside a tensor read 0; stores outside
it are skipped (testing.py:133-143).  Integer ``//`` and ``%`` use Python's floor semantics.
bfloat16 uses ``ml_dtypes`` (the reference's evaluator has no bfloat16).

It walks the program representation ``ntilang_b200.frontend`` reads (the tests build each
program once and hand the same reading to both sides); the golden vectors in ``tests/golden/``,
produced by the reference's own evaluator, pin it.  Only ``tests/`` may import this module.
"""

from __future__ import annotations


import numpy as np

try:  # bfloat16 values; absent -> bfloat16 programs are not evaluated
    import ml_dtypes

    _BF16 = np.dtype(ml_dtypes.bfloat16)
except ImportError:  # pragma: no cover
    _BF16 = None

_WIDTH = {"bool": 1, "int8": 1, "int16": 2, "int32": 4, "int64": 8, "uint8": 1, "uint16": 2, "uint32": 4,
          "uint64": 8, "float16": 2, "bfloat16": 2, "float32": 4, "float64": 8}
_FLOATS = ("float16", "bfloat16", "float32", "float64")


def np_dtype(name):
    return _BF16 if name == "bfloat16" else np.dtype(name)


def promote(left, right):
    """python/ntilang/scalar.py:60-78."""
    if left == right:
        return left
    if left == "bool":
        return right
    if right == "bool":
        return left
    lf, rf = left in _FLOATS, right in _FLOATS
    if lf and rf:
        return f"float{max(_WIDTH[left], _WIDTH[right]) * 8}"
    if lf or rf:
        return left if lf else right
    if left.startswith("uint") != right.startswith("uint"):
        uns, sig = (left, right) if left.startswith("uint") else (right, left)
        return uns if _WIDTH[uns] >= _WIDTH[sig] else sig
    return left if _WIDTH[left] >= _WIDTH[right] else right


def cast(value, dtype):
    with np.errstate(all="ignore"):
        return np.asarray(value).astype(np_dtype(dtype), casting="unsafe")[()]


def _const_dtype(value):
    if isinstance(value, bool):
        return "bool"
    if isinstance(value, int):
        return "int32" if -(2**31) <= value < 2**31 else "int64"
    return "float32"


_UNARY = {"exp": np.exp, "exp2": np.exp2, "log": np.log, "log2": np.log2, "log10": np.log10, "log1p": np.log1p,
          "sqrt": np.sqrt, "sin": np.sin, "cos": np.cos, "tan": np.tan, "tanh": np.tanh, "floor": np.floor,
          "ceil": np.ceil, "trunc": np.trunc, "round": np.round, "nearbyint": np.rint,
          "rsqrt": lambda v: 1 / np.sqrt(v), "exp10": lambda v: np.power(v.dtype.type(10), v)}


class _Break(Exception):
    pass


class _Continue(Exception):
    pass


class _Eval:
    def __init__(self, prog, arrays, scalars):
        self.prog = prog
        self.buffers = {}
        self.types = {}
        self.vars = {}
        it = iter(scalars)
        for p, a in zip((p for p in prog.params if hasattr(p, "type")), arrays):
            self.buffers[p.name] = a
        for p in prog.params:
            if not hasattr(p, "type"):
                self.vars[p.name] = cast(next(it), p.dtype)
                self.types[p.name] = p.dtype
        self.sym = {}
        for p in prog.params:
            if hasattr(p, "type"):
                for d, n in zip(p.type.shape, self.buffers[p.name].shape):
                    if type(d).__name__ == "SymDim":
                        self.sym[d.name] = n

    # ---------------------------------------------------------------- values
    def dtype(self, e):
        k = type(e).__name__
        if k == "Const":
            return _const_dtype(e.value)
        if k == "Var":
            return "int32" if e.name.startswith("$sym:") else self.types[e.name]
        if k == "Load":
            return self.buf_dtype(e.buf)
        if k == "Cmp":
            return "bool"
        if k == "Bin":
            if e.op in ("&", "|", "^", "<<", ">>"):
                return promote(*self._bit_operand_dtypes(e))
            return promote(self.dtype(e.a), self.dtype(e.b))
        if k == "Select":
            return promote(self.dtype(e.a), self.dtype(e.b))
        if k == "Call":
            if e.fn == "cast":
                return e.args[1].value
            if e.fn in ("and", "or", "not", "isnan", "isinf", "isfinite"):
                return "bool"
            if e.fn in ("max", "min", "maximum", "minimum", "pow"):
                d = self.dtype(e.args[0])
                for a in e.args[1:]:
                    d = promote(d, self.dtype(a))
                return d
            d = self.dtype(e.args[0])
            if e.fn == "exp" and d not in _FLOATS:
                return "float32"
            if e.fn == "neg" and d == "bool":
                return "int32"
            return d
        raise TypeError(k)

    def _bit_operand_dtypes(self, e):
        """An int literal takes the other operand's integer dtype (scalar.py:81-96)."""
        da, db = self.dtype(e.a), self.dtype(e.b)
        lit_a = type(e.a).__name__ == "Const" and type(e.a.value) is int
        lit_b = type(e.b).__name__ == "Const" and type(e.b.value) is int
        if lit_a and not lit_b and db not in _FLOATS:
            da = db
        elif lit_b and not lit_a and da not in _FLOATS:
            db = da
        return da, db

    def buf_dtype(self, name):
        b = self.prog.buffers[name]
        return b.dtype

    def ev(self, e):
        k = type(e).__name__
        if k == "Const":
            return e.value
        if k == "Var":
            if e.name.startswith("$sym:"):
                return np.int32(self.sym[e.name[5:]])
            return self.vars[e.name]
        if k == "Load":
            return self.read(e.buf, tuple(int(self.ev(i)) for i in e.idx))
        if k == "Cmp":
            d = promote(self.dtype(e.a), self.dtype(e.b))
            a, b = cast(self.ev(e.a), d), cast(self.ev(e.b), d)
            return bool({"<": a < b, "<=": a <= b, ">": a > b, ">=": a >= b, "==": a == b, "!=": a != b}[e.op])
        if k == "Bin" and e.op in ("&", "|", "^", "<<", ">>"):
            da, db = self._bit_operand_dtypes(e)
            d = promote(da, db)
            a, b = cast(self.ev(e.a), d), cast(self.ev(e.b), d)
            with np.errstate(all="ignore"):
                if d == "bool":
                    r = {"&": a & b, "|": a | b, "^": a ^ b}[e.op]
                else:
                    r = {"&": lambda: a & b, "|": lambda: a | b, "^": lambda: a ^ b,
                         "<<": lambda: a << b, ">>": lambda: a >> b}[e.op]()
            return cast(r, d)
        if k == "Bin":
            d = promote(self.dtype(e.a), self.dtype(e.b))
            a, b = self.ev(e.a), self.ev(e.b)
            if e.op in ("//", "%"):
                a, b = int(a), int(b)
                return cast(a // b if e.op == "//" else a % b, d)
            a, b = cast(a, d), cast(b, d)
            with np.errstate(all="ignore"):
                r = {"+": lambda: a + b, "-": lambda: a - b, "*": lambda: a * b, "/": lambda: a / b}[e.op]()
            return cast(r, d)
        if k == "Select":
            d = self.dtype(e)
            return cast(self.ev(e.a) if self.ev(e.cond) else self.ev(e.b), d)
        if k == "Call":
            return self.call(e)
        raise TypeError(k)

    def call(self, e):
        fn = e.fn
        if fn == "cast":
            return cast(self.ev(e.args[0]), e.args[1].value)
        if fn == "and":
            return bool(self.ev(e.args[0])) and bool(self.ev(e.args[1]))
        if fn == "or":
            return bool(self.ev(e.args[0])) or bool(self.ev(e.args[1]))
        if fn == "not":
            return not bool(self.ev(e.args[0]))
        if fn == "invert":
            d = self.dtype(e.args[0])
            v = cast(self.ev(e.args[0]), d)
            return (not bool(v)) if d == "bool" else cast(~v, d)
        d = self.dtype(e)
        vals = [self.ev(a) for a in e.args]
        if fn in ("max", "min", "maximum", "minimum"):
            a, b = (cast(v, d) for v in vals)
            if d in _FLOATS and a == 0 and b == 0:  # +0 above -0 (testing.py:186-194)
                neg = (np.signbit(a) and np.signbit(b)) if fn in ("max", "maximum") else (np.signbit(a) or np.signbit(b))
                return cast(np.copysign(0.0, -1.0 if neg else 1.0), d)
            op = {"max": np.fmax, "min": np.fmin, "maximum": np.maximum, "minimum": np.minimum}[fn]
            return cast(op(a, b), d)
        if fn == "neg":
            with np.errstate(all="ignore"):
                return cast(-cast(vals[0], d), d)
        if fn == "abs":
            with np.errstate(all="ignore"):
                return cast(np.abs(cast(vals[0], d)), d)
        if fn in ("isnan", "isinf", "isfinite"):
            return bool(getattr(np, fn)(vals[0]))
        compute = "float32" if d in ("float16", "bfloat16") else d
        with np.errstate(all="ignore"):
            if fn == "sigmoid":
                v = cast(vals[0], compute)
                ex = cast(np.exp(-v), d)
                den = cast(cast(1, d) + ex, d)
                return cast(cast(1, d) / den, d)
            if fn == "rcp":
                return cast(1 / cast(vals[0], compute), d)
            if fn in ("pow", "fmod"):
                a, b = cast(vals[0], compute), cast(vals[1], compute)
                return cast(np.power(a, b) if fn == "pow" else np.fmod(a, b), d)
            return cast(_UNARY[fn](cast(vals[0], compute)), d)

    # ---------------------------------------------------------------- memory
    def read(self, name, idx):
        arr = self.buffers[name]
        if all(0 <= i < s for i, s in zip(idx, arr.shape)):
            return arr[idx]
        return cast(0, self.buf_dtype(name))

    def write(self, name, idx, value):
        arr = self.buffers[name]
        if all(0 <= i < s for i, s in zip(idx, arr.shape)):
            arr[idx] = cast(value, self.buf_dtype(name))

    # ------------------------------------------------------------ statements
    def run(self):
        grid = []
        for g in self.prog.grid:
            grid.append(int(g) if isinstance(g, int) else int(self.ev(g)))
        for flat in np.ndindex(*reversed(grid)):
            for bv, v in zip(self.prog.block_vars, reversed(flat)):
                self.vars[bv] = np.int32(v)
                self.types[bv] = "int32"
            self.stmts(self.prog.body)

    def stmts(self, body):
        for s in body:
            self.stmt(s)

    def stmt(self, s):
        k = type(s).__name__
        if k == "Alloc":
            if s.scope == "var":
                self.types[s.name] = s.dtype
                self.vars[s.name] = cast(0, s.dtype)
            else:
                self.buffers[s.name] = np.zeros(s.shape, dtype=np_dtype(s.dtype))
        elif k == "Parallel":
            for point in np.ndindex(*s.extents):
                for v, x in zip(s.vars, point):
                    self.vars[v] = np.int32(x)
                    self.types[v] = "int32"
                self.stmts(s.body)
        elif k == "Loop":
            d = promote(promote(self.dtype(s.start), self.dtype(s.stop)), "int32")
            v, stop = int(self.ev(s.start)), int(self.ev(s.stop))  # range(start, stop, step): read once
            step = 1 if getattr(s, "step", None) is None else int(self.ev(s.step))
            self.types[s.var] = d
            while (step > 0 and v < stop) or (step < 0 and v > stop):
                self.vars[s.var] = cast(v, d)
                try:
                    self.stmts(s.body)
                except _Continue:
                    pass
                except _Break:
                    break
                v += step
        elif k == "While":
            while self.ev(s.cond):
                try:
                    self.stmts(s.body)
                except _Continue:
                    continue
                except _Break:
                    break
        elif k == "Break":
            raise _Break()
        elif k == "Continue":
            raise _Continue()
        elif k == "If":
            self.stmts(s.then if self.ev(s.cond) else s.orelse)
        elif k == "Let":
            self.vars[s.name] = cast(self.ev(s.value), self.types[s.name])
        elif k == "Store":
            b = self.prog.buffers[s.buf]
            if b.scope == "var":
                self.vars[s.buf] = cast(self.ev(s.value), b.dtype)
            else:
                self.write(s.buf, tuple(int(self.ev(i)) for i in s.idx), self.ev(s.value))
        elif k == "Atomic":
            idx = tuple(int(self.ev(i)) for i in s.idx)
            arr = self.buffers[s.buf]
            if all(0 <= i < n for i, n in zip(idx, arr.shape)):
                v = cast(self.ev(s.value), self.buf_dtype(s.buf))
                with np.errstate(all="ignore"):
                    old = arr[idx]
                    arr[idx] = old + v if s.op == "add" else (max(old, v) if s.op == "max" else min(old, v))
        elif k == "Copy":
            self.copy(s)
        elif k == "Fill":
            b = self.prog.buffers[s.buf]
            if b.scope == "var":
                self.vars[s.buf] = cast(s.value, b.dtype)
            else:
                self.buffers[s.buf][...] = cast(s.value, b.dtype)
        elif k == "Hint":
            pass
        else:
            raise NotImplementedError(k)

    def copy(self, s):
        src, dst = s.src, s.dst
        sb, db = self.prog.buffers[src.buf], self.prog.buffers[dst.buf]
        if sb.scope != "global":
            shape = tuple(sb.shape)
        elif db.scope != "global":
            shape = tuple(db.shape)
        elif not src.point:
            shape = tuple(src.extents)
        else:
            shape = tuple(dst.extents)

        def index(region, coord):
            rank = len(self.prog.buffers[region.buf].shape)
            starts = [int(self.ev(x)) for x in region.starts]
            if region.point:
                axes = list(range(rank - len(shape), rank))
                mapped = dict(zip(axes, coord))
            elif len(region.extents) == len(shape):
                mapped = dict(zip(range(rank), coord))
            else:
                axes = [k for k, ext in enumerate(region.extents) if ext != 1]
                mapped = dict(zip(axes, [c for c, ext in zip(coord, shape) if ext != 1]))
            return tuple(starts[k] + mapped.get(k, 0) for k in range(rank))

        values = [(c, self.read(src.buf, index(src, c))) for c in np.ndindex(*shape)]
        for c, v in values:
            self.write(dst.buf, index(dst, c), v)


def evaluate(prog, arrays, scalars=()):
    """Run ``prog`` (a ``ntilang_b200.frontend.Program``) on ``arrays`` (NumPy, one per tensor
    parameter, outputs updated in place) and ``scalars`` (one per scalar parameter)."""
    _Eval(prog, arrays, scalars).run()
    return arrays


__all__ = ["cast", "evaluate", "promote"]
