"""Op-family recognition: ``frontend.Program`` -> an ``OpSpec`` the C-ABI can launch.

The reference lowers any tile program through its CuTe emitter
(``python/ntilang/codegen.py:1997-2262``).  This package implements the kernels that
emitter produces for the hot path as hand-written sm_100a CUDA, so compilation is a
recognition problem: decide which family a program computes and extract its runtime
parameters.  Unrecognised programs raise ``CompileError`` — there is no fallback.

Families (reference program each matcher was written against):

* ``elementwise``  C[i] = A[i] (+|-|*) B[i]             examples/vector_add.py:5-10
* ``cumsum``       inclusive row scan, fwd / reverse     examples/cumsum.py:7-14, scan.py:87-240
* ``softmax``      exp(x - max) / sum                    examples/softmax.py:9-25
* ``rmsnorm``      x * rsqrt(sum(x^2) * inv_n + eps) * w examples/rmsnorm.py:13-37
* ``gemm``         C = epilogue(A @ B)                   examples/matmul.py:17-29, matmul_relu.py:17-38
* ``fa2``          FlashAttention-2 forward              examples/flash_attention.py:26-79

Row families are matched by evaluating the kernel symbolically per row (each buffer
element becomes an expression over the input row ``X[j]``, row reductions and 1-D
parameters) and comparing the stored expression with the family's canonical form.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

from .frontend import (
    Alloc, Bin, Call, Cmp, Const, Copy, Fill, Gemm, Hint, If, Let, Load, Loop, Parallel, Program,
    Reduce, Scan, Select, Store, Var, affine, simplify,
)
from .ir import CompileError, ScalarParameter, SymDim, TensorParameter


class NoMatch(Exception):
    pass


def need(cond, msg):
    if not cond:
        raise NoMatch(msg)


@dataclass
class OpSpec:
    family: str
    params: dict = field(default_factory=dict)  # family-specific static parameters
    args: dict = field(default_factory=dict)  # role -> kernel parameter index

    def describe(self) -> str:
        items = ", ".join(f"{k}={v}" for k, v in self.params.items())
        roles = ", ".join(f"{k}=arg{v}" for k, v in self.args.items())
        return f"{self.family}({items}; {roles})"


# --------------------------------------------------------------------------- utilities


def _body(stmts):
    """Statements with layout/schedule hints and allocations removed."""
    return [s for s in stmts if not isinstance(s, (Hint, Alloc))]


def _param_index(prog: Program, name: str) -> int:
    for i, p in enumerate(prog.params):
        if p.name == name:
            return i
    raise NoMatch(f"{name} is not a kernel parameter")


def _is_param(prog: Program, name: str) -> bool:
    return any(p.name == name and isinstance(p, TensorParameter) for p in prog.params)


def _dim(v):
    return v.name if isinstance(v, SymDim) else v


def _aff(e):
    f = affine(simplify(e)) if e is not None else None
    if f is None:
        raise NoMatch("index is not affine")
    return f


def _aff_is(e, expect: dict) -> bool:
    try:
        f = _aff(e)
    except NoMatch:
        return False
    f = {k: v for k, v in f.items() if v != 0}
    g = {k: v for k, v in expect.items() if v != 0}
    return f == g


def _grid_extent(prog: Program, var: str):
    if var not in prog.block_vars:
        return None
    g = prog.grid[prog.block_vars.index(var)]
    return g if isinstance(g, int) else None  # None: symbolic (covers its dimension by construction)


def _covers(prog, var, tile, extent) -> bool:
    """Does ``var * tile`` over the grid cover ``extent`` (symbolic dims always do)?"""
    if isinstance(extent, SymDim):
        return True
    g = _grid_extent(prog, var)
    if g is None:
        return True
    return g * tile >= extent


# ------------------------------------------------------------- symbolic row evaluation


@dataclass(frozen=True)
class X:  # element j of a 2-D input parameter row
    name: str


@dataclass(frozen=True)
class W:  # element j of a 1-D parameter (broadcast over rows)
    name: str


@dataclass(frozen=True)
class Pad:  # value for j < limit, else ``pad`` (tile padding)
    value: object
    pad: object
    limit: int


@dataclass(frozen=True)
class Red:  # a row reduction of an element expression
    kind: str
    expr: object


@dataclass(frozen=True)
class Acc:  # the GEMM accumulator element
    pass


def _fold(e):
    """Light algebraic clean-up on symbolic row/epilogue expressions."""
    if isinstance(e, Call):
        args = tuple(_fold(a) for a in e.args)
        if e.fn in ("max", "maximum") and len(args) == 2 and isinstance(args[1], Const) and args[1].value == -math.inf:
            return args[0]
        if e.fn == "neg" and isinstance(args[0], Const):
            return Const(-args[0].value)
        return Call(e.fn, args)
    if isinstance(e, Bin):
        a, b = _fold(e.a), _fold(e.b)
        if isinstance(a, Const) and isinstance(b, Const):
            try:
                return Const({"+": a.value + b.value, "-": a.value - b.value, "*": a.value * b.value,
                              "/": a.value / b.value}[e.op])
            except (KeyError, ZeroDivisionError):
                pass
        return Bin(e.op, a, b)
    if isinstance(e, Pad):
        return Pad(_fold(e.value), _fold(e.pad), e.limit)
    if isinstance(e, Red):
        return Red(e.kind, _fold(e.expr))
    return e


class RowEval:
    """Evaluate a 1-D-grid row kernel symbolically.

    Local 2-D tiles are indexed (local_row, col); local 1-D tiles (local_row,).
    Global 2-D parameters must be indexed (bx * rows_per_block + local_row, col).
    """

    def __init__(self, prog: Program):
        need(len(prog.grid) == 1, "row kernels use a 1-D grid")
        self.prog = prog
        self.bx = prog.block_vars[0]
        self.rb = None
        self.cols = None  # global row length
        self.tile = {}  # local buffer -> symbolic value
        self.out = {}  # global param name -> symbolic row value
        self.inputs2d = set()
        self.inputs1d = set()

    def shape(self, name):
        return self.prog.buffers[name].shape

    def is_global(self, name):
        return self.prog.buffers[name].scope == "global"

    def set_rows(self, rb):
        if self.rb is None:
            self.rb = rb
        need(self.rb == rb, "inconsistent rows per block")

    def global_row_ok(self, e, ivar):
        need(self.rb is not None, "row tile size unknown")
        need(_aff_is(e, {self.bx: self.rb, ivar: 1}) or (
            _grid_extent(self.prog, self.bx) == 1 and _aff_is(e, {ivar: 1})), "global row index must be bx*rows + i")

    def note_cols(self, n):
        n = _dim(n)
        if self.cols is None:
            self.cols = n
        need(self.cols == n, "inconsistent row lengths")

    # ---- expressions
    def ev(self, e, ivar, jvar, guard=None):
        if isinstance(e, Const):
            return e
        if isinstance(e, Load):
            buf = e.buf
            if self.is_global(buf):
                shp = self.shape(buf)
                if len(shp) == 2:
                    self.global_row_ok(e.idx[0], ivar)
                    need(jvar is not None and _aff_is(e.idx[1], {jvar: 1}), "global column index must be j")
                    self.note_cols(shp[1])
                    self.inputs2d.add(buf)
                    return X(buf)
                if len(shp) == 1:
                    need(jvar is not None and _aff_is(e.idx[0], {jvar: 1}), "1-D parameters are indexed by j")
                    self.inputs1d.add(buf)
                    return W(buf)
                raise NoMatch("unsupported global rank")
            shp = self.shape(buf)
            need(buf in self.tile, f"{buf} read before it is written")
            if len(shp) == 2:
                need(_aff_is(e.idx[0], {ivar: 1}) and jvar is not None and _aff_is(e.idx[1], {jvar: 1}),
                     "tiles are read at [i, j]")
                return self.tile[buf]
            if len(shp) == 1:
                need(_aff_is(e.idx[0], {ivar: 1}), "row vectors are read at [i]")
                return self.tile[buf]
            raise NoMatch("unsupported tile rank")
        if isinstance(e, Bin):
            return Bin(e.op, self.ev(e.a, ivar, jvar, guard), self.ev(e.b, ivar, jvar, guard))
        if isinstance(e, Call):
            return Call(e.fn, tuple(self.ev(a, ivar, jvar, guard) for a in e.args))
        if isinstance(e, Select):
            limit = self.col_guard(e.cond, jvar)
            return Pad(self.ev(e.a, ivar, jvar), self.ev(e.b, ivar, jvar), limit)
        raise NoMatch(f"unsupported row expression {type(e).__name__}")

    def col_guard(self, cond, jvar):
        need(isinstance(cond, Cmp) and cond.op == "<" and isinstance(cond.a, Var) and cond.a.name == jvar,
             "only `j < n` column guards are recognised")
        need(isinstance(cond.b, Const) or isinstance(cond.b, Var), "column guard bound")
        return cond.b.value if isinstance(cond.b, Const) else cond.b.name

    # ---- statements
    def run(self, stmts):
        for s in _body(stmts):
            self.stmt(s)

    def stmt(self, s):
        if isinstance(s, Parallel):
            need(len(s.vars) in (1, 2), "row kernels use T.Parallel(rows) or T.Parallel(rows, cols)")
            self.set_rows(s.extents[0])
            ivar = s.vars[0]
            jvar = s.vars[1] if len(s.vars) == 2 else None
            width = s.extents[1] if jvar else None
            self.parallel(s.body, ivar, jvar, width, None)
            return
        if isinstance(s, Reduce):
            need(s.dim == 1 and len(self.shape(s.src)) == 2, "row reductions reduce dim 1 of a 2-D tile")
            need(s.clear, "accumulating reductions are not recognised in row kernels")
            need(s.src in self.tile, "reduction of an unwritten tile")
            self.tile[s.dst] = Red(s.kind, self.tile[s.src])
            return
        if isinstance(s, Fill):
            self.tile[s.buf] = Const(s.value)
            return
        if isinstance(s, Copy):
            src, dst = s.src, s.dst
            if self.is_global(src.buf) and not self.is_global(dst.buf):
                need(len(self.shape(src.buf)) == 2, "row copies load 2-D rows")
                rows = self.shape(dst.buf)[0]
                self.set_rows(rows)
                need(_aff_is(src.starts[0], {self.bx: rows}) or (
                    _grid_extent(self.prog, self.bx) == 1 and _aff_is(src.starts[0], {})), "copy rows at bx*rows")
                need(_aff_is(src.starts[1], {}), "copies take whole rows")
                self.note_cols(self.shape(src.buf)[1])
                need(self.shape(dst.buf)[1] == self.cols, "tile width must equal the row length")
                self.inputs2d.add(src.buf)
                self.tile[dst.buf] = X(src.buf)
                return
            if not self.is_global(src.buf) and self.is_global(dst.buf):
                need(src.buf in self.tile, "copy of an unwritten tile")
                need(_aff_is(dst.starts[0], {self.bx: self.rb}) or (
                    _grid_extent(self.prog, self.bx) == 1 and _aff_is(dst.starts[0], {})), "copy rows at bx*rows")
                need(_aff_is(dst.starts[1], {}), "copies write whole rows")
                self.note_cols(self.shape(dst.buf)[1])
                self.out[dst.buf] = self.tile[src.buf]
                return
            if not self.is_global(src.buf) and not self.is_global(dst.buf):
                need(src.buf in self.tile, "copy of an unwritten tile")
                self.tile[dst.buf] = self.tile[src.buf]
                return
            raise NoMatch("global-to-global copy")
        raise NoMatch(f"unsupported statement {type(s).__name__} in a row kernel")

    def parallel(self, body, ivar, jvar, width, guard):
        for s in body:
            if isinstance(s, Store):
                self.store(s, ivar, jvar, guard)
            elif isinstance(s, If):
                limit = self.col_guard(s.cond, jvar)
                before = dict(self.tile)
                self.parallel(s.then, ivar, jvar, width, limit)
                then_tile = dict(self.tile)
                self.tile = dict(before)
                self.parallel(s.orelse, ivar, jvar, width, ("else", limit))
                else_tile = self.tile
                merged = dict(before)
                for name in set(then_tile) | set(else_tile):
                    t, e = then_tile.get(name), else_tile.get(name)
                    if t is e:
                        merged[name] = t
                    elif t is not None and e is not None and t != before.get(name) and e != before.get(name):
                        merged[name] = Pad(t, e, limit)
                    elif t is not None and t != before.get(name):
                        merged[name] = Pad(t, before.get(name, Const(math.nan)), limit)
                    else:
                        merged[name] = Pad(before.get(name, Const(math.nan)), e, limit)
                self.tile = merged
            elif isinstance(s, Let):
                raise NoMatch("scalar accumulation inside T.Parallel")
            else:
                raise NoMatch(f"unsupported {type(s).__name__} inside T.Parallel")

    def store(self, s, ivar, jvar, guard):
        value = self.ev(s.value, ivar, jvar, guard)
        buf = s.buf
        if self.is_global(buf):
            shp = self.shape(buf)
            need(len(shp) == 2, "row kernels store 2-D rows")
            self.global_row_ok(s.idx[0], ivar)
            need(jvar is not None and _aff_is(s.idx[1], {jvar: 1}), "stores index columns with j")
            need(not (isinstance(guard, tuple)), "stores in the padding branch")
            self.note_cols(shp[1])
            self.out[buf] = value
            return
        shp = self.shape(buf)
        if len(shp) == 2:
            need(jvar is not None and _aff_is(s.idx[0], {ivar: 1}) and _aff_is(s.idx[1], {jvar: 1}),
                 "tiles are written at [i, j]")
        else:
            need(_aff_is(s.idx[0], {ivar: 1}), "row vectors are written at [i]")
        self.tile[buf] = value


def _strip_pad(e, cols, pad_value):
    """X-like value with optional padding beyond ``cols`` equal to ``pad_value``."""
    if isinstance(e, Pad):
        need(e.limit == cols, "padding guard must be the row length")
        need(isinstance(e.pad, Const) and (e.pad.value == pad_value or (
            math.isnan(pad_value) is False and e.pad.value == pad_value)), "unexpected padding value")
        return e.value
    return e


def _match_softmax(prog: Program) -> OpSpec:
    ev = RowEval(prog)
    ev.run(prog.body)
    need(len(ev.out) == 1, "softmax writes one output")
    (out_name, y), = ev.out.items()
    y = _fold(y)
    need(isinstance(y, Bin) and y.op == "/", "softmax output is e / sum(e)")
    num, den = y.a, y.b
    need(isinstance(den, Red) and den.kind == "sum", "denominator is a row sum")
    num = _strip_pad(num, ev.cols, 0.0) if isinstance(num, Pad) else num
    need(num == _strip_pad(den.expr, ev.cols, 0.0) or num == den.expr, "numerator equals the summed term")
    need(isinstance(num, Call) and num.fn == "exp" and isinstance(num.args[0], Bin) and num.args[0].op == "-",
         "term is exp(x - max)")
    x, mx = num.args[0].a, num.args[0].b
    need(isinstance(mx, Red) and mx.kind == "max", "subtracted value is the row max")
    xs = _strip_pad(x, ev.cols, -math.inf)
    need(isinstance(xs, X), "softmax input is a row of a parameter")
    need(_strip_pad(mx.expr, ev.cols, -math.inf) == xs, "row max is over the same input")
    need(xs.name != out_name, "in-place softmax is not supported")
    rows = _dim(prog.buffers[xs.name].shape[0])
    need(prog.buffers[out_name].shape == prog.buffers[xs.name].shape, "input and output shapes match")
    need(_covers(prog, ev.bx, ev.rb, prog.buffers[xs.name].shape[0]), "grid must cover every row")
    need(prog.buffers[xs.name].dtype == "float32" and prog.buffers[out_name].dtype == "float32",
         "softmax kernels are float32")
    return OpSpec("softmax", {"rows": rows, "cols": ev.cols},
                  {"x": _param_index(prog, xs.name), "y": _param_index(prog, out_name)})


def _match_rmsnorm(prog: Program) -> OpSpec:
    ev = RowEval(prog)
    ev.run(prog.body)
    need(len(ev.out) == 1, "rmsnorm writes one output")
    (out_name, y), = ev.out.items()
    y = _fold(y)
    # (x * inv) * w   with  inv = rsqrt(sum(x*x) * inv_n + eps)
    need(isinstance(y, Bin) and y.op == "*", "rmsnorm output is (x * inv) * w")
    left, w = y.a, y.b
    if isinstance(left, W):
        left, w = w, left
    need(isinstance(w, W), "scale is a 1-D weight parameter")
    need(isinstance(left, Bin) and left.op == "*", "x * inv")
    x, inv = left.a, left.b
    if isinstance(x, Call):
        x, inv = inv, x
    xs = _strip_pad(x, ev.cols, 0.0)
    need(isinstance(xs, X), "normalised value is an input row")
    need(isinstance(inv, Call) and inv.fn == "rsqrt", "inverse RMS uses rsqrt")
    arg = inv.args[0]
    need(isinstance(arg, Bin) and arg.op == "+", "rsqrt(mean + eps)")
    mean, eps = arg.a, arg.b
    if isinstance(mean, Const):
        mean, eps = eps, mean
    need(isinstance(eps, Const), "eps is a constant")
    need(isinstance(mean, Bin) and mean.op in ("*", "/"), "mean = sum * inv_n")
    ss, scale = mean.a, mean.b
    if isinstance(ss, Const):
        ss, scale = scale, ss
    need(isinstance(scale, Const), "mean scale is a constant")
    inv_n = float(scale.value) if mean.op == "*" else 1.0 / float(scale.value)
    need(isinstance(ss, Red) and ss.kind == "sum", "sum of squares")
    sq = _strip_pad(ss.expr, ev.cols, 0.0)
    need(isinstance(sq, Bin) and sq.op == "*" and _strip_pad(sq.a, ev.cols, 0.0) == xs
         and _strip_pad(sq.b, ev.cols, 0.0) == xs, "squares of the same input row")
    shape = prog.buffers[xs.name].shape
    need(prog.buffers[out_name].shape == shape, "input and output shapes match")
    need(prog.buffers[w.name].shape == (shape[1],), "weight length equals the row length")
    need(_covers(prog, ev.bx, ev.rb, shape[0]), "grid must cover every row")
    need(all(prog.buffers[n].dtype == "float32" for n in (xs.name, w.name, out_name)), "rmsnorm kernels are float32")
    return OpSpec("rmsnorm", {"rows": _dim(shape[0]), "cols": ev.cols, "eps": float(eps.value), "inv_n": inv_n},
                  {"x": _param_index(prog, xs.name), "w": _param_index(prog, w.name), "y": _param_index(prog, out_name)})


def _mean_of(e, cols):
    """``Red(sum, row) * inv_n`` (or ``/ n``) -> (row, inv_n)."""
    need(isinstance(e, Bin) and e.op in ("*", "/"), "mean = sum * inv_n")
    red, scale = e.a, e.b
    if isinstance(red, Const) and e.op == "*":
        red, scale = scale, red
    need(isinstance(scale, Const), "mean scale is a constant")
    need(isinstance(red, Red) and red.kind == "sum", "mean of a row sum")
    inv_n = float(scale.value) if e.op == "*" else 1.0 / float(scale.value)
    return _strip_pad(red.expr, cols, 0.0), inv_n


def _match_layernorm(prog: Program) -> OpSpec:
    """examples/layernorm.py:18-43: y = ((x - mean) * rstd) * w + b, mean = sum(x) * (1/n),
    rstd = rsqrt(sum((x - mean)^2) * (1/n) + eps); padded columns contribute 0 to both sums."""
    ev = RowEval(prog)
    ev.run(prog.body)
    need(len(ev.out) == 1, "layernorm writes one output")
    (out_name, y), = ev.out.items()
    y = _fold(y)
    need(isinstance(y, Bin) and y.op == "+", "layernorm output is (...) * w + b")
    scaled, b = y.a, y.b
    if isinstance(scaled, W):
        scaled, b = b, scaled
    need(isinstance(b, W), "shift is a 1-D parameter")
    need(isinstance(scaled, Bin) and scaled.op == "*", "((x - mean) * rstd) * w")
    norm, w = scaled.a, scaled.b
    if isinstance(norm, W):
        norm, w = w, norm
    need(isinstance(w, W), "scale is a 1-D parameter")
    need(isinstance(norm, Bin) and norm.op == "*", "(x - mean) * rstd")
    centred, rstd = norm.a, norm.b
    if isinstance(centred, Call):
        centred, rstd = rstd, centred
    need(isinstance(centred, Bin) and centred.op == "-", "x - mean")
    xs = _strip_pad(centred.a, ev.cols, 0.0)
    need(isinstance(xs, X), "normalised value is an input row")
    row, inv_n = _mean_of(centred.b, ev.cols)
    need(row == xs, "mean of the same input row")
    need(isinstance(rstd, Call) and rstd.fn == "rsqrt", "rstd uses rsqrt")
    arg = rstd.args[0]
    need(isinstance(arg, Bin) and arg.op == "+", "rsqrt(var + eps)")
    var, eps = arg.a, arg.b
    if isinstance(var, Const):
        var, eps = eps, var
    need(isinstance(eps, Const), "eps is a constant")
    sq, inv_n2 = _mean_of(var, ev.cols)
    need(inv_n2 == inv_n, "mean and variance use the same 1/n")
    need(isinstance(sq, Bin) and sq.op == "*" and sq.a == sq.b, "variance of a square")
    d = sq.a
    need(isinstance(d, Bin) and d.op == "-" and _strip_pad(d.a, ev.cols, 0.0) == xs
         and _mean_of(d.b, ev.cols) == (xs, inv_n), "squares of x - mean")
    shape = prog.buffers[xs.name].shape
    need(prog.buffers[out_name].shape == shape, "input and output shapes match")
    need(prog.buffers[w.name].shape == (shape[1],) and prog.buffers[b.name].shape == (shape[1],),
         "weight and bias lengths equal the row length")
    need(xs.name != out_name, "in-place layernorm is not supported")
    need(_covers(prog, ev.bx, ev.rb, shape[0]), "grid must cover every row")
    need(all(prog.buffers[n].dtype == "float32" for n in (xs.name, w.name, b.name, out_name)),
         "layernorm kernels are float32")
    return OpSpec("layernorm", {"rows": _dim(shape[0]), "cols": ev.cols, "eps": float(eps.value), "inv_n": inv_n},
                  {"x": _param_index(prog, xs.name), "w": _param_index(prog, w.name), "b": _param_index(prog, b.name),
                   "y": _param_index(prog, out_name)})


# ------------------------------------------------------------------------------ transpose


def _match_transpose(prog: Program) -> OpSpec:
    """examples/transpose.py:5-15: B[by*T + i, bx*T + j] = tile[j, i] after
    tile[i, j] = A[bx*T + i, by*T + j], i.e. B = A^T (out-of-range elements untouched)."""
    need(len(prog.grid) == 2, "transpose uses a 2-D grid")
    bx, by = prog.block_vars
    body = _body(prog.body)
    need(len(body) == 2 and all(isinstance(s, Parallel) for s in body), "two T.Parallel loops")
    load, store = body
    need(len(load.vars) == 2 and len(store.vars) == 2 and load.extents == store.extents
         and load.extents[0] == load.extents[1], "square tile loops")
    t = load.extents[0]
    need(len(load.body) == 1 and len(store.body) == 1, "one statement per loop")
    li, lj = load.vars
    st0 = load.body[0]
    if isinstance(st0, Copy):
        need(st0.src.point and st0.dst.point, "element copies")
        src_buf, src_idx, tile, tile_idx = st0.src.buf, st0.src.starts, st0.dst.buf, st0.dst.starts
    else:
        need(isinstance(st0, Store) and isinstance(st0.value, Load), "tile[i, j] = A[...]")
        src_buf, src_idx, tile, tile_idx = st0.value.buf, st0.value.idx, st0.buf, st0.idx
    need(prog.buffers[tile].scope in ("shared", "fragment") and prog.buffers[tile].shape == (t, t), "a T x T tile")
    need(_aff_is(tile_idx[0], {li: 1}) and _aff_is(tile_idx[1], {lj: 1}), "tile written at [i, j]")
    need(_aff_is(src_idx[0], {bx: t, li: 1}) and _aff_is(src_idx[1], {by: t, lj: 1}), "A read at [bx*T + i, by*T + j]")
    si, sj = store.vars
    st1 = store.body[0]
    need(isinstance(st1, Store) and isinstance(st1.value, Load) and st1.value.buf == tile, "B[...] = tile[j, i]")
    need(_aff_is(st1.value.idx[0], {sj: 1}) and _aff_is(st1.value.idx[1], {si: 1}), "tile read at [j, i]")
    need(_aff_is(st1.idx[0], {by: t, si: 1}) and _aff_is(st1.idx[1], {bx: t, sj: 1}), "B written at [by*T + i, bx*T + j]")
    a, b = src_buf, st1.buf
    need(_is_param(prog, a) and _is_param(prog, b) and a != b, "distinct parameters A and B")
    m, n = prog.buffers[a].shape
    need(prog.buffers[b].shape == (n, m), "B has the transposed shape")
    need(_covers(prog, bx, t, m) and _covers(prog, by, t, n), "grid must cover A")
    need(prog.buffers[a].dtype == "float32" and prog.buffers[b].dtype == "float32", "transpose kernels are float32")
    return OpSpec("transpose", {"m": _dim(m), "n": _dim(n)}, {"a": _param_index(prog, a), "b": _param_index(prog, b)})


# ----------------------------------------------------------------------------- elementwise


def _match_elementwise(prog: Program) -> OpSpec:
    body = _body(prog.body)
    need(len(prog.grid) == 1 and len(body) == 1 and isinstance(body[0], Parallel), "one T.Parallel loop")
    par = body[0]
    need(len(par.vars) == 1 and len(par.body) == 1 and isinstance(par.body[0], Store), "one element store")
    st = par.body[0]
    block = par.extents[0]
    bx = prog.block_vars[0]
    v = st.value
    need(isinstance(v, Bin) and v.op in ("+", "-", "*") and isinstance(v.a, Load) and isinstance(v.b, Load),
         "C[i] = A[i] op B[i]")
    names = (v.a.buf, v.b.buf, st.buf)
    need(all(_is_param(prog, n) for n in names), "operands are kernel parameters")
    shapes = [prog.buffers[n].shape for n in names]
    need(all(len(s) == 1 for s in shapes) and shapes[0] == shapes[1] == shapes[2], "1-D operands of one length")
    need(all(prog.buffers[n].dtype == "float32" for n in names), "elementwise kernels are float32")
    expect = {bx: block, par.vars[0]: 1}
    for idx in (st.idx, v.a.idx, v.b.idx):
        need(len(idx) == 1 and (_aff_is(idx[0], expect) or (
            _grid_extent(prog, bx) == 1 and _aff_is(idx[0], {par.vars[0]: 1}))), "index bx*block + i")
    n = shapes[0][0]
    g = _grid_extent(prog, bx)
    count = _dim(n) if (g is None or isinstance(n, SymDim)) else min(n, g * block)
    need(st.buf not in (v.a.buf, v.b.buf), "in-place elementwise is not supported")
    return OpSpec("elementwise", {"op": v.op, "n": _dim(n), "count": count},
                  {"a": _param_index(prog, v.a.buf), "b": _param_index(prog, v.b.buf), "c": _param_index(prog, st.buf)})


# --------------------------------------------------------------------------------- cumsum


def _match_cumsum(prog: Program) -> OpSpec:
    """Row scans: one load copy of a parameter into a tile, T.cumsum / T.cummax calls on that
    loaded tile (in place or into another tile), and store copies of the scanned tiles
    (examples/cumsum.py:7-14, examples/scan.py:7-21)."""
    body = _body(prog.body)
    scans = [s for s in body if isinstance(s, Scan)]
    need(len(scans) >= 1, "one T.cumsum")
    need(len(prog.grid) == 1, "row scans use a 1-D grid")
    bx = prog.block_vars[0]
    first = body.index(scans[0])
    pre = body[:first]
    need(len(pre) == 1 and isinstance(pre[0], Copy), "one load copy before the scan")
    load = pre[0]
    src_param, tile = load.src.buf, load.dst.buf
    need(_is_param(prog, src_param) and not _is_param(prog, tile), "load copies a parameter into a tile")
    tshape = prog.buffers[tile].shape
    content = {tile: None}  # tile -> None (the loaded rows) or (kind, reverse)
    stores = []
    for s in body[first:]:
        if isinstance(s, Scan):
            need(s.src.buf in content and content[s.src.buf] is None, "scan reads the loaded tile")
            need(tuple(s.src.extents) == tuple(tshape) and tuple(s.dst.extents) == tuple(tshape),
                 "scan covers the whole tile")
            need(all(_aff_is(x, {}) for x in s.src.starts + s.dst.starts), "scan covers the whole tile")
            need(s.dim == len(tshape) - 1, "scans run along the last dimension")
            need(prog.buffers[s.dst.buf].dtype == "float32" and prog.buffers[s.dst.buf].shape == tshape,
                 "float32 scan tiles of one shape")
            content[s.dst.buf] = (s.kind, bool(s.reverse))
        elif isinstance(s, Copy):
            need(s.src.buf in content and content[s.src.buf] is not None and _is_param(prog, s.dst.buf),
                 "store copies the scanned tile out")
            stores.append((s, content[s.src.buf]))
        else:
            raise NoMatch(f"unsupported {type(s).__name__} in a scan kernel")
    need(stores, "store copies the scanned tile out")
    pshape = prog.buffers[src_param].shape
    outs = []
    for st, (kind, rev) in stores:
        dst_param = st.dst.buf
        need(prog.buffers[dst_param].shape == pshape, "input and output shapes match")
        need(prog.buffers[dst_param].dtype == "float32", "cumsum kernels are float32")
        need(dst_param != src_param, "in-place scans are not supported")
        outs.append((kind, rev, dst_param))
    need(prog.buffers[src_param].dtype == "float32" and prog.buffers[tile].dtype == "float32",
         "cumsum kernels are float32")
    need(len({d for _, _, d in outs}) == len(outs), "each output written once")
    if len(pshape) == 1:
        need(tshape == pshape and _grid_extent(prog, bx) == 1, "1-D scans take the whole vector")
        rows, cols = 1, _dim(pshape[0])
    else:
        need(len(pshape) == 2 and len(tshape) == 2, "2-D row scans")
        rb, cols = tshape[0], pshape[1]
        need(tshape[1] == cols, "tile width equals the row length")
        for region in [load.src] + [st.dst for st, _ in stores]:
            need(_aff_is(region.starts[0], {bx: rb}) or (_grid_extent(prog, bx) == 1 and _aff_is(region.starts[0], {})),
                 "copies move rows bx*rows .. +rows")
            need(_aff_is(region.starts[1], {}), "copies move whole rows")
            need(region.point or region.extents[0] in (rb, None), "copy row extent equals the tile rows")
        need(_covers(prog, bx, rb, pshape[0]), "grid must cover every row")
        rows, cols = _dim(pshape[0]), _dim(cols)
    x = _param_index(prog, src_param)
    if len(outs) == 1:
        kind, rev, dst = outs[0]
        family = "cumsum" if kind == "sum" else "cummax"
        return OpSpec(family, {"rows": rows, "cols": cols, "reverse": rev}, {"x": x, "y": _param_index(prog, dst)})
    return OpSpec("scans", {"rows": rows, "cols": cols, "scans": tuple((k, r) for k, r, _ in outs)},
                  {"x": x, **{f"y{i}": _param_index(prog, d) for i, (_, _, d) in enumerate(outs)}})


# ----------------------------------------------------------------------------------- GEMM


def _match_gemm(prog: Program) -> OpSpec:
    body = _body(prog.body)
    gemms = [s for s in _walk(body) if isinstance(s, Gemm)]
    need(len(gemms) == 1, "one T.gemm")
    g = gemms[0]
    need(not g.transpose_a, "transpose_A is not supported")
    buf = prog.buffers
    # K loop (or a single k-tile without a loop)
    loops = [s for s in body if isinstance(s, Loop)]
    need(len(loops) <= 1, "one K loop")
    if loops:
        loop = loops[0]
        need(isinstance(loop.start, Const) and loop.start.value == 0 and loop.step is None, "K loop starts at 0, step 1")
        kbody = _body(loop.body)
        kvar = loop.var
        trips = loop.stop.value if isinstance(loop.stop, Const) else None
    else:
        loop, kvar, trips = None, None, 1
        kbody = [s for s in body if isinstance(s, (Copy, Gemm))][:3]
    need(len(kbody) == 3 and isinstance(kbody[2], Gemm) and all(isinstance(s, Copy) for s in kbody[:2]),
         "K step = copy A tile, copy B tile, gemm")
    ca, cb = kbody[0], kbody[1]
    if ca.dst.buf != g.a:
        ca, cb = cb, ca
    need(ca.dst.buf == g.a and cb.dst.buf == g.b, "copies feed the gemm operands")
    A, B = ca.src.buf, cb.src.buf
    C_acc = g.c
    need(_is_param(prog, A) and _is_param(prog, B), "operands come from parameters")
    need(buf[A].dtype == "float16" and buf[B].dtype == "float16", "fp16 operands")
    need(buf[C_acc].dtype == "float32", "fp32 accumulator")
    need(len(buf[A].shape) == 2 and len(buf[B].shape) == 2, "2-D operands")
    M, K = buf[A].shape
    bm, bk = buf[g.a].shape
    if g.transpose_b:
        N, K2 = buf[B].shape
        bn, bk2 = buf[g.b].shape
    else:
        K2, N = buf[B].shape
        bk2, bn = buf[g.b].shape
    need(_dim(K) == _dim(K2) and bk == bk2, "A and B agree on K")
    need(buf[C_acc].shape == (bm, bn), "accumulator tile is block_m x block_n")

    def tile_var(e, size):
        f = _aff(e)
        f = {k: v for k, v in f.items() if v != 0}
        if not f:
            return None
        need(len(f) == 1, "tile origin uses one index variable")
        (var, coef), = f.items()
        need(coef == size and var != 1, "tile origin = index * tile")
        return var

    m_origin, k_origin_a = ca.src.starts
    if g.transpose_b:
        n_origin, k_origin_b = cb.src.starts
    else:
        k_origin_b, n_origin = cb.src.starts
    mvar, nvar = tile_var(m_origin, bm), tile_var(n_origin, bn)
    for ko in (k_origin_a, k_origin_b):
        kv = tile_var(ko, bk)
        need(kv == kvar, "K tile origin uses the K loop variable")
    need(mvar != nvar or mvar is None, "distinct M and N block indices")
    for var, tile, ext in ((mvar, bm, M), (nvar, bn, N)):
        if var is None:
            need(isinstance(ext, int) and tile >= ext, "a fixed tile must cover its dimension")
        else:
            need(var in prog.block_vars, "tile origins use block indices")
            need(_covers(prog, var, tile, ext), "grid must cover the output")
    if trips is not None and isinstance(K, int):
        need(trips * bk >= K, "K loop must cover K")
    # accumulator initialisation
    pre = body[: body.index(loop)] if loop is not None else [s for s in body if isinstance(s, Fill)]
    fills = [s for s in pre if isinstance(s, Fill) and s.buf == C_acc]
    if g.clear_accum:
        need(trips == 1, "clear_accum inside a multi-step K loop keeps only the last K tile")
    else:
        need(len(fills) == 1 and fills[0].value == 0.0, "accumulator cleared before the K loop")
    # epilogue
    post = body[body.index(loop) + 1:] if loop is not None else [s for s in body if not isinstance(s, (Copy, Gemm, Fill))] + [
        s for s in body if isinstance(s, Copy) and s.src.buf == C_acc]
    if loop is None:
        post = [s for s in body if s not in kbody and not (isinstance(s, Fill) and s.buf == C_acc)]
    ep = Epilogue(prog, C_acc, mvar, nvar, bm, bn)
    out_name = ep.run(post)
    need(out_name is not None and _is_param(prog, out_name), "result stored to a parameter")
    need(buf[out_name].dtype == "float32" and tuple(map(_dim, buf[out_name].shape)) == (_dim(M), _dim(N)),
         "C is float32 [M, N]")
    alpha, bias, relu = ep.canonical()
    params = {"M": _dim(M), "N": _dim(N), "K": _dim(K), "transpose_b": bool(g.transpose_b),
              "alpha": alpha, "bias_mode": bias[0] if bias else 0, "relu": relu}
    args = {"a": _param_index(prog, A), "b": _param_index(prog, B), "c": _param_index(prog, out_name)}
    if bias:
        args["bias"] = _param_index(prog, bias[1])
        need(buf[bias[1]].dtype == "float32", "float32 bias")
    return OpSpec("gemm", params, args)


BIAS_NONE, BIAS_N, BIAS_MN, BIAS_M = 0, 1, 2, 3


@dataclass(frozen=True)
class BiasRef:
    name: str
    mode: int


class Epilogue:
    """Symbolic per-element evaluation of what follows the K loop of a GEMM."""

    def __init__(self, prog, acc, mvar, nvar, bm, bn):
        self.prog, self.acc, self.mvar, self.nvar, self.bm, self.bn = prog, acc, mvar, nvar, bm, bn
        self.tile = {acc: Acc()}
        self.result = None

    def origin_ok(self, starts):
        m, n = starts
        em = {self.mvar: self.bm} if self.mvar else {}
        en = {self.nvar: self.bn} if self.nvar else {}
        return _aff_is(m, em) and _aff_is(n, en)

    def run(self, stmts):
        out = None
        for s in stmts:
            if isinstance(s, Copy):
                src, dst = s.src, s.dst
                gsrc = self.prog.buffers[src.buf].scope == "global"
                gdst = self.prog.buffers[dst.buf].scope == "global"
                if gsrc and not gdst:
                    need(self.prog.buffers[src.buf].shape.__len__() == 2 and self.origin_ok(src.starts),
                         "bias tiles are copied at the output tile origin")
                    self.tile[dst.buf] = BiasRef(src.buf, BIAS_MN)
                elif not gsrc and gdst:
                    need(src.buf in self.tile and self.origin_ok(dst.starts), "result copied at the tile origin")
                    self.result = self.tile[src.buf]
                    out = dst.buf
                else:
                    need(src.buf in self.tile, "copy of an unwritten tile")
                    self.tile[dst.buf] = self.tile[src.buf]
            elif isinstance(s, Parallel):
                need(len(s.vars) == 2 and tuple(s.extents) == (self.bm, self.bn), "epilogue runs over the tile")
                i, j = s.vars
                for st in s.body:
                    need(isinstance(st, Store), "epilogue statements are element stores")
                    v = self.ev(st.value, i, j)
                    if self.prog.buffers[st.buf].scope == "global":
                        em = {self.mvar: self.bm, i: 1} if self.mvar else {i: 1}
                        en = {self.nvar: self.bn, j: 1} if self.nvar else {j: 1}
                        need(_aff_is(st.idx[0], em) and _aff_is(st.idx[1], en), "stores at the tile origin + (i, j)")
                        self.result, out = v, st.buf
                    else:
                        need(_aff_is(st.idx[0], {i: 1}) and _aff_is(st.idx[1], {j: 1}), "tile stores at [i, j]")
                        self.tile[st.buf] = v
            else:
                raise NoMatch(f"unsupported epilogue statement {type(s).__name__}")
        return out

    def ev(self, e, i, j):
        if isinstance(e, Const):
            return e
        if isinstance(e, Load):
            b = self.prog.buffers[e.buf]
            if b.scope != "global":
                need(e.buf in self.tile, f"{e.buf} read before written")
                need(_aff_is(e.idx[0], {i: 1}) and _aff_is(e.idx[1], {j: 1}), "tile reads at [i, j]")
                return self.tile[e.buf]
            if len(b.shape) == 1:
                if _aff_is(e.idx[0], {self.nvar: self.bn, j: 1} if self.nvar else {j: 1}):
                    return BiasRef(e.buf, BIAS_N)
                if _aff_is(e.idx[0], {self.mvar: self.bm, i: 1} if self.mvar else {i: 1}):
                    return BiasRef(e.buf, BIAS_M)
                raise NoMatch("1-D epilogue operand must be indexed by the row or column")
            em = {self.mvar: self.bm, i: 1} if self.mvar else {i: 1}
            en = {self.nvar: self.bn, j: 1} if self.nvar else {j: 1}
            need(_aff_is(e.idx[0], em) and _aff_is(e.idx[1], en), "bias matrix read at the output element")
            return BiasRef(e.buf, BIAS_MN)
        if isinstance(e, Bin):
            return Bin(e.op, self.ev(e.a, i, j), self.ev(e.b, i, j))
        if isinstance(e, Call):
            return Call(e.fn, tuple(self.ev(a, i, j) for a in e.args))
        raise NoMatch("unsupported epilogue expression")

    def canonical(self):
        """result -> (alpha, (bias_mode, bias_name) | None, relu)."""
        e = _fold(self.result)
        relu = False
        if isinstance(e, Call) and e.fn in ("max", "maximum") and len(e.args) == 2:
            a, b = e.args
            if isinstance(a, Const):
                a, b = b, a
            need(isinstance(b, Const) and b.value == 0.0, "max(x, 0) is the only activation")
            relu, e = True, a
        bias = None
        if isinstance(e, Bin) and e.op == "+":
            a, b = e.a, e.b
            if isinstance(a, BiasRef):
                a, b = b, a
            need(isinstance(b, BiasRef), "epilogue adds a bias operand")
            bias = (b.mode, b.name)
            e = a
        alpha = 1.0
        if isinstance(e, Bin) and e.op == "*":
            a, b = e.a, e.b
            if isinstance(a, Const):
                a, b = b, a
            need(isinstance(b, Const), "accumulator scale is a constant")
            alpha, e = float(b.value), a
        need(isinstance(e, Acc), "epilogue = [relu](alpha * acc [+ bias])")
        return alpha, bias, relu


def _walk(stmts):
    for s in stmts:
        yield s
        for attr in ("body", "then", "orelse"):
            inner = getattr(s, attr, None)
            if isinstance(inner, list):
                yield from _walk(inner)


# ------------------------------------------------------------------------------------ FA2


def _match_fa2(prog: Program) -> OpSpec:
    body = _body(prog.body)
    gemms = [s for s in _walk(body) if isinstance(s, Gemm)]
    need(len(gemms) == 2, "two T.gemm calls (QK^T and PV)")
    qk, pv = gemms
    need(qk.transpose_b and qk.clear_accum and not pv.transpose_b, "S = Q K^T (cleared), O += P V")
    params = [p for p in prog.params if isinstance(p, TensorParameter)]
    need(len(params) == 4 and len(prog.params) == 4, "Q, K, V, Out parameters")
    buf = prog.buffers
    need(len(prog.grid) == 3, "grid (q_tiles, heads, batch)")
    bx, by, bz = prog.block_vars
    loops = [s for s in body if isinstance(s, Loop)]
    need(len(loops) == 1, "one KV loop")
    loop = loops[0]
    need(loop.step is None, "KV loop steps by 1")
    lbody = _body(loop.body)
    copies = [s for s in lbody if isinstance(s, Copy) and buf[s.src.buf].scope == "global"]
    need(len(copies) == 2, "KV loop copies K and V tiles")
    kcopy = next(c for c in copies if c.dst.buf == qk.b)
    vcopy = next(c for c in copies if c.dst.buf == pv.b)
    qcopy = next((s for s in body if isinstance(s, Copy) and s.dst.buf == qk.a), None)
    need(qcopy is not None, "Q tile copied before the loop")
    Q, Kp, V = qcopy.src.buf, kcopy.src.buf, vcopy.src.buf
    outs = [s for s in body[body.index(loop) + 1:] if isinstance(s, Copy) and buf[s.dst.buf].scope == "global"]
    need(len(outs) == 1, "output tile copied after the loop")
    O = outs[0].dst.buf
    need(len({Q, Kp, V, O}) == 4, "distinct Q, K, V, Out")
    shp = buf[Q].shape
    need(len(shp) == 4 and all(buf[n].shape == shp for n in (Kp, V, O)), "Q, K, V, Out share [B, H, S, D]")
    need(all(buf[n].dtype == "float16" for n in (Q, Kp, V, O)), "fp16 attention tensors")
    Bsz, H, S, D = shp
    bm = buf[qk.a].shape[0]
    bn = buf[qk.b].shape[0]
    need(buf[qk.a].shape[1] == D and buf[qk.b].shape[1] == D and buf[pv.b].shape == (bn, D), "tiles span head_dim")
    # index structure Q[bz, by, bx*bm : +bm, :]
    need(_aff_is(qcopy.src.starts[0], {bz: 1}) and _aff_is(qcopy.src.starts[1], {by: 1})
         and _aff_is(qcopy.src.starts[2], {bx: bm}), "Q tile at [bz, by, bx*block_m]")
    for c in (kcopy, vcopy):
        need(_aff_is(c.src.starts[0], {bz: 1}) and _aff_is(c.src.starts[1], {by: 1})
             and _aff_is(c.src.starts[2], {loop.var: bn}), "K/V tiles at [bz, by, k*block_n]")
    need(_aff_is(outs[0].dst.starts[2], {bx: bm}), "output tile at bx*block_m")
    need(_covers(prog, bx, bm, S) and _covers(prog, by, 1, H) and _covers(prog, bz, 1, Bsz), "grid covers B, H, S")
    # causal mask and scale
    causal = False
    scale = None
    for s in lbody:
        if isinstance(s, Parallel):
            for st in s.body:
                if not isinstance(st, Store):
                    continue
                if st.buf == qk.c and isinstance(st.value, Select):
                    cond = st.value.cond
                    need(isinstance(cond, Cmp) and cond.op == ">=", "causal mask keeps q >= k")
                    need(_aff_is(cond.a, {bx: bm, s.vars[0]: 1}) and _aff_is(cond.b, {loop.var: bn, s.vars[1]: 1}),
                         "causal mask compares query and key positions")
                    fill = _fold(st.value.b)
                    need(isinstance(fill, Const) and fill.value <= -1e30, "masked scores use a large negative fill")
                    causal = True
                if st.buf == qk.c and isinstance(st.value, Call) and st.value.fn == "exp2":
                    arg = st.value.args[0]
                    need(isinstance(arg, Bin) and arg.op == "-", "exp2(s*scale - max*scale)")
                    for side in (arg.a, arg.b):
                        need(isinstance(side, Bin) and side.op == "*", "scaled operands")
                        c = side.b if isinstance(side.b, Const) else side.a
                        need(isinstance(c, Const), "constant softmax scale")
                        scale = float(c.value) if scale is None else scale
                        need(abs(float(c.value) - scale) <= 1e-12 * abs(scale), "one softmax scale")
    need(scale is not None, "softmax exponent exp2(s*scale - m*scale) found")
    reduces = [s for s in lbody if isinstance(s, Reduce)]
    need([r.kind for r in reduces] == ["max", "sum"], "row max then row sum")
    need(not reduces[0].clear, "running max keeps the previous maximum")
    if isinstance(loop.stop, Const):
        trips = loop.stop.value
        need(isinstance(S, int) and trips * bn >= S, "KV loop covers the sequence")
    else:
        need(causal, "a block-dependent KV loop bound is the causal form")
    return OpSpec("fa2", {"batch": _dim(Bsz), "heads": _dim(H), "seq": _dim(S), "dim": _dim(D),
                          "scale_log2": scale, "causal": causal},
                  {"q": _param_index(prog, Q), "k": _param_index(prog, Kp), "v": _param_index(prog, V),
                   "o": _param_index(prog, O)})


MATCHERS = (
    ("fa2", _match_fa2),
    ("gemm", _match_gemm),
    ("cumsum", _match_cumsum),
    ("softmax", _match_softmax),
    ("rmsnorm", _match_rmsnorm),
    ("layernorm", _match_layernorm),
    ("transpose", _match_transpose),
    ("elementwise", _match_elementwise),
)


def recognize(prog: Program) -> OpSpec:
    if any(isinstance(p, ScalarParameter) for p in prog.params):
        raise CompileError(f"{prog.name}: scalar kernel parameters are not used by the recognised op families")
    reasons = []
    for name, matcher in MATCHERS:
        try:
            return matcher(prog)
        except NoMatch as exc:
            reasons.append(f"{name}: {exc}")
        except (IndexError, KeyError, StopIteration, ValueError, TypeError) as exc:
            reasons.append(f"{name}: {type(exc).__name__} {exc}")
    raise CompileError(
        f"{prog.name}: program is not one of the op families implemented by the sm_100a kernels "
        "(elementwise, cumsum / cummax, softmax, rmsnorm, layernorm, transpose, gemm, fa2):\n  " + "\n  ".join(reasons)
    )


__all__ = ["BIAS_M", "BIAS_MN", "BIAS_N", "BIAS_NONE", "OpSpec", "recognize"]
