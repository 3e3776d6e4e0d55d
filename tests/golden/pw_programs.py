"""Generic elementwise programs for the pointwise (NVRTC) path.

Each factory takes the ``T`` module and the ``compile`` function of the package that builds
it: ``make_golden.py`` builds them under the reference package to produce golden vectors with
its evaluator, the tests build them under ``ntilang_b200``.  Together with the reference's own
examples/fragment_affine.py, piecewise.py and window_sum.py they cover float32 / float16
arithmetic and promotion, Python-style integer floor division, bitwise operators and shifts,
Boolean logic and selects, while loops, break and continue,
scalar parameters, 2-D grids with partial tiles, fragment copies and atomics.
"""

from __future__ import annotations

import numpy as np


def scaled_shift(T, compile, n=300, block=128):
    @T.prim_func
    def scaled_shift(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), alpha: T.float32,
                     beta: T.float32):
        with T.Kernel(T.ceildiv(n, block), threads=128) as bx:
            for i in T.Parallel(block):
                B[bx * block + i] = A[bx * block + i] * alpha + beta

    return compile(scaled_shift)


def half_mix(T, compile, n=257, block=64):
    @T.prim_func
    def half_mix(A: T.Tensor((n,), "float16"), B: T.Tensor((n,), "float32"), C: T.Tensor((n,), "float16"),
                 D: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, block), threads=64) as bx:
            for i in T.Parallel(block):
                a = A[bx * block + i]
                b = B[bx * block + i]
                C[bx * block + i] = a * a - a / T.float16(3.0) + T.cast(b, "float16")
                D[bx * block + i] = b * a + T.cast(a, "float32") * 0.25

    return compile(half_mix)


def int_floor(T, compile, n=200, block=64):
    @T.prim_func
    def int_floor(X: T.Tensor((n,), "int32"), Q: T.Tensor((n,), "int32"), R: T.Tensor((n,), "int32")):
        with T.Kernel(T.ceildiv(n, block), threads=64) as bx:
            for i in T.Parallel(block):
                x = X[bx * block + i]
                Q[bx * block + i] = x // 7 - x // -3
                R[bx * block + i] = x % 7 + x % -3 + (x * 3 + 1) % 4

    return compile(int_floor)


def select_logic(T, compile, m=37, n=45, bm=8, bn=16):
    @T.prim_func
    def select_logic(A: T.Tensor((m, n), "float32"), B: T.Tensor((m, n), "float32"), C: T.Tensor((m, n), "float32")):
        with T.Kernel(T.ceildiv(n, bn), T.ceildiv(m, bm), threads=128) as (bx, by):
            for i, j in T.Parallel(bm, bn):
                a = A[by * bm + i, bx * bn + j]
                b = B[by * bm + i, bx * bn + j]
                C[by * bm + i, bx * bn + j] = T.if_then_else((a > b) and (a > 0.0), a - b,
                                                             T.if_then_else(a < -1.0 or b < -1.0, a * b, T.max(a, b)))

    return compile(select_logic)


def tile_copy(T, compile, m=50, n=70, bm=16, bn=32):
    @T.prim_func
    def tile_copy(A: T.Tensor((m, n), "float32"), B: T.Tensor((m, n), "float32")):
        with T.Kernel(T.ceildiv(n, bn), T.ceildiv(m, bm), threads=128) as (bx, by):
            tile = T.alloc_fragment((bm, bn), "float32")
            T.copy(A[by * bm, bx * bn], tile)
            for i, j in T.Parallel(bm, bn):
                tile[i, j] = tile[i, j] * 0.5 - 1.0
            T.copy(tile, B[by * bm, bx * bn])

    return compile(tile_copy)


def histogram(T, compile):
    @T.prim_func
    def histogram(X: T.Tensor((64,), "int32"), Out: T.Tensor((8,), "int32"), MaxOut: T.Tensor((8,), "int32")):
        with T.Kernel(1, threads=64):
            for i in T.Parallel(64):
                bucket = X[i] % 8
                T.atomic_add(Out[bucket], 1)
                T.atomic_max(MaxOut[bucket], i)

    return compile(histogram)


def bit_mix(T, compile, n=256):
    @T.prim_func
    def bit_mix(X: T.Tensor((n,), "int32"), U: T.Tensor((n,), "uint32"), Y: T.Tensor((n,), "int32"),
                V: T.Tensor((n,), "uint32")):
        with T.Kernel(T.ceildiv(n, 128), threads=128) as bx:
            for i in T.Parallel(128):
                x = X[bx * 128 + i]
                u = U[bx * 128 + i]
                Y[bx * 128 + i] = ((x & 255) | (x >> 3)) ^ (~x << 2)
                V[bx * 128 + i] = ((u >> 5) ^ (u << 7)) | (u & 3855)

    return compile(bit_mix)


def lane_loops(T, compile, n=90):
    """Per-point while loops with lane-dependent trip counts, and a serial loop with
    continue / break whose exit depends on the data."""

    @T.prim_func
    def lane_loops(X: T.Tensor((n,), "int32"), Tri: T.Tensor((n,), "int32"), Acc: T.Tensor((n,), "int32")):
        with T.Kernel(T.ceildiv(n, 32), threads=32) as bx:
            for i in T.Parallel(32):
                left = T.alloc_var("int32", X[bx * 32 + i])
                tri = T.alloc_var("int32", 0)
                while left > 0:
                    tri += left
                    left -= 1
                Tri[bx * 32 + i] = tri
                acc = T.alloc_var("int32", 0)
                for k in T.serial(24):
                    if k % 3 == 1:
                        continue
                    if acc > X[bx * 32 + i] * 4:
                        break
                    acc += k
                Acc[bx * 32 + i] = acc

    return compile(lane_loops)


def strided_rows(T, compile, rows=37, cols=50):
    """Serial loops with a start, a positive step and a negative step over each row."""

    @T.prim_func
    def strided_rows(X: T.Tensor((rows, cols), "float32"), Even: T.Tensor((rows,), "float32"),
                     Back: T.Tensor((rows,), "float32")):
        with T.Kernel(T.ceildiv(rows, 16), threads=16) as bx:
            for r in T.Parallel(16):
                even = T.alloc_var("float32", 0)
                back = T.alloc_var("float32", 0)
                for c in T.serial(1, cols, 2):
                    even += X[bx * 16 + r, c]
                for c in T.serial(cols - 1, 0, -3):
                    back = back * 0.5 + X[bx * 16 + r, c]
                Even[bx * 16 + r] = even
                Back[bx * 16 + r] = back

    return compile(strided_rows)


# name -> (factory, input builder(seed) -> list of arrays in parameter order (outputs NaN / 0 filled),
#          indices of output arrays, scalar arguments after the arrays)
def _f32(rng, *shape, scale=1.0):
    return (rng.normal(size=shape) * scale).astype(np.float32)


PROGRAMS = {
    "scaled_shift": (scaled_shift, lambda rng: [_f32(rng, 300), np.full(300, np.nan, np.float32)], (1,),
                     (1.75, -0.3)),
    "half_mix": (half_mix, lambda rng: [_f32(rng, 257, scale=4.0).astype(np.float16), _f32(rng, 257),
                                        np.full(257, np.nan, np.float16), np.full(257, np.nan, np.float32)], (2, 3), ()),
    "int_floor": (int_floor, lambda rng: [rng.integers(-1000, 1000, size=200).astype(np.int32),
                                          np.zeros(200, np.int32), np.zeros(200, np.int32)], (1, 2), ()),
    "select_logic": (select_logic, lambda rng: [_f32(rng, 37, 45, scale=2.0), _f32(rng, 37, 45, scale=2.0),
                                                np.full((37, 45), np.nan, np.float32)], (2,), ()),
    "tile_copy": (tile_copy, lambda rng: [_f32(rng, 50, 70), np.full((50, 70), np.nan, np.float32)], (1,), ()),
    "bit_mix": (bit_mix, lambda rng: [rng.integers(-2**31, 2**31 - 1, size=256, dtype=np.int64).astype(np.int32),
                                      rng.integers(0, 2**32 - 1, size=256, dtype=np.uint64).astype(np.uint32),
                                      np.zeros(256, np.int32), np.zeros(256, np.uint32)], (2, 3), ()),
    "lane_loops": (lane_loops, lambda rng: [rng.integers(-5, 30, size=90).astype(np.int32),
                                            np.zeros(90, np.int32), np.zeros(90, np.int32)], (1, 2), ()),
    "strided_rows": (strided_rows, lambda rng: [_f32(rng, 37, 50), np.full(37, np.nan, np.float32),
                                                np.full(37, np.nan, np.float32)], (1, 2), ()),
    "histogram": (histogram, lambda rng: [rng.integers(-50, 50, size=64).astype(np.int32),
                                          np.zeros(8, np.int32), np.full(8, -1, np.int32)], (1, 2), ()),
}


# The computations of the reference's examples/fragment_affine.py, piecewise.py and
# window_sum.py, written here so the GPU tests need no reference checkout; their outputs are
# checked against the goldens produced from the reference's own example programs.


def tile_affine(T, compile, n=257, block=96):
    @T.prim_func
    def tile_affine(X: T.Tensor((n,), "float32"), Y: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, block), threads=64) as b:
            frag = T.alloc_fragment((block,), "float32")
            T.copy(X[b * block], frag)
            for k in T.Parallel(block):
                Y[b * block + k] = frag[k] * 2.0 + 1.0

    return compile(tile_affine)


def three_piece(T, compile, n=93, width=32):
    @T.prim_func
    def three_piece(X: T.Tensor((n,), "float32"), Y: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, width), threads=width) as b:
            for k in T.Parallel(width):
                v = X[b * width + k]
                if v < 0.0:
                    Y[b * width + k] = -v
                elif v < 1.0:
                    Y[b * width + k] = v * v
                else:
                    Y[b * width + k] = v + 2.0

    return compile(three_piece)


def clipped_window(T, compile, batch=7, height=3, width=5, lanes=128):
    @T.prim_func
    def clipped_window(X: T.Tensor((batch, height, width), "float32"), Y: T.Tensor((batch,), "float32"),
                       nrows: T.int32, ncols: T.int32):
        with T.Kernel(T.ceildiv(batch, lanes), threads=lanes) as b:
            for k in T.Parallel(lanes):
                acc = T.alloc_var("float32", init=0)
                for r, c in T.grid(T.clamp(nrows, 0, height), T.clamp(ncols, 0, width)):
                    acc += X[b * lanes + k, r, c]
                Y[b * lanes + k] = acc

    return compile(clipped_window)


def generic_fma(T, compile, n=1 << 24, block=1024):
    """D = A * B + C, separately rounded: the bench workload of the generic path."""

    @T.prim_func
    def generic_fma(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), C: T.Tensor((n,), "float32"),
                    D: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, block), threads=256) as b:
            for k in T.Parallel(block):
                D[b * block + k] = A[b * block + k] * B[b * block + k] + C[b * block + k]

    return compile(generic_fma)
