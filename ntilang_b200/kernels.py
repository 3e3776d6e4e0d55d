"""Ready-made ``@jit(out_idx=[-1])`` factories for the hot-path op families.

Each factory returns a TileLang program; ``jit`` reads it, recognises the family and
returns a cached ``CompiledKernel`` whose call allocates the last parameter as the
output, e.g. ``y = softmax(16384, 512)(x)``.  The programs follow the operator semantics
of the reference's examples (vector_add.py, cumsum.py, softmax.py, rmsnorm.py,
layernorm.py, transpose.py, matmul.py, matmul_relu.py, flash_attention.py); the tile sizes written in them are
program-level hints only — the sm_100a kernels choose their own tiles.
"""

from __future__ import annotations

import math

from . import language as T
from .language import jit


@jit(out_idx=[-1])
def vector_add(n, block=256):
    @T.prim_func
    def vadd(X: T.Tensor((n,), "float32"), Y: T.Tensor((n,), "float32"), Z: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, block), threads=block) as b:
            for t in T.Parallel(block):
                Z[b * block + t] = X[b * block + t] + Y[b * block + t]

    return vadd


@jit(out_idx=[-1])
def cumsum(rows, cols, reverse=False, rows_per_block=4):
    @T.prim_func
    def row_scan(X: T.Tensor((rows, cols), "float32"), Y: T.Tensor((rows, cols), "float32")):
        with T.Kernel(T.ceildiv(rows, rows_per_block), threads=128) as b:
            buf = T.alloc_fragment((rows_per_block, cols), "float32")
            T.copy(X[b * rows_per_block : (b + 1) * rows_per_block, :], buf)
            T.cumsum(buf, dim=1, reverse=reverse)
            T.copy(buf, Y[b * rows_per_block : (b + 1) * rows_per_block, :])

    return row_scan


@jit(out_idx=[-1])
def cummax(rows, cols, reverse=False, rows_per_block=4):
    @T.prim_func
    def row_running_max(X: T.Tensor((rows, cols), "float32"), Y: T.Tensor((rows, cols), "float32")):
        with T.Kernel(T.ceildiv(rows, rows_per_block), threads=128) as b:
            buf = T.alloc_fragment((rows_per_block, cols), "float32")
            T.copy(X[b * rows_per_block : (b + 1) * rows_per_block, :], buf)
            T.cummax(buf, dim=1, reverse=reverse)
            T.copy(buf, Y[b * rows_per_block : (b + 1) * rows_per_block, :])

    return row_running_max


@jit(out_idx=[1, 2])
def sum_and_max_scans(rows, cols, reverse=False, rows_per_block=4):
    """Prefix sums and prefix maxima of one loaded tile (the shape of examples/scan.py)."""

    @T.prim_func
    def two_scans(X: T.Tensor((rows, cols), "float32"), Sums: T.Tensor((rows, cols), "float32"),
                  Maxima: T.Tensor((rows, cols), "float32")):
        with T.Kernel(T.ceildiv(rows, rows_per_block), threads=128) as b:
            loaded = T.alloc_fragment((rows_per_block, cols), "float32")
            sums = T.alloc_fragment((rows_per_block, cols), "float32")
            T.copy(X[b * rows_per_block : (b + 1) * rows_per_block, :], loaded)
            T.cumsum(loaded, sums, dim=1, reverse=reverse)
            T.cummax(loaded, dim=1, reverse=reverse)
            T.copy(sums, Sums[b * rows_per_block : (b + 1) * rows_per_block, :])
            T.copy(loaded, Maxima[b * rows_per_block : (b + 1) * rows_per_block, :])

    return two_scans


@jit(out_idx=[-1])
def softmax(rows, cols, rows_per_block=4):
    width = 1 << max(0, (cols - 1).bit_length())
    ninf = -T.infinity("float32")

    @T.prim_func
    def row_softmax(X: T.Tensor((rows, cols), "float32"), Y: T.Tensor((rows, cols), "float32")):
        with T.Kernel(T.ceildiv(rows, rows_per_block), threads=128) as b:
            vals = T.alloc_fragment((rows_per_block, width), "float32")
            peak = T.alloc_fragment((rows_per_block,), "float32")
            total = T.alloc_fragment((rows_per_block,), "float32")
            for r, c in T.Parallel(rows_per_block, width):
                vals[r, c] = X[b * rows_per_block + r, c] if c < cols else ninf
            T.reduce_max(vals, peak, dim=1)
            for r, c in T.Parallel(rows_per_block, width):
                vals[r, c] = T.exp(vals[r, c] - peak[r])
            T.reduce_sum(vals, total, dim=1)
            for r, c in T.Parallel(rows_per_block, width):
                if c < cols:
                    Y[b * rows_per_block + r, c] = vals[r, c] / total[r]

    return row_softmax


@jit(out_idx=[-1])
def rmsnorm(rows, cols, eps=1e-6, rows_per_block=4):
    width = 1 << max(0, (cols - 1).bit_length())
    scale = 1.0 / cols

    @T.prim_func
    def row_rmsnorm(X: T.Tensor((rows, cols), "float32"), G: T.Tensor((cols,), "float32"),
                    Y: T.Tensor((rows, cols), "float32")):
        with T.Kernel(T.ceildiv(rows, rows_per_block), threads=128) as b:
            xs = T.alloc_fragment((rows_per_block, width), "float32")
            sq = T.alloc_fragment((rows_per_block, width), "float32")
            acc = T.alloc_fragment((rows_per_block,), "float32")
            rinv = T.alloc_fragment((rows_per_block,), "float32")
            for r, c in T.Parallel(rows_per_block, width):
                xs[r, c] = X[b * rows_per_block + r, c] if c < cols else 0.0
                sq[r, c] = xs[r, c] * xs[r, c]
            T.reduce_sum(sq, acc, dim=1)
            for r in T.Parallel(rows_per_block):
                rinv[r] = T.rsqrt(acc[r] * scale + eps)
            for r, c in T.Parallel(rows_per_block, width):
                if c < cols:
                    Y[b * rows_per_block + r, c] = xs[r, c] * rinv[r] * G[c]

    return row_rmsnorm


@jit(out_idx=[-1])
def layernorm(rows, cols, eps=1e-5, rows_per_block=4):
    width = 1 << max(0, (cols - 1).bit_length())
    scale = 1.0 / cols

    @T.prim_func
    def row_layernorm(X: T.Tensor((rows, cols), "float32"), G: T.Tensor((cols,), "float32"),
                      Bb: T.Tensor((cols,), "float32"), Y: T.Tensor((rows, cols), "float32")):
        with T.Kernel(T.ceildiv(rows, rows_per_block), threads=128) as b:
            xs = T.alloc_fragment((rows_per_block, width), "float32")
            sq = T.alloc_fragment((rows_per_block, width), "float32")
            acc = T.alloc_fragment((rows_per_block,), "float32")
            var = T.alloc_fragment((rows_per_block,), "float32")
            mean = T.alloc_fragment((rows_per_block,), "float32")
            rstd = T.alloc_fragment((rows_per_block,), "float32")
            for r, c in T.Parallel(rows_per_block, width):
                xs[r, c] = X[b * rows_per_block + r, c] if c < cols else 0.0
            T.reduce_sum(xs, acc, dim=1)
            for r in T.Parallel(rows_per_block):
                mean[r] = acc[r] * scale
            for r, c in T.Parallel(rows_per_block, width):
                if c < cols:
                    d = xs[r, c] - mean[r]
                    sq[r, c] = d * d
                else:
                    sq[r, c] = 0.0
            T.reduce_sum(sq, var, dim=1)
            for r in T.Parallel(rows_per_block):
                rstd[r] = T.rsqrt(var[r] * scale + eps)
            for r, c in T.Parallel(rows_per_block, width):
                if c < cols:
                    Y[b * rows_per_block + r, c] = (xs[r, c] - mean[r]) * rstd[r] * G[c] + Bb[c]

    return row_layernorm


@jit(out_idx=[-1])
def transpose(m, n, tile=32):
    @T.prim_func
    def shared_transpose(A: T.Tensor((m, n), "float32"), B: T.Tensor((n, m), "float32")):
        with T.Kernel(T.ceildiv(m, tile), T.ceildiv(n, tile), threads=128) as (bx, by):
            t = T.alloc_shared((tile, tile), "float32")
            for i, j in T.Parallel(tile, tile):
                T.copy(A[bx * tile + i, by * tile + j], t[i, j])
            for i, j in T.Parallel(tile, tile):
                B[by * tile + i, bx * tile + j] = t[j, i]

    return shared_transpose


def _gemm_program(m, n, k, bm, bn, bk, stages, epilogue, trans_b=False):
    """GEMM program; ``epilogue`` in {None, "bias_relu" (bias[N]), "scaled_bias_relu" (Bias[M,N], 0.5)}."""
    b_shape = (n, k) if trans_b else (k, n)
    sb_shape = (bn, bk) if trans_b else (bk, bn)

    if epilogue is None:

        @T.prim_func
        def gemm(A: T.Tensor((m, k), "float16"), B: T.Tensor(b_shape, "float16"), C: T.Tensor((m, n), "float32")):
            with T.Kernel(T.ceildiv(n, bn), T.ceildiv(m, bm), threads=128) as (nx, my):
                a_s = T.alloc_shared((bm, bk), "float16")
                b_s = T.alloc_shared(sb_shape, "float16")
                acc = T.alloc_fragment((bm, bn), "float32")
                T.clear(acc)
                for kt in T.Pipelined(T.ceildiv(k, bk), num_stages=stages):
                    T.copy(A[my * bm, kt * bk], a_s)
                    if trans_b:
                        T.copy(B[nx * bn, kt * bk], b_s)
                    else:
                        T.copy(B[kt * bk, nx * bn], b_s)
                    T.gemm(a_s, b_s, acc, transpose_B=trans_b)
                T.copy(acc, C[my * bm, nx * bn])

        return gemm

    if epilogue == "bias_relu":

        @T.prim_func
        def gemm_bias_relu(A: T.Tensor((m, k), "float16"), B: T.Tensor(b_shape, "float16"),
                           bias: T.Tensor((n,), "float32"), C: T.Tensor((m, n), "float32")):
            with T.Kernel(T.ceildiv(n, bn), T.ceildiv(m, bm), threads=128) as (nx, my):
                a_s = T.alloc_shared((bm, bk), "float16")
                b_s = T.alloc_shared(sb_shape, "float16")
                acc = T.alloc_fragment((bm, bn), "float32")
                T.clear(acc)
                for kt in T.Pipelined(T.ceildiv(k, bk), num_stages=stages):
                    T.copy(A[my * bm, kt * bk], a_s)
                    if trans_b:
                        T.copy(B[nx * bn, kt * bk], b_s)
                    else:
                        T.copy(B[kt * bk, nx * bn], b_s)
                    T.gemm(a_s, b_s, acc, transpose_B=trans_b)
                for i, j in T.Parallel(bm, bn):
                    acc[i, j] = T.max(acc[i, j] + bias[nx * bn + j], 0.0)
                T.copy(acc, C[my * bm, nx * bn])

        return gemm_bias_relu

    @T.prim_func
    def gemm_scaled_bias_relu(A: T.Tensor((m, k), "float16"), B: T.Tensor(b_shape, "float16"),
                              Bias: T.Tensor((m, n), "float32"), C: T.Tensor((m, n), "float32")):
        with T.Kernel(T.ceildiv(n, bn), T.ceildiv(m, bm), threads=128) as (nx, my):
            a_s = T.alloc_shared((bm, bk), "float16")
            b_s = T.alloc_shared(sb_shape, "float16")
            acc = T.alloc_fragment((bm, bn), "float32")
            bias_t = T.alloc_fragment((bm, bn), "float32")
            T.clear(acc)
            for kt in T.Pipelined(T.ceildiv(k, bk), num_stages=stages):
                T.copy(A[my * bm, kt * bk], a_s)
                if trans_b:
                    T.copy(B[nx * bn, kt * bk], b_s)
                else:
                    T.copy(B[kt * bk, nx * bn], b_s)
                T.gemm(a_s, b_s, acc, transpose_B=trans_b)
            T.copy(Bias[my * bm, nx * bn], bias_t)
            for i, j in T.Parallel(bm, bn):
                acc[i, j] = T.maximum(acc[i, j] * 0.5 + bias_t[i, j], 0.0)
            T.copy(acc, C[my * bm, nx * bn])

    return gemm_scaled_bias_relu


@jit(out_idx=[-1])
def matmul(m, n, k, block_m=128, block_n=256, block_k=64, num_stages=4, trans_b=False):
    return _gemm_program(m, n, k, block_m, block_n, block_k, num_stages, None, trans_b)


@jit(out_idx=[-1])
def matmul_bias_relu(m, n, k, block_m=128, block_n=256, block_k=64, num_stages=4, trans_b=False):
    """C = relu(A @ B + bias[N]) — the fused-epilogue form of the GEMM benchmark."""
    return _gemm_program(m, n, k, block_m, block_n, block_k, num_stages, "bias_relu", trans_b)


@jit(out_idx=[-1])
def matmul_scaled_bias_relu(m, n, k, block_m=128, block_n=256, block_k=64, num_stages=4, trans_b=False):
    """C = relu(0.5 * (A @ B) + Bias[M, N]) — the epilogue of the reference's matmul_relu example."""
    return _gemm_program(m, n, k, block_m, block_n, block_k, num_stages, "scaled_bias_relu", trans_b)


@jit(out_idx=[-1])
def flash_attention(batch, heads, seq_len, dim, is_causal=False, block_m=128, block_n=128):
    qk_scale = math.log2(math.e) / math.sqrt(dim)
    masked = -1e30
    shape = (batch, heads, seq_len, dim)

    @T.prim_func
    def attention(Q: T.Tensor(shape, "float16"), K: T.Tensor(shape, "float16"), V: T.Tensor(shape, "float16"),
                  O: T.Tensor(shape, "float16")):
        with T.Kernel(T.ceildiv(seq_len, block_m), heads, batch, threads=256) as (qt, h, z):
            q_s = T.alloc_shared((block_m, dim), "float16")
            k_s = T.alloc_shared((block_n, dim), "float16")
            v_s = T.alloc_shared((block_n, dim), "float16")
            s = T.alloc_fragment((block_m, block_n), "float32")
            p16 = T.alloc_fragment((block_m, block_n), "float16")
            o = T.alloc_fragment((block_m, dim), "float32")
            m_cur = T.alloc_fragment((block_m,), "float32")
            m_old = T.alloc_fragment((block_m,), "float32")
            rescale = T.alloc_fragment((block_m,), "float32")
            psum = T.alloc_fragment((block_m,), "float32")
            l = T.alloc_fragment((block_m,), "float32")
            T.copy(Q[z, h, qt * block_m : (qt + 1) * block_m, :], q_s)
            T.fill(o, 0.0)
            T.fill(l, 0.0)
            T.fill(m_cur, -T.infinity("float32"))
            kv_tiles = T.ceildiv((qt + 1) * block_m, block_n) if is_causal else T.ceildiv(seq_len, block_n)
            for kt in T.Pipelined(kv_tiles, num_stages=2):
                T.copy(K[z, h, kt * block_n : (kt + 1) * block_n, :], k_s)
                T.copy(V[z, h, kt * block_n : (kt + 1) * block_n, :], v_s)
                T.gemm(q_s, k_s, s, transpose_B=True, clear_accum=True)
                if is_causal:
                    for i, j in T.Parallel(block_m, block_n):
                        s[i, j] = T.if_then_else(qt * block_m + i >= kt * block_n + j, s[i, j], masked)
                T.copy(m_cur, m_old)
                T.reduce_max(s, m_cur, dim=1, clear=False)
                for i in T.Parallel(block_m):
                    rescale[i] = T.exp2(m_old[i] * qk_scale - m_cur[i] * qk_scale)
                for i, d in T.Parallel(block_m, dim):
                    o[i, d] *= rescale[i]
                for i, j in T.Parallel(block_m, block_n):
                    s[i, j] = T.exp2(s[i, j] * qk_scale - m_cur[i] * qk_scale)
                T.reduce_sum(s, psum, dim=1)
                for i in T.Parallel(block_m):
                    l[i] = l[i] * rescale[i] + psum[i]
                T.copy(s, p16)
                T.gemm(p16, v_s, o)
            for i, d in T.Parallel(block_m, dim):
                o[i, d] /= l[i]
            T.copy(o, O[z, h, qt * block_m : (qt + 1) * block_m, :])

    return attention


__all__ = ["cummax", "cumsum", "flash_attention", "layernorm", "matmul", "matmul_bias_relu", "matmul_scaled_bias_relu", "rmsnorm",
           "softmax", "sum_and_max_scans", "transpose", "vector_add"]
