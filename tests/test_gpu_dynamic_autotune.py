"""On the GPU: ``T.dynamic`` family kernels compiled once and launched at several sizes
(``python/ntilang/compiler.py:203-337``; the reference's test is
``tests/test_m34_features.py:86-112``), and ``@autotune`` choosing among configurations of a
family kernel and of a generic kernel with scalar parameters (``tests/test_m34_features.py:150-181``).

Bars: cumsum bit-exact against the oracle (the reference's scan order); softmax and RMSNorm
within 1e-5 relative; GEMM within 1e-3 * (|ref| + max |ref|) of an fp32 product."""

from __future__ import annotations

import numpy as np
import pytest

import ntilang
import ntilang as tilelang
import ntilang.language as T
from oracle import ntl_oracle as O

pytestmark = pytest.mark.gpu
SIZES = (7, 131, 1029)


def to_gpu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dynamic_kernels():
    M = T.dynamic("m")

    @tilelang.jit(out_idx=[-1], target="auto")
    def dyn_cumsum(X: T.Tensor((M, 300), "float32"), Y: T.Tensor((M, 300), "float32")):
        with T.Kernel(T.ceildiv(M, 4), threads=128) as bx:
            tile = T.alloc_fragment((4, 300), "float32")
            T.copy(X[bx * 4 : bx * 4 + 4, :], tile)
            T.cumsum(tile, dim=1)
            T.copy(tile, Y[bx * 4 : bx * 4 + 4, :])

    @tilelang.jit(out_idx=[-1], target="auto")
    def dyn_softmax(A: T.Tensor((M, 128), "float32"), B: T.Tensor((M, 128), "float32")):
        with T.Kernel(T.ceildiv(M, 4), threads=128) as bx:
            tile = T.alloc_fragment((4, 128), "float32")
            row_max = T.alloc_fragment((4,), "float32")
            row_sum = T.alloc_fragment((4,), "float32")
            for i, j in T.Parallel(4, 128):
                tile[i, j] = A[bx * 4 + i, j]
            T.reduce_max(tile, row_max, dim=1)
            for i, j in T.Parallel(4, 128):
                tile[i, j] = T.exp(tile[i, j] - row_max[i])
            T.reduce_sum(tile, row_sum, dim=1)
            for i, j in T.Parallel(4, 128):
                B[bx * 4 + i, j] = tile[i, j] / row_sum[i]

    @tilelang.jit(out_idx=[-1], target="auto")
    def dyn_rmsnorm(X: T.Tensor((M, 1024), "float32"), G: T.Tensor((1024,), "float32"),
                    Y: T.Tensor((M, 1024), "float32")):
        with T.Kernel(T.ceildiv(M, 4), threads=128) as b:
            xs = T.alloc_fragment((4, 1024), "float32")
            sq = T.alloc_fragment((4, 1024), "float32")
            acc = T.alloc_fragment((4,), "float32")
            rinv = T.alloc_fragment((4,), "float32")
            for r, c in T.Parallel(4, 1024):
                xs[r, c] = X[b * 4 + r, c]
                sq[r, c] = xs[r, c] * xs[r, c]
            T.reduce_sum(sq, acc, dim=1)
            for r in T.Parallel(4):
                rinv[r] = T.rsqrt(acc[r] * (1.0 / 1024) + 1e-6)
            for r, c in T.Parallel(4, 1024):
                Y[b * 4 + r, c] = xs[r, c] * rinv[r] * G[c]

    @tilelang.jit(out_idx=[-1], target="auto")
    def dyn_gemm(A: T.Tensor((M, 256), "float16"), B: T.Tensor((256, 384), "float16"),
                 C: T.Tensor((M, 384), "float32")):
        with T.Kernel(T.ceildiv(384, 128), T.ceildiv(M, 128), threads=128) as (bx, by):
            sa = T.alloc_shared((128, 32), "float16")
            sb = T.alloc_shared((32, 128), "float16")
            acc = T.alloc_fragment((128, 128), "float32")
            T.clear(acc)
            for ko in T.Pipelined(T.ceildiv(256, 32), num_stages=3):
                T.copy(A[by * 128, ko * 32], sa)
                T.copy(B[ko * 32, bx * 128], sb)
                T.gemm(sa, sb, acc)
            T.copy(acc, C[by * 128, bx * 128])

    return {"cumsum": dyn_cumsum, "softmax": dyn_softmax, "rmsnorm": dyn_rmsnorm, "gemm": dyn_gemm}


@pytest.mark.parametrize("family", ["cumsum", "softmax", "rmsnorm", "gemm"])
def test_dynamic_family_compiles_once_for_three_sizes(torch_cuda, family):
    torch = torch_cuda
    kern = dynamic_kernels()[family]
    assert isinstance(kern, ntilang.DynamicJitKernel)
    rng = np.random.default_rng(hash(family) % 1000)
    for rows in SIZES:
        if family == "cumsum":
            x = rng.uniform(-1, 1, size=(rows, 300)).astype(np.float32)
            y = kern(to_gpu(torch, x)).cpu().numpy()
            assert np.array_equal(y.view(np.uint32), O.cumsum_rows(x).view(np.uint32))
        elif family == "softmax":
            x = (rng.normal(size=(rows, 128)) * 2).astype(np.float32)
            y = kern(to_gpu(torch, x)).cpu().numpy()
            np.testing.assert_allclose(y, O.softmax_rows(x), rtol=1e-5, atol=1e-30)
        elif family == "rmsnorm":
            x = rng.normal(size=(rows, 1024)).astype(np.float32)
            w = rng.normal(1, 0.1, size=1024).astype(np.float32)
            y = kern(to_gpu(torch, x), to_gpu(torch, w)).cpu().numpy()
            np.testing.assert_allclose(y, O.rmsnorm_rows(x, w, 1e-6, 1.0 / 1024), rtol=1e-5, atol=1e-7)
        else:
            a = (rng.normal(size=(rows, 256)) / 16).astype(np.float16)
            b = (rng.normal(size=(256, 384)) / 16).astype(np.float16)
            c = kern(to_gpu(torch, a), to_gpu(torch, b)).cpu().numpy()
            ref = a.astype(np.float32) @ b.astype(np.float32)
            assert np.all(np.abs(c - ref) <= 1e-3 * (np.abs(ref) + np.abs(ref).max()))
        assert kern.compile_count == 1, family
    # the one compile is the symbolic one: no per-size specialisation was made
    assert not kern._cache
    (sym,) = [k for k in kern._symbolic_cache.values() if k is not None]
    assert sym.spec.family == family


def test_autotune_family_gemm(torch_cuda):
    torch = torch_cuda
    configs = [
        {"block_m": 64, "block_n": 64, "block_k": 32, "num_stages": 2},
        {"block_m": 128, "block_n": 128, "block_k": 32, "num_stages": 3},
        {"block_m": 128, "block_n": 256, "block_k": 64, "num_stages": 4},
    ]

    @tilelang.autotune(configs=configs, warmup=3, rep=10)
    @tilelang.jit(out_idx=[-1], target="auto")
    def tuned_gemm(m, n, k, block_m=64, block_n=64, block_k=32, num_stages=2):
        @T.prim_func
        def main(A: T.Tensor((m, k), "float16"), B: T.Tensor((k, n), "float16"), C: T.Tensor((m, n), "float32")):
            with T.Kernel(T.ceildiv(n, block_n), T.ceildiv(m, block_m), threads=128) as (bx, by):
                sa = T.alloc_shared((block_m, block_k), "float16")
                sb = T.alloc_shared((block_k, block_n), "float16")
                acc = T.alloc_fragment((block_m, block_n), "float32")
                T.use_swizzle(panel_size=8, order="row")
                T.clear(acc)
                for ko in T.Pipelined(T.ceildiv(k, block_k), num_stages=num_stages):
                    T.copy(A[by * block_m, ko * block_k], sa)
                    T.copy(B[ko * block_k, bx * block_n], sb)
                    T.gemm(sa, sb, acc)
                T.copy(acc, C[by * block_m, bx * block_n])

        return main

    best = tuned_gemm(512, 512, 512)
    assert tuned_gemm.best_config in configs
    assert tuned_gemm.best_latency_ms > 0.0
    log = tuned_gemm.timings[((512, 512, 512), ())]
    assert [entry[0] for entry in log] == configs and all(ms is not None and ms > 0 for _, ms, _ in log)
    assert tuned_gemm(512, 512, 512) is best  # cached: no second tuning
    assert len(tuned_gemm.timings) == 1
    a = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    b = torch.randn(512, 512, device="cuda", dtype=torch.float16)
    c = best(a, b)
    torch.testing.assert_close(c, a.float() @ b.float(), rtol=1e-2, atol=1e-2)


def test_autotune_generic_kernel_with_scalar_parameters(torch_cuda):
    torch = torch_cuda

    @tilelang.autotune(configs=[{"block": 128}, {"block": 256}, {"block": 512}], warmup=2, rep=5, out_idx=[1])
    def tuned(n, block=128):
        @T.prim_func
        def scale_shift(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), alpha: T.float32,
                        flip: T.bool, k: T.int32):
            with T.Kernel(T.ceildiv(n, block), threads=128) as bx:
                for i in T.Parallel(block):
                    if flip:
                        B[bx * block + i] = -(A[bx * block + i] * alpha) + T.cast(k, "float32")
                    else:
                        B[bx * block + i] = A[bx * block + i] * alpha + T.cast(k, "float32")

        return scale_shift

    kern = tuned(1 << 20)
    assert kern.spec.family == "pointwise"
    assert tuned.best_config in ({"block": 128}, {"block": 256}, {"block": 512})
    assert tuned.best_latency_ms > 0.0
    assert all(err is None for _, _, err in tuned.timings[((1 << 20,), ())])
    a = torch.randn(1 << 20, device="cuda")
    for flip in (False, True):
        b = kern(a, 1.5, flip, 3)
        want = (-(a * 1.5) if flip else a * 1.5) + 3.0
        assert torch.equal(b, want)
