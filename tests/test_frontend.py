"""CPU tests of the drop-in surface: parsing, op recognition, out_idx, jit caching,
``patch_tilelang``, dynamic shapes and argument checks (no GPU needed)."""

from __future__ import annotations


import pytest

import ntilang
import ntilang as tilelang
import ntilang.language as T
from ntilang_b200 import kernels as K
from ntilang_b200.compat import normalize_out_idx
from ntilang_b200.ir import CompileError, ScalarParameter, TensorParameter, TensorType



def test_alias_package_is_the_implementation():
    import ntilang_b200

    assert ntilang is ntilang_b200
    assert T is ntilang_b200.language
    for name in ("jit", "compile", "CompiledKernel", "DynamicJitKernel", "autotune", "AutoTuner",
                 "patch_tilelang", "CompileError", "SymDim", "language", "layout"):
        assert hasattr(ntilang, name), name


def test_patch_tilelang_context_manager():
    with ntilang.patch_tilelang():
        import tilelang as patched
        import tilelang.language as patched_lang
        import tilelang.layout as patched_layout

        assert patched is ntilang
        assert patched_lang is T
        assert patched_layout is ntilang.layout


@pytest.mark.parametrize("factory,args,family,params", [
    (K.vector_add, (1000,), "elementwise", {"op": "+", "n": 1000}),
    (K.cumsum, (32768, 256), "cumsum", {"rows": 32768, "cols": 256, "reverse": False}),
    (K.cumsum, (7, 65, True), "cumsum", {"rows": 7, "cols": 65, "reverse": True}),
    (K.softmax, (16384, 512), "softmax", {"rows": 16384, "cols": 512}),
    (K.softmax, (9, 113), "softmax", {"rows": 9, "cols": 113}),
    (K.rmsnorm, (4096, 1024), "rmsnorm", {"rows": 4096, "cols": 1024, "eps": 1e-6}),
    (K.layernorm, (4096, 1024), "layernorm", {"rows": 4096, "cols": 1024, "eps": 1e-5, "inv_n": 1.0 / 1024}),
    (K.layernorm, (131, 100, 1e-6), "layernorm", {"rows": 131, "cols": 100, "eps": 1e-6}),
    (K.transpose, (65, 71), "transpose", {"m": 65, "n": 71}),
    (K.transpose, (4096, 4096), "transpose", {"m": 4096, "n": 4096}),
    (K.matmul, (4096, 4096, 4096), "gemm", {"M": 4096, "bias_mode": 0, "relu": False, "alpha": 1.0}),
    (K.matmul_bias_relu, (256, 512, 64), "gemm", {"bias_mode": 1, "relu": True}),
    (K.matmul_scaled_bias_relu, (65, 71, 37), "gemm", {"bias_mode": 2, "relu": True, "alpha": 0.5}),
    (K.flash_attention, (8, 32, 4096, 128), "fa2", {"causal": False, "dim": 128}),
    (K.flash_attention, (2, 4, 256, 64, True), "fa2", {"causal": True, "seq": 256}),
])
def test_factories_recognised(factory, args, family, params):
    kern = factory(*args)
    assert kern.spec.family == family
    for key, value in params.items():
        assert kern.spec.params[key] == value, key
    assert kern.out_idx == (len(kern.ir.params) - 1,)
    assert family in kern.source


def test_fa2_scale_is_log2e_over_sqrt_d():
    import math

    kern = K.flash_attention(1, 1, 128, 64)
    assert kern.spec.params["scale_log2"] == pytest.approx(math.log2(math.e) / 8.0, rel=1e-12)


def test_jit_factory_cache():
    assert K.softmax(64, 128) is K.softmax(64, 128)
    assert K.softmax(64, 128) is not K.softmax(64, 256)


def test_direct_jit_kernel():
    @tilelang.jit(out_idx=[-1], target="auto")
    def direct_add(A: T.Tensor((128,), "float32"), B: T.Tensor((128,), "float32"), C: T.Tensor((128,), "float32")):
        with T.Kernel(1, threads=128) as bx:
            for i in T.Parallel(128):
                C[bx * 128 + i] = A[bx * 128 + i] + B[bx * 128 + i]

    assert direct_add.out_idx == (2,)
    assert direct_add.spec.family == "elementwise"


def test_gemm_variants_recognised():
    @T.prim_func
    def single_tile(A: T.Tensor((32, 32), "float16"), B: T.Tensor((32, 32), "float16"),
                    C: T.Tensor((32, 32), "float32")):
        with T.Kernel(1, 1, threads=128):
            sa = T.alloc_shared((32, 32), "float16")
            sb = T.alloc_shared((32, 32), "float16")
            acc = T.alloc_local((32, 32), "float32")
            T.copy(A[0, 0], sa)
            T.copy(B[0, 0], sb)
            T.gemm(sa, sb, acc, clear_accum=True)
            for i, j in T.Parallel(32, 32):
                acc[i, j] = T.max(acc[i, j], -T.infinity("float32"))
            T.copy(acc, C[0, 0])

    k = ntilang.compile(single_tile)
    assert k.spec.family == "gemm" and k.spec.params["M"] == 32 and k.spec.params["relu"] is False

    @tilelang.jit(out_idx=[-1])
    def swizzled(m, n, kk):
        @T.prim_func
        def main(A: T.Tensor((m, kk), "float16"), B: T.Tensor((kk, n), "float16"), C: T.Tensor((m, n), "float32")):
            with T.Kernel(T.ceildiv(m, 32), T.ceildiv(n, 32), threads=128) as (bx, by):
                sa = T.alloc_shared((32, 32), "float16")
                sb = T.alloc_shared((32, 32), "float16")
                acc = T.alloc_fragment((32, 32), "float32")
                T.use_swizzle(panel_size=2, order="row")
                T.annotate_layout({sa: tilelang.layout.make_swizzled_layout(sa)})
                T.clear(acc)
                for ko in T.serial(T.ceildiv(kk, 32)):
                    T.copy(A[bx * 32, ko * 32], sa)
                    T.copy(B[ko * 32, by * 32], sb)
                    T.gemm(sa, sb, acc, policy=T.GemmWarpPolicy.Square)
                T.copy(acc, C[bx * 32, by * 32])

        return main

    assert swizzled(65, 71, 37).spec.params == {"M": 65, "N": 71, "K": 37, "transpose_b": False, "alpha": 1.0,
                                                 "bias_mode": 0, "relu": False}


def test_partial_k_loop_is_rejected():
    @T.prim_func
    def bad(A: T.Tensor((64, 128), "float16"), B: T.Tensor((128, 64), "float16"), C: T.Tensor((64, 64), "float32")):
        with T.Kernel(1, 1, threads=128) as (bx, by):
            sa = T.alloc_shared((64, 32), "float16")
            sb = T.alloc_shared((32, 64), "float16")
            acc = T.alloc_fragment((64, 64), "float32")
            T.clear(acc)
            for ko in T.serial(2):
                T.copy(A[bx * 64, ko * 32], sa)
                T.copy(B[ko * 32, by * 64], sb)
                T.gemm(sa, sb, acc)
            T.copy(acc, C[bx * 64, by * 64])

    with pytest.raises(CompileError, match="K loop must cover K"):
        ntilang.compile(bad)


def test_unsupported_program_raises_compile_error():
    @T.prim_func
    def fused_multiply_add(A: T.Tensor((1024,), "float32"), B: T.Tensor((1024,), "float32"),
                           C: T.Tensor((1024,), "float32"), D: T.Tensor((1024,), "float32")):
        with T.Kernel(4, threads=256) as bx:
            for i in T.Parallel(256):
                D[bx * 256 + i] = A[bx * 256 + i] * B[bx * 256 + i] + C[bx * 256 + i]

    # Not a recognised family: it runs on the generic elementwise (NVRTC) path.
    kern = ntilang.compile(fused_multiply_add)
    assert kern.spec.family == "pointwise"
    assert "ntl_pw_fused_multiply_add" in kern.get_kernel_source()

    @T.prim_func
    def shifted_fragment(A: T.Tensor((64,), "float32"), B: T.Tensor((64,), "float32")):
        with T.Kernel(1, threads=64):
            tile = T.alloc_fragment((64,), "float32")
            T.copy(A, tile)
            for i in T.Parallel(63):
                B[i] = tile[i + 1]

    with pytest.raises(CompileError, match="not one of the op families(.|\n)*pointwise: .*slot mapping"):
        ntilang.compile(shifted_fragment)


def test_transpose_with_store_load_form_is_recognised():
    @T.prim_func
    def transpose(A: T.Tensor((64, 96), "float32"), B: T.Tensor((96, 64), "float32")):
        with T.Kernel(2, 3, threads=128) as (bx, by):
            tile = T.alloc_shared((32, 32), "float32")
            for i, j in T.Parallel(32, 32):
                tile[i, j] = A[bx * 32 + i, by * 32 + j]
            for i, j in T.Parallel(32, 32):
                B[by * 32 + i, bx * 32 + j] = tile[j, i]

    kern = ntilang.compile(transpose)
    assert kern.spec.family == "transpose" and kern.spec.params == {"m": 64, "n": 96}


def test_softmax_without_padding_and_with_copy_load():
    @T.prim_func
    def sm(A: T.Tensor((64, 128), "float32"), B: T.Tensor((64, 128), "float32")):
        with T.Kernel(16, threads=128) as bx:
            tile = T.alloc_fragment((4, 128), "float32")
            mx = T.alloc_fragment((4,), "float32")
            sm_ = T.alloc_fragment((4,), "float32")
            T.copy(A[bx * 4 : bx * 4 + 4, :], tile)
            T.reduce_max(tile, mx, dim=1)
            for i, j in T.Parallel(4, 128):
                tile[i, j] = T.exp(tile[i, j] - mx[i])
            T.reduce_sum(tile, sm_, dim=1)
            for i, j in T.Parallel(4, 128):
                B[bx * 4 + i, j] = tile[i, j] / sm_[i]

    assert ntilang.compile(sm).spec.family == "softmax"


def test_wrong_math_is_not_softmax():
    @T.prim_func
    def not_sm(A: T.Tensor((64, 128), "float32"), B: T.Tensor((64, 128), "float32")):
        with T.Kernel(16, threads=128) as bx:
            tile = T.alloc_fragment((4, 128), "float32")
            mx = T.alloc_fragment((4,), "float32")
            sm_ = T.alloc_fragment((4,), "float32")
            T.copy(A[bx * 4 : bx * 4 + 4, :], tile)
            T.reduce_max(tile, mx, dim=1)
            for i, j in T.Parallel(4, 128):
                tile[i, j] = T.exp2(tile[i, j] - mx[i])
            T.reduce_sum(tile, sm_, dim=1)
            for i, j in T.Parallel(4, 128):
                B[bx * 4 + i, j] = tile[i, j] / sm_[i]

    with pytest.raises(CompileError):
        ntilang.compile(not_sm)


def test_grid_must_cover_rows():
    @T.prim_func
    def short(A: T.Tensor((64, 128), "float32"), B: T.Tensor((64, 128), "float32")):
        with T.Kernel(8, threads=128) as bx:
            tile = T.alloc_fragment((4, 128), "float32")
            T.copy(A[bx * 4 : bx * 4 + 4, :], tile)
            T.cumsum(tile, dim=1)
            T.copy(tile, B[bx * 4 : bx * 4 + 4, :])

    with pytest.raises(CompileError, match="cover"):
        ntilang.compile(short)


def test_dynamic_softmax_single_symbolic_compile():
    M = T.dynamic("m")

    @tilelang.jit(out_idx=[-1], target="sm_100a")
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

    assert isinstance(dyn_softmax, ntilang.DynamicJitKernel)
    kern = dyn_softmax._try_symbolic("sm_100a")
    assert kern is not None and kern.spec.family == "softmax" and kern.spec.params["rows"] == "m"

    import numpy as np

    k1 = dyn_softmax.specialize(np.ones((10, 128), np.float32))
    assert k1 is dyn_softmax.specialize(np.ones((10, 128), np.float32))
    assert k1 is not dyn_softmax.specialize(np.ones((18, 128), np.float32))
    assert k1.spec.params["rows"] == 10


def test_out_idx_normalisation():
    params = (TensorParameter("a", TensorType((4,), "float32")), TensorParameter("b", TensorType((4,), "float32")),
              ScalarParameter("s", "int32"))
    assert normalize_out_idx(-2, params) == (1,)
    assert normalize_out_idx([0, 1], params) == (0, 1)
    with pytest.raises(ValueError, match="scalar"):
        normalize_out_idx(-1, params)
    with pytest.raises(ValueError, match="Duplicate"):
        normalize_out_idx([0, -3], params)
    with pytest.raises(ValueError, match="out of range"):
        normalize_out_idx(3, params)
    with pytest.raises(TypeError):
        normalize_out_idx([0.5], params)


def test_call_checks_reject_cpu_tensors():
    torch = pytest.importorskip("torch")
    kern = K.vector_add(16)
    with pytest.raises(TypeError, match="CUDA tensor"):
        kern(torch.zeros(16), torch.zeros(16), torch.zeros(16))
    with pytest.raises(TypeError, match="Expected 3 arguments"):
        kern(torch.zeros(16))


def test_markers_raise_when_executed():
    with pytest.raises(RuntimeError, match="syntax"):
        T.copy(1, 2)
    with pytest.raises(TypeError):
        K.softmax(4, 4).ir  # noqa: B018 - attribute access works
        T.prim_func(lambda: None)()


def test_reference_examples_are_recognised():
    """The reference's own example programs compile unchanged under ``import ntilang``."""
    from tests.conftest import load_reference_example as load

    expect = {
        ("vector_add", ()): "elementwise", ("cumsum", ()): "cumsum", ("softmax", ()): "softmax",
        ("rmsnorm", ()): "rmsnorm", ("matmul", ()): "gemm", ("matmul_relu", ()): "gemm",
        ("flash_attention", ()): "fa2", ("layernorm", ()): "layernorm", ("transpose", ()): "transpose",
        ("scan", ()): "scans", ("fragment_affine", ()): "pointwise", ("piecewise", ()): "pointwise",
        ("window_sum", ()): "pointwise",
    }
    for (name, args), family in expect.items():
        kern = getattr(load(name), name)(*args)
        assert kern.spec.family == family, name
    fa = load("flash_attention").flash_attention(8, 32, 4096, 128, is_causal=True)
    assert fa.spec.params["causal"] is True


def test_layernorm_with_wrong_variance_is_not_recognised():
    """sum(x*x) in place of sum((x - mean)^2) is RMS-style, not LayerNorm: reject it."""
    width, cols, rows_per_block = 128, 100, 4

    @T.prim_func
    def not_layernorm(X: T.Tensor((8, cols), "float32"), G: T.Tensor((cols,), "float32"),
                      Bb: T.Tensor((cols,), "float32"), Y: T.Tensor((8, cols), "float32")):
        with T.Kernel(T.ceildiv(8, rows_per_block), threads=128) as b:
            xs = T.alloc_fragment((rows_per_block, width), "float32")
            sq = T.alloc_fragment((rows_per_block, width), "float32")
            acc = T.alloc_fragment((rows_per_block,), "float32")
            var = T.alloc_fragment((rows_per_block,), "float32")
            for r, c in T.Parallel(rows_per_block, width):
                xs[r, c] = X[b * rows_per_block + r, c] if c < cols else 0.0
                sq[r, c] = xs[r, c] * xs[r, c]
            T.reduce_sum(xs, acc, dim=1)
            T.reduce_sum(sq, var, dim=1)
            for r, c in T.Parallel(rows_per_block, width):
                if c < cols:
                    Y[b * rows_per_block + r, c] = ((xs[r, c] - acc[r] * 0.01) * T.rsqrt(var[r] * 0.01 + 1e-5)) * G[c] + Bb[c]

    with pytest.raises(CompileError):
        tilelang.compile(not_layernorm)


def test_transpose_with_untransposed_read_is_not_recognised():
    @T.prim_func
    def copy_not_transpose(A: T.Tensor((64, 64), "float32"), B: T.Tensor((64, 64), "float32")):
        with T.Kernel(2, 2, threads=128) as (bx, by):
            t = T.alloc_shared((32, 32), "float32")
            for i, j in T.Parallel(32, 32):
                T.copy(A[bx * 32 + i, by * 32 + j], t[i, j])
            for i, j in T.Parallel(32, 32):
                B[by * 32 + i, bx * 32 + j] = t[i, j]

    with pytest.raises(CompileError):
        tilelang.compile(copy_not_transpose)
