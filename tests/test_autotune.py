"""``@autotune`` on the CPU: the configuration rules of the reference's tuner
(``python/ntilang/autotune.py:96-137``, used as in ``tests/test_m34_features.py:163-196``), the
untimed choice without CUDA, and the sample arguments (scalar parameters included)."""

from __future__ import annotations

import pytest

import ntilang
import ntilang as tilelang
import ntilang.language as T
from ntilang_b200.autotune import SYMBOLIC_SIZE, sample_arguments
from ntilang_b200.ir import CompileError

torch = pytest.importorskip("torch")
needs_no_cuda = pytest.mark.skipif(torch.cuda.is_available(), reason="checks the untimed path")


def scaled(n, block=128):
    @T.prim_func
    def scale_shift(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), alpha: T.float32,
                    flip: T.bool, k: T.int32):
        with T.Kernel(T.ceildiv(n, block), threads=128) as bx:
            for i in T.Parallel(block):
                B[bx * block + i] = A[bx * block + i] * alpha + T.cast(k, "float32")

    return scale_shift


def test_empty_configuration_list_is_rejected():
    tuner = tilelang.autotune(configs=[])(lambda n: scaled(n))
    with pytest.raises(ValueError, match="at least one configuration"):
        tuner(64)


@needs_no_cuda
def test_without_cuda_first_compiling_candidate_is_chosen_and_cached():
    calls = []

    @tilelang.autotune(configs=lambda: [{"block": 64}, {"block": 128}], out_idx=[1])
    def tuned(n, block=32):
        calls.append(block)
        return scaled(n, block)

    first = tuned.tune(256)
    assert first.config == {"block": 64} and first.latency_ms == 0.0
    assert tuned.best_config == {"block": 64} and tuned.best_latency_ms == 0.0
    assert first.kernel.out_idx == (1,)
    assert tuned.tune(256) is first and calls == [64]  # cache hit: nothing rebuilt
    tuned.tune(512)
    assert calls == [64, 64]


@needs_no_cuda
def test_failing_candidates_are_skipped_and_the_last_error_is_reported():
    def factory(n, block=0):
        if block == 1:
            raise CompileError("candidate one does not compile")
        return scaled(n, block)

    ok = tilelang.autotune(configs=[{"block": 1}, {"block": 128}])(factory)
    assert ok.tune(256).config == {"block": 128}
    log = ok.timings[((256,), ())]
    assert log[0][2].startswith("CompileError") and log[1][2] is None

    bad = tilelang.autotune(configs=[{"block": 1}])(factory)
    with pytest.raises(CompileError, match="All autotune configurations failed; last error: candidate one"):
        bad(256)


def test_factory_must_return_a_kernel_or_program():
    tuner = tilelang.autotune(configs=[{"x": 1}])(lambda x: 42)
    with pytest.raises(TypeError, match="CompiledKernel or @T.prim_func"):
        tuner()


def test_jit_factory_under_autotune_keeps_its_out_idx():
    @tilelang.autotune(configs=[{"block_m": 128}, {"block_m": 64}])
    @tilelang.jit(out_idx=[-1], target="sm_100a")
    def tuned_gemm(m, n, k, block_m=64):
        from ntilang_b200.kernels import _gemm_program

        return _gemm_program(m, n, k, block_m, 128, 32, 3, None)

    kern = tuned_gemm.compile_candidate((256, 256, 256), {}, {"block_m": 128})
    assert isinstance(kern, ntilang.CompiledKernel) and kern.out_idx == (2,) and kern.spec.family == "gemm"


def test_sample_arguments_cover_scalars_and_symbolic_sizes():
    kern = ntilang.compile(scaled(96), out_idx=[1])
    a, b, alpha, flip, k = sample_arguments(kern, torch, device="cpu")
    assert a.shape == (96,) and b.shape == (96,) and a.dtype == torch.float32
    assert alpha == 0.0 and isinstance(alpha, float)
    assert flip is False
    assert k == 0 and type(k) is int

    M = T.dynamic("m")

    @T.prim_func
    def dyn(A: T.Tensor((M, 128), "float32"), B: T.Tensor((M, 128), "float32")):
        with T.Kernel(T.ceildiv(M, 4), threads=128) as bx:
            tile = T.alloc_fragment((4, 128), "float32")
            T.copy(A[bx * 4 : bx * 4 + 4, :], tile)
            T.cumsum(tile, dim=1)
            T.copy(tile, B[bx * 4 : bx * 4 + 4, :])

    x, y = sample_arguments(ntilang.compile(dyn, out_idx=[-1]), torch, device="cpu")
    assert x.shape == (SYMBOLIC_SIZE, 128) and y.shape == (SYMBOLIC_SIZE, 128)
