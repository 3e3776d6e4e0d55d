"""CPU checks of the generic elementwise path: the oracle against the reference's golden
vectors, CUDA generation and NVRTC compilation for sm_100a (no GPU needed), the standalone
export module and the staged Compiler API.  GPU parity is in test_gpu_pointwise.py."""

from __future__ import annotations

import ast
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import ntilang
import ntilang.language as T
from ntilang_b200 import _lib
from ntilang_b200.ir import CompileError
from oracle import pointwise_eval
from tests.conftest import golden

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import pw_programs  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]


def _nvrtc_available() -> bool:
    try:
        import ctypes

        h = ctypes.c_uint64(0)
        _lib.call("ntl_rtc_build", b'extern "C" __global__ void ntl_probe() {}', b"ntl_probe", ctypes.byref(h))
        return True
    except Exception:
        return False


needs_nvrtc = pytest.mark.skipif(not _nvrtc_available(), reason="NVRTC or libntl_kernels.so unavailable")


def _example(name):
    from tests.conftest import load_reference_example

    return load_reference_example(name)


# ------------------------------------------------------------------ oracle vs golden


@pytest.mark.parametrize("name", sorted(pw_programs.PROGRAMS))
def test_oracle_matches_reference_evaluator(name):
    factory, _, outs, scalars = pw_programs.PROGRAMS[name]
    g = golden(f"pw_{name}")
    arrays = [g[f"in{i}"].copy() for i in range(len([k for k in g if k.startswith("in")]))]
    kern = factory(T, ntilang.compile)
    assert kern.spec.family == "pointwise"
    pointwise_eval.evaluate(kern.ir, arrays, scalars)
    for i in outs:
        np.testing.assert_array_equal(arrays[i], g[f"out{i}"])


def test_oracle_on_reference_examples():
    g = golden("pw_fragment_affine_257")
    b = np.full_like(g["a"], np.nan)
    pointwise_eval.evaluate(_example("fragment_affine").fragment_affine().ir, [g["a"], b])
    np.testing.assert_array_equal(b, g["b"])
    g = golden("pw_piecewise_93")
    b = np.full_like(g["a"], np.nan)
    pointwise_eval.evaluate(_example("piecewise").piecewise().ir, [g["a"], b])
    np.testing.assert_array_equal(b, g["b"])
    g = golden("pw_window_sum_7x3x5")
    kern = _example("window_sum").window_sum()
    for (rows, cols), expect in zip(g["windows"], g["b"]):
        b = np.full(7, np.nan, np.float32)
        pointwise_eval.evaluate(kern.ir, [g["a"], b], (int(rows), int(cols)))
        np.testing.assert_array_equal(b, expect)


def test_oracle_plants_are_caught():
    """A wrong promotion in the oracle (float16 product computed in float16 instead of the
    float32 the literal promotes it to) changes the golden-checked output."""
    factory, build, outs, _ = pw_programs.PROGRAMS["half_mix"]
    g = golden("pw_half_mix")
    kern = factory(T, ntilang.compile)
    arrays = [g[f"in{i}"].copy() for i in range(4)]
    saved = pointwise_eval.promote
    try:
        pointwise_eval.promote = lambda a, b: a if a == b else ("float16" if "float16" in (a, b) else saved(a, b))
        pointwise_eval.evaluate(kern.ir, arrays)
    finally:
        pointwise_eval.promote = saved
    assert not np.array_equal(arrays[3], g["out3"])


# ------------------------------------------------------------------ generation + NVRTC


@needs_nvrtc
@pytest.mark.parametrize("name", sorted(pw_programs.PROGRAMS))
def test_generated_cuda_compiles_for_sm100a(name):
    kern = pw_programs.PROGRAMS[name][0](T, ntilang.compile)
    assert kern.spec.params["kernel"].build() > 0


def test_vector_groups_only_where_four_points_are_contiguous():
    """Which accesses the generic lowering turns into 4-point vector groups: unit stride in the
    innermost T.Parallel variable, read-only loads, top-level stores to write-only tensors."""
    n = 4096

    @T.prim_func
    def shapes(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), C: T.Tensor((n,), "float32"),
               D: T.Tensor((64, 64), "float32"), E: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, 256), threads=128) as b:
            for k in T.Parallel(256):
                B[b * 256 + k] = A[b * 256 + k] * 2.0          # vector load and store
                C[b * 256 + k] = C[b * 256 + k] + A[k * 2 % n]  # in place, stride 2: per point
                D[b % 64, k % 64] = A[b * 256 + 1 + k]         # D per point; A a group (misaligned at run time)
                acc = T.alloc_var("float32", 0)
                for t in T.serial(3):
                    acc += E[b * 256 + k + t]                   # depends on the loop: per point
                if k > 3:
                    E[b * 256 + k] = acc                        # E is read too: per point

    src = ntilang.compile(shapes).get_cuda_source()
    assert src.count("reinterpret_cast<const float4*>") == 2  # A[b*256 + k] and A[b*256 + 1 + k]
    assert src.count("reinterpret_cast<float4*>") == 1  # B only
    assert "(long long)threadIdx.x * 4" in src  # the 4-consecutive-points mapping

    @T.prim_func
    def odd_extent(A: T.Tensor((300,), "float32"), B: T.Tensor((300,), "float32")):
        with T.Kernel(T.ceildiv(300, 30), threads=32) as b:
            for k in T.Parallel(30):
                B[b * 30 + k] = A[b * 30 + k] + 1.0

    src = ntilang.compile(odd_extent).get_cuda_source()
    assert "float4" not in src and "+ threadIdx.x;" in src  # 30 points: the strided mapping


@needs_nvrtc
def test_reference_examples_compile_on_the_generic_path():
    for name in ("fragment_affine", "piecewise", "window_sum"):
        kern = getattr(_example(name), name)()
        assert kern.spec.family == "pointwise", name
        kern.build()


def test_reference_control_flow_programs():
    """The reference's control-flow programs (tests/test_control_flow.py:12-60) lower, and
    the invalid ones are rejected with the reference's reasons."""

    @T.prim_func
    def conditional_fragment(A: T.Tensor((93,), "float32"), B: T.Tensor((93,), "float32")):
        with T.Kernel(3, threads=32) as bx:
            tile = T.alloc_fragment((32,), "float32")
            for i in T.Parallel(32):
                x = A[bx * 32 + i]
                if x > 0.0:
                    tile[i] = x
                else:
                    tile[i] = -x
                if i < 16:
                    tile[i] += 1.0
            T.copy(tile, B[bx * 32])

    @T.prim_func
    def uniform_collective(A: T.Tensor((93,), "float32"), B: T.Tensor((93,), "float32")):
        with T.Kernel(3, threads=32) as bx:
            tile = T.alloc_shared((32,), "float32")
            if bx % 2 == 0:
                T.copy(A[bx * 32], tile)
            else:
                T.fill(tile, -2.0)
            T.copy(tile, B[bx * 32])

    a = np.linspace(-2, 2, 93, dtype=np.float32)
    for prog, expect in ((conditional_fragment, np.abs(a) + (np.arange(93) % 32 < 16)),
                         (uniform_collective, np.where(np.arange(93) // 32 % 2 == 0, a, -2))):
        kern = ntilang.compile(prog)
        assert kern.spec.family == "pointwise"
        b = np.full_like(a, np.nan)
        pointwise_eval.evaluate(kern.ir, [a, b])
        np.testing.assert_array_equal(b, expect.astype(np.float32))

    @T.prim_func
    def divergent_collective(A: T.Tensor((32,), "float32")):
        with T.Kernel(1, threads=32) as _bx:
            tile = T.alloc_shared((32,), "float32")
            for i in T.Parallel(32):
                if i < 16:
                    T.clear(tile)
            T.copy(tile, A)

    with pytest.raises(CompileError, match="Collective"):
        ntilang.compile(divergent_collective)

    @T.prim_func
    def collision(A: T.Tensor((32,), "float32")):
        with T.Kernel(1, threads=32) as _bx:
            for i in T.Parallel(32):
                if i < 16:
                    A[i] = 1.0
                else:
                    A[i - 16] = 2.0

    with pytest.raises(CompileError, match="identical ownership"):
        ntilang.compile(collision)

    @T.prim_func
    def escaping_local(A: T.Tensor((32,), "float32")):
        with T.Kernel(1, threads=32) as _bx:
            for i in T.Parallel(32):
                if i < 16:
                    value = i + 2.0
                A[i] = value

    with pytest.raises(CompileError, match="defining region"):
        ntilang.compile(escaping_local)


def test_cross_point_reduction_through_a_scalar_is_rejected():
    @T.prim_func
    def racy_sum(A: T.Tensor((64,), "float32"), B: T.Tensor((1,), "float32")):
        with T.Kernel(1, threads=64):
            total = T.alloc_var("float32", init=0)
            for i in T.Parallel(64):
                total += A[i]
            B[0] = total

    with pytest.raises(CompileError, match="reduction across parallel points"):
        ntilang.compile(racy_sum)


def test_integer_true_division_is_rejected():
    @T.prim_func
    def int_div(X: T.Tensor((8,), "int32"), Y: T.Tensor((8,), "int32")):
        with T.Kernel(1, threads=8):
            for i in T.Parallel(8):
                Y[i] = X[i] / 2

    with pytest.raises(CompileError, match="Integer '/' is ambiguous"):
        ntilang.compile(int_div)


# ------------------------------------------------------------------ export + Compiler API


def _imports(text):
    tree = ast.parse(text)
    return {n.names[0].name if isinstance(n, ast.Import) else n.module for n in ast.walk(tree)
            if isinstance(n, (ast.Import, ast.ImportFrom))}


def test_saved_module_is_standalone(tmp_path):
    """The exported launcher imports only ctypes and os (python/ntilang/compiler.py:44-49 and
    the reference's tests/test_compiler.py:63-71 for its CuTe module)."""
    kern = pw_programs.scaled_shift(T, ntilang.compile)
    path = kern.save(tmp_path / "scaled_shift.py")
    text = path.read_text(encoding="utf-8")
    assert _imports(text) == {"ctypes", "os"}
    assert "def compile_kernel" in text and "ntl_pw_scaled_shift" in text
    first, second = (pw_programs.scaled_shift(T, ntilang.compile) for _ in range(2))
    assert first.source == second.source and first.cache_key == second.cache_key
    assert pw_programs.scaled_shift(T, ntilang.compile, n=301).cache_key != first.cache_key
    from ntilang_b200 import kernels as K

    fam = K.vector_add(1024)
    assert _imports(fam.source) == {"ctypes", "os"} and "CALLS = (('ntl_binary_f32'" in fam.source


@needs_nvrtc
def test_saved_module_compiles_without_ntilang(tmp_path):
    """Mirrors the reference's tests/test_compiler.py:177-188: the saved module loads and
    builds in an isolated interpreter that never imports ntilang."""
    for kern, stem in ((pw_programs.scaled_shift(T, ntilang.compile), "pw"),
                       (__import__("ntilang_b200.kernels", fromlist=["x"]).vector_add(1024), "fam")):
        path = kern.save(tmp_path / f"{stem}.py")
        code = ("import runpy, sys; m = runpy.run_path(sys.argv[1]); f = m['compile_kernel'](); "
                "assert f.has_gpu_module; assert 'ntilang' not in sys.modules and 'ntilang_b200' not in sys.modules; "
                "print('ok')")
        out = subprocess.run([sys.executable, "-I", "-c", code, str(path)], capture_output=True, text=True,
                             timeout=120)
        assert out.returncode == 0 and out.stdout.strip() == "ok", out.stderr


def test_program_listing_and_runtime_module_lookup():
    """``Program.as_text`` lists parameters with types and the launch shape (symbolic sizes by
    name); ``RuntimeModule`` is a read-only mapping from program name to kernel."""
    from ntilang_b200.pipeline import RuntimeModule

    M = T.dynamic("m")

    @T.prim_func
    def rows(A: T.Tensor((M, 128), "float32"), B: T.Tensor((M, 128), "float32"), alpha: T.float32):
        with T.Kernel(T.ceildiv(M, 4), threads=128) as bx:
            for i, j in T.Parallel(4, 128):
                B[bx * 4 + i, j] = A[bx * 4 + i, j] * alpha

    compiler = ntilang.Compiler()
    text = compiler.import_program(rows).as_text().splitlines()
    assert text == ["program rows [frontend tilelang]", "  A: float32[m, 128]", "  B: float32[m, 128]",
                    "  alpha: float32", "  launch: grid (((m + 3) // 4)), 128 threads per block"]

    @T.prim_func
    def scale(A: T.Tensor((64,), "float32"), B: T.Tensor((64,), "float32")):
        with T.Kernel(1, threads=64):
            for i in T.Parallel(64):
                B[i] = A[i] * 2.0

    bundle = compiler.compile(compiler.lower(compiler.import_program(scale), out_idx=[-1]))
    module = RuntimeModule(bundle)
    assert list(module) == ["scale"] and len(module) == 1 and "scale" in module
    assert module["scale"] is bundle.kernel and module.get("other") is None
    with pytest.raises(KeyError, match="no kernel named 'other'"):
        module["other"]


def test_staged_compiler_api_and_artifact_save(tmp_path):
    """The reference's tests/test_m34_features.py:53-68 under import ntilang."""

    @T.prim_func
    def scale(A: T.Tensor((64,), "float32"), B: T.Tensor((64,), "float32")):
        with T.Kernel(1, threads=64):
            for i in T.Parallel(64):
                B[i] = A[i] * 2.0

    compiler = ntilang.Compiler()
    program = compiler.import_program(scale, frontend="tilelang")
    assert "scale" in program.as_text()
    lowered = compiler.lower(program, backend="cute", target="cuda:sm_80", out_idx=[-1])
    saved = lowered.emit(format="python").save(tmp_path / "scale_cute.py")
    assert saved.exists()
    assert "def compile_kernel" in saved.read_text(encoding="utf-8")
    assert "ntl_pw_scale" in lowered.emit(format="cuda").content
    bundle = compiler.compile(lowered)
    assert bundle.kernel.out_idx == (1,)
    with pytest.raises(CompileError, match="Unknown backend"):
        compiler.lower(program, backend="nope")
    with pytest.raises(CompileError, match="Unknown frontend"):
        compiler.import_program(scale, frontend="nope")
    with pytest.raises(CompileError, match="Unsupported emit format"):
        lowered.emit(format="ptx")

    @T.prim_func
    def vadd(A: T.Tensor((1024,), "float32"), B: T.Tensor((1024,), "float32"), C: T.Tensor((1024,), "float32")):
        with T.Kernel(4, threads=256) as bx:
            for i in T.Parallel(256):
                C[bx * 256 + i] = A[bx * 256 + i] + B[bx * 256 + i]

    fam = compiler.lower(compiler.import_program(vadd))
    assert fam.kernel.spec.family == "elementwise"
    with pytest.raises(CompileError, match="prebuilt"):
        fam.emit(format="cuda")


def test_compiler_registers_frontends_and_backends():
    compiler = ntilang.Compiler()
    seen = []

    def backend(ir, target, out_idx):
        seen.append((ir.name, target, out_idx))
        return ntilang.compile(ir_source, target=target, out_idx=list(out_idx))

    @T.prim_func
    def ir_source(A: T.Tensor((64,), "float32"), B: T.Tensor((64,), "float32")):
        with T.Kernel(1, threads=64):
            for i in T.Parallel(64):
                B[i] = A[i] + 1.0

    compiler.register_backend("mine", backend)
    lowered = compiler.lower(compiler.import_program(ir_source), backend="mine", target="sm_100a", out_idx=[1])
    assert seen == [("ir_source", "sm_100a", (1,))] and lowered.out_idx == (1,)
    jitted = compiler.jit(ir_source, out_idx=[-1])
    assert jitted.spec.family == "pointwise"


def test_example_computations_match_reference_goldens_on_the_oracle():
    """tests/golden/pw_programs.py restates the three reference examples' computations; on the
    oracle they reproduce the goldens made from the reference's own example programs."""
    g = golden("pw_fragment_affine_257")
    b = np.full_like(g["a"], np.nan)
    pointwise_eval.evaluate(pw_programs.tile_affine(T, ntilang.compile).ir, [g["a"], b])
    np.testing.assert_array_equal(b, g["b"])
    g = golden("pw_piecewise_93")
    b = np.full_like(g["a"], np.nan)
    pointwise_eval.evaluate(pw_programs.three_piece(T, ntilang.compile).ir, [g["a"], b])
    np.testing.assert_array_equal(b, g["b"])
    g = golden("pw_window_sum_7x3x5")
    kern = pw_programs.clipped_window(T, ntilang.compile)
    for (rows, cols), expect in zip(g["windows"], g["b"]):
        b = np.full(7, np.nan, np.float32)
        pointwise_eval.evaluate(kern.ir, [g["a"], b], (int(rows), int(cols)))
        np.testing.assert_array_equal(b, expect)


def test_break_directly_in_parallel_is_rejected():
    @T.prim_func
    def early_exit(A: T.Tensor((32,), "float32")):
        with T.Kernel(1, threads=32):
            for i in T.Parallel(32):
                if i > 3:
                    break
                A[i] = 1.0

    with pytest.raises(CompileError, match="inside a serial loop"):
        ntilang.compile(early_exit)
