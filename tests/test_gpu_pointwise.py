"""GPU parity of the generic elementwise path (CUDA C generated per program, NVRTC for sm_100a).

Bar: bit-exact against the reference evaluator's golden vectors for programs without
transcendental functions (fp32 / fp16 / int arithmetic, selects, copies, atomics); the oracle
(``oracle.pointwise_eval``) for bfloat16 and symbolic sizes; transcendental functions within
2 ulp of fp32 (CUDA's library vs NumPy's).
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import ntilang
import ntilang as tilelang
import ntilang.language as T
from oracle import pointwise_eval
from tests.conftest import golden

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import pw_programs  # noqa: E402

pytestmark = pytest.mark.gpu



def to_gpu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("name", sorted(pw_programs.PROGRAMS))
def test_program_matches_reference_golden(torch_cuda, name):
    torch = torch_cuda
    factory, _, outs, scalars = pw_programs.PROGRAMS[name]
    g = golden(f"pw_{name}")
    n_in = len([k for k in g if k.startswith("in")])
    tensors = [to_gpu(torch, g[f"in{i}"]) for i in range(n_in)]
    kern = factory(T, ntilang.compile)
    assert kern.spec.family == "pointwise"
    kern(*tensors, *scalars)
    torch.cuda.synchronize()
    for i in outs:
        np.testing.assert_array_equal(tensors[i].cpu().numpy(), g[f"out{i}"])


def test_reference_example_computations_match_reference_golden(torch_cuda):
    """The computations of examples/fragment_affine.py, piecewise.py and window_sum.py
    (tests/golden/pw_programs.py) against the reference evaluator's outputs for its examples."""
    torch = torch_cuda
    g = golden("pw_fragment_affine_257")
    a = to_gpu(torch, g["a"])
    b = torch.full_like(a, float("nan"))
    pw_programs.tile_affine(T, ntilang.compile)(a, b)
    np.testing.assert_array_equal(b.cpu().numpy(), g["b"])
    g = golden("pw_piecewise_93")
    a = to_gpu(torch, g["a"])
    b = torch.full_like(a, float("nan"))
    pw_programs.three_piece(T, ntilang.compile)(a, b)
    np.testing.assert_array_equal(b.cpu().numpy(), g["b"])
    g = golden("pw_window_sum_7x3x5")
    kern = pw_programs.clipped_window(T, ntilang.compile)
    a = to_gpu(torch, g["a"])
    for (rows, cols), expect in zip(g["windows"], g["b"]):
        b = torch.full((7,), float("nan"), device="cuda")
        kern(a, b, int(rows), int(cols))
        np.testing.assert_array_equal(b.cpu().numpy(), expect)


def test_symbolic_size_single_compile(torch_cuda):
    """One compile serves every M (the reference's tests/test_m34_features.py:89-110 pattern)."""
    torch = torch_cuda
    M = T.dynamic("m")

    @tilelang.jit(out_idx=[-1], target="auto")
    def dyn_affine(A: T.Tensor((M, 64), "float32"), B: T.Tensor((M, 64), "float32")):
        with T.Kernel(T.ceildiv(M, 4), threads=128) as bx:
            for i, j in T.Parallel(4, 64):
                B[bx * 4 + i, j] = A[bx * 4 + i, j] * 3.0 + 1.0

    for rows in (1, 7, 19, 131, 4097):
        x = torch.randn(rows, 64, device="cuda")
        y = dyn_affine(x)
        torch.cuda.synchronize()
        torch.testing.assert_close(y, x * 3.0 + 1.0, rtol=0, atol=0)
    assert dyn_affine.compile_count == 1


def test_bfloat16_and_transcendentals_against_oracle(torch_cuda):
    torch = torch_cuda

    @T.prim_func
    def mixed(A: T.Tensor((1000,), "bfloat16"), B: T.Tensor((1000,), "float32"), C: T.Tensor((1000,), "bfloat16"),
              D: T.Tensor((1000,), "float32")):
        with T.Kernel(T.ceildiv(1000, 256), threads=256) as bx:
            for i in T.Parallel(256):
                a = A[bx * 256 + i]
                b = B[bx * 256 + i]
                C[bx * 256 + i] = a * a + a - T.cast(b, "bfloat16")
                D[bx * 256 + i] = T.exp(b) + T.sigmoid(b) * T.sqrt(T.abs(b)) + T.tanh(b * 0.5)

    import ml_dtypes

    rng = np.random.default_rng(5)
    a = (rng.normal(size=1000) * 3).astype(ml_dtypes.bfloat16)
    b = (rng.normal(size=1000) * 2).astype(np.float32)
    kern = ntilang.compile(mixed)
    ta = to_gpu(torch, a.view(np.uint16)).view(torch.bfloat16)
    tb = to_gpu(torch, b)
    tc = torch.empty(1000, device="cuda", dtype=torch.bfloat16)
    td = torch.empty(1000, device="cuda")
    kern(ta, tb, tc, td)
    c = np.zeros(1000, ml_dtypes.bfloat16)
    d = np.zeros(1000, np.float32)
    pointwise_eval.evaluate(kern.ir, [a, b, c, d])
    np.testing.assert_array_equal(tc.view(torch.int16).cpu().numpy(), c.view(np.int16))
    np.testing.assert_allclose(td.cpu().numpy(), d, rtol=4e-7, atol=1e-7)


def test_scalar_argument_checks(torch_cuda):
    torch = torch_cuda
    kern = pw_programs.scaled_shift(T, ntilang.compile)
    a = torch.randn(300, device="cuda")
    b = torch.empty_like(a)
    with pytest.raises(TypeError, match="real scalar"):
        kern(a, b, "x", 1.0)
    with pytest.raises(TypeError, match="real scalar"):
        kern(a, b, True, 1.0)
    g = golden("pw_window_sum_7x3x5")
    ws = pw_programs.clipped_window(T, ntilang.compile)
    with pytest.raises(TypeError, match="integer scalar"):
        ws(to_gpu(torch, g["a"]), torch.empty(7, device="cuda"), 1.5, 2)
    with pytest.raises(ValueError, match="outside the int32 range"):
        ws(to_gpu(torch, g["a"]), torch.empty(7, device="cuda"), 2**31, 2)


def test_saved_module_runs_without_ntilang(torch_cuda, tmp_path):
    """The standalone launcher (CompiledKernel.save) launches on the GPU in an isolated
    interpreter that never imports ntilang (the reference's tests/test_compiler.py:177-188)."""
    kern = pw_programs.scaled_shift(T, ntilang.compile)
    from ntilang_b200 import kernels as K

    fam = K.vector_add(4096)
    pw_path = kern.save(tmp_path / "scaled_shift.py")
    fam_path = fam.save(tmp_path / "vector_add.py")
    code = f"""
import runpy, sys, torch
pw = runpy.run_path({str(pw_path)!r})['compile_kernel']()
fam = runpy.run_path({str(fam_path)!r})['compile_kernel']()
a = torch.randn(300, device='cuda'); b = torch.empty_like(a)
pw(a, b, 1.75, -0.3, stream=torch.cuda.current_stream().cuda_stream)
x, y = torch.randn(4096, device='cuda'), torch.randn(4096, device='cuda'); z = torch.empty_like(x)
fam(x, y, z, stream=torch.cuda.current_stream().cuda_stream)
torch.cuda.synchronize()
assert torch.equal(b, a * 1.75 + (-0.3)), 'pointwise'
assert torch.equal(z, x + y), 'family'
assert 'ntilang' not in sys.modules and 'ntilang_b200' not in sys.modules
print('ok')
"""
    out = subprocess.run([sys.executable, "-I", "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stderr[-2000:]


def test_compiler_load_runtime_module(torch_cuda):
    """The reference's tests/test_m34_features.py:184-196."""
    torch = torch_cuda

    @T.prim_func
    def gpu_scale(A: T.Tensor((128,), "float32"), B: T.Tensor((128,), "float32")):
        with T.Kernel(1, threads=128):
            for i in T.Parallel(128):
                B[i] = A[i] + 5.0

    compiler = ntilang.Compiler()
    prog = compiler.import_program(gpu_scale, frontend="tilelang")
    lowered = compiler.lower(prog, backend="cute", target="auto", out_idx=[-1])
    module = compiler.load(compiler.compile(lowered), device="cuda:0")
    x = torch.randn(128, device="cuda")
    y = module["gpu_scale"](x)
    torch.cuda.synchronize()
    torch.testing.assert_close(y, x + 5.0, rtol=0, atol=0)


def test_large_generic_fma_matches_oracle_sample(torch_cuda):
    """16M elements through the generic path (the bench workload): separately rounded
    multiply and add, bit-exact against torch's two-kernel a * b + c."""
    torch = torch_cuda
    n = 1 << 24
    kern = pw_programs.generic_fma(T, ntilang.compile, n)
    g = torch.Generator(device="cuda").manual_seed(0)
    a, b, c = (torch.randn(n, device="cuda", generator=g) for _ in range(3))
    d = torch.empty_like(a)
    kern(a, b, c, d)
    torch.cuda.synchronize()
    assert torch.equal(d, a * b + c)


def _run_against_oracle(torch, kern, arrays, scalars=()):
    """Run a generic kernel on the GPU and the oracle evaluator on copies; compare bitwise."""
    gpu_args = [to_gpu(torch, a) for a in arrays]
    kern(*gpu_args, *scalars)
    torch.cuda.synchronize()
    expect = [a.copy() for a in arrays]
    pointwise_eval.evaluate(kern.ir, expect, scalars)
    for got, want in zip(gpu_args, expect):
        np.testing.assert_array_equal(got.cpu().numpy(), want)


def test_three_d_grid_symbolic_rows_and_two_loop_shapes(torch_cuda):
    """A 3-D grid whose first extent is symbolic, an integer scalar, and two T.Parallel loops
    of different shapes in one kernel (each thread covers the larger domain)."""
    torch = torch_cuda
    R = T.dynamic("r")

    @T.prim_func
    def grid3(X: T.Tensor((R, 6, 40), "float32"), Y: T.Tensor((R, 6, 40), "float32"),
              Z: T.Tensor((R, 6), "int32"), shift: T.int32):
        with T.Kernel(T.ceildiv(40, 16), 6, R, threads=64) as (bx, by, bz):
            for i in T.Parallel(16):
                Y[bz, by, bx * 16 + i] = X[bz, by, bx * 16 + i] * 2.0 - T.cast(shift, "float32")
            for j in T.Parallel(4):
                if bx == 0 and j == 0:
                    Z[bz, by] = bz * 100 + by * 10 + shift

    kern = ntilang.compile(grid3)
    assert kern.spec.family == "pointwise"
    for rows in (1, 5):
        rng = np.random.default_rng(rows)
        arrays = [rng.normal(size=(rows, 6, 40)).astype(np.float32), np.full((rows, 6, 40), np.nan, np.float32),
                  np.zeros((rows, 6), np.int32)]
        _run_against_oracle(torch, kern, arrays, (7,))


def test_region_copy_and_narrow_and_wide_dtypes(torch_cuda):
    """A global-to-global T.copy of a tile region, int8/uint8 wrap-around arithmetic and float64."""
    torch = torch_cuda

    @T.prim_func
    def mixed_types(A: T.Tensor((50, 70), "float32"), B: T.Tensor((50, 70), "float32"),
                    C: T.Tensor((300,), "int8"), D: T.Tensor((300,), "uint8"), E: T.Tensor((300,), "float64"),
                    F: T.Tensor((300,), "float64")):
        with T.Kernel(T.ceildiv(70, 32), T.ceildiv(50, 16), threads=128) as (bx, by):
            T.copy(A[by * 16:by * 16 + 16, bx * 32:bx * 32 + 32], B[by * 16:by * 16 + 16, bx * 32:bx * 32 + 32])
            for k in T.Parallel(128):
                idx = (by * 3 + bx) * 128 + k
                c = C[idx]
                C[idx] = c * c + T.cast(7, "int8")
                d = D[idx]
                D[idx] = d * T.cast(3, "uint8") + d
                F[idx] = E[idx] * E[idx] / 3.0 + E[idx]

    kern = ntilang.compile(mixed_types)
    assert kern.spec.family == "pointwise"
    rng = np.random.default_rng(11)
    arrays = [rng.normal(size=(50, 70)).astype(np.float32), np.full((50, 70), np.nan, np.float32),
              rng.integers(-128, 127, size=300).astype(np.int8), rng.integers(0, 255, size=300).astype(np.uint8),
              rng.normal(size=300), np.full(300, np.nan)]
    _run_against_oracle(torch, kern, arrays)


def test_vector_groups_and_their_per_point_fallbacks(torch_cuda):
    """Unit-stride accesses of a T.Parallel point run as 4-point vector groups (16-byte fp32,
    8-byte fp16, 4-byte int8 accesses); a group that is misaligned, crosses the tensor's end or
    starts at a negative index falls back to per-point accesses, and a store inside a branch
    stays per point.  Bit-exact against the oracle."""
    torch = torch_cuda
    n = 1003

    @T.prim_func
    def groups(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), C: T.Tensor((n,), "float32"),
               H: T.Tensor((n,), "float16"), G: T.Tensor((n,), "float16"), I: T.Tensor((n,), "int8"),
               J: T.Tensor((n,), "int8"), lo: T.int32):
        with T.Kernel(T.ceildiv(n, 128), threads=128) as b:
            for k in T.Parallel(128):
                B[b * 128 + k] = A[k + (b * 128 + 1)] + A[k + (b * 128 + 4)]
                if k >= lo:
                    C[b * 128 + k] = A[k + b * 128] * 2.0
                G[b * 128 + k] = H[b * 128 + k] * T.float16(1.5) + H[k + (b * 128 + 2)]
                J[b * 128 + k] = I[b * 128 + k] * T.cast(3, "int8") + I[k + (b * 128 - 1)]

    kern = ntilang.compile(groups)
    assert kern.spec.family == "pointwise"
    src = kern.get_cuda_source()
    for vt in ("float4", "ushort4", "char4"):  # vector loads and stores for each element size
        assert f"reinterpret_cast<const {vt}*>" in src and f"reinterpret_cast<{vt}*>" in src, vt
    rng = np.random.default_rng(5)
    for lo in (0, 37):
        arrays = [rng.normal(size=n).astype(np.float32), np.full(n, np.nan, np.float32), np.full(n, np.nan, np.float32),
                  (rng.normal(size=n) * 8).astype(np.float16), np.full(n, np.nan, np.float16),
                  rng.integers(-128, 127, size=n).astype(np.int8), np.zeros(n, np.int8)]
        _run_against_oracle(torch, kern, arrays, (lo,))
