"""GPU parity for the memory-bound families: vector add, cumsum, softmax, RMSNorm, LayerNorm, transpose.

Every kernel runs through the reference-compatible surface (``ntilang.compile`` / ``jit``
factories -> ``CompiledKernel.__call__`` -> the C ABI of libntl_kernels.so) and is compared
with the CPU oracle (``oracle/``) and the golden vectors generated from the reference.

Bars (north star): vector add and cumsum bit-exact; softmax and RMSNorm within 1e-5
relative (an absolute floor of 1e-30 covers results that underflow to subnormals).
"""

from __future__ import annotations

import numpy as np
import pytest

from ntilang_b200 import kernels as K
from oracle import ntl_oracle as O
from oracle import rowops
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def bits_equal(actual, expected):
    a = np.ascontiguousarray(actual, np.float32)
    e = np.ascontiguousarray(expected, np.float32)
    same = (a.view(np.uint32) == e.view(np.uint32)) | (np.isnan(a) & np.isnan(e))
    return bool(same.all()), int((~same).sum())


def to_gpu(torch, arr):
    return torch.from_numpy(np.ascontiguousarray(arr)).cuda()


# --------------------------------------------------------------------------- vector add


def test_vector_add_golden(torch_cuda):
    torch = torch_cuda
    g = golden("vadd_1000")
    out = K.vector_add(1000)(to_gpu(torch, g["a"]), to_gpu(torch, g["b"]))
    ok, bad = bits_equal(out.cpu().numpy(), g["c"])
    assert ok, bad


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 4099, 16 * 1024 * 1024 + 3])
def test_vector_add_bit_exact(torch_cuda, n):
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(n)
    a = torch.randn(n, device="cuda", generator=g)
    b = torch.randn(n, device="cuda", generator=g)
    c = K.vector_add(n)(a, b)
    torch.testing.assert_close(c, a + b, rtol=0, atol=0)


def test_vector_add_unaligned_pointers_abi(torch_cuda):
    """The C ABI also serves unaligned pointers (scalar path); results stay bit-exact."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    base = torch.randn(3 * 1001 + 8, device="cuda")
    a, b, c = base[1:1001], base[1002:2002], torch.empty(1003, device="cuda")[3:1003]
    _lib.call("ntl_vadd_f32", a.data_ptr(), b.data_ptr(), c.data_ptr(), 1000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    torch.testing.assert_close(c, a + b, rtol=0, atol=0)


def test_nondefault_stream(torch_cuda):
    torch = torch_cuda
    kernel = K.vector_add(1000)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        a = torch.full((1000,), 2.0, device="cuda")
        b = torch.full_like(a, 3.0)
        c = kernel(a, b)
        expected = a + b
    stream.synchronize()
    torch.testing.assert_close(c, expected, rtol=0, atol=0)


def test_launch_follows_the_current_stream(torch_cuda):
    """The kernel runs on torch's current stream: ordered after work queued on that stream
    (here a ~50 ms sleep, then the fills), never on the legacy stream."""
    torch = torch_cuda
    n = 1 << 20
    kernel = K.vector_add(n)
    a = torch.zeros(n, device="cuda")
    b = torch.zeros_like(a)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        torch.cuda._sleep(100_000_000)
        a.fill_(1.0)
        b.fill_(2.0)
        c = kernel(a, b)
    side.synchronize()
    assert bool(torch.all(c == 3.0))


# ------------------------------------------------------------------------------- cumsum


@pytest.mark.parametrize("case", [
    "cumsum_7x65_fwd", "cumsum_7x65_rev", "cumsum_4x256_fwd", "cumsum_4x256_rev",
    "cumsum_special_fwd", "cumsum_special_rev", "cumsum_eval_64x1000_fwd", "cumsum_eval_64x1000_rev",
])
def test_cumsum_golden_bit_exact(torch_cuda, case):
    torch = torch_cuda
    g = golden(case)
    rows, cols = g["x"].shape
    y = K.cumsum(rows, cols, bool(g["reverse"]))(to_gpu(torch, g["x"]))
    ok, bad = bits_equal(y.cpu().numpy(), g["y"])
    assert ok, f"{bad} elements differ"


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 2), (5, 3), (2, 31), (9, 33), (4, 127), (3, 129),
                                       (6, 1000), (2, 1025), (3, 4097), (2, 70001)])
@pytest.mark.parametrize("reverse", [False, True])
def test_cumsum_ragged_bit_exact(torch_cuda, rows, cols, reverse):
    torch = torch_cuda
    rng = np.random.default_rng(rows * 7919 + cols)
    x = rng.uniform(-1, 1, size=(rows, cols)).astype(np.float32)
    y = K.cumsum(rows, cols, reverse)(to_gpu(torch, x)).cpu().numpy()
    ok, bad = bits_equal(y, O.cumsum_rows(x, reverse))
    assert ok, f"{bad} elements differ"


@pytest.mark.parametrize("reverse", [False, True])
def test_cumsum_baseline_size_bit_exact(torch_cuda, reverse):
    """BASELINE config: X f32 [32768, 256] ~ U(-1, 1)."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.rand(32768, 256, device="cuda", generator=g) * 2 - 1
    y = K.cumsum(32768, 256, reverse)(x)
    ok, bad = bits_equal(y.cpu().numpy(), rowops.cumsum(x.cpu().numpy(), reverse))
    assert ok, f"{bad} elements differ"


@pytest.mark.parametrize("case", ["scan_9x113_fwd", "scan_9x113_rev"])
def test_sum_and_max_scans_golden_bit_exact(torch_cuda, case):
    """examples/scan.py's two outputs (cumsum and cummax of one tile) against the reference
    evaluator, through the factory with the same program shape."""
    torch = torch_cuda
    g = golden(case)
    rows, cols = g["x"].shape
    kern = K.sum_and_max_scans(rows, cols, bool(g["reverse"]))
    assert kern.spec.family == "scans"
    sums, maxima = kern(to_gpu(torch, g["x"]))
    for got, want in ((sums, g["prefix"]), (maxima, g["maximum"])):
        ok, bad = bits_equal(got.cpu().numpy(), want)
        assert ok, f"{bad} elements differ"


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 2), (2, 31), (9, 33), (3, 129), (6, 1000), (2, 1025),
                                       (3, 4097), (2, 70001)])
@pytest.mark.parametrize("reverse", [False, True])
def test_cummax_ragged_bit_exact(torch_cuda, rows, cols, reverse):
    torch = torch_cuda
    rng = np.random.default_rng(rows * 131 + cols)
    x = rng.normal(size=(rows, cols)).astype(np.float32)
    x[:, ::17] = 0.0
    x[:, ::23] = -0.0
    y = K.cummax(rows, cols, reverse)(to_gpu(torch, x)).cpu().numpy()
    ok, bad = bits_equal(y, O.cummax_rows(x, reverse))
    assert ok, f"{bad} elements differ"


def test_cumsum_1d_program(torch_cuda):
    """A rank-1 tile scan (one row) written directly with ntilang.compile."""
    torch = torch_cuda
    import ntilang
    import ntilang.language as T

    @T.prim_func
    def scan1d(A: T.Tensor((300,), "float32"), B: T.Tensor((300,), "float32")):
        with T.Kernel(1, threads=128):
            t = T.alloc_shared((300,), "float32")
            T.copy(A, t)
            T.cumsum(t, dim=0)
            T.copy(t, B)

    k = ntilang.compile(scan1d)
    x = np.random.default_rng(1).normal(size=300).astype(np.float32)
    out = torch.empty(300, device="cuda")
    k(to_gpu(torch, x), out)
    ok, bad = bits_equal(out.cpu().numpy(), O.cumsum_rows(x))
    assert ok, bad


# ------------------------------------------------------------------------------ softmax


@pytest.mark.parametrize("case", ["softmax_9x113", "softmax_4x512"])
def test_softmax_golden(torch_cuda, case):
    torch = torch_cuda
    g = golden(case)
    rows, cols = g["x"].shape
    y = K.softmax(rows, cols)(to_gpu(torch, g["x"])).cpu().numpy()
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-30)


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 2), (4, 3), (9, 113), (8, 128), (5, 2047), (7, 2048),
                                       (3, 2049), (2, 5000), (2, 16384)])
def test_softmax_shapes(torch_cuda, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows + cols)
    x = (rng.normal(size=(rows, cols)) * 2.0).astype(np.float32)
    y = K.softmax(rows, cols)(to_gpu(torch, x)).cpu().numpy()
    np.testing.assert_allclose(y, O.softmax_rows(x), rtol=1e-5, atol=1e-30)


def test_softmax_baseline_size(torch_cuda):
    """BASELINE config: X f32 [16384, 512] ~ N(0, 4)."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(16384, 512, device="cuda", generator=g) * 2.0
    y = K.softmax(16384, 512)(x).cpu().numpy()
    np.testing.assert_allclose(y, rowops.softmax(x.cpu().numpy()), rtol=1e-5, atol=1e-30)
    np.testing.assert_allclose(y.sum(axis=1), 1.0, rtol=1e-5)


def test_softmax_large_magnitude_like_reference(torch_cuda):
    torch = torch_cuda
    a = torch.randn(9, 113, device="cuda") * 30
    y = K.softmax(9, 113)(a)
    torch.testing.assert_close(y, torch.softmax(a, dim=1), rtol=2e-5, atol=2e-6)


# ------------------------------------------------------------------------------ RMSNorm


@pytest.mark.parametrize("case", ["rmsnorm_6x1024", "rmsnorm_5x768"])
def test_rmsnorm_golden(torch_cuda, case):
    torch = torch_cuda
    g = golden(case)
    rows, cols = g["x"].shape
    y = K.rmsnorm(rows, cols, float(g["eps"]))(to_gpu(torch, g["x"]), to_gpu(torch, g["w"])).cpu().numpy()
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (131, 256), (131, 512), (131, 768), (4, 2048), (3, 3000),
                                       (2, 16384)])
def test_rmsnorm_shapes(torch_cuda, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows * cols)
    x = rng.normal(size=(rows, cols)).astype(np.float32)
    w = rng.normal(1.0, 0.1, size=cols).astype(np.float32)
    y = K.rmsnorm(rows, cols, 1e-6)(to_gpu(torch, x), to_gpu(torch, w)).cpu().numpy()
    np.testing.assert_allclose(y, O.rmsnorm_rows(x, w, 1e-6), rtol=1e-5, atol=1e-7)


def test_rmsnorm_baseline_size(torch_cuda):
    """BASELINE config: X f32 [4096, 1024] ~ N(0,1), gamma ~ N(1, 0.1), eps 1e-6."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4096, 1024, device="cuda", generator=g)
    w = torch.randn(1024, device="cuda", generator=g) * 0.1 + 1.0
    y = K.rmsnorm(4096, 1024, 1e-6)(x, w)
    np.testing.assert_allclose(y.cpu().numpy(), rowops.rmsnorm(x.cpu().numpy(), w.cpu().numpy(), 1e-6),
                               rtol=1e-5, atol=1e-7)
    ref = x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + 1e-6) * w
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=1e-5)


# ---------------------------------------------------------------------------- LayerNorm
# Bar: within 1e-5 relative plus 1e-6 absolute of the oracle and of the reference evaluator's
# golden vectors (the evaluator sums pairwise, the kernel and oracle with the emitted kernel's
# tree; outputs near zero come from cancellation in d * rstd * w + b).


@pytest.mark.parametrize("case", ["layernorm_6x1024", "layernorm_5x768", "layernorm_3x100"])
def test_layernorm_golden(torch_cuda, case):
    torch = torch_cuda
    g = golden(case)
    rows, cols = g["x"].shape
    kern = K.layernorm(rows, cols, float(g["eps"]))
    y = kern(to_gpu(torch, g["x"]), to_gpu(torch, g["w"]), to_gpu(torch, g["b"])).cpu().numpy()
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 5), (131, 256), (131, 768), (4, 2048), (37, 1030), (40, 999),
                                       (3, 3000), (2, 16384)])
def test_layernorm_shapes(torch_cuda, rows, cols):
    torch = torch_cuda
    rng = np.random.default_rng(rows * cols + 1)
    x = (rng.normal(size=(rows, cols)) * 3.0 + 1.0).astype(np.float32)
    w = rng.normal(1.0, 0.1, size=cols).astype(np.float32)
    b = rng.normal(0.0, 0.1, size=cols).astype(np.float32)
    y = K.layernorm(rows, cols, 1e-5)(to_gpu(torch, x), to_gpu(torch, w), to_gpu(torch, b)).cpu().numpy()
    np.testing.assert_allclose(y, rowops.layernorm(x, w, b, 1e-5), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n", [256, 512, 768])
def test_layernorm_reference_test_shape(torch_cuda, n):
    """The reference's GPU test shape and bar (tests/test_llm_operators.py:76-100)."""
    torch = torch_cuda
    import torch.nn.functional as F

    x = torch.randn(131, n, device="cuda")
    w = torch.randn(n, device="cuda")
    b = torch.randn(n, device="cuda")
    y = torch.empty_like(x)
    K.layernorm(131, n, 1e-5)(x, w, b, y)
    torch.testing.assert_close(y, F.layer_norm(x, (n,), weight=w, bias=b, eps=1e-5), rtol=1e-4, atol=1e-5)


def test_layernorm_baseline_size(torch_cuda):
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4096, 1024, device="cuda", generator=g)
    w = torch.randn(1024, device="cuda", generator=g) * 0.1 + 1.0
    b = torch.randn(1024, device="cuda", generator=g) * 0.1
    y = K.layernorm(4096, 1024, 1e-5)(x, w, b)
    np.testing.assert_allclose(y.cpu().numpy(), rowops.layernorm(x.cpu().numpy(), w.cpu().numpy(), b.cpu().numpy(),
                                                                1e-5), rtol=1e-5, atol=1e-6)


# ---------------------------------------------------------------------------- transpose (bit-exact)


@pytest.mark.parametrize("case", ["transpose_65x71", "transpose_33x130"])
def test_transpose_golden(torch_cuda, case):
    torch = torch_cuda
    g = golden(case)
    m, n = g["a"].shape
    out = K.transpose(m, n)(to_gpu(torch, g["a"])).cpu().numpy()
    assert np.array_equal(out, g["b"])


# (n % 4, m % 4) select the vector or scalar side of the kernel: all four pairings, partial
# 64x64 tiles on either edge, and a full-size square.
@pytest.mark.parametrize("m,n", [(1, 1), (1, 100), (100, 1), (65, 71), (64, 71), (65, 72), (1000, 33), (130, 260),
                                 (4096, 4096)])
def test_transpose_shapes(torch_cuda, m, n):
    torch = torch_cuda
    a = torch.randn(m, n, device="cuda")
    b = K.transpose(m, n)(a)
    torch.testing.assert_close(b, a.T, rtol=0, atol=0)


@pytest.mark.parametrize("a_off,b_off", [(1, 0), (0, 1), (1, 1)])
def test_transpose_unaligned_pointers(torch_cuda, a_off, b_off):
    """Buffers that start 4 bytes past a 16-byte boundary take the element-wise side."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    m, n = 72, 136
    abuf = torch.randn(m * n + 1, device="cuda")
    bbuf = torch.full((m * n + 1,), -1.0, device="cuda")
    _lib.call("ntl_transpose_f32", abuf.data_ptr() + 4 * a_off, bbuf.data_ptr() + 4 * b_off, m, n,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    a = abuf[a_off:a_off + m * n].view(m, n)
    assert torch.equal(bbuf[b_off:b_off + m * n].view(n, m), a.T)
    assert bbuf[0 if b_off else m * n].item() == -1.0  # nothing written outside B


def test_native_launches_counted(torch_cuda):
    torch = torch_cuda
    from ntilang_b200 import _lib

    before = _lib.launch_count()
    K.softmax(4, 64)(torch.randn(4, 64, device="cuda"))
    torch.cuda.synchronize()
    assert _lib.launch_count() == before + 1


# ------------------------------------------------------------- back-to-back dependent launches
#
# The HBM-bound kernels are launched with programmatic stream serialization: the next kernel on
# the stream may start while the previous one runs, and waits (griddepcontrol.wait) before its
# first global access.  These tests chain kernels whose inputs are the previous kernel's output
# (read after write) or whose outputs overwrite the previous kernel's input (write after read),
# with no synchronisation in between, eagerly and inside a CUDA graph.


def _ping_pong(torch, x, y, rows, cols, rounds, stream):
    """Bit-exact ops only: y = cumsum(x); x = y - x (x is rewritten right after being read)."""
    from ntilang_b200 import _lib

    s = stream.cuda_stream
    for _ in range(rounds):
        _lib.call("ntl_cumsum_f32", x.data_ptr(), y.data_ptr(), rows, cols, 0, s)
        _lib.call("ntl_binary_f32", 1, y.data_ptr(), x.data_ptr(), x.data_ptr(), rows * cols, s)


def _four_ops(torch, x, y, w, rows, cols, stream):
    """y = x + x; x = cumsum(y); y = softmax(x); x = rmsnorm(y, w): each reads the previous
    output and overwrites a buffer the previous kernel read."""
    from ntilang_b200 import _lib

    s = stream.cuda_stream
    _lib.call("ntl_vadd_f32", x.data_ptr(), x.data_ptr(), y.data_ptr(), rows * cols, s)
    _lib.call("ntl_cumsum_f32", y.data_ptr(), x.data_ptr(), rows, cols, 0, s)
    _lib.call("ntl_softmax_f32", x.data_ptr(), y.data_ptr(), rows, cols, s)
    _lib.call("ntl_rmsnorm_f32", y.data_ptr(), w.data_ptr(), x.data_ptr(), rows, cols, 1e-6, 1.0 / cols, s)


def _run(torch, graph, body):
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    torch.cuda.synchronize()
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            body(stream)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            g.replay()
    else:
        body(stream)
    torch.cuda.synchronize()


@pytest.mark.parametrize("graph", [False, True])
def test_dependent_launches_bit_exact_ping_pong(torch_cuda, graph):
    torch = torch_cuda
    rows, cols, rounds = 8192, 256, 4
    x0 = np.random.default_rng(17).uniform(-1, 1, size=(rows, cols)).astype(np.float32)
    expect = x0
    for _ in range(rounds):
        y = rowops.cumsum(expect)
        expect = O.binary("-", y, expect)
    x = to_gpu(torch, x0)
    y = torch.empty_like(x)
    _run(torch, graph, lambda st: _ping_pong(torch, x, y, rows, cols, rounds, st))
    ok, bad = bits_equal(x.cpu().numpy(), expect)
    assert ok, f"{bad} elements differ"


@pytest.mark.parametrize("graph", [False, True])
def test_dependent_launches_four_op_chain(torch_cuda, graph):
    torch = torch_cuda
    rows, cols = 8192, 256
    rng = np.random.default_rng(18)
    x0 = rng.uniform(-1, 1, size=(rows, cols)).astype(np.float32)
    w0 = rng.normal(1.0, 0.1, size=cols).astype(np.float32)
    expect = rowops.rmsnorm(rowops.softmax(rowops.cumsum(rowops.vadd(x0, x0))), w0, 1e-6)
    x, w = to_gpu(torch, x0), to_gpu(torch, w0)
    y = torch.empty_like(x)
    _run(torch, graph, lambda st: _four_ops(torch, x, y, w, rows, cols, st))
    # vadd and cumsum are bit-exact; softmax then RMSNorm each within 1e-5 of the oracle.
    np.testing.assert_allclose(x.cpu().numpy(), expect, rtol=5e-5, atol=1e-7)
