"""The reference's own example programs, unchanged, on the GPU.

Each hot-path ``examples/*.py`` of the reference (``vector_add.py:5-10``, ``cumsum.py:7-14``,
``scan.py:7-22``, ``softmax.py:9-25``, ``rmsnorm.py:13-37``, ``layernorm.py:9-45``,
``transpose.py:5-15``, ``matmul.py:17-31``, ``matmul_relu.py:17-38``,
``flash_attention.py:26-79``), and the generic elementwise programs ``piecewise.py``,
``fragment_affine.py`` and ``window_sum.py``, is imported from the reference's tree (``tests.conftest.
reference_examples_dir``) with ``import ntilang`` resolving to this repository, built with its
own function at the BASELINE shapes for ``target="auto"`` and launched on the B200.  The outputs
are checked at the north-star bars: bit-exact (vector add, scans, transpose), 1e-5 relative
(softmax, RMSNorm, LayerNorm), 1e-3 * (|ref| + max |ref|) of an fp32 product (GEMMs, the
example's ``relu(0.5 * acc + Bias[M, N])`` epilogue for matmul_relu), 2e-3 absolute against fp32
attention on sampled heads; the generic programs bit-exact against the outputs the reference's
own evaluator gave for the same inputs (``tests/golden/pw_*.npz``)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ntl_oracle as O
from tests.conftest import golden, load_reference_example
from tests.test_gpu_fa2 import ATOL, sdpa_fp32

pytestmark = pytest.mark.gpu
TARGET = "auto"


def to_gpu(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_vector_add_example(torch_cuda):
    torch = torch_cuda
    n = 16 * 1024 * 1024
    kern = load_reference_example("vector_add").vector_add(n, target=TARGET)
    rng = np.random.default_rng(1)
    a, b = (rng.normal(size=n).astype(np.float32) for _ in range(2))
    c = torch.empty(n, device="cuda")
    kern(to_gpu(torch, a), to_gpu(torch, b), c)
    assert np.array_equal(bits(c.cpu().numpy()), bits(O.vadd(a, b)))


@pytest.mark.parametrize("reverse", [False, True])
def test_cumsum_example(torch_cuda, reverse):
    torch = torch_cuda
    rows, cols = (32768, 256) if not reverse else (1029, 300)
    kern = load_reference_example("cumsum").cumsum(rows, cols, reverse=reverse, target=TARGET)
    x = np.random.default_rng(2).uniform(-1, 1, size=(rows, cols)).astype(np.float32)
    y = torch.empty(rows, cols, device="cuda")
    kern(to_gpu(torch, x), y)
    assert np.array_equal(bits(y.cpu().numpy()), bits(O.cumsum_rows(x, reverse)))


def test_scan_example(torch_cuda):
    torch = torch_cuda
    rows, cols = 515, 113
    kern = load_reference_example("scan").scan(rows, cols, target=TARGET)
    x = np.random.default_rng(3).normal(size=(rows, cols)).astype(np.float32)
    prefix, maxima = torch.empty(rows, cols, device="cuda"), torch.empty(rows, cols, device="cuda")
    kern(to_gpu(torch, x), prefix, maxima)
    assert np.array_equal(bits(prefix.cpu().numpy()), bits(O.cumsum_rows(x)))
    assert np.array_equal(bits(maxima.cpu().numpy()), bits(O.cummax_rows(x)))


def test_softmax_example(torch_cuda):
    torch = torch_cuda
    rows, cols = 16384, 512
    kern = load_reference_example("softmax").softmax(rows, cols, target=TARGET)
    x = (np.random.default_rng(4).normal(size=(rows, cols)) * 2).astype(np.float32)
    y = torch.empty(rows, cols, device="cuda")
    kern(to_gpu(torch, x), y)
    np.testing.assert_allclose(y.cpu().numpy(), O.softmax_rows(x), rtol=1e-5, atol=1e-30)


def test_rmsnorm_example(torch_cuda):
    torch = torch_cuda
    rows, cols, eps = 4096, 1024, 1e-6
    kern = load_reference_example("rmsnorm").rmsnorm(rows, cols, eps=eps, target=TARGET)
    rng = np.random.default_rng(5)
    x = rng.normal(size=(rows, cols)).astype(np.float32)
    w = rng.normal(1, 0.1, size=cols).astype(np.float32)
    y = torch.empty(rows, cols, device="cuda")
    kern(to_gpu(torch, x), to_gpu(torch, w), y)
    np.testing.assert_allclose(y.cpu().numpy(), O.rmsnorm_rows(x, w, eps, 1.0 / cols), rtol=1e-5, atol=1e-7)


def test_layernorm_example(torch_cuda):
    torch = torch_cuda
    rows, cols, eps = 4096, 1024, 1e-5
    kern = load_reference_example("layernorm").layernorm(rows, cols, eps=eps, target=TARGET)
    rng = np.random.default_rng(6)
    x = rng.normal(size=(rows, cols)).astype(np.float32)
    w = rng.normal(1, 0.1, size=cols).astype(np.float32)
    b = rng.normal(0, 0.1, size=cols).astype(np.float32)
    y = torch.empty(rows, cols, device="cuda")
    kern(to_gpu(torch, x), to_gpu(torch, w), to_gpu(torch, b), y)
    np.testing.assert_allclose(y.cpu().numpy(), O.layernorm_rows(x, w, b, eps, 1.0 / cols), rtol=1e-5,
                               atol=1e-6)


def test_transpose_example(torch_cuda):
    torch = torch_cuda
    m, n = 4096, 4096
    kern = load_reference_example("transpose").transpose(m, n, target=TARGET)
    a = torch.randn(m, n, device="cuda")
    b = torch.empty(n, m, device="cuda")
    kern(a, b)
    assert torch.equal(b, a.t())


def _gemm_inputs(torch, m, n, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn(m, k, device="cuda", generator=g) / k ** 0.5).half()
    b = (torch.randn(k, n, device="cuda", generator=g) / k ** 0.5).half()
    return a, b


def _close(got, ref):
    bound = 1e-3 * (ref.abs() + ref.abs().max())
    assert bool(((got - ref).abs() <= bound).all())


def test_matmul_example_readme_tiles(torch_cuda):
    torch = torch_cuda
    m = n = k = 4096
    kern = load_reference_example("matmul").matmul(m, n, k, block_m=128, block_n=128, block_k=32, num_stages=3,
                                                   swizzle_panel=8, target=TARGET)
    a, b = _gemm_inputs(torch, m, n, k, 7)
    c = torch.empty(m, n, device="cuda")
    kern(a, b, c)
    _close(c, a.float() @ b.float())


def test_matmul_relu_example_epilogue(torch_cuda):
    torch = torch_cuda
    m = n = k = 4096
    kern = load_reference_example("matmul_relu").matmul_relu(m, n, k, block_m=128, block_n=128, block_k=32,
                                                             num_stages=3, swizzle_panel=8, target=TARGET)
    a, b = _gemm_inputs(torch, m, n, k, 8)
    bias = torch.randn(m, n, device="cuda") * 0.1
    c = torch.empty(m, n, device="cuda")
    kern(a, b, bias, c)
    _close(c, torch.relu(0.5 * (a.float() @ b.float()) + bias))


@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_example(torch_cuda, causal):
    torch = torch_cuda
    shape = (8, 32, 4096, 128)
    kern = load_reference_example("flash_attention").flash_attention(*shape, is_causal=causal, target=TARGET)
    g = torch.Generator(device="cuda").manual_seed(9)
    q, k, v = (torch.randn(shape, device="cuda", generator=g, dtype=torch.float16) for _ in range(3))
    o = torch.empty_like(q)
    kern(q, k, v, o)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all()
    for b, h in ((0, 0), (2, 17), (7, 31)):
        ref = sdpa_fp32(torch, q[b:b + 1, h:h + 1], k[b:b + 1, h:h + 1], v[b:b + 1, h:h + 1], causal)
        torch.testing.assert_close(o[b:b + 1, h:h + 1].float(), ref, rtol=0, atol=ATOL)


def test_generic_elementwise_examples(torch_cuda):
    """examples/piecewise.py, fragment_affine.py and window_sum.py at their default sizes, through
    the NVRTC path, against the reference evaluator's golden outputs."""
    torch = torch_cuda
    g = golden("pw_piecewise_93")
    kern = load_reference_example("piecewise").piecewise(target=TARGET)
    b = torch.full((93,), float("nan"), device="cuda")
    kern(to_gpu(torch, g["a"]), b)
    assert np.array_equal(bits(b.cpu().numpy()), bits(g["b"]))

    g = golden("pw_fragment_affine_257")
    kern = load_reference_example("fragment_affine").fragment_affine(target=TARGET)
    b = torch.full((257,), float("nan"), device="cuda")
    kern(to_gpu(torch, g["a"]), b)
    assert np.array_equal(bits(b.cpu().numpy()), bits(g["b"]))

    g = golden("pw_window_sum_7x3x5")
    kern = load_reference_example("window_sum").window_sum(target=TARGET)
    a = to_gpu(torch, g["a"])
    for (rows, cols), expect in zip(g["windows"], g["b"]):
        b = torch.full((7,), float("nan"), device="cuda")
        kern(a, b, int(rows), int(cols))
        assert np.array_equal(bits(b.cpu().numpy()), bits(expect)), (rows, cols)
