"""GPU parity for the FP16 GEMM family (tcgen05 path and the CUDA-core path for unaligned shapes).

Bar (north star): within 1e-2 relative of an fp32-accumulated product.  The checks below are
tighter — every element within rtol + atol * max|C| of ``A.float() @ B.float()`` computed
in fp32 with TF32 disabled — because both sides accumulate exact fp16 products in fp32.
"""

from __future__ import annotations

import numpy as np
import pytest

from ntilang_b200 import kernels as K
from oracle import ntl_oracle as O
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def ref_gemm(torch, a, b, trans_b=False):
    torch.backends.cuda.matmul.allow_tf32 = False
    bb = b.float().t() if trans_b else b.float()
    return a.float() @ bb


def check(torch, c, ref, rtol=1e-3):
    scale = float(ref.abs().max()) + 1e-30
    err = (c - ref).abs()
    bound = rtol * ref.abs() + rtol * scale
    assert bool((err <= bound).all()), f"max err {float(err.max()):.3e} (scale {scale:.3e})"


def test_gemm_golden_unaligned_shape(torch_cuda):
    torch = torch_cuda
    g = golden("gemm_65x71x37")
    a = torch.from_numpy(g["a"]).cuda()
    b = torch.from_numpy(g["b"]).cuda()
    c = K.matmul(65, 71, 37)(a, b)
    np.testing.assert_allclose(c.cpu().numpy(), g["c"], rtol=1e-4, atol=1e-4)


def test_gemm_relu_golden(torch_cuda):
    torch = torch_cuda
    g = golden("gemm_relu_65x71x37")
    args = [torch.from_numpy(g[k]).cuda() for k in ("a", "b", "bias")]
    c = K.matmul_scaled_bias_relu(65, 71, 37)(*args)
    np.testing.assert_allclose(c.cpu().numpy(), g["c"], rtol=1e-4, atol=1e-4)


SHAPES = [
    (128, 256, 64),    # one tile, one k-block
    (128, 256, 128),
    (256, 512, 256),
    (200, 264, 72),    # ragged M, N, K (TMA zero fill + predicated stores)
    (1024, 1024, 1024),
    (129, 8, 8),       # tiny N, K
    (4096, 4096, 4096),
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_tcgen05(torch_cuda, m, n, k):
    torch = torch_cuda
    gen = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
    b = torch.randn(k, n, device="cuda", generator=gen).half()
    c = K.matmul(m, n, k)(a, b)
    check(torch, c, ref_gemm(torch, a, b))


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 520, 136), (2048, 2048, 512)])
def test_gemm_tcgen05_transpose_b(torch_cuda, m, n, k):
    torch = torch_cuda
    gen = torch.Generator(device="cuda").manual_seed(7)
    a = torch.randn(m, k, device="cuda", generator=gen).half()
    b = torch.randn(n, k, device="cuda", generator=gen).half()
    c = K.matmul(m, n, k, trans_b=True)(a, b)
    check(torch, c, ref_gemm(torch, a, b, trans_b=True))


def test_gemm_bias_relu_baseline(torch_cuda):
    """BASELINE variant: C = relu(A @ B + bias[N]), A, B ~ N(0,1)/sqrt(K), bias ~ N(0, 0.1)."""
    torch = torch_cuda
    m = n = k = 4096
    gen = torch.Generator(device="cuda").manual_seed(0)
    a = (torch.randn(m, k, device="cuda", generator=gen) / 64).half()
    b = (torch.randn(k, n, device="cuda", generator=gen) / 64).half()
    bias = torch.randn(n, device="cuda", generator=gen) * 0.1
    c = K.matmul_bias_relu(m, n, k)(a, b, bias)
    check(torch, c, torch.relu(ref_gemm(torch, a, b) + bias))


@pytest.mark.parametrize("m,n,k", [(256, 256, 128), (200, 264, 72)])
def test_gemm_scaled_bias_matrix_relu(torch_cuda, m, n, k):
    torch = torch_cuda
    gen = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(m, k, device="cuda", generator=gen).half()
    b = torch.randn(k, n, device="cuda", generator=gen).half()
    bias = torch.randn(m, n, device="cuda", generator=gen)
    c = K.matmul_scaled_bias_relu(m, n, k)(a, b, bias)
    check(torch, c, torch.relu(ref_gemm(torch, a, b) * 0.5 + bias))


@pytest.mark.parametrize("m,n,k", [(65, 71, 37), (1, 1, 1), (33, 17, 9), (100, 200, 30)])
def test_gemm_cuda_core_path(torch_cuda, m, n, k):
    torch = torch_cuda
    gen = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(m, k, device="cuda", generator=gen).half()
    b = torch.randn(k, n, device="cuda", generator=gen).half()
    c = K.matmul(m, n, k)(a, b)
    check(torch, c, ref_gemm(torch, a, b), rtol=1e-4)


def test_gemm_against_cpu_oracle(torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    a = rng.normal(size=(384, 128)).astype(np.float16)
    b = rng.normal(size=(128, 512)).astype(np.float16)
    bias = rng.normal(0, 0.1, size=512).astype(np.float32)
    c = K.matmul_bias_relu(384, 512, 128)(*(torch.from_numpy(x).cuda() for x in (a, b, bias)))
    expect = O.gemm(a, b, bias, O.BIAS_N, relu=True)
    np.testing.assert_allclose(c.cpu().numpy(), expect, rtol=1e-3, atol=1e-3)


def test_gemm_timeout_path_reports_error(torch_cuda):
    """A 1-poll wait limit makes the bounded waits give up; the kernel must return (no hang),
    report a status code and leave the context usable."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    a = torch.randn(512, 512, device="cuda").half()
    b = torch.randn(512, 512, device="cuda").half()
    c = torch.empty(512, 512, device="cuda")
    _lib.clear_device_status()
    _lib.set_wait_limit(1)
    try:
        _lib.call("ntl_gemm_f16_f32", a.data_ptr(), b.data_ptr(), c.data_ptr(), None, 0, 1.0, 0, 512, 512, 512, 0,
                  torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        status = _lib.device_status()
    finally:
        _lib.set_wait_limit(1 << 26)
        _lib.clear_device_status()
    assert status != 0
    # the context still works
    c2 = K.matmul(512, 512, 512)(a, b)
    check(torch, c2, ref_gemm(torch, a, b))


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (512, 4096, 4096), (1000, 1024, 1032), (384, 768, 4096)])
def test_gemm_stream_k_repeated_calls(torch_cuda, m, n, k):
    """Shapes whose last wave is split along K (stream-K through the cached workspace), called
    three times in a row: the contributor flags must be back to zero after every call."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    from ntilang_b200.launch import gemm_workspace

    need = _lib.gemm_workspace_size(m, n, k, 0)
    assert need > 0
    ws = gemm_workspace(torch.device("cuda"), need)
    gen = torch.Generator(device="cuda").manual_seed(m + k)
    a = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
    b = torch.randn(k, n, device="cuda", generator=gen).half()
    bias = torch.randn(n, device="cuda", generator=gen) * 0.1
    ref = torch.relu(ref_gemm(torch, a, b) + bias)
    for _ in range(3):
        c = torch.full((m, n), float("nan"), device="cuda")
        _lib.call("ntl_gemm_f16_f32_ws", a.data_ptr(), b.data_ptr(), c.data_ptr(), bias.data_ptr(), 1, 1.0, 1, m, n,
                  k, 0, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        check(torch, c, ref)


@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (520, 2048, 1024), (96, 4096, 2048)])
def test_gemm_split_tail_transpose_b_row_bias(torch_cuda, m, n, k):
    """The split tail with B given as [N, K], a per-row bias and alpha = 0.5 (CTA-pair kernel for
    M > 128, one-SM stream-K for M <= 128)."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    from ntilang_b200.launch import gemm_workspace

    need = _lib.gemm_workspace_size(m, n, k, 1)
    ws = gemm_workspace(torch.device("cuda"), need)
    gen = torch.Generator(device="cuda").manual_seed(m)
    a = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
    b = torch.randn(n, k, device="cuda", generator=gen).half()
    bias = torch.randn(m, device="cuda", generator=gen)
    ref = torch.relu(ref_gemm(torch, a, b, trans_b=True) * 0.5 + bias[:, None])
    for _ in range(2):
        c = torch.full((m, n), float("nan"), device="cuda")
        _lib.call("ntl_gemm_f16_f32_ws", a.data_ptr(), b.data_ptr(), c.data_ptr(), bias.data_ptr(), 3, 0.5, 1, m, n,
                  k, 1, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        check(torch, c, ref)


def test_gemm_stream_k_matches_data_parallel_entry(torch_cuda):
    torch = torch_cuda
    from ntilang_b200 import _lib

    m = n = k = 2048
    a = torch.randn(m, k, device="cuda").half()
    b = torch.randn(k, n, device="cuda").half()
    from ntilang_b200.launch import gemm_workspace

    c_dp = torch.empty(m, n, device="cuda")
    c_sk = torch.empty(m, n, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    ws = gemm_workspace(torch.device("cuda"), _lib.gemm_workspace_size(m, n, k, 0))
    _lib.call("ntl_gemm_f16_f32", a.data_ptr(), b.data_ptr(), c_dp.data_ptr(), None, 0, 1.0, 0, m, n, k, 0, s)
    _lib.call("ntl_gemm_f16_f32_ws", a.data_ptr(), b.data_ptr(), c_sk.data_ptr(), None, 0, 1.0, 0, m, n, k, 0,
              ws.data_ptr(), ws.numel(), s)
    check(torch, c_sk, c_dp, rtol=1e-5)
    check(torch, c_dp, ref_gemm(torch, a, b))


def test_gemm_workspace_too_small_is_rejected(torch_cuda):
    torch = torch_cuda
    from ntilang_b200 import _lib

    m = n = k = 4096
    need = _lib.gemm_workspace_size(m, n, k, 0)
    a = torch.zeros(m, k, device="cuda").half()
    b = torch.zeros(k, n, device="cuda").half()
    c = torch.empty(m, n, device="cuda")
    ws = torch.zeros(need // 2, dtype=torch.uint8, device="cuda")
    with pytest.raises(_lib.KernelError, match="workspace"):
        _lib.call("ntl_gemm_f16_f32_ws", a.data_ptr(), b.data_ptr(), c.data_ptr(), None, 0, 1.0, 0, m, n, k, 0,
                  ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,n,k,trans_b,bias_mode", [
    (2560, 4096, 512, 0, 1),   # 160 pair tiles: two full waves on 74 pairs, 12 tail tiles split along N
    (2560, 4096, 512, 1, 3),   # the same with B given as [N, K] and a per-row bias
    (1536, 1000, 264, 1, 1),   # 24 tiles, all split; ragged N: the last tile's second half is empty
    (1536, 1000, 264, 0, 0),
    (384, 520, 136, 0, 1),     # 6 tiles on 12 pairs, ragged M / N / K
])
def test_gemm_n_split_tail_tiles(torch_cuda, m, n, k, trans_b, bias_mode):
    """Data-parallel entry: the last partial wave's 256x256 tiles run as two 256x128 halves on
    otherwise idle CTA pairs (every tile when there are fewer tiles than half the pairs)."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    gen = torch.Generator(device="cuda").manual_seed(m + n)
    a = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
    b = torch.randn(n, k, device="cuda", generator=gen).half() if trans_b else \
        torch.randn(k, n, device="cuda", generator=gen).half()
    bias = torch.randn(m if bias_mode == 3 else n, device="cuda", generator=gen)
    ref = ref_gemm(torch, a, b, trans_b=bool(trans_b)) * 0.75
    if bias_mode == 1:
        ref = ref + bias[None, :]
    elif bias_mode == 3:
        ref = ref + bias[:, None]
    ref = torch.relu(ref)
    for _ in range(2):
        c = torch.full((m, n), float("nan"), device="cuda")
        _lib.call("ntl_gemm_f16_f32", a.data_ptr(), b.data_ptr(), c.data_ptr(), bias.data_ptr(), bias_mode, 0.75, 1,
                  m, n, k, trans_b, torch.cuda.current_stream().cuda_stream)
        check(torch, c, ref)


@pytest.mark.parametrize("m,n,k", [(1024, 1024, 1024), (512, 4096, 1024), (96, 512, 256)])
def test_gemm_dependent_launches_in_one_stream(torch_cuda, m, n, k):
    """The tcgen05 GEMMs start their setup while the previous kernel on the stream runs, and
    touch global memory only after it completes.  Twenty rounds, with no synchronisation, of
    C = A B; D = C + E (a vector add, which also overlaps its predecessor); C = A2 B2: every D is
    exactly A B + E, so no GEMM wrote C while the add still read it, and no add read C before the
    GEMM finished writing it."""
    torch = torch_cuda
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a, a2 = ((torch.randn(m, k, device="cuda", generator=g) / k ** 0.5).half() for _ in range(2))
    b, b2 = ((torch.randn(k, n, device="cuda", generator=g) / k ** 0.5).half() for _ in range(2))
    e = torch.randn(m * n, device="cuda", generator=g)
    gemm = K.matmul(m, n, k)
    add = K.vector_add(m * n)
    want = gemm(a, b).view(-1) + e
    assert not torch.equal(gemm(a2, b2).view(-1) + e, want)
    c = torch.empty(m, n, device="cuda")
    outs = []
    for _ in range(20):
        gemm(a, b, c)
        d = torch.empty(m * n, device="cuda")
        add(c.view(-1), e, d)
        gemm(a2, b2, c)
        outs.append(d)
    torch.cuda.synchronize()
    for d in outs:
        assert torch.equal(d, want)
