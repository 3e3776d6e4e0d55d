"""The allocation-free GEMM entry point, ntl_gemm_f16_f32_noalloc.

It exists for callers that cannot allocate device memory for a workspace: a plugin host
that hands a kernel only tensors and a stream (the reference's TVM-FFI launch path has no
workspace argument), or a runtime that runs with the device allocator switched off.  It
runs the same split-K GEMM as ntl_gemm_f16_f32_ws, with the scratch in a fixed 16 MiB
device array inside the library instead of a caller buffer.

The test calls it through the C ABI twice in a row (the array keeps the previous call's
contents, so the second call checks that the flags are cleared) and compares each output
with the workspace entry point's, within the GEMM tolerance of the other GPU tests.  A
second test first makes one call give up (a 1-poll wait limit, as the GEMM timeout test
does: contributor flags raised, finaliser gone, so flags stay set in the array), then
checks that the next call clears them and is correct.  It also checks that a shape whose
plan needs more scratch than the array holds is refused, and that operands only the
CUDA-core path can address are run without scratch whatever the shape.
This file sorts last so a failure here cannot hide earlier tests; it passes on its own in
a fresh process as well.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _check(c, ref, rtol=1e-3):
    scale = float(ref.abs().max()) + 1e-30
    err = (c - ref).abs()
    assert bool((err <= rtol * ref.abs() + rtol * scale).all()), f"max err {float(err.max()):.3e}"


def test_noalloc_gemm_matches_workspace_entry_point(torch_cuda):
    torch = torch_cuda
    from ntilang_b200 import _lib

    m, n, k = 1536, 4096, 1024  # one wave of 74 pair tiles, then 22 tail tiles split in 3 along K
    need = _lib.gemm_workspace_size(m, n, k, 0)
    assert 0 < need <= 16 << 20
    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(123)
    for call in range(2):
        a = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
        b = torch.randn(k, n, device="cuda", generator=gen).half()
        bias = torch.randn(n, device="cuda", generator=gen) * 0.1
        c_noalloc = torch.full((m, n), float("nan"), device="cuda")
        c_ws = torch.empty(m, n, device="cuda")
        _lib.call("ntl_gemm_f16_f32_noalloc", a.data_ptr(), b.data_ptr(), c_noalloc.data_ptr(), bias.data_ptr(), 1,
                  1.0, 1, m, n, k, 0, stream)
        _lib.call("ntl_gemm_f16_f32_ws", a.data_ptr(), b.data_ptr(), c_ws.data_ptr(), bias.data_ptr(), 1, 1.0, 1, m,
                  n, k, 0, ws.data_ptr(), ws.numel(), stream)
        torch.cuda.synchronize()
        assert torch.isfinite(c_noalloc).all(), f"call {call}: output not fully written"
        _check(c_noalloc, c_ws)
        torch.backends.cuda.matmul.allow_tf32 = False
        _check(c_noalloc, torch.relu(a.float() @ b.float() + bias))


def test_noalloc_gemm_refuses_plans_larger_than_its_scratch(torch_cuda):
    torch = torch_cuda
    from ntilang_b200 import _lib

    m, n, k = 128, 25600, 4096  # one-SM stream-K plan over every SM: 148 slots of 128 KB
    if _lib.gemm_workspace_size(m, n, k, 0) <= 16 << 20:
        pytest.skip("this device's plan for 128x25600x4096 fits the static scratch")
    a = torch.zeros(m, k, device="cuda").half()
    b = torch.zeros(k, n, device="cuda").half()
    c = torch.empty(m, n, device="cuda")
    with pytest.raises(_lib.KernelError, match="scratch"):
        _lib.call("ntl_gemm_f16_f32_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), None, 0, 1.0, 0, m, n, k, 0,
                  torch.cuda.current_stream().cuda_stream)


def test_noalloc_gemm_after_an_aborted_call(torch_cuda):
    torch = torch_cuda
    from ntilang_b200 import _lib

    m, n, k = 1536, 4096, 1024
    stream = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator(device="cuda").manual_seed(321)
    a = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
    b = torch.randn(k, n, device="cuda", generator=gen).half()
    c = torch.empty(m, n, device="cuda")
    _lib.clear_device_status()
    _lib.set_wait_limit(1)
    try:
        _lib.call("ntl_gemm_f16_f32_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), None, 0, 1.0, 0, m, n, k, 0,
                  stream)
        torch.cuda.synchronize()
        status = _lib.device_status()
    finally:
        _lib.set_wait_limit(1 << 26)
        _lib.clear_device_status()
    assert status != 0
    a2 = (torch.randn(m, k, device="cuda", generator=gen) / k**0.5).half()
    b2 = torch.randn(k, n, device="cuda", generator=gen).half()
    c2 = torch.full((m, n), float("nan"), device="cuda")
    _lib.call("ntl_gemm_f16_f32_noalloc", a2.data_ptr(), b2.data_ptr(), c2.data_ptr(), None, 0, 1.0, 0, m, n, k, 0,
              stream)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    torch.backends.cuda.matmul.allow_tf32 = False
    _check(c2, a2.float() @ b2.float())


def test_noalloc_gemm_unaligned_operands_need_no_scratch(torch_cuda):
    """The shape the previous test sees refused (its stream-K plan needs more than the array) runs
    when A is not 16-byte aligned: that launch takes the CUDA-core path and uses no scratch."""
    torch = torch_cuda
    from ntilang_b200 import _lib

    m, n, k = 128, 25600, 4096
    a_buf = torch.randn(m * k + 8, device="cuda").half()
    a = a_buf[4:4 + m * k].view(m, k)  # 8-byte offset: TMA cannot address it
    assert a.data_ptr() % 16 != 0
    b = (torch.randn(k, n, device="cuda") / k**0.5).half()
    c = torch.empty(m, n, device="cuda")
    _lib.call("ntl_gemm_f16_f32_noalloc", a.data_ptr(), b.data_ptr(), c.data_ptr(), None, 0, 1.0, 0, m, n, k, 0,
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    torch.backends.cuda.matmul.allow_tf32 = False
    _check(c, a.float() @ b.float())
