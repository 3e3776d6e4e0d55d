"""The C ABI library: it builds, loads without a GPU, exports every symbol the header
declares, and rejects bad arguments on the host before any CUDA call."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "ntl_kernels.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_0-9]+\**\s+\**(ntl_[a-z0-9_]+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    names = declared_symbols()
    for must in ("ntl_vadd_f32", "ntl_cumsum_f32", "ntl_softmax_f32", "ntl_rmsnorm_f32", "ntl_gemm_f16_f32",
                 "ntl_fa2_fwd_f16", "ntl_last_error", "ntl_device_status"):
        assert must in names


def test_library_exports_every_declared_symbol(built_library):
    handle = ctypes.CDLL(str(built_library))
    missing = [n for n in declared_symbols() if not hasattr(handle, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    from ntilang_b200._lib import SIGNATURES

    assert set(declared_symbols()) == set(SIGNATURES)


def test_host_side_validation_without_gpu(built_library):
    from ntilang_b200 import _lib

    h = _lib.lib()
    assert h.ntl_version() >= 100
    assert h.ntl_cumsum_f32(None, None, -1, 4, 0, None) == 1
    assert b"negative" in h.ntl_last_error()
    assert h.ntl_gemm_f16_f32(16, 16, 16, None, 7, 1.0, 0, 8, 8, 8, 0, None) == 1
    assert b"bias_mode" in h.ntl_last_error()
    assert h.ntl_gemm_f16_f32(16, 16, 16, None, 1, 1.0, 0, 8, 8, 8, 0, None) == 1
    assert h.ntl_softmax_f32(16, 32, 4, 1 << 20, None) == 2
    assert h.ntl_set_wait_limit(0) == 1
    assert h.ntl_fa2_set_causal_grid(3) == 1 and b"causal grid" in h.ntl_last_error()
    for mode in (_lib.FA2_GRID_PERSISTENT, _lib.FA2_GRID_PER_BLOCK, _lib.FA2_GRID_AUTO):
        assert h.ntl_fa2_set_causal_grid(mode) == 0
    # empty problems are no-ops that succeed without touching the device
    assert h.ntl_vadd_f32(None, None, None, 0, None) == 0
    assert h.ntl_rmsnorm_f32(None, None, None, 0, 128, 1e-6, 1 / 128, None) == 0
    with pytest.raises(_lib.KernelError, match="negative"):
        _lib.call("ntl_softmax_f32", None, None, -2, 4, None)


def test_no_cpu_fallback_in_product_path():
    """The package never imports the oracle and has no CPU compute path."""
    pkg = ROOT / "ntilang_b200"
    for path in pkg.rglob("*.py"):
        text = path.read_text()
        assert "oracle" not in text.replace("oracle/", ""), path
