"""Pin the CPU oracle against golden vectors produced by the reference implementation.

The ``tests/golden/*.npz`` files were written by ``tests/golden/make_golden.py`` from the
reference's own NumPy evaluator (``ntilang.testing.reference``) and scan evaluator
(``ntilang.scan.evaluate``).  Integer-free fp32 scans and vector add must match
bit-for-bit; reductions within 1e-5 relative; GEMM / attention within the tolerances the
north-star states.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ntl_oracle as O
from oracle import rowops
from tests.conftest import golden


def assert_bits(actual, expected):
    a = np.asarray(actual, np.float32)
    e = np.asarray(expected, np.float32)
    assert a.shape == e.shape
    same = (a.view(np.uint32) == e.view(np.uint32)) | (np.isnan(a) & np.isnan(e))
    assert same.all(), f"{(~same).sum()} of {a.size} elements differ bitwise"


def test_vadd_bit_exact():
    g = golden("vadd_1000")
    assert_bits(O.vadd(g["a"], g["b"]), g["c"])
    assert_bits(rowops.vadd(g["a"], g["b"]), g["c"])


CUMSUM_CASES = [
    "cumsum_7x65_fwd", "cumsum_7x65_rev", "cumsum_4x256_fwd", "cumsum_4x256_rev",
    "cumsum_special_fwd", "cumsum_special_rev", "cumsum_eval_64x1000_fwd", "cumsum_eval_64x1000_rev",
]


@pytest.mark.parametrize("case", CUMSUM_CASES)
def test_cumsum_bit_exact(case):
    g = golden(case)
    rev = bool(g["reverse"])
    with np.errstate(over="ignore", invalid="ignore"):
        assert_bits(O.cumsum_rows(g["x"], rev), g["y"])
        assert_bits(rowops.cumsum(g["x"], rev), g["y"])


@pytest.mark.parametrize("case", ["scan_9x113_fwd", "scan_9x113_rev"])
def test_sum_and_max_scans_bit_exact(case):
    """examples/scan.py (T.cumsum into a second tile, T.cummax in place) with signed zeros,
    infinities and a NaN, from the reference evaluator."""
    g = golden(case)
    rev = bool(g["reverse"])
    with np.errstate(over="ignore", invalid="ignore"):
        assert_bits(O.cumsum_rows(g["x"], rev), g["prefix"])
    assert_bits(O.cummax_rows(g["x"], rev), g["maximum"])
    zeros = g["maximum"][3]  # an all -0 row stays -0; a row mixing signed zeros rises to +0
    assert np.all(np.signbit(zeros))


def test_cumsum_order_differs_from_sequential():
    """The reference's segment order is not a sequential prefix sum: torch/np.cumsum is no oracle."""
    g = golden("cumsum_eval_64x1000_fwd")
    seq = np.cumsum(g["x"], axis=1, dtype=np.float32)
    assert not np.array_equal(seq.view(np.uint32), g["y"].view(np.uint32))


@pytest.mark.parametrize("case", ["softmax_9x113", "softmax_4x512"])
def test_softmax_within_1e5(case):
    g = golden(case)
    for got in (O.softmax_rows(g["x"]), rowops.softmax(g["x"])):
        np.testing.assert_allclose(got, g["y"], rtol=1e-5, atol=1e-30)


@pytest.mark.parametrize("case", ["rmsnorm_6x1024", "rmsnorm_5x768"])
def test_rmsnorm_within_1e5(case):
    g = golden(case)
    eps = float(g["eps"])
    for got in (O.rmsnorm_rows(g["x"], g["w"], eps), rowops.rmsnorm(g["x"], g["w"], eps)):
        np.testing.assert_allclose(got, g["y"], rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("case", ["layernorm_6x1024", "layernorm_5x768", "layernorm_3x100"])
def test_layernorm_within_tolerance(case):
    """The reference evaluator sums with NumPy's pairwise add.reduce; the oracle (and the GPU
    kernel) follow the emitted kernel's perfect tree, so they agree to rounding: 1e-5 relative
    plus 1e-6 absolute (outputs near zero come from cancellation in d * rstd * w + b)."""
    g = golden(case)
    eps = float(g["eps"])
    oracle_np = O.layernorm_rows(g["x"], g["w"], g["b"], eps)
    oracle_c = rowops.layernorm(g["x"], g["w"], g["b"], eps)
    np.testing.assert_array_equal(oracle_np.view(np.uint32), oracle_c.view(np.uint32))
    np.testing.assert_allclose(oracle_np, g["y"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", ["transpose_65x71", "transpose_33x130"])
def test_transpose_bit_exact(case):
    g = golden(case)
    np.testing.assert_array_equal(O.transpose(g["a"]), g["b"])
    np.testing.assert_array_equal(rowops.transpose(g["a"]), g["b"])


def test_gemm_against_reference_evaluator():
    g = golden("gemm_65x71x37")
    np.testing.assert_allclose(O.gemm(g["a"], g["b"]), g["c"], rtol=1e-5, atol=1e-4)


def test_gemm_relu_against_reference_evaluator():
    g = golden("gemm_relu_65x71x37")
    got = O.gemm(g["a"], g["b"], g["bias"], O.BIAS_MN, alpha=float(g["alpha"]), relu=True)
    np.testing.assert_allclose(got, g["c"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("case", ["fa2_1x2x128x64_full", "fa2_1x2x128x64_causal"])
def test_fa2_blockwise_against_reference_evaluator(case):
    g = golden(case)
    got = O.fa2_blockwise(g["q"], g["k"], g["v"], float(g["scale_log2"]), bool(g["causal"]))
    np.testing.assert_allclose(got.astype(np.float32), g["o"].astype(np.float32), rtol=0, atol=2e-3)
    sdpa = O.attention_reference(g["q"], g["k"], g["v"], bool(g["causal"]))
    np.testing.assert_allclose(g["o"].astype(np.float32), sdpa.astype(np.float32), rtol=0, atol=2e-3)


def test_c_and_numpy_oracles_agree_on_larger_rows():
    rng = np.random.default_rng(9)
    x = rng.normal(size=(33, 1500)).astype(np.float32) * 3
    for rev in (False, True):
        assert_bits(rowops.cumsum(x, rev), O.cumsum_rows(x, rev))
    np.testing.assert_allclose(rowops.softmax(x), O.softmax_rows(x), rtol=1e-6, atol=1e-30)
    w = rng.normal(1, 0.1, 1500).astype(np.float32)
    np.testing.assert_allclose(rowops.rmsnorm(x, w, 1e-6), O.rmsnorm_rows(x, w, 1e-6), rtol=1e-6)


def test_tree_sum_is_the_reference_tree():
    # 8 values where pairwise and sequential summation round differently.
    v = np.array([[1e8, 1.0, -1e8, 1.0, 3.0, 5.0, 7.0, 1e-3]], np.float32)
    t = O.tree_sum_rows(v)[0]
    expect = np.float32((np.float32(1e8) + np.float32(1.0)) + (np.float32(-1e8) + np.float32(1.0)))
    expect = np.float32(expect + np.float32(np.float32(3 + 5) + np.float32(np.float32(7) + np.float32(1e-3))))
    assert t == expect
