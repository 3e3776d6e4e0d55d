"""Shared pytest configuration.

Markers: ``gpu`` — needs a CUDA device (run with ``-m gpu`` on a B200); everything else
runs on CPU.  The GPU tests call the sm_100a kernels through the C ABI of
libntl_kernels.so (via the ntilang-compatible Python surface) and compare with the CPU
oracle under ``oracle/`` and the golden vectors under ``tests/golden/``.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an NVIDIA GPU (sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def reference_examples_dir() -> Path:
    """Where the reference's own ``examples/*.py`` are read from: ``$NTL_REFERENCE_EXAMPLES``, else
    the reference install beside the bench (``baseline/_ref/examples``, git-ignored; it travels
    with the repository to the GPU box)."""
    env = os.environ.get("NTL_REFERENCE_EXAMPLES")
    return Path(env) if env else ROOT / "baseline" / "_ref" / "examples"


def load_reference_example(name: str):
    """Import the reference's ``examples/<name>.py`` unchanged.  Its ``import ntilang`` resolves to
    this repository's alias package (the repository root is first on ``sys.path``); skip when the
    examples are absent."""
    import importlib.util

    path = reference_examples_dir() / f"{name}.py"
    if not path.exists():
        pytest.skip(f"reference example {path} not present")
    spec = importlib.util.spec_from_file_location(f"_ref_example_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("No NVIDIA GPU available")
    from ntilang_b200 import _lib

    _lib.lib()  # the CUDA path must be the one that runs: fail loudly if the library is missing
    return torch


@pytest.fixture(scope="session")
def built_library():
    """Build (if needed) and return the path of libntl_kernels.so (CPU-safe: no device calls)."""
    from ntilang_b200.build import LIB, build_library

    if os.environ.get("NTL_SKIP_BUILD") != "1":
        build_library()
    if not LIB.exists():
        pytest.skip("libntl_kernels.so is not built")
    return LIB
