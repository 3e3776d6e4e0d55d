"""The bench's ``--impl reference-gpu`` leg on the CPU: its ``unavailable`` line when the
reference package is missing, and, when a copy of the reference is present under
baseline/_ref, that every bench op maps to one of the reference's example programs with the
bench's shapes (program generation only; building and launching need a GPU)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"


def test_reference_gpu_leg_reports_unavailable_without_the_package(tmp_path):
    env = dict(os.environ, NTL_REFERENCE_DIR=str(tmp_path / "missing"))
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference-gpu"], env=env, cwd=tmp_path,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference-gpu" and "unavailable" in line


_PROBE = r"""
import sys
sys.path.insert(0, sys.argv[1])
import bench
sys.path.insert(0, str(bench.REF_INSTALL))
import ntilang
assert str(bench.REF_INSTALL) in ntilang.__file__, ntilang.__file__
builders = bench.reference_builders("sm_100a")
assert set(builders) == set(bench.OPS), sorted(set(builders) ^ set(bench.OPS))
for name in bench.OPS:
    kern = builders[name][0](bench.OPS[name](None, None, 0))
    assert "def " in kern.source, name
print("ok")
"""


@pytest.mark.skipif(not (REF / "ntilang" / "__init__.py").exists() or not (REF / "examples").is_dir(),
                    reason="no copy of the reference under baseline/_ref")
def test_reference_gpu_builders_cover_every_bench_op(tmp_path):
    pytest.importorskip("cutlass")  # the reference's code generation imports the CuTe DSL lazily
    out = subprocess.run([sys.executable, "-c", _PROBE, str(ROOT)], cwd=tmp_path, capture_output=True, text=True,
                         timeout=600, env=dict(os.environ, NTL_REFERENCE_DIR=str(REF)))
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip().endswith("ok"), out.stdout
