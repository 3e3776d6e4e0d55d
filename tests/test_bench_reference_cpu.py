"""The driver's reference arm, ``bench.py --impl reference``, on the CPU: the reference's algorithm
(the oracle port) timed on the host cores, one JSON line with the contract's fields, and nothing
printed by ranks other than 0."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
ARGS = ["--impl", "reference", "--steps", "1", "--warmup", "1", "--ops", "cumsum,vadd", "--cpu-seconds", "0.2",
        "--detail", ""]


def run(env_extra, tmp_path):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *ARGS], env=env, cwd=tmp_path,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_line(tmp_path):
    out = run({}, tmp_path)
    assert out.returncode == 0, out.stderr
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["config"]["op"] == "cumsum" and set(line["ops"]) == {"cumsum", "vadd"}
    # one step is one whole workload (67,108,864 bytes for the cumsum) at the sampled rate
    assert abs(line["ms_per_step"] - 67108864 / (line["value"] * 1e9) * 1e3) <= 1e-3 * line["ms_per_step"] + 1e-6
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing(tmp_path):
    out = run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, tmp_path)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == ""
