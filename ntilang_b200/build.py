"""Build libntl_kernels.so in-tree with nvcc for sm_100a.

``python -m ntilang_b200.build`` (or ``__graft_entry__.build()``) compiles every
``csrc/*.cu`` to an object under ``ntilang_b200/_build/`` and links
``ntilang_b200/libntl_kernels.so``.  The library is plain C ABI (``include/ntl_kernels.h``);
Python reaches it through ctypes (``ntilang_b200._lib``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libntl_kernels.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; install the CUDA toolkit or set NVCC")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    headers = list(CSRC.glob("*.cuh")) + [ROOT / "include" / "ntl_kernels.h"]
    srcs = sources()
    if not force and not _stale(LIB, srcs + headers + [Path(__file__)]):
        return LIB
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)
    procs = []
    objects = []
    for src in srcs:
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if not force and not _stale(obj, [src] + headers):
            continue
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failures = []
    for src, proc in procs:
        out, _ = proc.communicate()
        if proc.returncode != 0:
            failures.append(f"{src.name}:\n{out}")
        elif verbose and out.strip():
            print(out, file=sys.stderr)
    if failures:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failures))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "--cudart", "static", "-o", str(tmp), *map(str, objects), "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("link failed:\n" + res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True))
