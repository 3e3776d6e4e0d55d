#!/usr/bin/env python
"""Throughput of the hot-path kernels on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-gpu] [--ops a,b,...]

A *step* is one pass of an op over one batch of synthetic input with BASELINE.json's
shapes and distributions.  The headline is the configuration BASELINE.json's metric is
normally quoted on (configs[1]: row cumsum, X f32 [32768, 256]); every op family's figures
are in the same line under ``"ops"`` (value, roofline fraction, ms per step, end-to-end and
CPU baselines), and the full per-op records go to a side file the line names.

value      K steps replayed from one CUDA graph (inputs resident in HBM, rotated over
           enough buffer sets that no set is reused within 3x L2 of other traffic, L2
           flushed before the timed replay), timed with CUDA events on the launching
           stream between barriers; max over ranks.
e2e        the same metric through the public call (``CompiledKernel.__call__`` -> C ABI)
           with pinned host buffers: every step copies its inputs host->device and its
           output device->host inside the timed region (steps alternate between two
           streams, so uploads and downloads of neighbouring steps overlap).
roofline   algorithmic bytes (or FLOPs) per launch / average launch time, against the
           measured HBM copy bandwidth or dense bf16 GEMM rate in MEASURED_PEAKS.json.
cpu_baseline  the CPU oracle (a restatement of the reference's algorithm; ``kind: port``)
           on the host cores, bounded sample, rank 0 at N=1 only; beside it the same op in
           torch on all host cores (``cpu_torch``).
Multi-GPU (``scaling: strong``): one BASELINE job is split across the N ranks -- contiguous
row blocks for the row ops, M-panels of A and C (B and bias replicated) for the GEMMs,
batches of (batch, head) pairs for attention -- with no collective on the data path.  The
value is the whole job's algorithmic work / the slowest rank's time per step.  After the
timed region the shards' outputs are all-gathered over NCCL and rank 0 compares them
bit-for-bit with the same kernels run on the whole job on one GPU.  ``weak`` repeats the
timing with a full-size job on every rank.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BASELINE_METRIC = "achieved GB/s or TFLOPS per op at 1/2/4/8 B200 and % of HBM/tensor roofline"
HEADLINE = "cumsum"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
DETAIL_DEFAULT = "gpurun_out/bench_detail_n{n}.json"


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return data, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    path = ROOT / "profiles" / "ncu_traffic.json"
    if path.exists():
        try:
            return json.loads(path.read_text())
        except json.JSONDecodeError:
            return {}
    return {}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def shard_bounds(total, rank, world):
    from ntilang_b200.dist import shard_bounds as bounds

    return bounds(total, rank, world)


# ---------------------------------------------------------------------------- workloads


class Op:
    """One bench workload.  ``world`` > 1 makes this rank's instance a shard of the job."""

    name = ""
    bound = "hbm"
    unit = "GB/s"
    dtype = "f32"

    def __init__(self, torch, device, rank=0, world=1):
        self.torch, self.device, self.rank, self.world = torch, device, rank, world
        self.localize()

    def localize(self):
        """Set this rank's share of the job."""

    def sets_needed(self, footprint):
        """Distinct buffer sets so that a set is reused only after > 3x L2 of other traffic
        (bounded to about 2 GiB of buffers)."""
        want = math.ceil(3 * L2_BYTES / max(1, footprint))
        cap = max(1, (2 << 30) // max(1, footprint))
        return max(1, min(want, cap, 256))

    def units(self):  # algorithmic bytes or FLOPs of this rank's share, per step
        return self.units_of_rank(self.rank)

    def units_of_rank(self, r):
        return self.units_of_rows(self.rows_of_rank(r))

    def whole_job_units(self):  # the job on one GPU (what the ncu captures cover)
        return self.units_of_rows(self.full_rows)

    def total_units(self):  # of the whole job (all ranks), per step
        return sum(self.units_of_rank(r) for r in range(self.world))

    def per_unit(self):
        return 1e9 if self.unit == "GB/s" else 1e12

    def g(self, seed):
        return self.torch.Generator(device=self.device).manual_seed(seed)

    # -- the generic setup: set 0 is this rank's slice of one seeded global input (so the
    # gathered outputs can be checked against a one-GPU run of the whole job); the other
    # sets are independent local inputs.
    def setup(self):
        self.kernel = self.make_kernel(local=True)
        ins0 = self.slice_inputs(self.global_inputs())
        foot = sum(t.numel() * t.element_size() for t in ins0) + self.out_bytes(ins0)
        self.sets = []
        for s in range(self.sets_needed(foot)):
            ins = ins0 if s == 0 else self.local_inputs(s)
            out = self.alloc_out(ins)
            self.sets.append((ins + (out,), ins, out))

    def out_bytes(self, ins):
        return ins[0].numel() * 4

    def alloc_out(self, ins):
        return self.torch.empty_like(ins[0])

    def gather_view(self, y):  # the rank's output as rows of the shard axis
        return y

    def ungather(self, g):
        return g


class RowOp(Op):
    full_rows = cols = 0

    def localize(self):
        b, e = shard_bounds(self.full_rows, self.rank, self.world)
        self.r0, self.rows = b, e - b

    def rows_of_rank(self, r):
        b, e = shard_bounds(self.full_rows, r, self.world)
        return e - b

    def gen(self, shape, dist, seed):
        torch = self.torch
        g = self.g(seed)
        if dist == "uniform":
            return torch.rand(shape, device=self.device, generator=g) * 2 - 1
        return torch.randn(shape, device=self.device, generator=g) * dist

    def take(self, x):
        return x[self.r0:self.r0 + self.rows].contiguous()


class RMSNormOp(RowOp):
    name = "rmsnorm"
    full_rows, cols, eps = 4096, 1024, 1e-6
    config = "RMSNorm X f32 [4096,1024] ~N(0,1), gamma f32 [1024] ~N(1,0.1), eps 1e-6"

    def units_of_rows(self, rows):
        return 2 * rows * self.cols * 4 + self.cols * 4

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return K.rmsnorm(self.rows if local else self.full_rows, self.cols, self.eps)

    def global_inputs(self):
        return self.gen((self.full_rows, self.cols), 1.0, 0), self.gen((self.cols,), 0.1, 7) + 1.0

    def slice_inputs(self, full):
        return self.take(full[0]), full[1]

    def local_inputs(self, s):
        return self.gen((self.rows, self.cols), 1.0, 1000 * self.rank + s), self.gen((self.cols,), 0.1, 7 + s) + 1.0

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = self.full_rows
        x = np.random.default_rng(0).normal(size=(rows, self.cols)).astype(np.float32)
        w = np.random.default_rng(1).normal(1, 0.1, size=self.cols).astype(np.float32)
        return timed(lambda: rowops.rmsnorm(x, w, self.eps), seconds,
                     2 * rows * self.cols * 4 + self.cols * 4, 1e9, f"RMSNorm [{rows},{self.cols}]")

    def cpu_torch(self, torch, seconds):
        rows = self.full_rows
        g = torch.Generator().manual_seed(0)
        x = torch.randn(rows, self.cols, generator=g)
        w = torch.randn(self.cols, generator=g) * 0.1 + 1

        def run():
            return x * torch.rsqrt((x * x).mean(dim=1, keepdim=True) + self.eps) * w

        return timed(run, seconds, 2 * rows * self.cols * 4 + self.cols * 4, 1e9, f"RMSNorm [{rows},{self.cols}]")


class LayerNormOp(RowOp):
    name = "layernorm"
    full_rows, cols, eps = 4096, 1024, 1e-5
    config = "LayerNorm X f32 [4096,1024] ~N(0,1), gamma ~N(1,0.1), beta ~N(0,0.1), eps 1e-5"

    def units_of_rows(self, rows):
        return 2 * rows * self.cols * 4 + 2 * self.cols * 4

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return K.layernorm(self.rows if local else self.full_rows, self.cols, self.eps)

    def global_inputs(self):
        return (self.gen((self.full_rows, self.cols), 1.0, 0), self.gen((self.cols,), 0.1, 7) + 1.0,
                self.gen((self.cols,), 0.1, 17))

    def slice_inputs(self, full):
        return self.take(full[0]), full[1], full[2]

    def local_inputs(self, s):
        return (self.gen((self.rows, self.cols), 1.0, 1000 * self.rank + s), self.gen((self.cols,), 0.1, 7 + s) + 1.0,
                self.gen((self.cols,), 0.1, 17 + s))

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = self.full_rows
        x = np.random.default_rng(0).normal(size=(rows, self.cols)).astype(np.float32)
        w = np.random.default_rng(1).normal(1, 0.1, size=self.cols).astype(np.float32)
        b = np.random.default_rng(2).normal(0, 0.1, size=self.cols).astype(np.float32)
        return timed(lambda: rowops.layernorm(x, w, b, self.eps), seconds,
                     2 * rows * self.cols * 4 + 2 * self.cols * 4, 1e9, f"LayerNorm [{rows},{self.cols}]")

    def cpu_torch(self, torch, seconds):
        rows = self.full_rows
        g = torch.Generator().manual_seed(0)
        x = torch.randn(rows, self.cols, generator=g)
        w = torch.randn(self.cols, generator=g) * 0.1 + 1
        b = torch.randn(self.cols, generator=g) * 0.1
        return timed(lambda: torch.nn.functional.layer_norm(x, (self.cols,), w, b, self.eps), seconds,
                     2 * rows * self.cols * 4 + 2 * self.cols * 4, 1e9, f"LayerNorm [{rows},{self.cols}]")


class TransposeOp(RowOp):
    """A [m, n] -> B [n, m]; a rank transposes a block of A's rows into its own [n, m/N] block."""

    name = "transpose"
    full_rows, cols = 4096, 4096
    config = "shared transpose A f32 [4096,4096] ~N(0,1) -> B [4096,4096] (README config)"

    def units_of_rows(self, rows):
        return 2 * rows * self.cols * 4

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return K.transpose(self.rows if local else self.full_rows, self.cols)

    def global_inputs(self):
        return (self.gen((self.full_rows, self.cols), 1.0, 0),)

    def slice_inputs(self, full):
        return (self.take(full[0]),)

    def local_inputs(self, s):
        return (self.gen((self.rows, self.cols), 1.0, 1000 * self.rank + s),)

    def alloc_out(self, ins):
        return self.torch.empty((self.cols, ins[0].shape[0]), device=self.device)

    def gather_view(self, y):
        return y.t().contiguous()

    def ungather(self, g):
        return g.t()

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        m = self.full_rows
        a = np.random.default_rng(0).normal(size=(m, self.cols)).astype(np.float32)
        return timed(lambda: rowops.transpose(a), seconds, 2 * m * self.cols * 4, 1e9, f"transpose [{m},{self.cols}]")

    def cpu_torch(self, torch, seconds):
        m = self.full_rows
        a = torch.randn(m, self.cols, generator=torch.Generator().manual_seed(0))
        return timed(lambda: a.t().contiguous(), seconds, 2 * m * self.cols * 4, 1e9, f"transpose [{m},{self.cols}]")


class CumsumOp(RowOp):
    name = "cumsum"
    full_rows, cols = 32768, 256
    config = "row inclusive cumsum X f32 [32768,256] ~U(-1,1)"

    def units_of_rows(self, rows):
        return 2 * rows * self.cols * 4

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return K.cumsum(self.rows if local else self.full_rows, self.cols)

    def global_inputs(self):
        return (self.gen((self.full_rows, self.cols), "uniform", 0),)

    def slice_inputs(self, full):
        return (self.take(full[0]),)

    def local_inputs(self, s):
        return (self.gen((self.rows, self.cols), "uniform", 1000 * self.rank + s),)

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = self.full_rows
        x = np.random.default_rng(0).uniform(-1, 1, size=(rows, self.cols)).astype(np.float32)
        return timed(lambda: rowops.cumsum(x), seconds, 2 * rows * self.cols * 4, 1e9, f"cumsum [{rows},{self.cols}]")

    def cpu_torch(self, torch, seconds):
        rows = self.full_rows
        x = torch.rand(rows, self.cols, generator=torch.Generator().manual_seed(0)) * 2 - 1
        return timed(lambda: torch.cumsum(x, dim=1), seconds, 2 * rows * self.cols * 4, 1e9,
                     f"cumsum [{rows},{self.cols}]")


class SoftmaxOp(RowOp):
    name = "softmax"
    full_rows, cols = 16384, 512
    config = "row softmax X f32 [16384,512] ~N(0,4)"

    def units_of_rows(self, rows):
        return 2 * rows * self.cols * 4

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return K.softmax(self.rows if local else self.full_rows, self.cols)

    def global_inputs(self):
        return (self.gen((self.full_rows, self.cols), 2.0, 0),)

    def slice_inputs(self, full):
        return (self.take(full[0]),)

    def local_inputs(self, s):
        return (self.gen((self.rows, self.cols), 2.0, 1000 * self.rank + s),)

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = self.full_rows
        x = (np.random.default_rng(0).normal(size=(rows, self.cols)) * 2).astype(np.float32)
        return timed(lambda: rowops.softmax(x), seconds, 2 * rows * self.cols * 4, 1e9, f"softmax [{rows},{self.cols}]")

    def cpu_torch(self, torch, seconds):
        rows = self.full_rows
        x = torch.randn(rows, self.cols, generator=torch.Generator().manual_seed(0)) * 2
        return timed(lambda: torch.softmax(x, dim=1), seconds, 2 * rows * self.cols * 4, 1e9,
                     f"softmax [{rows},{self.cols}]")


class VaddOp(RowOp):
    name = "vadd"
    full_rows, cols = 16 * 1024 * 1024, 1
    config = "vector add A,B f32 [16777216] ~N(0,1)"

    def units_of_rows(self, rows):
        return 3 * rows * 4

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return K.vector_add(self.rows if local else self.full_rows)

    def global_inputs(self):
        return self.gen((self.full_rows,), 1.0, 0), self.gen((self.full_rows,), 1.0, 1)

    def slice_inputs(self, full):
        return self.take(full[0]), self.take(full[1])

    def local_inputs(self, s):
        return (self.gen((self.rows,), 1.0, 1000 * self.rank + 2 * s),
                self.gen((self.rows,), 1.0, 1000 * self.rank + 2 * s + 1))

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        m = self.full_rows
        a = np.random.default_rng(0).normal(size=m).astype(np.float32)
        b = np.random.default_rng(1).normal(size=m).astype(np.float32)
        return timed(lambda: rowops.vadd(a, b), seconds, 3 * m * 4, 1e9, f"vector add [{m}]")

    def cpu_torch(self, torch, seconds):
        m = self.full_rows
        g = torch.Generator().manual_seed(0)
        a, b = torch.randn(m, generator=g), torch.randn(m, generator=g)
        c = torch.empty(m)
        return timed(lambda: torch.add(a, b, out=c), seconds, 3 * m * 4, 1e9, f"vector add [{m}]")


def generic_fma_program(T, n, block=1024):
    """D = A * B + C as a TileLang program, built with whichever package's ``T`` is passed."""

    @T.prim_func
    def generic_fma(A: T.Tensor((n,), "float32"), B: T.Tensor((n,), "float32"), C: T.Tensor((n,), "float32"),
                    D: T.Tensor((n,), "float32")):
        with T.Kernel(T.ceildiv(n, block), threads=256) as b:
            for k in T.Parallel(block):
                D[b * block + k] = A[b * block + k] * B[b * block + k] + C[b * block + k]

    return generic_fma


class GenericFmaOp(RowOp):
    """A program outside the recognised families: CUDA C generated per program, NVRTC-compiled."""

    name = "pointwise"
    full_rows, cols = 16 * 1024 * 1024, 1
    config = "generic elementwise D = A*B + C (separately rounded), A,B,C f32 [16777216] ~N(0,1), NVRTC path"

    def units_of_rows(self, rows):
        return 4 * rows * 4

    def make_kernel(self, local):
        import ntilang_b200
        from ntilang_b200 import language as T

        kern = ntilang_b200.compile(generic_fma_program(T, self.rows if local else self.full_rows), out_idx=[-1])
        assert kern.spec.family == "pointwise"
        return kern

    def global_inputs(self):
        return tuple(self.gen((self.full_rows,), 1.0, j) for j in range(3))

    def slice_inputs(self, full):
        return tuple(self.take(t) for t in full)

    def local_inputs(self, s):
        return tuple(self.gen((self.rows,), 1.0, 1000 * self.rank + 3 * s + j) for j in range(3))

    def cpu(self, seconds):
        import numpy as np

        m = self.full_rows
        a, b, c = (np.random.default_rng(j).normal(size=m).astype(np.float32) for j in range(3))
        return timed(lambda: np.add(np.multiply(a, b), c), seconds, 4 * m * 4, 1e9,
                     f"numpy a*b+c [{m}] (float32, separately rounded)")

    def cpu_torch(self, torch, seconds):
        m = self.full_rows
        g = torch.Generator().manual_seed(0)
        a, b, c = (torch.randn(m, generator=g) for _ in range(3))
        return timed(lambda: a * b + c, seconds, 4 * m * 4, 1e9, f"a*b+c [{m}]")


class GemmOp(RowOp):
    """C = A @ B; a rank computes an M-panel of C from its rows of A and the whole of B."""

    name = "gemm"
    bound = "tensor"
    unit = "TFLOP/s"
    dtype = "f16xf16->f32"
    m = n = k = 4096
    epilogue = False
    config = "FP16 GEMM 4096x4096x4096, A,B ~N(0,1)/sqrt(K), C f32"

    def localize(self):
        self.full_rows = self.m
        super().localize()

    def units_of_rows(self, rows):
        return 2 * rows * self.n * self.k

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        return (K.matmul_bias_relu if self.epilogue else K.matmul)(self.rows if local else self.m, self.n, self.k)

    def _ab(self, rows, seed):
        torch = self.torch
        g = self.g(seed)
        a = (torch.randn(rows, self.k, device=self.device, generator=g) / math.sqrt(self.k)).half()
        b = (torch.randn(self.k, self.n, device=self.device, generator=g) / math.sqrt(self.k)).half()
        if not self.epilogue:
            return a, b
        return a, b, torch.randn(self.n, device=self.device, generator=g) * 0.1

    def global_inputs(self):
        return self._ab(self.m, 0)

    def slice_inputs(self, full):
        return (self.take(full[0]),) + tuple(full[1:])

    def local_inputs(self, s):
        return self._ab(self.rows, 1000 * self.rank + s)

    def out_bytes(self, ins):
        return ins[0].shape[0] * self.n * 4

    def alloc_out(self, ins):
        return self.torch.empty(ins[0].shape[0], self.n, device=self.device)

    def cpu(self, seconds):
        import numpy as np

        from oracle import ntl_oracle as O

        rows = self.full_rows
        rng = np.random.default_rng(0)
        a = (rng.normal(size=(rows, self.k)) / 64).astype(np.float16)
        b = (rng.normal(size=(self.k, self.n)) / 64).astype(np.float16)
        bias = rng.normal(0, 0.1, self.n).astype(np.float32)
        if self.epilogue:
            fn = lambda: O.gemm(a, b, bias, O.BIAS_N, relu=True, accumulate=np.float32)  # noqa: E731
        else:
            fn = lambda: O.gemm(a, b, accumulate=np.float32)  # noqa: E731
        return timed(fn, seconds, 2 * rows * self.n * self.k, 1e12, f"fp32 matmul [{rows},{self.k}]x[{self.k},{self.n}]")

    def cpu_torch(self, torch, seconds):
        rows = self.full_rows
        g = torch.Generator().manual_seed(0)
        a = (torch.randn(rows, self.k, generator=g) / 64).half()
        b = (torch.randn(self.k, self.n, generator=g) / 64).half()
        bias = torch.randn(self.n, generator=g) * 0.1
        if self.epilogue:
            fn = lambda: torch.relu(a.float() @ b.float() + bias)  # noqa: E731
        else:
            fn = lambda: a.float() @ b.float()  # noqa: E731
        return timed(fn, seconds, 2 * rows * self.n * self.k, 1e12, f"fp32 matmul [{rows},{self.k}]x[{self.k},{self.n}]")


class GemmBiasReluOp(GemmOp):
    name = "gemm_bias_relu"
    epilogue = True
    config = "FP16 GEMM 4096^3 + fused C=relu(A@B+bias[N]), bias ~N(0,0.1)"


class FA2Op(RowOp):
    """Attention over [B, H, S, D]; a rank takes a contiguous block of the batch (N | B), else of
    the flattened (batch, head) pairs."""

    name = "fa2"
    bound = "tensor"
    unit = "TFLOP/s"
    dtype = "f16xf16->f32"
    B, H, S, D = 8, 32, 4096, 128
    causal = False
    config = "FlashAttention-2 fwd Q,K,V f16 [8,32,4096,128] ~N(0,1), scale 1/sqrt(128), non-causal"

    def localize(self):
        self.by_batch = self.B % max(1, self.world) == 0
        self.full_rows = self.B if self.by_batch else self.B * self.H
        super().localize()

    def local_shape(self, rows=None):
        rows = self.rows if rows is None else rows
        return (rows, self.H, self.S, self.D) if self.by_batch else (rows, 1, self.S, self.D)

    def units_of_rows(self, rows):
        f = 4 * rows * (self.H if self.by_batch else 1) * self.S * self.S * self.D
        return f // 2 if self.causal else f

    def make_kernel(self, local):
        from ntilang_b200 import kernels as K

        if not local:
            return K.flash_attention(self.B, self.H, self.S, self.D, self.causal)
        b, h = self.local_shape()[:2]
        return K.flash_attention(b, h, self.S, self.D, self.causal)

    def _qkv(self, shape, seed):
        g = self.g(seed)
        return tuple(self.torch.randn(shape, device=self.device, generator=g).half() for _ in range(3))

    def global_inputs(self):
        return self._qkv((self.B, self.H, self.S, self.D), 0)

    def slice_inputs(self, full):
        if self.by_batch:
            return tuple(self.take(t) for t in full)
        return tuple(self.take(t.reshape(self.B * self.H, 1, self.S, self.D)) for t in full)

    def local_inputs(self, s):
        return self._qkv(self.local_shape(), 1000 * self.rank + s)

    def out_bytes(self, ins):
        return ins[0].numel() * 2

    def ungather(self, g):
        return g.reshape(self.B, self.H, self.S, self.D)

    def cpu(self, seconds):
        import numpy as np

        from oracle import ntl_oracle as O

        rng = np.random.default_rng(0)
        rows = 256
        q = rng.normal(size=(1, 1, rows, self.D)).astype(np.float16)
        k, v = (rng.normal(size=(1, 1, self.S, self.D)).astype(np.float16) for _ in range(2))
        c = math.log2(math.e) / math.sqrt(self.D)
        # causal: the last `rows` queries of a head attend to (almost) all keys, the same work
        return timed(lambda: O.fa2_blockwise(q, k, v, c, False), seconds, 4 * rows * self.S * self.D, 1e12,
                     f"attention [1,1,{rows} queries,{self.S} keys,{self.D}]")

    def cpu_torch(self, torch, seconds):
        rows = 256
        g = torch.Generator().manual_seed(0)
        q = torch.randn(1, 1, rows, self.D, generator=g).half().float()
        k, v = (torch.randn(1, 1, self.S, self.D, generator=g).half().float() for _ in range(2))
        fn = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v)  # noqa: E731
        return timed(fn, seconds, 4 * rows * self.S * self.D, 1e12,
                     f"fp32 SDPA [1,1,{rows} queries,{self.S} keys,{self.D}]")


class FA2CausalOp(FA2Op):
    name = "fa2_causal"
    causal = True
    config = "FlashAttention-2 fwd Q,K,V f16 [8,32,4096,128] ~N(0,1), scale 1/sqrt(128), causal"


OPS = {c.name: c for c in (CumsumOp, RMSNormOp, SoftmaxOp, VaddOp, GemmOp, GemmBiasReluOp, FA2Op, FA2CausalOp,
                           LayerNormOp, TransposeOp, GenericFmaOp)}


def timed(fn, seconds, units_per_call, per_unit, what):
    """Repeat ``fn`` for about ``seconds``; (throughput, sample description)."""
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return n * units_per_call / dt / per_unit, f"{n} x {what}"


# ------------------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi samples (every 20 ms) of the SM clock, power and throttle reasons during the
    run: ``stop()`` summarises the whole run, ``window(t0, t1)`` the samples inside one op's
    timed region (host wall-clock bounds)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.rows = []  # (unix time, sm MHz, max MHz, power W, active reasons)

    def start(self):
        import tempfile

        self.path = tempfile.NamedTemporaryFile(prefix="ntl_clocks_", suffix=".csv", delete=False).name
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", str(self.gpu)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    @staticmethod
    def _num(x):
        try:
            return float(x)
        except ValueError:
            return None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        import datetime

        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                continue
            active = tuple(n for n, v in zip(self.REASONS, parts[6:10]) if v.lower() == "active")
            self.rows.append((ts, self._num(parts[2]), self._num(parts[3]), self._num(parts[4]), active))
        os.unlink(self.path)
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [r[1] for r in self.rows if r[1] is not None]
        mx = [r[2] for r in self.rows if r[2] is not None]
        power = [r[3] for r in self.rows if r[3] is not None]
        reasons = sorted({n for r in self.rows for n in r[4]})
        loaded = sorted(r[1] for r in self.rows if r[1] is not None and r[3] is not None and r[3] > 300) or sorted(sm)
        return {"sm_mhz": loaded[len(loaded) // 2] if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "power_w_max": max(power) if power else None}

    def window(self, t0, t1):
        """Median SM clock and power of the samples taken in [t0, t1]."""
        sel = [r for r in self.rows if t0 <= r[0] <= t1 and r[1] is not None]
        if not sel:
            return {"samples": 0}
        sm = sorted(r[1] for r in sel)
        pw = sorted(r[3] for r in sel if r[3] is not None)
        return {"sm_mhz": sm[len(sm) // 2], "power_w": pw[len(pw) // 2] if pw else None, "samples": len(sel),
                "reasons": sorted({n for r in sel for n in r[4]})}


# ----------------------------------------------------------------------------- measure


class Timer:
    """Device time of work on ``stream`` between a barrier and a synchronize, max over ranks."""

    def __init__(self, torch, dist, device):
        self.torch, self.dist, self.device = torch, dist, device

    def max_over_ranks(self, ms):
        if self.dist is None:
            return ms
        t = self.torch.tensor([ms], device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def flush_l2(torch, device, scratch={}):  # noqa: B006 - one scratch buffer per device and process
    """Evict L2 before a timed region by reading a buffer of twice its size.  Reading (not
    writing) leaves the cache holding clean lines, so the timed launches pay no write-back of
    the flush itself."""
    buf = scratch.get(device)
    if buf is None:
        buf = scratch[device] = torch.ones(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
    return buf.amax()


def time_graph(op, torch, dist, steps, stream, timer):
    """K launches (rotating input sets) captured into one CUDA graph; one untimed replay, then
    an L2 flush and the timed replay between CUDA events.  Returns (ms per step, launches)."""
    from ntilang_b200 import _lib

    kern = op.kernel
    nsets = len(op.sets)
    before = _lib.launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            kern(*op.sets[i % nsets][0])
    launches = _lib.launch_count() - before
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay() launches on the current stream
        graph.replay()  # untimed replay
        stream.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        # The L2-evicting read (~40 us of GPU work) is queued ahead of the start event, so the
        # GPU is still busy with it while the host submits the graph: the host's submission
        # latency stays outside the timed region.
        flush_l2(torch, op.device)
        t0 = time.time()
        start.record(stream)
        graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    op.timed_window = (t0, time.time())
    if dist is not None:
        dist.barrier()
    ms = timer.max_over_ranks(start.elapsed_time(end))
    del graph
    return ms / steps, launches


def warm(op, torch, stream, warmup):
    kern = op.kernel
    with torch.cuda.stream(stream):
        for i in range(max(3, warmup)):
            kern(*op.sets[i % len(op.sets)][0])
    stream.synchronize()


def run_op(op, torch, dist, steps, warmup, stream, peaks, peak_kind, traffic, timer, want_e2e, want_call_path=True):
    op.setup()
    warm(op, torch, stream, warmup)
    ms_step, launches = time_graph(op, torch, dist, steps, stream, timer)
    units = op.units()
    total = op.total_units()
    value = total / (ms_step / 1e3) / op.per_unit()
    per_launch = units / (ms_step / 1e3) / op.per_unit()
    if op.bound == "hbm":
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        punit = "GB/s"
    else:
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        punit = "TFLOP/s"
    tr = traffic.get(op.name)
    tr_bytes = None
    if isinstance(tr, dict) and tr.get("bytes_per_launch") is not None:
        # the captured launch covers the full single-GPU job; a shard moves its share of it
        tr_bytes = int(round(tr["bytes_per_launch"] * units / op.whole_job_units()))
    result = {
        "window": op.timed_window,
        "metric": f"{op.name} achieved {op.unit}", "value": round(value, 3), "unit": op.unit,
        "ms_per_step": round(ms_step, 6), "steps": steps, "buffer_sets": len(op.sets), "gpu_launches": launches,
        "config": op.config, "dtype": op.dtype, "shard": shard_desc(op),
        "roofline": {"bound": op.bound, "achieved": round(per_launch, 3), "peak": peak, "unit": punit,
                     "frac": round(per_launch / peak, 4),
                     "peak_source": "measured, burst" if peak_kind == "measured" else "fallback",
                     "traffic": tr_bytes, "algorithmic_per_launch": units},
    }
    if want_call_path:
        result["python_call"] = measure_call_path(op, torch, stream)
    if want_e2e:
        result["e2e"] = measure_e2e(op, torch, dist, steps, stream, timer)
    return result


def whole_job_op(cls, torch, device):
    """The weak-scaling leg's op on any rank: the whole BASELINE job, as the only rank of one."""
    return cls(torch, device, 0, 1)


def shard_desc(op):
    if op.world == 1:
        return "whole job"
    return f"rank {op.rank}: {op.rows} of {op.full_rows} {'rows' if op.bound == 'hbm' else 'panel rows'}"


def verify_shards(op, torch, dist, stream):
    """All-gather the shards' outputs for input set 0 (one seeded global input) and compare
    them on rank 0, bit for bit, with the same kernels run on the whole job on one GPU."""
    from ntilang_b200.dist import gather_rows

    with torch.cuda.stream(stream):
        y = op.kernel(*op.sets[0][1])
    stream.synchronize()
    gathered = gather_rows(op.gather_view(y), op.world)
    if op.rank != 0:
        return None
    whole = op.ungather(gathered)
    full_in = op.global_inputs()
    kern = op.make_kernel(local=False)
    with torch.cuda.stream(stream):
        ref = kern(*full_in)
    stream.synchronize()
    same = bool(torch.equal(whole, ref))
    return {"bit_identical": same, "max_abs_diff": 0.0 if same else float((whole.float() - ref.float()).abs().max())}


def measure_call_path(op, torch, stream, calls=200):
    """The drop-in call path: CompiledKernel.__call__ (argument checks, ctypes, launch) on
    device-resident tensors, timed on the host over back-to-back calls.  When the host cost
    per call exceeds the kernel time the GPU waits on Python, and us_per_call is the host cost."""
    kern = op.kernel
    nsets = len(op.sets)
    n = calls if op.bound == "hbm" else max(5, min(calls, 20))
    with torch.cuda.stream(stream):
        for i in range(3):
            kern(*op.sets[i % nsets][0])
        stream.synchronize()
        t0 = time.perf_counter()
        for i in range(n):
            kern(*op.sets[i % nsets][0])
        t_issue = time.perf_counter() - t0
        stream.synchronize()
        t_all = time.perf_counter() - t0
    return {"us_per_call": round(1e6 * t_all / n, 2), "host_us_per_call": round(1e6 * t_issue / n, 2), "calls": n}


def measure_e2e(op, torch, dist, steps, stream, timer):
    """Public-call path with host buffers.  Every step copies its inputs host->device from pinned
    memory, makes the public call (``CompiledKernel.__call__``) and copies its output
    device->host.  Steps alternate between two streams, each with its own device and host
    buffers, so a step's host->device copy can overlap the previous step's device->host copy on
    the full-duplex PCIe link; the timed region spans every step on both streams."""
    kern = op.kernel
    _, ins, out = op.sets[0]
    host_in = [t.cpu().pin_memory() for t in ins]
    lanes = [stream, torch.cuda.Stream(device=op.device)]
    dev_in = [[torch.empty_like(t) for t in ins] for _ in lanes]
    host_out = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in lanes]
    bi = sum(t.numel() * t.element_size() for t in host_in)
    bo = host_out[0].numel() * host_out[0].element_size()
    n = max(4, min(steps, 20))

    def one(k):
        lane = k % 2
        with torch.cuda.stream(lanes[lane]):
            for h, d in zip(host_in, dev_in[lane]):
                d.copy_(h, non_blocking=True)
            y = kern(*dev_in[lane])
            host_out[lane].copy_(y, non_blocking=True)

    one(0)
    one(1)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    lanes[1].wait_event(start)
    for k in range(n):
        one(k)
    stream.wait_stream(lanes[1])
    end.record(stream)
    torch.cuda.synchronize()
    ms_step = timer.max_over_ranks(start.elapsed_time(end)) / n
    value = op.total_units() / (ms_step / 1e3) / op.per_unit()
    return {"value": round(value, 3), "unit": op.unit, "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "ms_per_step": round(ms_step, 4), "steps": n, "streams": 2}


def cpu_baselines(op, seconds):
    """The oracle port (``kind: port``) and torch on all host cores, each a bounded sample."""
    try:
        import oracle.rowops as rowops

        threads = rowops.threads()
    except Exception:  # noqa: BLE001 - report what ran
        threads = os.cpu_count() or 1
    value, sample = op.cpu(seconds)
    cores = threads if op.bound == "hbm" else (os.cpu_count() or 1)
    port = {"value": round(value, 4), "unit": op.unit, "cores": cores, "kind": "port", "sample": sample}
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    tval, tsample = op.cpu_torch(torch, seconds)
    return port, {"value": round(tval, 4), "unit": op.unit, "cores": torch.get_num_threads(), "sample": tsample,
                  "torch": torch.__version__}


# ------------------------------------------------------------------------------ the reference's kernels on the GPU

REF_INSTALL = Path(os.environ.get("NTL_REFERENCE_DIR", str(ROOT / "baseline" / "_ref")))


def reference_builders(target):
    """The reference's own kernels for each op at the bench shapes.

    Each is built by the reference's unmodified examples/*.py through its own ``compile``
    (CuTe DSL code generation, then cute.compile for ``target``) and launched through its own
    ``CompiledKernel.__call__`` (TVM-FFI on torch's current stream).  The GEMMs use the tiles
    of the reference's README benchmark (README.md:38-58: 128x128x32, 3 stages, swizzle panel
    8); everything else uses the examples' defaults.  name -> (make(op) -> kernel,
    args(our argument tuple, op) -> the reference's argument tuple, expected(args) -> the
    output to compare against or None to compare with our kernel's output)."""
    import importlib

    import ntilang as R
    import ntilang.language as RT

    def ex(module, fn=None):
        return getattr(importlib.import_module(f"examples.{module}"), fn or module)

    same = lambda a, op: a  # noqa: E731

    def relu_args(a, op):
        x, w, bias, c = a
        return x, w, bias.expand(op.m, op.n).contiguous(), c

    gemm_tiles = dict(block_m=128, block_n=128, block_k=32, num_stages=3, swizzle_panel=8, target=target)
    return {
        "cumsum": (lambda op: ex("cumsum")(op.full_rows, op.cols, target=target), same, None),
        "rmsnorm": (lambda op: ex("rmsnorm")(op.full_rows, op.cols, eps=op.eps, target=target), same, None),
        "layernorm": (lambda op: ex("layernorm")(op.full_rows, op.cols, eps=op.eps, target=target), same, None),
        "softmax": (lambda op: ex("softmax")(op.full_rows, op.cols, target=target), same, None),
        "vadd": (lambda op: ex("vector_add")(op.full_rows, target=target), same, None),
        "transpose": (lambda op: ex("transpose")(op.full_rows, op.cols, target=target), same, None),
        "gemm": (lambda op: ex("matmul")(op.m, op.n, op.k, **gemm_tiles), same, None),
        # The example's epilogue is relu(0.5 * acc + Bias[M, N]) (examples/matmul_relu.py:35-38):
        # bias[N] is broadcast to a full [M, N] operand and the result checked against torch.
        "gemm_bias_relu": (lambda op: ex("matmul_relu")(op.m, op.n, op.k, **gemm_tiles), relu_args,
                           lambda a: (0.5 * (a[0].float() @ a[1].float()) + a[2]).relu()),
        "fa2": (lambda op: ex("flash_attention")(op.B, op.H, op.S, op.D, is_causal=False, target=target), same,
                None),
        "fa2_causal": (lambda op: ex("flash_attention")(op.B, op.H, op.S, op.D, is_causal=True, target=target),
                       same, None),
        "pointwise": (lambda op: R.compile(generic_fma_program(RT, op.full_rows), target=target), same, None),
    }


# max |ref - expected| allowed per op (atol + rtol * |expected|): bit-exact where both follow one
# operation order.  For the generic D = A*B + C the reference's compiled kernel may contract the
# multiply-add into one FMA (its evaluator and ours round twice): up to a few fp32 ulps apart.
REF_TOLERANCE = {"cumsum": (0.0, 0.0), "vadd": (0.0, 0.0), "transpose": (0.0, 0.0), "pointwise": (4.8e-7, 1e-6),
                 "rmsnorm": (1e-5, 1e-6), "layernorm": (1e-5, 1e-6), "softmax": (1e-5, 1e-7),
                 "gemm": (1e-3, 1e-5), "gemm_bias_relu": (1e-3, 1e-5), "fa2": (0.0, 2e-3), "fa2_causal": (0.0, 2e-3)}


def run_reference_gpu(args, ops):
    """The reference's own GPU kernels (CuTe DSL, sm_80-style mma.sync / cp.async code compiled
    for sm_100a) timed on this GPU beside ours: same shapes, inputs and buffer rotation.

    The reference launches through TVM-FFI and takes no stream argument, so everything here
    runs on torch's default stream and every check synchronises the whole device.  Timing:
    K eager launches through ``CompiledKernel.__call__`` between CUDA events, queued behind a
    short ``torch.cuda._sleep`` so the host's call overhead does not show in the kernel time
    (its host cost per call is reported separately).  Needs the reference package and its
    examples under baseline/_ref."""
    if not (REF_INSTALL / "ntilang" / "__init__.py").exists() or not (REF_INSTALL / "examples").is_dir():
        print(json.dumps({"impl": "reference-gpu", "unavailable": f"no reference package under {REF_INSTALL}"}))
        return 0
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sys.path.insert(0, str(REF_INSTALL))
    os.environ.setdefault("NTILANG_CACHE_DIR", str(Path("/tmp") / "ntilang_ref_cache"))
    import ntilang
    import torch

    if not Path(ntilang.__file__).resolve().is_relative_to(REF_INSTALL.resolve()):
        raise SystemExit(f"ntilang resolved to {ntilang.__file__}, not the reference under {REF_INSTALL}")
    torch.cuda.set_device(0)
    device = torch.device("cuda:0")
    major, minor = torch.cuda.get_device_capability(device)
    target = f"sm_{major}{minor}a" if major >= 9 else f"sm_{major}{minor}"
    builders = reference_builders(target)
    peaks, peak_kind = load_peaks()
    stream = torch.cuda.current_stream(device)
    sampler = ClockSampler(0)
    sampler.start()
    results = {}
    steps = max(1, args.steps)
    for name in ops:
        op = OPS[name](torch, device, 0)
        make, to_ref, expected = builders[name]
        t0 = time.perf_counter()
        try:
            kern = make(op)
            kern.build()
        except Exception as exc:  # noqa: BLE001 - a kernel the reference cannot build is reported
            results[name] = {"unavailable": f"reference build failed: {type(exc).__name__}: {str(exc)[:160]}"}
            continue
        build_s = time.perf_counter() - t0
        op.setup()
        sets = [to_ref(s[0], op) for s in op.sets]
        kern(*sets[0])
        torch.cuda.synchronize()
        want = op.kernel(*op.sets[0][1]) if expected is None else expected(sets[0])
        torch.cuda.synchronize()
        got = sets[0][-1]
        diff = (got.float() - want.float()).abs()
        rtol, atol = REF_TOLERANCE[name]
        bound = atol + rtol * want.float().abs()
        check = {"max_abs_diff": float(diff.max().item()), "within": bool((diff <= bound).all().item()),
                 "mismatches": int((diff > bound).sum().item()), "against": "ours" if expected is None else "torch",
                 "rtol": rtol, "atol": atol}
        del want, diff, bound
        for i in range(max(3, args.warmup)):
            kern(*sets[i % len(sets)])
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        for i in range(steps):
            kern(*sets[i % len(sets)])
        host_us = 1e6 * (time.perf_counter() - t1) / steps
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        # a head start of ~2x the host time of K calls (at <= 2 GHz), so the launches queue up
        torch.cuda._sleep(int(min(2e8, 2 * host_us * steps * 2000)))
        start.record(stream)
        for i in range(steps):
            kern(*sets[i % len(sets)])
        end.record(stream)
        torch.cuda.synchronize()
        ms_step = start.elapsed_time(end) / steps
        units = op.units()
        value = units / (ms_step / 1e3) / op.per_unit()
        key = "hbm_gbs" if op.bound == "hbm" else "bf16_tflops"
        peak = float(peaks.get(key, FALLBACK_PEAKS[key]))
        results[name] = {"value": round(value, 3), "unit": op.unit, "ms_per_step": round(ms_step, 6),
                         "frac_of_peak": round(value / peak, 4), "peak": peak, "peak_source": peak_kind,
                         "config": op.config, "build_seconds": round(build_s, 2), "check": check,
                         "host_us_per_call": round(host_us, 2), "buffer_sets": len(sets),
                         "timing": "K eager launches through CompiledKernel.__call__ on the default stream, "
                                   "queued behind torch.cuda._sleep, CUDA events"}
        op.sets = sets = None
        torch.cuda.empty_cache()
    clocks = sampler.stop()
    print(json.dumps({"impl": "reference-gpu", "target": target, "n_gpus": 1, "steps": steps,
                      "warmup": args.warmup, "clocks": clocks, "ops": results}), flush=True)
    return 0


# ------------------------------------------------------------------------------ driver


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference", "reference-gpu"), default="ours")
    ap.add_argument("--ops", default=",".join(OPS))
    ap.add_argument("--cpu-seconds", type=float, default=1.5, help="CPU-baseline sample per op and path (0 = skip)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-call-path", action="store_true",
                    help="skip the Python call-path timing (200 extra launches per op; for launch lists)")
    ap.add_argument("--no-weak", action="store_true", help="N > 1: skip the full-job-per-rank (weak) timing")
    ap.add_argument("--detail", default=os.environ.get("NTL_BENCH_DETAIL", DETAIL_DEFAULT),
                    help="side file for the full per-op records ({n} = number of GPUs; '' = none)")
    ap.add_argument("--gemm-shape", default=None, help="M,N,K override (profiling a small case)")
    ap.add_argument("--fa2-shape", default=None, help="B,H,S,D override (profiling a small case)")
    args = ap.parse_args()
    if args.gemm_shape:
        m, n, k = (int(x) for x in args.gemm_shape.split(","))
        for cls in (GemmOp, GemmBiasReluOp):
            cls.m, cls.n, cls.k = m, n, k
            cls.config = cls.config + f" [override M,N,K={m},{n},{k}]"
    if args.fa2_shape:
        b, h, s_, d = (int(x) for x in args.fa2_shape.split(","))
        for cls in (FA2Op, FA2CausalOp):
            cls.B, cls.H, cls.S, cls.D = b, h, s_, d
            cls.config = cls.config + f" [override B,H,S,D={b},{h},{s_},{d}]"

    ops = [o for o in args.ops.split(",") if o]
    for o in ops:
        if o not in OPS:
            raise SystemExit(f"unknown op {o}; choose from {', '.join(OPS)}")
    if HEADLINE not in ops:
        ops.insert(0, HEADLINE)
    if args.impl == "reference":
        return run_reference(args, ops)
    if args.impl == "reference-gpu":
        return run_reference_gpu(args, ops)
    return run_ours(args, ops)


def write_detail(path_tpl, n, record):
    if not path_tpl:
        return None
    path = Path(path_tpl.format(n=n))
    if not path.is_absolute():
        path = ROOT / path
    try:
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(record, indent=1))
    except OSError:
        return None
    return str(path.relative_to(ROOT)) if path.is_relative_to(ROOT) else str(path)


def run_reference(args, ops):
    """The reference's CPU path (the oracle port of its algorithm) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch

    per, detail = {}, {}
    head = None
    steps = max(1, args.steps)
    for name in ops:
        op = OPS[name](None, None, 0)
        vals = []
        for _ in range(max(0, min(args.warmup, 1))):
            op.cpu(0.05)
        seconds = max(0.05, min(args.cpu_seconds, 30.0 / (len(ops) * steps)))
        sample = ""
        for _ in range(steps if name == HEADLINE else 1):
            v, sample = op.cpu(seconds)
            vals.append(v)
        vals.sort()
        v = vals[len(vals) // 2]
        cb = {"value": round(v, 4), "unit": op.unit, "cores": os.cpu_count() or 1, "kind": "port", "sample": sample,
              "cpu": cpu_model()}
        per[name] = round(v, 4)
        detail[name] = {"value": round(v, 4), "unit": op.unit, "config": op.config, "cpu_baseline": cb}
        if name == HEADLINE:
            head = (op, v, cb)
    op, v, cb = head
    # one step = one whole BASELINE workload, at the rate the bounded sample measured
    ms = round(op.total_units() / (v * op.per_unit()) * 1e3, 6) if v > 0 else None
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": round(v, 4), "unit": op.unit, "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE.json distributions)",
        "config": {"workload": op.config, "op": op.name,
                   "path": "CPU oracle port of the reference algorithm; ms_per_step = one whole workload at the "
                           "sampled rate", "torch": torch.__version__},
        "cpu_baseline": cb, "e2e": {"value": round(v, 4), "unit": op.unit, "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0},
        "ops": per,
    }
    where = write_detail(args.detail.replace("bench_detail", "bench_reference_detail") if args.detail else "",
                         args.gpus, detail)
    if where:
        line["detail"] = where
    print(json.dumps(line), flush=True)
    return 0


def compact(r):
    """The per-op figures the one-line record carries."""
    if "unavailable" in r:
        return {"unavailable": r["unavailable"][:80]}
    out = {"value": r["value"], "frac": r["roofline"]["frac"], "ms_per_step": r["ms_per_step"]}
    if r.get("e2e"):
        out["e2e"] = r["e2e"]["value"]
    if r.get("cpu_baseline"):
        out["cpu"] = r["cpu_baseline"]["value"]
    if r.get("cpu_torch"):
        out["cpu_torch"] = r["cpu_torch"]["value"]
    if r.get("weak"):
        out["weak"] = r["weak"]["value"]
    if r.get("verify"):
        out["verified"] = r["verify"]["bit_identical"]
    return out


def run_ours(args, ops):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device(f"cuda:{local}"))
        dist = tdist
    else:
        torch.cuda.set_device(0)
    device = torch.device(f"cuda:{torch.cuda.current_device()}")
    from ntilang_b200 import _lib

    _lib.lib()
    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    stream = torch.cuda.Stream(device=device)
    timer = Timer(torch, dist, device)
    flush_l2(torch, device)  # allocate (and write) the eviction buffer before any timing
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    results = {}
    for name in ops:
        op = OPS[name](torch, device, rank, world)
        try:
            r = run_op(op, torch, dist, args.steps, args.warmup, stream, peaks, peak_kind, traffic, timer,
                       want_e2e=not args.no_e2e, want_call_path=not args.no_call_path)
            if world > 1:
                r["verify"] = verify_shards(op, torch, dist, stream)
            op.sets = None
            if world > 1 and not args.no_weak:
                full = whole_job_op(OPS[name], torch, device)
                full.setup()
                warm(full, torch, stream, args.warmup)
                ms_w, launches_w = time_graph(full, torch, dist, args.steps, stream, timer)
                r["weak"] = {"value": round(world * full.total_units() / (ms_w / 1e3) / full.per_unit(), 3),
                             "ms_per_step": round(ms_w, 6), "gpu_launches": launches_w,
                             "what": "the whole job on every rank"}
                full.sets = None
            results[name] = r
        except _lib.KernelError as exc:
            if exc.code != 2:
                raise
            results[name] = {"unavailable": str(exc)}
            op.sets = None
        torch.cuda.empty_cache()
    clocks = sampler.stop()
    for name, r in results.items():
        if "window" in r:
            r["clocks"] = sampler.window(*r.pop("window"))
            if r["roofline"]["bound"] == "tensor":
                # the tensor kernels run at the power cap inside their timed region: beside the burst
                # fraction, the fraction of the sustained (seconds-long, power-capped) GEMM rate
                sus = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
                r["roofline"]["peak_sustained"] = sus
                r["roofline"]["frac_sustained"] = round(r["roofline"]["achieved"] / sus, 4)
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        for name in ops:
            if "unavailable" not in results[name]:
                port, tcpu = cpu_baselines(OPS[name](None, None, 0), args.cpu_seconds)
                results[name]["cpu_baseline"], results[name]["cpu_torch"] = port, tcpu
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    where = write_detail(args.detail, world, {"n_gpus": world, "peaks": peak_kind, "cpu": cpu_model(),
                                              "clocks": clocks, "ops": results})
    print(json.dumps(assemble_line(args.steps, args.warmup, world, results, clocks, where)), flush=True)
    return 0


def assemble_line(steps, warmup, world, results, clocks, detail_path):
    """The one JSON record rank 0 prints: the headline op's figures at the top level, every op's
    compact figures under ``ops``.  It must fit the last ~3,000 characters of stdout that the
    driver keeps (``tests/test_bench_shards.py`` checks the worst case)."""
    head = results[HEADLINE]
    total_launches = sum(r.get("gpu_launches", 0) + r.get("weak", {}).get("gpu_launches", 0)
                         for r in results.values())
    cb = head.get("cpu_baseline")
    if cb is not None:
        cb = dict(cb, cpu=cpu_model(), torch_value=head["cpu_torch"]["value"],
                  torch_cores=head["cpu_torch"]["cores"])
    roof = {k: head["roofline"][k] for k in ("bound", "achieved", "peak", "unit", "frac", "traffic")}
    e2e = head.get("e2e")
    if e2e is not None:
        e2e = {k: e2e[k] for k in ("value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step")}
    line = {
        "metric": BASELINE_METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic, seeded, BASELINE shapes",
        "config": {"workload": OPS[HEADLINE].config + " (configs[1])", "op": HEADLINE,
                   "parallelism": f"rows split over {world} GPUs, no collective" if world > 1 else "single GPU",
                   "l2": "buffer sets > 3x L2 between reuses; L2 flushed before timing",
                   "timing": "CUDA graph of K launches, CUDA events, max over ranks"},
        "roofline": roof, "e2e": e2e, "gpu_launches": total_launches, "clocks": clocks, "cpu_baseline": cb,
    }
    if world > 1:
        line["weak"] = {k: head["weak"][k] for k in ("value", "ms_per_step")} if head.get("weak") else None
        checked = [r["verify"]["bit_identical"] for r in results.values() if r.get("verify")]
        line["verify"] = {"gathered_ops": len(checked), "bit_identical": sum(checked),
                          "against": "whole job on one GPU"}
    line["op_units"] = "GB/s; TFLOP/s for gemm*, fa2*"
    line["ops"] = {name: compact(r) for name, r in results.items()}
    if detail_path:
        line["detail"] = detail_path
    return line


if __name__ == "__main__":
    sys.exit(main())
