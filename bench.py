#!/usr/bin/env python
"""Throughput of the hot-path kernels on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-gpu] [--ops a,b,...]

A *step* is one launch of an op over one batch of synthetic input with BASELINE.json's
shapes and distributions.  The headline line is the configuration BASELINE.json's metric
is normally quoted on (configs[1]: row cumsum, X f32 [32768, 256]); every op family's
measurement is in the same line under ``"ops"``.

value      K steps replayed from one CUDA graph (inputs resident in HBM, rotated over
           enough buffer sets that the working set exceeds L2 between reuses), timed with
           CUDA events on the launching stream between barriers; max over ranks.
e2e        the same metric through the public call (``CompiledKernel.__call__`` -> C ABI)
           with pinned host buffers: every step copies its inputs host->device and its
           output device->host inside the timed region (steps alternate between two
           streams, so uploads and downloads of neighbouring steps overlap).
roofline   algorithmic bytes (or FLOPs) per launch / average launch time, against the
           measured HBM copy bandwidth or dense bf16 GEMM rate in MEASURED_PEAKS.json.
cpu_baseline  the CPU oracle (a restatement of the reference's algorithm; ``kind: port``)
           on the host cores, bounded sample, rank 0 at N=1 only.
Multi-GPU: each rank runs a full config-sized shard of an N-times larger job (row blocks,
M-panels or (batch, head) slices; no collective on the data path): ``scaling: weak``.
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


# ---------------------------------------------------------------------------- workloads


class Op:
    name = ""
    bound = "hbm"
    unit = "GB/s"
    dtype = "f32"

    def __init__(self, torch, device, rank):
        self.torch, self.device, self.rank = torch, device, rank

    def sets_needed(self, footprint):
        return max(1, min(8, math.ceil(3 * L2_BYTES / max(1, footprint))))

    def units(self):  # algorithmic bytes or FLOPs per step
        raise NotImplementedError

    def per_unit(self):
        return 1e9 if self.unit == "GB/s" else 1e12


class RowOp(Op):
    def gen(self, shape, dist, seed):
        torch = self.torch
        g = torch.Generator(device=self.device).manual_seed(seed)
        if dist == "uniform":
            return torch.rand(shape, device=self.device, generator=g) * 2 - 1
        return torch.randn(shape, device=self.device, generator=g) * dist


class RMSNormOp(RowOp):
    name = "rmsnorm"
    rows, cols, eps = 4096, 1024, 1e-6
    config = "RMSNorm X f32 [4096,1024] ~N(0,1), gamma f32 [1024] ~N(1,0.1), eps 1e-6"

    def setup(self):
        from ntilang_b200 import kernels as K

        self.kernel = K.rmsnorm(self.rows, self.cols, self.eps)
        n = self.sets_needed(2 * self.rows * self.cols * 4)
        self.sets = []
        for s in range(n):
            x = self.gen((self.rows, self.cols), 1.0, 1000 * self.rank + s)
            w = self.gen((self.cols,), 0.1, 7 + s) + 1.0
            y = self.torch.empty_like(x)
            self.sets.append(((x, w, y), (x, w), y))

    def units(self):
        return 2 * self.rows * self.cols * 4 + self.cols * 4

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = 1024
        x = np.random.default_rng(0).normal(size=(rows, self.cols)).astype(np.float32)
        w = np.random.default_rng(1).normal(1, 0.1, size=self.cols).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rowops.rmsnorm(x, w, self.eps)
            n += 1
        dt = time.perf_counter() - t0
        return n * (2 * rows * self.cols * 4 + self.cols * 4) / dt / 1e9, f"{n} x RMSNorm [{rows},{self.cols}]"


class LayerNormOp(RowOp):
    name = "layernorm"
    rows, cols, eps = 4096, 1024, 1e-5
    config = "LayerNorm X f32 [4096,1024] ~N(0,1), gamma f32 [1024] ~N(1,0.1), beta f32 [1024] ~N(0,0.1), eps 1e-5"

    def setup(self):
        from ntilang_b200 import kernels as K

        self.kernel = K.layernorm(self.rows, self.cols, self.eps)
        n = self.sets_needed(2 * self.rows * self.cols * 4)
        self.sets = []
        for s in range(n):
            x = self.gen((self.rows, self.cols), 1.0, 1000 * self.rank + s)
            w = self.gen((self.cols,), 0.1, 7 + s) + 1.0
            b = self.gen((self.cols,), 0.1, 17 + s)
            y = self.torch.empty_like(x)
            self.sets.append(((x, w, b, y), (x, w, b), y))

    def units(self):
        return 2 * self.rows * self.cols * 4 + 2 * self.cols * 4

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = 1024
        x = np.random.default_rng(0).normal(size=(rows, self.cols)).astype(np.float32)
        w = np.random.default_rng(1).normal(1, 0.1, size=self.cols).astype(np.float32)
        b = np.random.default_rng(2).normal(0, 0.1, size=self.cols).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rowops.layernorm(x, w, b, self.eps)
            n += 1
        dt = time.perf_counter() - t0
        return n * (2 * rows * self.cols * 4 + 2 * self.cols * 4) / dt / 1e9, f"{n} x LayerNorm [{rows},{self.cols}]"


class TransposeOp(RowOp):
    name = "transpose"
    m, n = 4096, 4096
    config = "shared transpose A f32 [4096,4096] ~N(0,1) -> B [4096,4096] (README config)"

    def setup(self):
        from ntilang_b200 import kernels as K

        self.kernel = K.transpose(self.m, self.n)
        k = self.sets_needed(2 * self.m * self.n * 4)
        self.sets = []
        for s in range(k):
            a = self.gen((self.m, self.n), 1.0, 1000 * self.rank + s)
            b = self.torch.empty((self.n, self.m), device=self.device)
            self.sets.append(((a, b), (a,), b))

    def units(self):
        return 2 * self.m * self.n * 4

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        m = 1024
        a = np.random.default_rng(0).normal(size=(m, self.n)).astype(np.float32)
        k, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rowops.transpose(a)
            k += 1
        dt = time.perf_counter() - t0
        return k * 2 * m * self.n * 4 / dt / 1e9, f"{k} x transpose [{m},{self.n}]"


class CumsumOp(RowOp):
    name = "cumsum"
    rows, cols = 32768, 256
    config = "row inclusive cumsum X f32 [32768,256] ~U(-1,1)"

    def setup(self):
        from ntilang_b200 import kernels as K

        self.kernel = K.cumsum(self.rows, self.cols)
        n = self.sets_needed(2 * self.rows * self.cols * 4)
        self.sets = []
        for s in range(n):
            x = self.gen((self.rows, self.cols), "uniform", 1000 * self.rank + s)
            y = self.torch.empty_like(x)
            self.sets.append(((x, y), (x,), y))

    def units(self):
        return 2 * self.rows * self.cols * 4

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = 4096
        x = np.random.default_rng(0).uniform(-1, 1, size=(rows, self.cols)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rowops.cumsum(x)
            n += 1
        dt = time.perf_counter() - t0
        return n * 2 * rows * self.cols * 4 / dt / 1e9, f"{n} x cumsum [{rows},{self.cols}]"


class SoftmaxOp(RowOp):
    name = "softmax"
    rows, cols = 16384, 512
    config = "row softmax X f32 [16384,512] ~N(0,4)"

    def setup(self):
        from ntilang_b200 import kernels as K

        self.kernel = K.softmax(self.rows, self.cols)
        n = self.sets_needed(2 * self.rows * self.cols * 4)
        self.sets = []
        for s in range(n):
            x = self.gen((self.rows, self.cols), 2.0, 1000 * self.rank + s)
            y = self.torch.empty_like(x)
            self.sets.append(((x, y), (x,), y))

    def units(self):
        return 2 * self.rows * self.cols * 4

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        rows = 2048
        x = (np.random.default_rng(0).normal(size=(rows, self.cols)) * 2).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rowops.softmax(x)
            n += 1
        dt = time.perf_counter() - t0
        return n * 2 * rows * self.cols * 4 / dt / 1e9, f"{n} x softmax [{rows},{self.cols}]"


class VaddOp(RowOp):
    name = "vadd"
    n = 16 * 1024 * 1024
    config = "vector add A,B f32 [16777216] ~N(0,1)"

    def setup(self):
        from ntilang_b200 import kernels as K

        self.kernel = K.vector_add(self.n)
        k = self.sets_needed(3 * self.n * 4)
        self.sets = []
        for s in range(k):
            a = self.gen((self.n,), 1.0, 1000 * self.rank + 2 * s)
            b = self.gen((self.n,), 1.0, 1000 * self.rank + 2 * s + 1)
            c = self.torch.empty_like(a)
            self.sets.append(((a, b, c), (a, b), c))

    def units(self):
        return 3 * self.n * 4

    def cpu(self, seconds):
        import numpy as np

        from oracle import rowops

        m = 4 * 1024 * 1024
        a = np.random.default_rng(0).normal(size=m).astype(np.float32)
        b = np.random.default_rng(1).normal(size=m).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            rowops.vadd(a, b)
            n += 1
        dt = time.perf_counter() - t0
        return n * 3 * m * 4 / dt / 1e9, f"{n} x vector add [{m}]"


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
    n = 16 * 1024 * 1024
    config = "generic elementwise D = A*B + C (separately rounded), A,B,C f32 [16777216] ~N(0,1), NVRTC path"

    def setup(self):
        import ntilang_b200
        from ntilang_b200 import language as T

        self.kernel = ntilang_b200.compile(generic_fma_program(T, self.n), out_idx=[-1])
        assert self.kernel.spec.family == "pointwise"
        k = self.sets_needed(4 * self.n * 4)
        self.sets = []
        for s in range(k):
            a, b, c = (self.gen((self.n,), 1.0, 1000 * self.rank + 3 * s + j) for j in range(3))
            d = self.torch.empty_like(a)
            self.sets.append(((a, b, c, d), (a, b, c), d))

    def units(self):
        return 4 * self.n * 4

    def cpu(self, seconds):
        import numpy as np

        m = 4 * 1024 * 1024
        a, b, c = (np.random.default_rng(j).normal(size=m).astype(np.float32) for j in range(3))
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            np.add(np.multiply(a, b), c)
            n += 1
        dt = time.perf_counter() - t0
        return n * 4 * m * 4 / dt / 1e9, f"{n} x numpy a*b+c [{m}] (float32, separately rounded)"


class GemmOp(Op):
    name = "gemm"
    bound = "tensor"
    unit = "TFLOP/s"
    dtype = "f16xf16->f32"
    m = n = k = 4096
    epilogue = False
    config = "FP16 GEMM 4096x4096x4096, A,B ~N(0,1)/sqrt(K), C f32"

    def setup(self):
        from ntilang_b200 import kernels as K

        torch = self.torch
        self.kernel = (K.matmul_bias_relu if self.epilogue else K.matmul)(self.m, self.n, self.k)
        foot = (self.m * self.k + self.k * self.n) * 2 + self.m * self.n * 4
        self.sets = []
        for s in range(self.sets_needed(foot)):
            g = torch.Generator(device=self.device).manual_seed(1000 * self.rank + s)
            a = (torch.randn(self.m, self.k, device=self.device, generator=g) / math.sqrt(self.k)).half()
            b = (torch.randn(self.k, self.n, device=self.device, generator=g) / math.sqrt(self.k)).half()
            c = torch.empty(self.m, self.n, device=self.device)
            if self.epilogue:
                bias = torch.randn(self.n, device=self.device, generator=g) * 0.1
                self.sets.append(((a, b, bias, c), (a, b, bias), c))
            else:
                self.sets.append(((a, b, c), (a, b), c))

    def units(self):
        return 2 * self.m * self.n * self.k

    def cpu(self, seconds):
        import numpy as np

        from oracle import ntl_oracle as O

        rows = 256
        rng = np.random.default_rng(0)
        a = (rng.normal(size=(rows, self.k)) / 64).astype(np.float16)
        b = (rng.normal(size=(self.k, self.n)) / 64).astype(np.float16)
        bias = rng.normal(0, 0.1, self.n).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            if self.epilogue:
                O.gemm(a, b, bias, O.BIAS_N, relu=True, accumulate=np.float32)
            else:
                O.gemm(a, b, accumulate=np.float32)
            n += 1
        dt = time.perf_counter() - t0
        return n * 2 * rows * self.n * self.k / dt / 1e12, f"{n} x fp32 matmul [{rows},{self.k}]x[{self.k},{self.n}]"


class GemmBiasReluOp(GemmOp):
    name = "gemm_bias_relu"
    epilogue = True
    config = "FP16 GEMM 4096^3 + fused C=relu(A@B+bias[N]), bias ~N(0,0.1)"


class FA2Op(Op):
    name = "fa2"
    bound = "tensor"
    unit = "TFLOP/s"
    dtype = "f16xf16->f32"
    B, H, S, D = 8, 32, 4096, 128
    causal = False
    config = "FlashAttention-2 fwd Q,K,V f16 [8,32,4096,128] ~N(0,1), scale 1/sqrt(128), non-causal"

    def setup(self):
        from ntilang_b200 import kernels as K

        torch = self.torch
        self.kernel = K.flash_attention(self.B, self.H, self.S, self.D, self.causal)
        g = torch.Generator(device=self.device).manual_seed(1000 * self.rank)
        shape = (self.B, self.H, self.S, self.D)
        q, k, v = (torch.randn(shape, device=self.device, generator=g).half() for _ in range(3))
        o = torch.empty_like(q)
        self.sets = [((q, k, v, o), (q, k, v), o)]

    def units(self):
        f = 4 * self.B * self.H * self.S * self.S * self.D
        return f // 2 if self.causal else f

    def cpu(self, seconds):
        import numpy as np

        from oracle import ntl_oracle as O

        rng = np.random.default_rng(0)
        rows = 256
        q = rng.normal(size=(1, 1, rows, self.D)).astype(np.float16)
        k, v = (rng.normal(size=(1, 1, self.S, self.D)).astype(np.float16) for _ in range(2))
        c = math.log2(math.e) / math.sqrt(self.D)
        n, t0 = 0, time.perf_counter()
        flops = 0
        while time.perf_counter() - t0 < seconds:
            if self.causal:
                # the last `rows` queries of a causal head attend to (almost) all keys
                qq = np.zeros((1, 1, self.S, self.D), np.float16)
                qq[0, 0, -rows:] = q[0, 0]
                O.fa2_blockwise(qq[:, :, -rows:], k, v, c, False)
                flops += 4 * rows * self.S * self.D
            else:
                O.fa2_blockwise(q, k, v, c, False)
                flops += 4 * rows * self.S * self.D
            n += 1
        dt = time.perf_counter() - t0
        return flops / dt / 1e12, f"{n} x attention [1,1,{rows} queries,{self.S} keys,{self.D}]"


class FA2CausalOp(FA2Op):
    name = "fa2_causal"
    causal = True
    config = "FlashAttention-2 fwd Q,K,V f16 [8,32,4096,128] ~N(0,1), scale 1/sqrt(128), causal"


OPS = {c.name: c for c in (CumsumOp, RMSNormOp, SoftmaxOp, VaddOp, GemmOp, GemmBiasReluOp, FA2Op, FA2CausalOp,
                           LayerNormOp, TransposeOp, GenericFmaOp)}


# ------------------------------------------------------------------------------ clocks


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        import tempfile

        self.path = tempfile.NamedTemporaryFile(prefix="ntl_clocks_", suffix=".csv", delete=False).name
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        power = [num(r[3]) for r in rows if num(r[3]) is not None]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s, p in zip(sm, power) if p is not None and p > 300] or sm
        loaded.sort()
        return {"sm_mhz": loaded[len(loaded) // 2] if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "power_w_max": max(power) if power else None}


# ----------------------------------------------------------------------------- measure


def run_op(op, torch, dist, world, steps, warmup, stream, peaks, peak_kind, traffic, want_e2e, want_call_path=True):
    from ntilang_b200 import _lib

    op.setup()
    kern = op.kernel
    nsets = len(op.sets)
    # warm-up through the public call
    with torch.cuda.stream(stream):
        for i in range(max(3, warmup)):
            kern(*op.sets[i % nsets][0])
    stream.synchronize()
    # capture K steps (rotating input sets) into one graph
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
        start.record(stream)
        graph.replay()
        end.record(stream)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device=op.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    del graph
    ms_step = ms / steps
    units = op.units()
    value = world * units / (ms_step / 1e3) / op.per_unit()
    per_launch = units / (ms_step / 1e3) / op.per_unit()
    if op.bound == "hbm":
        peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        punit = "GB/s"
    else:
        peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
        punit = "TFLOP/s"
    tr = traffic.get(op.name)
    result = {
        "metric": f"{op.name} achieved {op.unit}", "value": round(value, 3), "unit": op.unit,
        "ms_per_step": round(ms_step, 6), "steps": steps, "buffer_sets": nsets, "gpu_launches": launches,
        "config": op.config, "dtype": op.dtype,
        "roofline": {"bound": op.bound, "achieved": round(per_launch, 3), "peak": peak, "unit": punit,
                     "frac": round(per_launch / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json burst)"
                     if peak_kind == "measured" else "fallback",
                     "traffic": tr.get("bytes_per_launch") if isinstance(tr, dict) else None,
                     "algorithmic_per_launch": units},
    }
    if want_call_path:
        result["python_call"] = measure_call_path(op, torch, stream)
    if want_e2e:
        result["e2e"] = measure_e2e(op, torch, dist, world, steps, stream)
    op.sets = None
    torch.cuda.empty_cache()
    return result


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


def measure_e2e(op, torch, dist, world, steps, stream):
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
    ms = start.elapsed_time(end)
    if dist is not None:
        t = torch.tensor([ms], device=op.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / n
    value = world * op.units() / (ms_step / 1e3) / op.per_unit()
    return {"value": round(value, 3), "unit": op.unit, "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
            "ms_per_step": round(ms_step, 4), "steps": n, "streams": 2}


def cpu_baseline(op, seconds):
    try:
        import oracle.rowops as rowops

        threads = rowops.threads()
    except Exception:  # noqa: BLE001 - report what ran
        threads = os.cpu_count() or 1
    value, sample = op.cpu(seconds)
    cores = threads if op.bound == "hbm" else (os.cpu_count() or 1)
    return {"value": round(value, 4), "unit": op.unit, "cores": cores, "kind": "port", "sample": sample}


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
        "cumsum": (lambda op: ex("cumsum")(op.rows, op.cols, target=target), same, None),
        "rmsnorm": (lambda op: ex("rmsnorm")(op.rows, op.cols, eps=op.eps, target=target), same, None),
        "layernorm": (lambda op: ex("layernorm")(op.rows, op.cols, eps=op.eps, target=target), same, None),
        "softmax": (lambda op: ex("softmax")(op.rows, op.cols, target=target), same, None),
        "vadd": (lambda op: ex("vector_add")(op.n, target=target), same, None),
        "transpose": (lambda op: ex("transpose")(op.m, op.n, target=target), same, None),
        "gemm": (lambda op: ex("matmul")(op.m, op.n, op.k, **gemm_tiles), same, None),
        # The example's epilogue is relu(0.5 * acc + Bias[M, N]) (examples/matmul_relu.py:35-38):
        # bias[N] is broadcast to a full [M, N] operand and the result checked against torch.
        "gemm_bias_relu": (lambda op: ex("matmul_relu")(op.m, op.n, op.k, **gemm_tiles), relu_args,
                           lambda a: (0.5 * (a[0].float() @ a[1].float()) + a[2]).relu()),
        "fa2": (lambda op: ex("flash_attention")(op.B, op.H, op.S, op.D, is_causal=False, target=target), same,
                None),
        "fa2_causal": (lambda op: ex("flash_attention")(op.B, op.H, op.S, op.D, is_causal=True, target=target),
                       same, None),
        "pointwise": (lambda op: R.compile(generic_fma_program(RT, op.n), target=target), same, None),
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
    ap.add_argument("--cpu-seconds", type=float, default=2.0, help="CPU-baseline sample per op (0 = skip)")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--no-call-path", action="store_true",
                    help="skip the Python call-path timing (200 extra launches per op; for launch lists)")
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


def run_reference(args, ops):
    """The reference's CPU path (the oracle port of its algorithm) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch  # noqa: F401  (same environment as our arm)

    per = {}
    head = None
    steps = max(1, args.steps)
    for name in ops:
        op = OPS[name](None, None, 0)
        vals = []
        warm = max(0, min(args.warmup, 1))
        for _ in range(warm):
            op.cpu(0.05)
        seconds = max(0.05, min(args.cpu_seconds, 30.0 / (len(ops) * steps)))
        sample = ""
        for _ in range(steps if name == HEADLINE else 1):
            v, sample = op.cpu(seconds)
            vals.append(v)
        vals.sort()
        v = vals[len(vals) // 2]
        cb = {"value": round(v, 4), "unit": op.unit, "cores": os.cpu_count() or 1, "kind": "port", "sample": sample}
        per[name] = {"value": round(v, 4), "unit": op.unit, "config": op.config, "cpu_baseline": cb}
        if name == HEADLINE:
            head = (op, v, cb)
    op, v, cb = head
    line = {
        "impl": "reference", "metric": BASELINE_METRIC, "value": round(v, 4), "unit": op.unit, "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE.json distributions)",
        "config": {"workload": op.config, "op": op.name, "path": "CPU oracle port of the reference algorithm"},
        "cpu_baseline": cb, "e2e": {"value": round(v, 4), "unit": op.unit, "h2d_bytes_per_step": 0,
                                    "d2h_bytes_per_step": 0},
        "ops": per,
    }
    print(json.dumps(line), flush=True)
    return 0


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
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
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
    sampler = ClockSampler(torch.cuda.current_device())
    sampler.start()
    results = {}
    for name in ops:
        op = OPS[name](torch, device, rank)
        try:
            results[name] = run_op(op, torch, dist, world, args.steps, args.warmup, stream, peaks, peak_kind, traffic,
                                   want_e2e=not args.no_e2e, want_call_path=not args.no_call_path)
        except _lib.KernelError as exc:
            if exc.code != 2:
                raise
            results[name] = {"unavailable": str(exc)}
            op.sets = None
    clocks = sampler.stop()
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        for name in ops:
            if "unavailable" not in results[name]:
                results[name]["cpu_baseline"] = cpu_baseline(OPS[name](None, None, 0), args.cpu_seconds)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    head = results[HEADLINE]
    total_launches = sum(r.get("gpu_launches", 0) for r in results.values())
    line = {
        "metric": BASELINE_METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, BASELINE.json shapes and distributions)",
        "config": {"workload": OPS[HEADLINE].config + " (BASELINE.json configs[1])", "op": HEADLINE,
                   "parallelism": f"row-sharded x{world}, no collective" if world > 1 else "single GPU",
                   "l2": "inputs rotated over buffer sets larger than L2 between reuses",
                   "timing": "K launches replayed from one CUDA graph, CUDA events, max over ranks"},
        "roofline": head["roofline"], "e2e": head.get("e2e"), "gpu_launches": total_launches, "clocks": clocks,
        "cpu_baseline": head.get("cpu_baseline"), "ops": results,
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
