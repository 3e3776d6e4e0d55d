"""``@autotune``: compile each candidate configuration, time it on the GPU, keep the fastest.

The public surface is the reference's (``python/ntilang/autotune.py:23-153``): ``autotune(configs,
warmup=, rep=, target=, out_idx=)`` wraps a kernel factory in an ``AutoTuner``; calling it with the
factory's arguments returns the fastest ``CompiledKernel`` (cached per argument tuple), and
``best_config`` / ``best_latency_ms`` / ``tune()`` -> ``TuneResult`` report the choice.  Same
rules: ``configs`` is a list of dicts or a callable returning one, an empty list is a
``ValueError``, a candidate that fails to compile or launch (``CompileError``, ``RuntimeError``,
``ValueError``) is skipped, and when every candidate fails the last error is raised as a
``CompileError``.  Without CUDA the first candidate that compiles is returned untimed.

How a candidate is timed here:

* Its arguments come from the kernel's own parameter list: a zero-filled tensor of the declared
  shape and dtype for every tensor (outputs included, so no allocation is timed), a zero of the
  declared type for every scalar (``False`` for bool).  A symbolic dimension is bound to
  ``SYMBOLIC_SIZE``.
* Candidates that compile to the same kernel (the sm_100a family kernels choose their own tiles,
  so tile hints often change nothing) are timed once.
* ``rep`` launches are captured into one CUDA graph; after ``warmup`` eager launches and one
  untimed replay, the graph is replayed ``TRIALS`` times between CUDA events and the median
  per-launch time is kept.  This measures the kernel, not the Python call path.  A kernel whose
  launches cannot be captured is timed eagerly instead.
"""

from __future__ import annotations

import importlib
import statistics
import sys
from dataclasses import dataclass

from .compiler import CompiledKernel
from .compiler import compile as compile_kernel
from .ir import CompileError, ScalarParameter, SymDim
from .language import PrimFunc

SYMBOLIC_SIZE = 1024
TRIALS = 3
_SKIPPED = (CompileError, RuntimeError, ValueError)


@dataclass(frozen=True)
class TuneResult:
    config: dict
    kernel: CompiledKernel
    latency_ms: float


def _torch_or_none():
    torch = sys.modules.get("torch")
    if torch is not None:
        return torch
    try:
        return importlib.import_module("torch")
    except ImportError:
        return None


def sample_arguments(kernel: CompiledKernel, torch, device="cuda") -> tuple:
    """One value per kernel parameter (outputs included) for timing launches."""
    from .compat import torch_dtype_for

    values = []
    for param in kernel.user_parameters:
        if isinstance(param, ScalarParameter):
            dtype = param.dtype
            values.append(False if dtype == "bool" else 0.0 if dtype.startswith(("float", "bfloat")) else 0)
            continue
        shape = tuple(SYMBOLIC_SIZE if isinstance(d, SymDim) else int(d) for d in param.type.shape)
        values.append(torch.zeros(shape, dtype=torch_dtype_for(param.type.dtype, torch), device=device))
    return tuple(values)


def time_kernel(kernel: CompiledKernel, arguments: tuple, torch, *, warmup: int, rep: int) -> float:
    """Median milliseconds per launch of ``kernel(*arguments)`` (see the module docstring)."""
    rep = max(1, int(rep))
    for _ in range(max(1, int(warmup))):
        kernel(*arguments)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph):
            for _ in range(rep):
                kernel(*arguments)
    except RuntimeError:
        graph = None
        torch.cuda.synchronize()
    samples = []
    for trial in range(TRIALS + 1):
        start.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(rep):
                kernel(*arguments)
        end.record()
        torch.cuda.synchronize()
        if trial:  # the first replay is untimed
            samples.append(start.elapsed_time(end) / rep)
    return float(statistics.median(samples))


class AutoTuner:
    """Chooses, per factory argument tuple, the configuration whose kernel runs fastest."""

    def __init__(self, fn, configs, *, warmup=5, rep=20, target="auto", out_idx=None):
        self.fn = fn
        self.configs = configs
        self.warmup = warmup
        self.rep = rep
        self.target = target
        self.out_idx = out_idx
        self.best_config = None
        self.best_latency_ms = None
        self.results: dict = {}  # argument key -> TuneResult
        self.timings: dict = {}  # argument key -> [(config, ms or None, error or None)]

    def candidates(self) -> list:
        listed = self.configs() if callable(self.configs) else self.configs
        out = [dict(c) for c in listed]
        if not out:
            raise ValueError("autotune requires at least one configuration")
        return out

    def compile_candidate(self, args, kwargs, config) -> CompiledKernel:
        made = self.fn(*args, **dict(kwargs, **config))
        if isinstance(made, PrimFunc):
            return compile_kernel(made, target=self.target, out_idx=self.out_idx)
        if isinstance(made, CompiledKernel):
            return made
        raise TypeError("autotune factory must return a CompiledKernel or @T.prim_func")

    def tune(self, *args, **kwargs) -> TuneResult:
        key = (args, tuple(sorted(kwargs.items())))
        hit = self.results.get(key)
        if hit is not None:
            return hit
        torch = _torch_or_none()
        timed = torch is not None and torch.cuda.is_available()
        best, error, log = None, None, []
        seen: dict = {}  # kernel identity -> ms, so identical kernels are timed once
        for config in self.candidates():
            try:
                kernel = self.compile_candidate(args, kwargs, config)
                if not timed:
                    best = TuneResult(config, kernel, 0.0)
                    log.append((config, None, None))
                    break
                identity = (kernel.cache_key, kernel.out_idx)
                if identity not in seen:
                    seen[identity] = time_kernel(kernel, sample_arguments(kernel, torch), torch,
                                                 warmup=self.warmup, rep=self.rep)
                ms = seen[identity]
                log.append((config, ms, None))
                if best is None or ms < best.latency_ms:
                    best = TuneResult(config, kernel, ms)
            except _SKIPPED as exc:
                error = exc
                log.append((config, None, f"{type(exc).__name__}: {exc}"))
        self.timings[key] = log
        if best is None:
            raise CompileError(f"All autotune configurations failed; last error: {error}") from error
        self.results[key] = best
        self.best_config, self.best_latency_ms = best.config, best.latency_ms
        return best

    def __call__(self, *args, **kwargs) -> CompiledKernel:
        return self.tune(*args, **kwargs).kernel


def autotune(configs, *, warmup=5, rep=20, target="auto", out_idx=None):
    """Decorator: ``@autotune(configs=[...])`` over a kernel factory (see ``AutoTuner``)."""

    def wrap(fn):
        return AutoTuner(fn, configs, warmup=warmup, rep=rep, target=target, out_idx=out_idx)

    return wrap


__all__ = ["AutoTuner", "TuneResult", "autotune", "sample_arguments", "time_kernel"]
