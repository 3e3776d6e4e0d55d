"""``@autotune``: time candidate configurations with CUDA events and keep the fastest.

Same surface as the reference's ``python/ntilang/autotune.py:23-153`` (``AutoTuner``,
``TuneResult``, ``autotune(configs, warmup=, rep=, target=, out_idx=)``).  Tile hints in
the configurations reach the recognised kernels only as program parameters; the sm_100a
kernels pick their own tiles, so candidates usually time alike.
"""

from __future__ import annotations

import importlib
import sys
from dataclasses import dataclass

from .compiler import CompiledKernel
from .compiler import compile as compile_kernel
from .ir import CompileError
from .language import PrimFunc


@dataclass(frozen=True)
class TuneResult:
    config: dict
    kernel: CompiledKernel
    latency_ms: float


class AutoTuner:
    def __init__(self, fn, configs, *, warmup=5, rep=20, target="auto", out_idx=None):
        self.fn = fn
        self._configs = configs
        self.warmup = warmup
        self.rep = rep
        self.target = target
        self.out_idx = out_idx
        self._cache = {}
        self.best_config = None
        self.best_latency_ms = None

    def _resolve_configs(self):
        raw = self._configs() if callable(self._configs) else self._configs
        configs = [dict(c) for c in raw]
        if not configs:
            raise ValueError("autotune requires at least one configuration")
        return configs

    def _build_candidate(self, args, kwargs, cfg):
        result = self.fn(*args, **{**kwargs, **cfg})
        if isinstance(result, CompiledKernel):
            return result
        if isinstance(result, PrimFunc):
            return compile_kernel(result, target=self.target, out_idx=self.out_idx)
        raise TypeError("autotune factory must return a CompiledKernel or @T.prim_func")

    @staticmethod
    def _make_dummy_args(kernel, torch):
        from .compat import torch_dtype_for

        out_set = set(kernel.out_idx)
        args = []
        for idx, param in enumerate(kernel.user_parameters):
            if idx in out_set:
                continue
            args.append(torch.zeros(param.type.shape, dtype=torch_dtype_for(param.type.dtype, torch), device="cuda"))
        return tuple(args)

    def _measure_ms(self, kernel, sample_args, torch):
        for _ in range(self.warmup):
            kernel(*sample_args)
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(self.rep):
            kernel(*sample_args)
        end.record()
        torch.cuda.synchronize()
        return float(start.elapsed_time(end)) / max(1, self.rep)

    def tune(self, *args, **kwargs) -> TuneResult:
        key = (args, tuple(sorted(kwargs.items())))
        if key in self._cache:
            return self._cache[key]
        torch = sys.modules.get("torch")
        if torch is None:
            try:
                torch = importlib.import_module("torch")
            except ImportError:
                torch = None
        has_cuda = torch is not None and torch.cuda.is_available()
        best, last_error = None, None
        for cfg in self._resolve_configs():
            try:
                kernel = self._build_candidate(args, kwargs, cfg)
                if not has_cuda:
                    best = TuneResult(cfg, kernel, 0.0)
                    break
                ms = self._measure_ms(kernel, self._make_dummy_args(kernel, torch), torch)
                if best is None or ms < best.latency_ms:
                    best = TuneResult(cfg, kernel, ms)
            except (CompileError, RuntimeError, ValueError) as exc:
                last_error = exc
        if best is None:
            raise CompileError(f"All autotune configurations failed; last error: {last_error}") from last_error
        self._cache[key] = best
        self.best_config = best.config
        self.best_latency_ms = best.latency_ms
        return best

    def __call__(self, *args, **kwargs) -> CompiledKernel:
        return self.tune(*args, **kwargs).kernel


def autotune(configs, *, warmup=5, rep=20, target="auto", out_idx=None):
    def decorator(fn):
        return AutoTuner(fn, configs, warmup=warmup, rep=rep, target=target, out_idx=out_idx)

    return decorator


__all__ = ["AutoTuner", "TuneResult", "autotune"]
