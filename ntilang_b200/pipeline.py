"""The staged ``Compiler`` API: import_program -> lower -> emit / compile -> load -> jit.

Same stages, names and return types as the reference's python/ntilang/pipeline.py:18-158
(``Artifact.save``, ``Program.as_text``, ``LoweredProgram.emit``, ``ArtifactBundle``,
``RuntimeModule[name]``, ``register_frontend`` / ``register_backend``).  What the stages do
differs: the ``tilelang`` front end is this package's reader (``frontend.read_program``),
and the back end picks the op's kernel (``compiler.lower_program``) instead of writing CuTe
DSL source.  The back end is registered as ``sm100a``; ``cute`` names the same back end so
code written for the reference keeps working.  ``emit(format="python")`` is the standalone
launcher module (``CompiledKernel.save()`` writes the same text); ``emit(format="cuda")`` is
the CUDA C of a generic elementwise program (recognised families run prebuilt kernels and
have no per-program CUDA source).
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from pathlib import Path

from . import frontend
from .compat import normalize_out_idx, resolve_target
from .compiler import CompiledKernel, DynamicJitKernel, lower_program, make_kernel
from .ir import CompileError
from .language import PrimFunc, has_symbolic_annotations


@dataclass(frozen=True)
class Artifact:
    format: str
    content: str

    def save(self, path) -> Path:
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        target.write_text(self.content, encoding="utf-8", newline="\n")
        return target


@dataclass(frozen=True)
class Program:
    ir: frontend.Program
    frontend: str
    name: str

    def as_text(self) -> str:
        params = ", ".join(p.name for p in self.ir.params)
        return f"Program(frontend={self.frontend!r}, name={self.name!r}, params=({params}), threads={self.ir.threads})"


@dataclass(frozen=True)
class LoweredProgram:
    program: Program
    backend: str
    target: str
    source: str
    out_idx: tuple = ()
    kernel: CompiledKernel = None

    def emit(self, *, format: str = "python") -> Artifact:
        if format == "python":
            return Artifact(format=format, content=self.source)
        if format == "cuda":
            spec = self.kernel.spec
            if spec is None or spec.family != "pointwise":
                raise CompileError(f"{self.program.name}: runs the prebuilt `{spec.family}` kernel of "
                                   "libntl_kernels.so; there is no per-program CUDA source to emit")
            return Artifact(format=format, content=spec.params["kernel"].source)
        raise CompileError(f"Unsupported emit format {format!r} for backend {self.backend!r}")


@dataclass(frozen=True)
class ArtifactBundle:
    lowered: LoweredProgram
    kernel: CompiledKernel


class RuntimeModule:
    """Loaded executable container exposing entry points by kernel name."""

    def __init__(self, bundle: ArtifactBundle, device: str = "cuda:0"):
        self.bundle = bundle
        self.device = device
        self._entries = {bundle.lowered.program.name: bundle.kernel}

    def __getitem__(self, name: str) -> CompiledKernel:
        return self._entries[name]

    def __contains__(self, name: str) -> bool:
        return name in self._entries


def _sm100a_backend(ir: frontend.Program, target: str, out_idx) -> CompiledKernel:
    return make_kernel(ir, lower_program(ir), target, out_idx)


class Compiler:
    """Staged compiler: import_program -> lower -> compile -> load, plus jit."""

    def __init__(self):
        self._frontends: dict[str, Callable] = {"tilelang": frontend.read_program}
        self._backends: dict[str, Callable] = {"sm100a": _sm100a_backend, "cute": _sm100a_backend}

    def register_frontend(self, name: str, parser_fn: Callable) -> None:
        """``parser_fn(source) -> frontend.Program``."""
        self._frontends[name] = parser_fn

    def register_backend(self, name: str, emitter_fn: Callable) -> None:
        """``emitter_fn(ir, target, out_idx) -> CompiledKernel``."""
        self._backends[name] = emitter_fn

    def import_program(self, source, *, frontend: str = "tilelang") -> Program:
        if frontend not in self._frontends:
            raise CompileError(f"Unknown frontend {frontend!r}; registered: {', '.join(sorted(self._frontends))}")
        ir = self._frontends[frontend](source)
        return Program(ir=ir, frontend=frontend, name=ir.name)

    def lower(self, program: Program, *, backend: str = "sm100a", target: str = "auto", out_idx=None) -> LoweredProgram:
        if backend not in self._backends:
            raise CompileError(f"Unknown backend {backend!r}; registered: {', '.join(sorted(self._backends))}")
        resolved = resolve_target(target)
        normalized = normalize_out_idx(out_idx, program.ir.params)
        kernel = self._backends[backend](program.ir, resolved, normalized)
        return LoweredProgram(program=program, backend=backend, target=resolved, source=kernel.source,
                              out_idx=normalized, kernel=kernel)

    def compile(self, lowered: LoweredProgram) -> ArtifactBundle:
        return ArtifactBundle(lowered=lowered, kernel=lowered.kernel)

    def load(self, bundle: ArtifactBundle, *, device: str = "cuda:0") -> RuntimeModule:
        bundle.kernel.build()
        return RuntimeModule(bundle, device=device)

    def jit(self, source, *, frontend: str = "tilelang", backend: str = "sm100a", target: str = "auto",
            out_idx=None):
        if (isinstance(source, PrimFunc) and frontend == "tilelang" and backend in ("sm100a", "cute")
                and has_symbolic_annotations(source)):
            return DynamicJitKernel(source, target=target, out_idx=out_idx)
        program = self.import_program(source, frontend=frontend)
        return self.compile(self.lower(program, backend=backend, target=target, out_idx=out_idx)).kernel


__all__ = ["Artifact", "ArtifactBundle", "Compiler", "LoweredProgram", "Program", "RuntimeModule"]
