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

from collections.abc import Callable, Mapping
from dataclasses import dataclass
from pathlib import Path
from types import MappingProxyType

from . import frontend
from .compat import normalize_out_idx, resolve_target
from .compiler import CompiledKernel, DynamicJitKernel, lower_program, make_kernel
from .ir import CompileError, ScalarParameter, SymDim
from .language import PrimFunc, has_symbolic_annotations


def _dim_text(n) -> str:
    return n.name if isinstance(n, SymDim) else str(n)


def _expr_text(e) -> str:
    """Infix text of a launch-shape expression (integers, symbolic sizes, + - * // %)."""
    if isinstance(e, frontend.Const):
        return str(e.value)
    if isinstance(e, frontend.Var):
        return e.name.rsplit(":", 1)[-1]
    if isinstance(e, frontend.Bin):
        return f"({_expr_text(e.a)} {e.op} {_expr_text(e.b)})"
    return str(e)


@dataclass(frozen=True)
class Artifact:
    """One emitted text (``format`` is ``"python"`` or ``"cuda"``)."""

    format: str
    content: str

    def save(self, path) -> Path:
        """Write the text as UTF-8 with ``\\n`` line ends, creating missing folders; returns the path."""
        out = Path(path)
        if not out.parent.is_dir():
            out.parent.mkdir(parents=True)
        with open(out, "w", encoding="utf-8", newline="\n") as fh:
            fh.write(self.content)
        return out


@dataclass(frozen=True)
class Program:
    """A parsed program and the front end that read it."""

    ir: frontend.Program
    frontend: str
    name: str

    def as_text(self) -> str:
        """A short listing: the program's name, its parameters with types, and its launch shape."""
        lines = [f"program {self.name} [frontend {self.frontend}]"]
        for prm in self.ir.params:
            if isinstance(prm, ScalarParameter):
                lines.append(f"  {prm.name}: {prm.dtype}")
            else:
                dims = ", ".join(_dim_text(n) for n in prm.type.shape)
                lines.append(f"  {prm.name}: {prm.type.dtype}[{dims}]")
        grid = ", ".join(_expr_text(g) for g in self.ir.grid)
        lines.append(f"  launch: grid ({grid}), {self.ir.threads} threads per block")
        return "\n".join(lines)


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
        raise CompileError(f"Unsupported emit format {format!r}: the {self.backend!r} back end writes 'python' "
                           "(the launcher module) or 'cuda' (a generated elementwise kernel)")


@dataclass(frozen=True)
class ArtifactBundle:
    lowered: LoweredProgram
    kernel: CompiledKernel


class RuntimeModule(Mapping):
    """The built kernels of one bundle, looked up by program name (``module["scale"]``).

    A read-only mapping: ``in``, ``len``, iteration over names and ``keys()`` work as for a dict.
    """

    def __init__(self, bundle: ArtifactBundle, device: str = "cuda:0"):
        self.bundle = bundle
        self.device = device
        self._by_name = MappingProxyType({bundle.lowered.program.name: bundle.kernel})

    def __getitem__(self, name: str) -> CompiledKernel:
        try:
            return self._by_name[name]
        except KeyError:
            raise KeyError(f"no kernel named {name!r} in this module (it holds {', '.join(self._by_name)})") from None

    def __iter__(self):
        return iter(self._by_name)

    def __len__(self) -> int:
        return len(self._by_name)


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

    @staticmethod
    def _lookup(table: dict, kind: str, name: str) -> Callable:
        fn = table.get(name)
        if fn is None:
            raise CompileError(f"Unknown {kind} {name!r}: this Compiler knows {sorted(table)}")
        return fn

    def import_program(self, source, *, frontend: str = "tilelang") -> Program:
        ir = self._lookup(self._frontends, "frontend", frontend)(source)
        return Program(ir=ir, frontend=frontend, name=ir.name)

    def lower(self, program: Program, *, backend: str = "sm100a", target: str = "auto", out_idx=None) -> LoweredProgram:
        emit = self._lookup(self._backends, "backend", backend)
        resolved = resolve_target(target)
        normalized = normalize_out_idx(out_idx, program.ir.params)
        kernel = emit(program.ir, resolved, normalized)
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
