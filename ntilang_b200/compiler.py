"""``compile`` / ``CompiledKernel`` / ``DynamicJitKernel``: the drop-in launch path.

Same contract as the reference's ``python/ntilang/compiler.py``:

* ``compile(prim_func, target=, out_idx=)`` (:340-355) reads the program and normalises
  ``out_idx``; instead of generating CuTe source it recognises the op family
  (``recognize.recognize``, a prebuilt sm_100a kernel) or, for any other elementwise
  program, generates CUDA C compiled by NVRTC (``pointwise.lower``).  ``source`` /
  ``save()`` give a standalone launcher module (``export.standalone_module``).
* ``CompiledKernel.__call__`` (:134-200) allocates ``out_idx`` outputs with
  ``torch.empty`` on the first CUDA input's device (:109-132), checks every tensor
  (CUDA device, shape, dtype, row-major contiguity, 16-byte alignment, disjoint
  storage, one device) with the same exception types, then launches — through the
  C ABI of ``libntl_kernels.so`` on ``torch.cuda.current_stream()`` instead of TVM-FFI.
* ``DynamicJitKernel`` (:203-337): one symbolic compile when the op family accepts
  runtime sizes (all of them do — the C ABI takes sizes per call), else per-shape
  specialisation cached by the bound symbolic dimensions.
"""

from __future__ import annotations

import hashlib
import importlib
import inspect
import sys
from dataclasses import dataclass, field
from pathlib import Path

from . import _lib
from .compat import normalize_out_idx, resolve_target, torch_dtype_for
from .frontend import Program, read_program
from .ir import DTYPES, CompileError, ScalarParameter, SymDim
from .language import PrimFunc, SymbolicDim, SymbolicTensorSpec
from .export import standalone_module
from .launch import describe, make_launcher
from .pointwise import lower as lower_pointwise
from .pointwise import validate_scalar
from .recognize import OpSpec, recognize


def _current_stream(torch, index):
    """torch's current CUDA stream on device ``index`` as a raw cudaStream_t (the stream TVM-FFI's
    environment stream follows in the reference)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(index)
    return torch.cuda.current_stream(index).cuda_stream


def _torch():
    torch = sys.modules.get("torch")
    return torch if torch is not None else importlib.import_module("torch")


@dataclass
class CompiledKernel:
    ir: Program
    target: str
    source: str  # the standalone launcher module save() writes (ntilang_b200.export)
    out_idx: tuple = ()
    spec: OpSpec = None
    _built: bool = field(default=False, init=False, repr=False)
    _state: object = field(default=None, init=False, repr=False)
    _run: object = field(default=None, init=False, repr=False)

    has_gpu_module = True

    @property
    def cache_key(self) -> str:
        return hashlib.sha256(self.source.encode("utf-8")).hexdigest()

    def get_kernel_source(self) -> str:
        """The standalone launcher module (``source``), as the reference returns its generated
        module here (python/ntilang/compiler.py:36-42)."""
        return self.source

    def get_host_source(self) -> str:
        return self.source

    def get_cuda_source(self) -> str:
        """Device code: the generated CUDA C of a generic elementwise program, else the launch
        plan of the prebuilt sm_100a kernel in libntl_kernels.so."""
        if self.spec is not None and self.spec.family == "pointwise":
            return self.spec.params["kernel"].source
        return describe(self.spec, self.ir.name, self.target)

    def save(self, path) -> Path:
        """Write the standalone launcher module (python/ntilang/compiler.py:44-49)."""
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(self.source, encoding="utf-8", newline="\n")
        return path

    def build(self):
        """Load libntl_kernels.so (the recognised kernels are compiled ahead of time for
        sm_100a); a generic elementwise program is also compiled by NVRTC here."""
        handle = _lib.lib()
        if self.spec is not None and self.spec.family == "pointwise":
            self.spec.params["kernel"].build()
        self._built = True
        return handle

    @property
    def user_parameters(self):
        return self.ir.params

    @property
    def family(self) -> str:
        return self.spec.family

    # ------------------------------------------------------------------ launch
    def _bind_symbols(self, arguments) -> dict:
        bindings = {}
        for param, arg in zip(self.ir.params, arguments):
            if isinstance(param, ScalarParameter) or not hasattr(arg, "shape"):
                continue
            if len(arg.shape) != len(param.type.shape):
                raise ValueError(f"{param.name}: expected rank {len(param.type.shape)}, got {len(arg.shape)}")
            for spec_dim, actual in zip(param.type.shape, arg.shape):
                if isinstance(spec_dim, SymDim):
                    actual = int(actual)
                    if actual <= 0:
                        raise ValueError(f"Symbolic dimension {spec_dim.name!r} must be positive")
                    prev = bindings.get(spec_dim.name)
                    if prev is not None and prev != actual:
                        raise ValueError(f"Symbolic dimension {spec_dim.name!r} mismatch: {prev} vs {actual}")
                    bindings[spec_dim.name] = actual
        return bindings

    @staticmethod
    def _resolve(shape, bindings):
        return tuple(bindings[d.name] if isinstance(d, SymDim) else d for d in shape)

    def _allocate_outputs(self, inputs, bindings):
        torch = _torch()
        device = None
        for arg in inputs:
            if hasattr(arg, "device") and hasattr(arg, "__dlpack_device__") and arg.__dlpack_device__()[0] == 2:
                device = arg.device
                break
        if device is None:
            device = torch.device("cuda")
        outs = []
        for idx in self.out_idx:
            param = self.ir.params[idx]
            shape = self._resolve(param.type.shape, bindings)
            outs.append(torch.empty(shape, dtype=torch_dtype_for(param.type.dtype, torch), device=device))
        return outs

    def _call_state(self):
        """Per-kernel state of the call path, built on the first call: for each parameter its
        static shape (None when symbolic), torch dtype and byte size."""
        torch = _torch()
        plan = []
        for p in self.ir.params:
            if isinstance(p, ScalarParameter):
                plan.append(None)
                continue
            shape = tuple(p.type.shape)
            static = not any(isinstance(d, SymDim) for d in shape)
            size = DTYPES[p.type.dtype]
            for d in shape if static else ():
                size *= d
            plan.append((p, shape if static else None, torch_dtype_for(p.type.dtype, torch), size if static else None))
        return plan

    def __call__(self, *arguments):
        params = self.ir.params
        allocated = None
        bindings = {}
        if self.out_idx and len(arguments) == len(params) - len(self.out_idx):
            out_set = set(self.out_idx)
            ins = [p for i, p in enumerate(params) if i not in out_set]
            if self.ir.sym_dims:
                bindings = self._bind_symbols_pairs(zip(ins, arguments))
            allocated = self._allocate_outputs(arguments, bindings)
            out_map = dict(zip(self.out_idx, allocated))
            it = iter(arguments)
            arguments = tuple(out_map[i] if i in out_map else next(it) for i in range(len(params)))
        if len(arguments) != len(params):
            raise TypeError(f"Expected {len(params)} arguments, received {len(arguments)}")
        if self.ir.sym_dims:
            bindings = self._bind_symbols(arguments)
            missing = [s.name for s in self.ir.sym_dims if s.name not in bindings]
            if missing:
                raise ValueError(f"Unbound symbolic dimensions: {', '.join(missing)}")
        if self._state is None:
            self._state = self._call_state()
        plan = self._state
        torch = _torch()
        tensor_type = torch.Tensor
        devices = set()
        ranges = []
        checked = []
        first = None
        for tensor, param, entry in zip(arguments, params, plan):
            if entry is None:
                checked.append(validate_scalar(tensor, param))
                continue
            checked.append(tensor)
            _, static_shape, tdtype, static_size = entry
            if type(tensor) is tensor_type:  # fast path: a torch tensor
                if not tensor.is_cuda:
                    raise TypeError(f"{param.name} must be a CUDA tensor supporting DLPack")
                devices.add(tensor.get_device())
                expected = static_shape if static_shape is not None else self._resolve(param.type.shape, bindings)
                if tensor.shape != expected:
                    raise ValueError(f"{param.name}: expected shape {expected}, got {tuple(tensor.shape)}")
                if tensor.dtype is not tdtype:
                    raise ValueError(f"{param.name}: expected dtype {param.type.dtype}, got {tensor.dtype}")
            else:
                if not hasattr(tensor, "__dlpack_device__") or tensor.__dlpack_device__()[0] != 2:
                    raise TypeError(f"{param.name} must be a CUDA tensor supporting DLPack")
                devices.add(tensor.__dlpack_device__()[1])
                expected = self._resolve(param.type.shape, bindings)
                if tuple(tensor.shape) != expected:
                    raise ValueError(f"{param.name}: expected shape {expected}, got {tuple(tensor.shape)}")
                if str(tensor.dtype).split(".")[-1] != param.type.dtype:
                    raise ValueError(f"{param.name}: expected dtype {param.type.dtype}, got {tensor.dtype}")
            if not tensor.is_contiguous():
                raise ValueError(f"{param.name} must be contiguous in row-major order")
            pointer = tensor.data_ptr()
            if pointer % 16:
                raise ValueError(f"{param.name} requires a tensor with an inspectable, 16-byte-aligned data pointer")
            size = static_size
            if size is None:
                size = DTYPES[param.type.dtype]
                for d in expected:
                    size *= d
            for start, end, name in ranges:
                if pointer < end and start < pointer + size:
                    raise ValueError(f"Tensor arguments {name} and {param.name} must have disjoint storage")
            ranges.append((pointer, pointer + size, param.name))
            if first is None:
                first = tensor
        if len(devices) > 1:
            raise ValueError("All tensor arguments must be on the same CUDA device")
        if not devices:
            raise TypeError("a kernel launch needs at least one CUDA tensor argument")
        if not self._built:
            self.build()
        run = self._run
        if run is None:
            run = self._run = make_launcher(self.spec)
        (index,) = devices
        if index == torch.cuda.current_device():
            run(checked, _current_stream(torch, index), bindings)
        else:
            with torch.cuda.device(first.device):
                run(checked, _current_stream(torch, index), bindings)
        if allocated is not None:
            return allocated[0] if len(allocated) == 1 else tuple(allocated)
        return None

    @staticmethod
    def _bind_symbols_pairs(pairs) -> dict:
        """Bind symbolic dimensions from (parameter, argument) pairs of the inputs only."""
        bindings = {}
        for param, arg in pairs:
            if isinstance(param, ScalarParameter) or not hasattr(arg, "shape"):
                continue
            for spec_dim, actual in zip(param.type.shape, arg.shape):
                if isinstance(spec_dim, SymDim):
                    bindings[spec_dim.name] = int(actual)
        return bindings


def lower_program(prog: Program) -> OpSpec:
    """The op a program runs: a recognised family (prebuilt sm_100a kernel), else a generic
    elementwise kernel generated as CUDA C for NVRTC; ``CompileError`` when neither applies."""
    try:
        return recognize(prog)
    except CompileError as family_error:
        try:
            kernel = lower_pointwise(prog)
        except CompileError as pointwise_error:
            raise CompileError(f"{family_error}\n  pointwise: {pointwise_error}") from None
        return OpSpec("pointwise", {"kernel": kernel, "points": kernel.points}, {})


def make_kernel(prog: Program, spec: OpSpec, target: str, out_idx) -> CompiledKernel:
    normalized = normalize_out_idx(out_idx, prog.params)
    source = standalone_module(spec, prog, prog.name, target, str(_lib.library_path()))
    return CompiledKernel(prog, target, source, out_idx=normalized, spec=spec)


def compile(program: PrimFunc, *, target="sm_100a", out_idx=None, pass_configs=None) -> CompiledKernel:
    """Read a ``@T.prim_func`` and pick its kernel: a recognised op family (prebuilt for
    sm_100a, nothing compiled per program) or a generic elementwise kernel (CUDA C, compiled
    by NVRTC on first launch).  Other programs raise ``CompileError``."""
    del pass_configs
    resolved = resolve_target(target)
    prog = read_program(program)
    return make_kernel(prog, lower_program(prog), resolved, out_idx)


class DynamicJitKernel:
    """Kernels with ``T.dynamic`` dimensions.

    The first call tries one symbolic compile (sizes are runtime arguments of the C ABI);
    if recognition needs a concrete size it falls back to per-shape specialisation.
    """

    def __init__(self, program: PrimFunc, *, target="auto", out_idx=None, pass_configs=None, symbolic=True):
        self.program = program
        self.target = target
        self.out_idx = out_idx
        self.pass_configs = pass_configs
        self.symbolic = symbolic
        self._cache: dict = {}
        self._symbolic_cache: dict = {}
        self._param_names = tuple(inspect.signature(program.function).parameters)
        self._annotations = self._resolve_annotations()

    @property
    def compile_count(self) -> int:
        return sum(1 for v in self._symbolic_cache.values() if v is not None) + len(self._cache)

    def _env(self):
        fn = self.program.function
        env = dict(fn.__globals__)
        env.update(dict(self.program.annotation_locals))
        try:
            env.update(inspect.getclosurevars(fn).nonlocals)
        except (TypeError, ValueError):
            pass
        return env

    def _resolve_annotations(self):
        env = self._env()
        out = {}
        for name in self._param_names:
            ann = self.program.function.__annotations__.get(name)
            if isinstance(ann, str):
                try:
                    ann = eval(ann, env)  # noqa: S307 - the user's own annotation
                except Exception:
                    pass
            out[name] = ann
        return out

    def _out_set(self):
        if self.out_idx is None:
            return set()
        raw = (self.out_idx,) if isinstance(self.out_idx, int) else tuple(self.out_idx)
        n = len(self._param_names)
        return {i + n if i < 0 else i for i in raw}

    def _try_symbolic(self, target):
        if not self.symbolic:
            return None
        if target not in self._symbolic_cache:
            try:
                self._symbolic_cache[target] = compile(self.program, target=target, out_idx=self.out_idx)
            except CompileError:
                self._symbolic_cache[target] = None
        return self._symbolic_cache[target]

    def specialize(self, *arguments) -> CompiledKernel:
        n = len(self._param_names)
        out_set = self._out_set()
        if len(arguments) == n:
            pairs = list(zip(self._param_names, arguments))
        elif out_set and len(arguments) == n - len(out_set):
            pairs = list(zip([p for i, p in enumerate(self._param_names) if i not in out_set], arguments))
        else:
            expected = n - len(out_set) if out_set else n
            raise TypeError(f"Expected {expected} arguments, received {len(arguments)}")
        bindings = {}
        for name, arg in pairs:
            ann = self._annotations.get(name)
            if not isinstance(ann, SymbolicTensorSpec):
                continue
            if not hasattr(arg, "shape"):
                raise TypeError(f"{name}: expected tensor argument with .shape")
            shape = tuple(int(d) for d in arg.shape)
            if len(shape) != len(ann.shape):
                raise ValueError(f"{name}: expected rank {len(ann.shape)}, got {len(shape)}")
            for spec_dim, actual in zip(ann.shape, shape):
                if isinstance(spec_dim, SymbolicDim):
                    prev = bindings.get(spec_dim.name)
                    if prev is not None and prev != actual:
                        raise ValueError(f"Symbolic dimension {spec_dim.name!r} mismatch: {prev} vs {actual}")
                    bindings[spec_dim.name] = actual
                elif spec_dim != actual:
                    raise ValueError(f"{name}: expected static dim {spec_dim}, got {actual}")
        target = resolve_target(self.target)
        key = (tuple(sorted(bindings.items())), target)
        if key not in self._cache:
            special = dict(bindings)
            for var, val in self._env().items():
                if isinstance(val, SymbolicDim) and val.name in bindings:
                    special[var] = bindings[val.name]
            prog = PrimFunc(self.program.function, self.program.annotation_locals, tuple(sorted(special.items())))
            self._cache[key] = compile(prog, target=target, out_idx=self.out_idx)
        return self._cache[key]

    def __call__(self, *arguments):
        kernel = self._try_symbolic(resolve_target(self.target))
        if kernel is not None:
            return kernel(*arguments)
        return self.specialize(*arguments)(*arguments)


__all__ = ["CompiledKernel", "DynamicJitKernel", "compile"]
