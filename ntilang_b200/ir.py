"""Tensor/dtype vocabulary shared by the front end, the recognizer and the launcher.

Mirrors the names the reference exposes from ``python/ntilang/ir.py``:
``DTYPES`` (ir.py:8-22), ``CompileError`` (ir.py:51-55), ``SymDim`` (ir.py:58-63) and
``TensorType`` (ir.py:66-86, including the 2**31-1 element cap).  The rest of the
reference's tile IR (Buffer/Region/Statement/Kernel) is not reproduced: this package
recognises whole-kernel op families instead of lowering an arbitrary tile program.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import prod

# dtype name -> size in bytes
DTYPES = {
    "bool": 1,
    "int8": 1,
    "int16": 2,
    "int32": 4,
    "int64": 8,
    "uint8": 1,
    "uint16": 2,
    "uint32": 4,
    "uint64": 8,
    "float16": 2,
    "bfloat16": 2,
    "float32": 4,
    "float64": 8,
}

DTYPE_ALIASES = {
    "short": "int16",
    "int": "int32",
    "uint": "uint32",
    "long": "int64",
    "ulong": "uint64",
    "half": "float16",
    "float": "float32",
    "double": "float64",
}

FLOAT_DTYPES = ("float16", "bfloat16", "float32", "float64")


def canonical_dtype(name) -> str:
    name = str(name)
    name = DTYPE_ALIASES.get(name, name)
    if name not in DTYPES:
        raise CompileError(f"Unsupported dtype {name!r}; supported: {', '.join(DTYPES)}")
    return name


def integer_limits(dtype: str) -> tuple[int, int]:
    if dtype == "bool":
        return 0, 1
    bits = DTYPES[dtype] * 8
    if dtype.startswith("uint"):
        return 0, 2**bits - 1
    if dtype.startswith("int"):
        return -(2 ** (bits - 1)), 2 ** (bits - 1) - 1
    raise ValueError(f"{dtype} is not an integer dtype")


@dataclass(frozen=True)
class SourceLocation:
    filename: str
    line: int
    column: int = 0


class CompileError(ValueError):
    """Raised for programs outside the recognised op families or with invalid structure."""

    def __init__(self, message: str, location: SourceLocation | None = None):
        self.location = location
        prefix = f"{location.filename}:{location.line}:{location.column + 1}: " if location else ""
        super().__init__(prefix + message)


@dataclass(frozen=True)
class SymDim:
    """A symbolic tensor dimension bound from argument shapes at call time."""

    name: str
    divisibility: int = 1


@dataclass(frozen=True)
class TensorType:
    shape: tuple
    dtype: str

    def __post_init__(self):
        object.__setattr__(self, "dtype", canonical_dtype(self.dtype))
        if not self.shape or any(
            not isinstance(n, SymDim) and (type(n) is not int or n <= 0) for n in self.shape
        ):
            raise CompileError("Tensor dimensions must be positive static integers")
        if not self.is_symbolic and prod(self.shape) > 2**31 - 1:
            raise CompileError("Tensor sizes exceeding signed 32-bit indexing are not supported")

    @property
    def is_symbolic(self) -> bool:
        return any(isinstance(n, SymDim) for n in self.shape)


@dataclass(frozen=True)
class TensorParameter:
    name: str
    type: TensorType


@dataclass(frozen=True)
class ScalarParameter:
    name: str
    dtype: str


__all__ = [
    "DTYPES",
    "DTYPE_ALIASES",
    "CompileError",
    "ScalarParameter",
    "SourceLocation",
    "SymDim",
    "TensorParameter",
    "TensorType",
    "canonical_dtype",
    "integer_limits",
]
