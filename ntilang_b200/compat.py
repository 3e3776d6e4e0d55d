"""Drop-in helpers: target resolution, ``out_idx`` normalisation, ``import tilelang`` patching
and dtype mapping.

Behaviour follows the reference's ``python/ntilang/compat.py``: ``resolve_target``
(:11-25), ``normalize_out_idx`` (:28-50), ``patch_tilelang`` (:53-88) and
``torch_dtype_for`` (:91-111).
"""

from __future__ import annotations

import sys

from .ir import CompileError, ScalarParameter


def resolve_target(target="auto") -> str:
    """'auto' / 'cuda' / None -> 'sm_XY' of the current device; 'cuda:sm_XY' -> 'sm_XY'."""
    if target is None or target in ("auto", "cuda"):
        torch = sys.modules.get("torch")
        if torch is not None:
            try:
                if torch.cuda.is_available():
                    major, minor = torch.cuda.get_device_capability()
                    return f"sm_{major}{minor}"
            except Exception:
                pass
        return "sm_100a"
    if isinstance(target, str) and target.startswith("cuda:"):
        return target[5:]
    return target


def normalize_out_idx(out_idx, parameters) -> tuple:
    """int or sequence of ints, negatives allowed; no scalars, no duplicates."""
    if out_idx is None:
        return ()
    raw = (out_idx,) if isinstance(out_idx, int) else tuple(out_idx)
    count = len(parameters)
    result = []
    for index in raw:
        if type(index) is not int:
            raise TypeError(f"out_idx entries must be integers, got {index!r}")
        resolved = index + count if index < 0 else index
        if not 0 <= resolved < count:
            raise ValueError(f"out_idx {index} is out of range for {count} kernel parameters")
        if isinstance(parameters[resolved], ScalarParameter):
            raise ValueError(f"out_idx {index} cannot refer to scalar parameter {parameters[resolved].name!r}")
        if resolved in result:
            raise ValueError(f"Duplicate out_idx {index}")
        result.append(resolved)
    return tuple(result)


class _TileLangPatch:
    """Routes ``import tilelang`` (and ``.language`` / ``.layout``) to this package.

    Usable directly or as a context manager that restores the previous modules.
    """

    KEYS = ("tilelang", "tilelang.language", "tilelang.layout")

    def __init__(self):
        import ntilang_b200 as package
        from ntilang_b200 import language, layout

        pkg = sys.modules.get("ntilang", package)
        self._previous = {key: sys.modules.get(key) for key in self.KEYS}
        sys.modules["tilelang"] = pkg
        sys.modules["tilelang.language"] = language
        sys.modules["tilelang.layout"] = layout
        self._active = True

    def restore(self) -> None:
        if not self._active:
            return
        for key, prev in self._previous.items():
            if prev is None:
                sys.modules.pop(key, None)
            else:
                sys.modules[key] = prev
        self._active = False

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        self.restore()
        return False


def patch_tilelang() -> _TileLangPatch:
    return _TileLangPatch()


def torch_dtype_for(dtype_name: str, torch_module):
    mapping = {
        "bool": torch_module.bool,
        "int8": torch_module.int8,
        "int16": torch_module.int16,
        "int32": torch_module.int32,
        "int64": torch_module.int64,
        "uint8": torch_module.uint8,
        "uint16": getattr(torch_module, "uint16", None),
        "uint32": getattr(torch_module, "uint32", None),
        "uint64": getattr(torch_module, "uint64", None),
        "float16": torch_module.float16,
        "bfloat16": torch_module.bfloat16,
        "float32": torch_module.float32,
        "float64": torch_module.float64,
    }
    resolved = mapping.get(dtype_name)
    if resolved is None:
        raise CompileError(f"PyTorch does not expose dtype {dtype_name!r} for out_idx allocation")
    return resolved


__all__ = ["normalize_out_idx", "patch_tilelang", "resolve_target", "torch_dtype_for"]
