"""Drop-in helpers: target strings, ``out_idx`` normalisation, ``import tilelang`` redirection and
the dtype used to allocate outputs.

Interface points with the reference (``python/ntilang/compat.py``): ``resolve_target`` accepts
the same spellings (:11-25), ``normalize_out_idx`` keeps the reference's rules and exception
messages (:28-50; its tests and users' error handling see them), ``patch_tilelang`` is usable
directly or as a context manager (:53-88), and ``torch_dtype_for`` raises ``CompileError`` for a
dtype torch cannot allocate (:91-111).
"""

from __future__ import annotations

import re
import sys

from .ir import DTYPES, CompileError, ScalarParameter

# The kernels in libntl_kernels.so are built for this architecture only.
NATIVE_TARGET = "sm_100a"
_ARCH = re.compile(r"^(?:cuda:)?(sm_\d+[a-z]?)$")


def _device_arch():
    """``sm_<major><minor>`` of torch's current CUDA device, with the ``a`` suffix this library
    compiles for on sm_100; None without a usable device."""
    torch = sys.modules.get("torch")
    if torch is None:
        return None
    try:
        if not torch.cuda.is_available():
            return None
        major, minor = torch.cuda.get_device_capability()
    except Exception:  # noqa: BLE001 - no driver, no device: the default target applies
        return None
    arch = f"sm_{major}{minor}"
    return arch + "a" if (major, minor) == (10, 0) else arch


def resolve_target(target="auto") -> str:
    """'auto', 'cuda' and None name the current device (sm_100a without one); 'cuda:sm_XY' and
    'sm_XY' name that architecture; any other string is returned unchanged."""
    if target is None or target in ("auto", "cuda"):
        return _device_arch() or NATIVE_TARGET
    if isinstance(target, str):
        match = _ARCH.match(target)
        if match:
            return match.group(1)
    return target


def normalize_out_idx(out_idx, parameters) -> tuple:
    """``out_idx`` as a tuple of non-negative parameter indices.

    An int or a sequence of ints; negative values count from the end.  Each must name a tensor
    parameter, once."""
    if out_idx is None:
        return ()
    requested = [out_idx] if isinstance(out_idx, int) else list(out_idx)
    total = len(parameters)
    chosen: list = []
    for entry in requested:
        if type(entry) is not int:
            raise TypeError(f"out_idx entries must be integers, got {entry!r}")
        position = entry % total if -total <= entry < 0 else entry
        if not 0 <= position < total:
            raise ValueError(f"out_idx {entry} is out of range for {total} kernel parameters")
        target = parameters[position]
        if isinstance(target, ScalarParameter):
            raise ValueError(f"out_idx {entry} cannot refer to scalar parameter {target.name!r}")
        if position in chosen:
            raise ValueError(f"Duplicate out_idx {entry}")
        chosen.append(position)
    return tuple(chosen)


_REDIRECTED = ("tilelang", "tilelang.language", "tilelang.layout")


class TileLangRedirect:
    """Points ``tilelang``, ``tilelang.language`` and ``tilelang.layout`` in ``sys.modules`` at
    this package while active; ``restore()`` (or leaving a ``with`` block) puts back whatever was
    there before, removing entries that did not exist."""

    def __init__(self):
        import ntilang_b200
        from ntilang_b200 import language, layout

        package = sys.modules.get("ntilang", ntilang_b200)
        replacement = dict(zip(_REDIRECTED, (package, language, layout)))
        self._saved = {name: sys.modules.get(name) for name in _REDIRECTED}
        sys.modules.update(replacement)
        self.active = True

    def restore(self) -> None:
        if self.active:
            self.active = False
            for name, module in self._saved.items():
                if module is not None:
                    sys.modules[name] = module
                else:
                    sys.modules.pop(name, None)

    def __enter__(self):
        return self

    def __exit__(self, *exc_info):
        self.restore()
        return False


def patch_tilelang() -> TileLangRedirect:
    """Make ``import tilelang`` load this package (see ``TileLangRedirect``)."""
    return TileLangRedirect()


def torch_dtype_for(dtype_name: str, torch_module):
    """The torch dtype for one of the canonical dtype names (they are torch's attribute names:
    bool, int8…int64, uint8…uint64, float16, bfloat16, float32, float64).  Older torch builds
    lack the wide unsigned types; asking for one there raises ``CompileError``."""
    found = getattr(torch_module, dtype_name, None) if dtype_name in DTYPES else None
    if found is None:
        raise CompileError(f"cannot allocate an output of dtype {dtype_name!r}: this PyTorch has no such dtype")
    return found


__all__ = ["NATIVE_TARGET", "TileLangRedirect", "normalize_out_idx", "patch_tilelang", "resolve_target",
           "torch_dtype_for"]
