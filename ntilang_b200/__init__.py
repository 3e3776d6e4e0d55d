"""ntilang_b200: the kernels Ntilang's compiler emits, rebuilt as hand-written sm_100a CUDA
behind Ntilang's own ``jit`` / ``compile`` operator surface.

``import ntilang`` (the sibling alias package) and ``ntilang.patch_tilelang()`` expose this
package under the reference's names (python/ntilang/__init__.py:1-25).
"""

from . import language, layout
from .autotune import AutoTuner, autotune
from .compat import patch_tilelang
from .compiler import CompiledKernel, DynamicJitKernel, compile
from .ir import CompileError, SymDim
from .language import jit
from .pipeline import Compiler

__version__ = "0.1.0"
__all__ = [
    "AutoTuner",
    "CompileError",
    "CompiledKernel",
    "Compiler",
    "DynamicJitKernel",
    "SymDim",
    "autotune",
    "compile",
    "jit",
    "language",
    "layout",
    "patch_tilelang",
]
