"""``import ntilang`` / ``import ntilang.language as T``: the reference's package name.

This module replaces itself (and its ``language`` / ``layout`` submodules) in
``sys.modules`` with ``ntilang_b200`` so programs written for Ntilang run unchanged.
"""

import sys

import ntilang_b200 as _impl
from ntilang_b200 import autotune as _autotune
from ntilang_b200 import compat as _compat
from ntilang_b200 import compiler as _compiler
from ntilang_b200 import ir as _ir
from ntilang_b200 import language as _language
from ntilang_b200 import layout as _layout
from ntilang_b200 import pipeline as _pipeline

sys.modules[__name__] = _impl
for _name, _mod in (("language", _language), ("layout", _layout), ("compiler", _compiler), ("ir", _ir),
                    ("compat", _compat), ("autotune", _autotune), ("pipeline", _pipeline)):
    sys.modules[f"{__name__}.{_name}"] = _mod
