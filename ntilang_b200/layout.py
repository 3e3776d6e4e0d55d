"""``tilelang.layout`` helpers.  Layout hints are accepted and ignored: the sm_100a
kernels stage their operands in the 128-byte-swizzled layouts TMA and tcgen05 use.

Same names as the reference's ``python/ntilang/layout.py:8-22``.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class SwizzledLayout:
    buffer: object
    is_a: bool = False
    is_b: bool = False


def make_swizzled_layout(buffer, is_a: bool = False, is_b: bool = False) -> SwizzledLayout:
    return SwizzledLayout(buffer=buffer, is_a=is_a, is_b=is_b)


__all__ = ["SwizzledLayout", "make_swizzled_layout"]
