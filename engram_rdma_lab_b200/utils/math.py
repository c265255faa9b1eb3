"""Integer helpers shared by the memory plan (reference: ``deepep/deep_ep/utils/math.py``)."""

from __future__ import annotations


def ceil_div(x: int, y: int) -> int:
    return (x + y - 1) // y


def align(x: int, y: int) -> int:
    return ceil_div(x, y) * y
