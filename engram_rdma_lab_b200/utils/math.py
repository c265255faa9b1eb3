"""Small numeric helpers (reference: ``deepep/deep_ep/utils/math.py``)."""

from __future__ import annotations

import torch


def ceil_div(x: int, y: int) -> int:
    return (x + y - 1) // y


def align(x: int, y: int) -> int:
    return ceil_div(x, y) * y


def safe_div(a, b):
    """``a / b`` that maps ``0 / 0`` to 0 and raises on other divisions by zero."""
    if b == 0:
        if a == 0:
            return 0
        raise ZeroDivisionError(f"{a} / 0")
    return a / b


def calc_diff(x: torch.Tensor, y: torch.Tensor) -> float:
    """1 - cosine-style similarity of ``x + 1`` and ``y + 1`` (0 means identical)."""
    x, y = x.double() + 1, y.double() + 1
    denominator = (x * x + y * y).sum()
    return float((1 - 2 * (x * y).sum() / denominator).item())


def count_bytes(*tensors) -> int:
    total = 0
    for t in tensors:
        if isinstance(t, (tuple, list)):
            total += count_bytes(*t)
        elif t is not None:
            total += t.numel() * t.element_size()
    return total


def hash_tensors(*tensors) -> int:
    """Order-insensitive XOR of per-tensor byte sums (a cheap change detector)."""
    value = 0
    for t in tensors:
        if isinstance(t, (tuple, list)):
            value ^= hash_tensors(*t)
        elif isinstance(t, torch.Tensor):
            value ^= int(t.contiguous().view(torch.uint8).to(torch.int64).sum().item())
    return value
