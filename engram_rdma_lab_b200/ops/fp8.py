"""FP8 e4m3 block quantisation used to build FP8 vocabularies (torch ops only).

Each row is split into blocks of ``block`` columns (128 by default, the
granularity of one scale pack).  A block's scale is ``amax / 448`` (448 is the
largest finite e4m3 value), optionally rounded up to a power of two so that
dequantisation is exact in binary floating point (the UE8M0 convention).  The
codes are ``round_to_e4m3(x / scale)``; dequantisation multiplies back.
``calc_diff`` measures how far a dequantised table is from its source.
Parity: ``deepep/deep_ep/utils/math.py:30-56`` (``per_token_cast_to_fp8`` /
``per_token_cast_back``, ``calc_diff``), rewritten without ``torch.compile``.
"""

from __future__ import annotations

import torch

E4M3_MAX = 448.0


def quantize_fp8_blockwise(x: torch.Tensor, block: int = 128, power_of_two: bool = False, eps: float = 1e-4):
    """Quantise ``x [m, n]`` to ``(codes [m, n] e4m3, scales [m, ceil(n/block)] fp32)``."""
    if x.dim() != 2:
        raise ValueError("expected a 2-D tensor")
    m, n = x.shape
    blocks = (n + block - 1) // block
    padded = torch.nn.functional.pad(x.float(), (0, blocks * block - n))
    view = padded.view(m, blocks, block)
    amax = view.abs().amax(dim=2).clamp_min(eps)
    scale = amax / E4M3_MAX
    if power_of_two:
        scale = torch.pow(2.0, torch.ceil(torch.log2(scale)))
    codes = (view / scale[:, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return codes.view(m, blocks * block)[:, :n].contiguous(), scale.contiguous()


def dequantize_fp8_blockwise(codes: torch.Tensor, scales: torch.Tensor, block: int = 128,
                             dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """Inverse of :func:`quantize_fp8_blockwise` (scales may be strided)."""
    m, n = codes.shape
    if codes.numel() == 0:
        return codes.to(dtype)
    blocks = (n + block - 1) // block
    padded = torch.nn.functional.pad(codes.float(), (0, blocks * block - n)).view(m, blocks, block)
    out = padded * scales.float().reshape(m, blocks, 1)
    return out.view(m, blocks * block)[:, :n].to(dtype)


def calc_diff(x: torch.Tensor, y: torch.Tensor) -> float:
    """Dissimilarity of ``x`` and ``y``: 1 - 2<x', y'> / (|x'|^2 + |y'|^2) with x' = x + 1, y' = y + 1.

    0 means identical; a blockwise FP8 round trip of N(0, 1) data stays below 1e-3.
    """
    x, y = x.double() + 1, y.double() + 1
    denominator = (x * x + y * y).sum()
    return float((1 - 2 * (x * y).sum() / denominator).item())
