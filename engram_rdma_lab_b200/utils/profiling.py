"""NVTX ranges and torch.profiler helpers (reference: ``benchmarks/test_write.py:315-389``).

``nvtx_range`` marks host submission scopes (fetch issue, hook wait, owner
service launches) so they show up in a torch.profiler / Nsight timeline.
"""

from __future__ import annotations

import contextlib

import torch


@contextlib.contextmanager
def nvtx_range(name: str, enabled: bool = True):
    if not enabled or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def record_function(name: str, enabled: bool = True):
    return torch.profiler.record_function(name) if enabled else contextlib.nullcontext()


def cuda_profiler(enabled: bool = True):
    """A torch.profiler collecting CPU and CUDA activity (or a null context)."""
    if not enabled:
        return contextlib.nullcontext()
    return torch.profiler.profile(
        activities=[torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA],
        record_shapes=True,
    )
