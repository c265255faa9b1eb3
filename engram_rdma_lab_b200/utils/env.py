"""Scoped environment overrides (reference: ``deepep/deep_ep/utils/envs.py:22-37``)
and the table of the buffer's ``ENGRAM_*`` knobs."""

from __future__ import annotations

import os


class EnvOverride:
    """Set ``(name, value, enabled)`` entries for the duration of a ``with`` block."""

    def __init__(self, envs):
        self.envs = {name: value for name, value, enabled in envs if enabled}
        self._saved = {}

    def __enter__(self):
        self._saved = {name: os.environ.get(name) for name in self.envs}
        os.environ.update(self.envs)
        return self

    def __exit__(self, *_):
        for name, value in self._saved.items():
            if value is None:
                os.environ.pop(name, None)
            else:
                os.environ[name] = value
        return False


# Every environment knob the buffer reads, with its default and meaning.
KNOBS = {
    "ENGRAM_EGM_ENABLE": ("0", "1 = prefer the peer-HBM route (adds an HBM mirror of the shard)"),
    "ENGRAM_WRITE_LOCAL_SF": ("= ENGRAM_EGM_ENABLE", "1 = full local FP8 scale table, 0 = each owner's rows only"),
    "ENGRAM_DEDUP": ("auto", "move each distinct row once per fetch: auto, 1 or 0"),
    "ENGRAM_GATHER_KERNEL": ("auto", "gather variant: auto = simt (vector loads), or bulk (TMA ring; bulk copies "
                                     "read peers' memory, opt-in)"),
    "ENGRAM_GATHER_CTAS_PER_SM": ("0", "SIMT grid cap per SM (0 = 2)"),
    "ENGRAM_GATHER_UNROLL": ("0", "SIMT row steps in flight for 256-byte rows (0 = 4)"),
    "ENGRAM_GATHER_STRIDED": ("0", "1 = SIMT warps stride over 32-row groups instead of equal ranges"),
    "ENGRAM_GATHER_VECTOR": ("auto", "SIMT bytes per load and store: auto (32 when rows come over NVLink, else 16), "
                                     "32 (256-bit, rows of 256 B and up) or 16"),
    "ENGRAM_GATHER_L2_PREFETCH": ("0", "1 = the SIMT gather's 32-byte loads carry the 256-byte L2 prefetch-size hint"),
    "ENGRAM_PEER_TRANSPORT": ("pull", "peer-HBM pairs: pull (requester loads from the owner's mirror) or push "
                                      "(the owner pushes from its mirror after a dispatch)"),
    "ENGRAM_SERVE_CHUNK_ROWS": ("512", "rows per claimed chunk of host-route and owner-push serving (multiple of 16, "
                                       "at most 512)"),
    "ENGRAM_HOST_VMM": ("1", "host shards as CUDA-VMM HOST_NUMA allocations (else memfd + cudaHostRegister)"),
    "ENGRAM_HOT_ROWS": ("", "replicate global ids [0, H) of each layer on every rank (H or H0,H1,...)"),
    "ENGRAM_NVTX": ("0", "1 = NVTX ranges around fetch, hooks, write and owner-service launches"),
    "ENGRAM_INDEX_STAGING": ("1", "1 = copy pinned host indices to the GPU on a side stream (overlaps the next "
                                  "step's H2D with this step's gather); 0 = the kernels read them in place"),
}


def describe_knobs(environ=None) -> dict:
    """``{name: value}`` of every ``ENGRAM_*`` knob: the set value, or ``default:<d>``."""
    environ = os.environ if environ is None else environ
    return {name: environ.get(name, f"default:{default}") for name, (default, _) in KNOBS.items()}
