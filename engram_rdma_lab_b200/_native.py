"""Loader for the in-tree native extension ``engram_rdma_lab_b200._C``.

On a machine with a CUDA device the native runtime is mandatory: a missing or
stale build raises instead of silently falling back to a slower path.  On a
CPU-only machine the module may be absent; :func:`load` then raises
``ImportError`` and only the pure-torch oracle is usable.
"""

from __future__ import annotations

import importlib

_C = None
_ERROR = None


def load():
    """Return the extension module or raise ImportError with a build hint."""
    global _C, _ERROR
    if _C is not None:
        return _C
    try:
        _C = importlib.import_module("engram_rdma_lab_b200._C")
    except ImportError as error:  # pragma: no cover - exercised on unbuilt trees
        _ERROR = error
        raise ImportError(
            "engram_rdma_lab_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"in the repository root ({error})"
        ) from error
    return _C


def available() -> bool:
    try:
        load()
        return True
    except ImportError:
        return False
