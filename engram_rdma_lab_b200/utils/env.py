"""Scoped environment overrides (reference: ``deepep/deep_ep/utils/envs.py:22-37``)."""

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
