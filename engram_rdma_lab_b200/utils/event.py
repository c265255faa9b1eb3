"""Stream/event helper for overlapping work with a fetch.

``EventOverlap`` wraps a CUDA event recorded on one stream; entering it as a
context manager lets the caller queue independent work, and leaving it makes the
current stream wait for the event.  Tensors passed as ``extra_tensors`` stay
alive until the wait, which replaces ``record_stream`` under CUDA Graph capture.
Parity: ``deepep/deep_ep/utils/event.py:8-106`` (not used by the Engram path
there either; kept for callers that build on it).
"""

from __future__ import annotations

import torch


class EventOverlap:
    def __init__(self, event: torch.cuda.Event | None = None, extra_tensors=None):
        self.event = event
        self.extra_tensors = extra_tensors
        self.hook_after_wait = None
        self._release = False

    @classmethod
    def record(cls, stream: torch.cuda.Stream | None = None, extra_tensors=None) -> "EventOverlap":
        event = torch.cuda.Event()
        event.record(stream or torch.cuda.current_stream())
        return cls(event, extra_tensors)

    def current_stream_wait(self, release_handle: bool = False):
        if self.event is None:
            raise RuntimeError("EventOverlap has no event")
        torch.cuda.current_stream().wait_event(self.event)
        result = None
        if self.hook_after_wait is not None:
            result, self.hook_after_wait = self.hook_after_wait(), None
        if release_handle:
            self.event, self.extra_tensors = None, None
        return result

    def wait(self):
        return self.current_stream_wait()

    def register_hook_after_wait(self, hook):
        if self.hook_after_wait is not None:
            raise RuntimeError("A hook is already registered on this EventOverlap")
        self.hook_after_wait = hook

    def __call__(self, release_handle: bool = False) -> "EventOverlap":
        self._release = release_handle
        return self

    def __enter__(self):
        return self

    def __exit__(self, *_):
        if self.event is not None:
            self.current_stream_wait(release_handle=self._release)
        self._release = False
        return False
