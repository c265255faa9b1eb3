"""Device timing, L2 flushing and clock sampling for benchmarks.

* :class:`L2Flusher` writes a buffer larger than the 126 MB L2 so that the next
  timed step starts cold.
* :func:`event_ms` times a callable with CUDA events on the current stream.
* :class:`ClockSampler` runs ``nvidia-smi`` in the background during a timed
  region and summarises SM clocks and active throttle reasons.  It only reads
  GPU state.
"""

from __future__ import annotations

import statistics
import subprocess
import tempfile
import time

import torch

L2_FLUSH_BYTES = 256 << 20


class L2Flusher:
    """Evict the L2 between timed steps.

    Writes a buffer twice the L2 size, then reads it back: the write evicts
    every line the previous step left behind, and the read makes the flush's
    own dirty lines drain to DRAM here, outside the timed region, instead of
    during the next step.
    """

    def __init__(self, nbytes: int = L2_FLUSH_BYTES, device=None):
        self.buffer = torch.empty(nbytes // 4, dtype=torch.int32, device=device or "cuda")
        self.sink = torch.empty((), dtype=torch.int64, device=device or "cuda")
        self._value = 0

    def __call__(self):
        self._value ^= 1
        self.buffer.fill_(self._value)
        torch.sum(self.buffer, dim=0, dtype=torch.int64, out=self.sink)


def event_ms(fn, stream=None) -> float:
    stream = stream or torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def percentile(values, q: float) -> float:
    if not values:
        return float("nan")
    ordered = sorted(values)
    k = (len(ordered) - 1) * q
    lo, hi = int(k), min(int(k) + 1, len(ordered) - 1)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (k - lo)


_QUERY = (
    "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
    "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
    "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
)
_REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """Background ``nvidia-smi`` sampler (200 ms period) for one GPU index."""

    def __init__(self, gpu_index: int | None = None, period_ms: int = 200):
        self.gpu_index, self.period_ms = gpu_index, period_ms
        self.proc, self.file = None, None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={_QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"],
                stdout=self.file, stderr=subprocess.DEVNULL,
            )
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *_):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if self.file is None or self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.seek(0)
        sm, sm_max, reasons = [], [], set()
        for line in self.file.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                index = int(parts[0])
            except ValueError:
                continue
            if self.gpu_index is not None and index != self.gpu_index:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(_REASONS, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        self.file.close()
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(sm_max) if sm_max else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }
