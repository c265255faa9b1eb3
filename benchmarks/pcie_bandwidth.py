"""PCIe envelope of one GPU: copy-engine H2D against SM zero-copy reads of pinned host memory.

The kernels that read host memory (the gather over pinned host indices, the
host route's owner push from a pinned shard) are bounded by this envelope.
For each size, pinned host memory is moved to the GPU back to back (a) by the
copy engine (``Tensor.copy_`` from pinned memory) and (b) by SM 16-byte loads
through the memory's device mapping (``_C.host_read``), timed with CUDA events
after warm-up; then both again from write-combined pinned memory
(``_C.alloc_pinned``, the allocation behind ``EngramBuffer.pinned_indices``).
One JSON line per size.

Run: ``python benchmarks/pcie_bandwidth.py``.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from engram_rdma_lab_b200 import _native  # noqa: E402


def timed_us(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) * 1e3 / iters


def main():
    C = _native.load()
    torch.cuda.set_device(0)
    for size in (786432, 6 << 20, 48 << 20):
        src = torch.randint(0, 255, (size,), dtype=torch.uint8).pin_memory()
        dst = torch.empty(size, dtype=torch.uint8, device="cuda")
        iters = 50 if size < (8 << 20) else 10
        row = {"bytes": size, "copy_engine_us": round(timed_us(lambda: dst.copy_(src, non_blocking=True), iters), 1)}
        for blocks in (148, 592, 2368):
            row[f"sm_read_{blocks}_us"] = round(timed_us(lambda: C.host_read(src, dst, blocks), iters), 1)
        torch.cuda.synchronize()
        assert torch.equal(dst.cpu(), src), "host_read copied wrong bytes"
        # The same source bytes in write-combined pinned memory (_C.alloc_pinned).
        wc = C.alloc_pinned(size, True)
        wc.copy_(src)
        row["copy_engine_wc_us"] = round(timed_us(lambda: dst.copy_(wc, non_blocking=True), iters), 1)
        row["sm_read_wc_592_us"] = round(timed_us(lambda: C.host_read(wc, dst, 592), iters), 1)
        torch.cuda.synchronize()
        assert torch.equal(dst.cpu(), src), "write-combined copy moved wrong bytes"
        best = min(v for k, v in row.items() if k.endswith("_us"))
        row["best_gbs"] = round(size / best / 1e3, 1)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
