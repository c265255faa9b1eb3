"""Measure this node's peer-memory envelope through the EngramBuffer's own mappings.

Every rank streams 50 MiB to or from the next rank at the same time (a ring,
so every GPU both sends and receives), once with SM loads from the peer
("pull", what the peer-HBM gather does) and once with SM stores into the peer
("push", what the owner push does).  The device time is the maximum over
ranks.  These are the roofline denominators for the NVLink-bound kernels.

Run: ``python -m torch.distributed.run --nnodes 1 --nproc-per-node N
--master-addr 127.0.0.1 benchmarks/peer_bandwidth.py``; rank 0 prints one JSON
line per measurement.
"""

from __future__ import annotations

import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from engram_rdma_lab_b200 import EngramBuffer  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    os.environ["ENGRAM_EGM_ENABLE"] = "1"
    group = dist.group.WORLD
    # The output region (2 x 4096 x 24 x 512 B = 96 MiB) is the copy window.
    entries, hidden, tokens, ept = (4096, 4096), 256, 4096, 24
    sizes = EngramBuffer.get_storage_size_hint(group, entries, hidden, tokens, ept, torch.bfloat16, 0)
    buf = EngramBuffer(group, *sizes, True, 4, 1024, explicitly_destroy=True)
    buf.set_config(entries, hidden, tokens, ept, torch.bfloat16, 0)
    nbytes = 50 << 20
    peer = (rank + 1) % world
    for mode in ("pull", "push", "local"):
        for blocks in (296, 1184):
            samples = []
            for _ in range(8):
                dist.barrier()
                target = rank if mode == "local" else peer
                samples.append(buf.runtime.debug_peer_copy(target, nbytes, mode == "push", blocks))
            samples = sorted(samples[2:])
            us = torch.tensor([samples[len(samples) // 2]])
            dist.all_reduce(us, op=dist.ReduceOp.MAX)
            if rank == 0:
                print(json.dumps({"mode": mode, "ranks": world, "blocks": blocks, "bytes": nbytes,
                                  "us": round(float(us), 2),
                                  "gbs_per_gpu": round(nbytes / (float(us) * 1e-6) / 1e9, 1)}), flush=True)
    dist.barrier()
    buf.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
