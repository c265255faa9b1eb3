"""Measure this node's peer-memory envelope through the EngramBuffer's own mappings.

Two families of measurements, every rank at the same time, device time as the
maximum over ranks:

* ``stream``: every rank streams 50 MiB to or from the next rank (a ring, so
  every GPU both sends and receives) with 16-byte SM loads from the peer
  ("pull") or SM stores into it ("push").
* ``rows``: every rank moves random 256-byte rows to or from pseudo-random
  remote peers (all-to-all, the traffic of a uniform fetch) with each access
  mechanism of ``csrc/kernels/peer_probe.cu``: 16- and 32-byte register
  loads, 16-byte cp.async into a shared ring, 16- and 32-byte stores, bulk
  stores from shared memory, stores into consecutive peer rows (a staging
  pattern), streaming row loads; plus pull and push sharing one launch.

These are the roofline denominators of the NVLink-bound kernels.

Run: ``python -m torch.distributed.run --nnodes 1 --nproc-per-node N
--master-addr 127.0.0.1 benchmarks/peer_bandwidth.py [--family rows]``;
rank 0 prints one JSON line per measurement.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from engram_rdma_lab_b200 import EngramBuffer  # noqa: E402

MODES = {"pull_v4": 0, "pull_v4_deep": 1, "pull_v8": 2, "pull_ldgsts": 3, "push_v4": 4, "push_v8": 5,
         "push_bulk": 6, "push_seq_v8": 7, "pull_seq_v8": 8, "pull_v8_l2": 9}
ROW_CASES = [("pull_v4", "pull_v4"), ("pull_v8", "pull_v8"), ("pull_v8_l2", "pull_v8_l2"), ("pull_ldgsts", "pull_ldgsts"), ("push_v4", "push_v4"),
             ("push_v8", "push_v8"), ("push_bulk", "push_bulk"), ("push_seq_v8", "push_seq_v8"),
             ("pull_seq_v8", "pull_seq_v8"), ("pull_v8", "push_v8")]


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--family", choices=["stream", "rows", "all"], default="all")
    p.add_argument("--rows", type=int, default=172032, help="rows per rank per launch (rows family)")
    p.add_argument("--repeats", type=int, default=8)
    p.add_argument("--blocks", default="296", help="comma-separated grid sizes (rows family)")
    return p.parse_args()


def timed(fn, repeats):
    samples = []
    for _ in range(repeats):
        dist.barrier()
        samples.append(fn())
    samples = sorted(samples[2:])
    us = torch.tensor([samples[len(samples) // 2]])
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    return float(us)


def main():
    args = parse()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    os.environ["ENGRAM_EGM_ENABLE"] = "1"
    group = dist.group.WORLD
    # The headline table (268 MB of 256-byte rows per rank, larger than L2) and
    # its output region (2 x 4096 x 24 rows = 48 MiB) are the probe's windows.
    entries, hidden, tokens, ept = (524288, 524309), 256, 4096, 24
    dtype, packs = torch.float8_e4m3fn, 2
    sizes = EngramBuffer.get_storage_size_hint(group, entries, hidden, tokens, ept, dtype, packs)
    buf = EngramBuffer(group, *sizes, True, 4, 1024, explicitly_destroy=True)
    buf.set_config(entries, hidden, tokens, ept, dtype, packs)
    rt = buf.runtime
    if args.family in ("stream", "all"):
        nbytes = 50 << 20
        peer = (rank + 1) % world
        for mode in ("pull", "push", "local"):
            for blocks in (296, 1184):
                target = rank if mode == "local" else peer
                us = timed(lambda: rt.debug_peer_copy(target, nbytes, mode == "push", blocks), args.repeats)
                if rank == 0:
                    print(json.dumps({"family": "stream", "mode": mode, "ranks": world, "blocks": blocks,
                                      "bytes": nbytes, "us": round(us, 2),
                                      "gbs_per_gpu": round(nbytes / (us * 1e-6) / 1e9, 1)}), flush=True)
    if args.family in ("rows", "all"):
        nbytes = args.rows * hidden
        for even, odd in ROW_CASES:
            for blocks in (int(b) for b in args.blocks.split(",")):
                seed = [0]

                def once():
                    seed[0] += 1
                    return rt.debug_peer_probe(MODES[even], MODES[odd], args.rows, blocks, 50, seed[0])

                us = timed(once, args.repeats)
                if rank == 0:
                    name = even if even == odd else f"{even}+{odd}"
                    print(json.dumps({"family": "rows", "mode": name, "ranks": world, "blocks": blocks,
                                      "rows": args.rows, "row_bytes": hidden, "us": round(us, 2),
                                      "gbs_per_gpu": round(nbytes / (us * 1e-6) / 1e9, 1)}), flush=True)
    dist.barrier()
    buf.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
