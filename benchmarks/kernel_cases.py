"""Single-GPU cases of the Engram kernels, for CUDA-event timing and ncu captures.

Each case builds a one-rank EngramBuffer on ``cuda:0`` with the headline
table shape (2 layers x 524288 / 524309 rows of 256 bytes, 268 MB per rank,
larger than the L2) and runs one kernel ``--launches`` times, printing one
JSON line per case with the median CUDA-event time and the bytes moved:

* ``gather``: ``fetch_all`` of 4096 tokens x 24 uniform entries (FP8 with
  two scale packs): the SIMT gather, 256-bit or 128-bit vectors
  (``ENGRAM_GATHER_VECTOR``), or the TMA ring (``ENGRAM_GATHER_KERNEL=bulk``);
* ``dedup``: the same fetch with Zipf(1.1) indices, so the dedup and expand
  kernels run around the gather;
* ``push`` / ``hook``: the host route's serving code moving one request of
  ``--rows`` rows of this rank to itself, read zero-copy from the pinned host
  shard (or, with ``--mirror``, from the HBM mirror) by the push kernel
  (``--blocks`` CTAs) or by a serving hook kernel.

Run: ``python benchmarks/kernel_cases.py --case gather [--launches 20]``.  Under
ncu, capture one launch after the warm-up ones (``-k regex:<kernel> -s 3 -c 1``).
"""

from __future__ import annotations

import argparse
import json
import os
import socket
import statistics
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from engram_rdma_lab_b200 import EngramBuffer  # noqa: E402
from engram_rdma_lab_b200.models import make_indices, normal_bf16_shard, quantized_fp8_shard  # noqa: E402

ENTRIES, HIDDEN, TOKENS, EPT = (524288, 524309), 256, 4096, 24


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--case", choices=["gather", "dedup", "push", "hook"], required=True)
    p.add_argument("--launches", type=int, default=20)
    p.add_argument("--rows", type=int, default=98304, help="rows of the served request (push / hook)")
    p.add_argument("--blocks", default="8", help="push CTAs, comma-separated for a sweep")
    p.add_argument("--mirror", action="store_true",
                   help="push / hook: serve from the HBM mirror (ENGRAM_EGM_ENABLE=1) instead of the pinned shard")
    return p.parse_args()


def buffer(fp8: bool, mirror: bool):
    os.environ["ENGRAM_EGM_ENABLE"] = "1" if mirror else "0"
    os.environ.setdefault("ENGRAM_WRITE_LOCAL_SF", "1")
    group = dist.group.WORLD
    dtype, packs = (torch.float8_e4m3fn, 2) if fp8 else (torch.bfloat16, 0)
    sizes = EngramBuffer.get_storage_size_hint(group, ENTRIES, HIDDEN, TOKENS, EPT, dtype, packs)
    cfg = EngramBuffer.get_theoretical_config(group, len(ENTRIES), TOKENS, EPT)
    buf = EngramBuffer(group, *sizes, True, *cfg, num_gpu_timeout_secs=2, explicitly_destroy=True)
    buf.set_config(ENTRIES, HIDDEN, TOKENS, EPT, dtype, packs)
    if fp8:
        storages, scales = quantized_fp8_shard(0, 1, ENTRIES, HIDDEN, packs, "cuda")
    else:
        storages, scales = normal_bf16_shard(0, 1, ENTRIES, HIDDEN, "cuda"), None
    buf.write(storages, scales)
    return buf


def time_fetches(buf, distribution, launches):
    pool = [make_indices(0, 1, ENTRIES, TOKENS, EPT, epoch=e + 1, distribution=distribution, device="cuda")
            for e in range(4)]
    samples = []
    for k in range(launches):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        buf.fetch_all(pool[k % len(pool)])
        b.record()
        torch.cuda.synchronize()
        samples.append(a.elapsed_time(b) * 1e3)
    return statistics.median(samples[2:] if len(samples) > 4 else samples)


def main():
    args = parse()
    torch.cuda.set_device(0)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("gloo", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{port}")
    line = {"case": args.case}
    if args.case in ("gather", "dedup"):
        os.environ["ENGRAM_DEDUP"] = "1" if args.case == "dedup" else os.environ.get("ENGRAM_DEDUP", "0")
        buf = buffer(fp8=True, mirror=True)
        us = time_fetches(buf, "zipf" if args.case == "dedup" else "uniform", args.launches)
        mem = buf.memory_usage()
        rows = len(ENTRIES) * TOKENS * EPT
        # rows read + written, indices, scales read + written (2 packs of fp32)
        nbytes = rows * HIDDEN * 2 + rows * 4 + rows * 2 * 4 * 2
        line.update(us=round(us, 2), kernel=mem["gather_kernel"], vector_bytes=mem["gather_vector_bytes"],
                    algorithmic_bytes=nbytes, gbs=round(nbytes / (us * 1e-6) / 1e9, 1),
                    dedup_unique_ratio=mem["dedup_last_unique_ratio"])
        print(json.dumps(line), flush=True)
    else:
        buf = buffer(fp8=False, mirror=args.mirror)
        line["source"] = "hbm_mirror" if args.mirror else "pinned_host_shard"
        line["chunk_rows"] = buf.memory_usage()["serve_chunk_rows"]
        for blocks in (int(b) for b in args.blocks.split(",")):
            runs = [buf.runtime.debug_serve_local(args.rows, args.case, blocks) for _ in range(args.launches)]
            bad = sum(r["mismatched_rows"] for r in runs)
            us = statistics.median(r["us"] for r in (runs[2:] if len(runs) > 4 else runs))
            nbytes = runs[0]["bytes"]
            print(json.dumps(dict(line, blocks=blocks if args.case == "push" else None, rows=args.rows,
                                  us=round(us, 2), bytes=nbytes, gbs=round(nbytes / (us * 1e-6) / 1e9, 2),
                                  mismatched_rows=bad)), flush=True)
    buf.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
