"""Scaling sweep: fetch GB/s per requester and fetch->hook latency over token counts and distributions.

The sweep shape of the project's benchmark configuration 4: FP8 e4m3, hidden 256,
2 scale packs, ept 24, 2 layers of 524288 rows per rank; tokens 256 / 1024 /
4096 / 16384; uniform and Zipf(1.1) requests.  Every point uses fresh indices per
step, flushes the L2 between steps, times each step with CUDA events and takes
the maximum over ranks.  With ``--with-baseline`` the torch NCCL all_to_all
baseline is measured on the same points.

Run: ``python -m torch.distributed.run --nnodes 1 --nproc-per-node N
--master-addr 127.0.0.1 benchmarks/scaling_sweep.py``; rank 0 prints one JSON
line per point.
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

from engram_rdma_lab_b200 import EngramBuffer, TorchEngramBuffer  # noqa: E402
from engram_rdma_lab_b200.models import make_indices, quantized_fp8_shard  # noqa: E402
from engram_rdma_lab_b200.utils.timing import L2Flusher, percentile  # noqa: E402


def measure(buf, entries, tokens, ept, dist_name, rank, world, steps, warmup, flush):
    pool = [make_indices(rank, world, entries, tokens, ept, epoch=e + 1, distribution=dist_name, device="cuda")
            for e in range(4)]
    times = []
    for k in range(warmup + steps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        [h() for h in buf.fetch(pool[k % len(pool)])]
        b.record()
        b.synchronize()
        if k >= warmup:
            times.append(a.elapsed_time(b))
    t = torch.tensor(times, dtype=torch.float64, device="cuda")
    gathered = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(gathered, t)
    per_step = torch.stack(gathered).max(dim=0).values.tolist()
    mean = sum(per_step) / len(per_step)
    return mean, percentile(per_step, 0.5), percentile(per_step, 0.99)


def main():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--tokens", default="256,1024,4096,16384")
    p.add_argument("--distributions", default="uniform,zipf")
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--with-baseline", action="store_true")
    p.add_argument("--hot-rows", default="", help="ENGRAM_HOT_ROWS for our buffer (hot-prefix replica)")
    p.add_argument("--kernels", default="auto",
                   help="comma-separated ENGRAM_GATHER_KERNEL values to compare for our buffer, e.g. bulk,simt")
    args = p.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                            timeout=datetime.timedelta(seconds=300))
    os.environ["ENGRAM_EGM_ENABLE"] = "1"
    os.environ.setdefault("ENGRAM_WRITE_LOCAL_SF", "1")
    if args.hot_rows:
        os.environ["ENGRAM_HOT_ROWS"] = args.hot_rows
    entries, hidden, ept, packs, dtype = (524288, 524288), 256, 24, 2, torch.float8_e4m3fn
    token_list = [int(t) for t in args.tokens.split(",")]
    cap = max(token_list)
    storages, scales = quantized_fp8_shard(rank, world, entries, hidden, packs, "cuda")
    flush = L2Flusher()
    impls = [(f"ours:{k}" if k != "auto" else "ours", EngramBuffer, k) for k in args.kernels.split(",")]
    impls += [("nccl_all_to_all", TorchEngramBuffer, None)] if args.with_baseline else []
    group = dist.group.WORLD
    for name, cls, kernel in impls:
        if kernel:
            os.environ["ENGRAM_GATHER_KERNEL"] = kernel
        sizes = cls.get_storage_size_hint(group, entries, hidden, cap, ept, dtype, packs)
        buf = cls(group, *sizes, True, 4, 1024, explicitly_destroy=True)
        buf.set_config(entries, hidden, cap, ept, dtype, packs)
        buf.write(storages, scales)
        for dist_name in args.distributions.split(","):
            for tokens in token_list:
                mean, p50, p99 = measure(buf, entries, tokens, ept, dist_name, rank, world, args.steps,
                                         args.warmup, flush)
                nbytes = len(entries) * tokens * ept * hidden
                if rank == 0:
                    print(json.dumps({"impl": name, "gpus": world, "tokens": tokens, "distribution": dist_name,
                                      "hot_rows": getattr(buf, "hot_rows", None) or None,
                                      "per_requester_gbs": round(nbytes / (mean * 1e-3) / 1e9, 1),
                                      "mean_us": round(mean * 1e3, 1), "p50_us": round(p50 * 1e3, 1),
                                      "p99_us": round(p99 * 1e3, 1)}), flush=True)
        dist.barrier()
        buf.destroy()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
