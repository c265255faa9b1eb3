"""Every benchmark configuration of the project at the launched world size.

One process per GPU (``python -m torch.distributed.run --nnodes 1
--nproc-per-node N --master-addr 127.0.0.1 benchmarks/baseline_configs.py``);
rank 0 prints one JSON line per measured point.  Every point builds its own
buffer through the public API, writes random-init tables, checks one fetch
bit-exactly against every owner's tables, then times steps with CUDA events.
Before each step a device barrier lines the ranks up (the L2 flush runs before
it, outside the events); the step time is the maximum over ranks.  Clocks are
sampled with nvidia-smi during each point.

* ``1``  BF16, host shards, owner-push route: 2 layers x 524288 / 524309 rows,
  hidden 256, ept 24, 4096 tokens, 2% padding.  Roofline: the bytes each owner
  reads from its pinned host shard per step at the PCIe rate measured here
  (SM zero-copy reads of 48 MiB, every rank at once).
* ``2``  the FP8 headline shape with mixed routes: the pair (requester, owner)
  is on the host route when requester + owner is odd, else on the peer-HBM
  route (probe results altered on the host, as a failed mapping would).
* ``3`` / ``3h``  FP8 CUDA-graph replay: 4 layers x 2,097,143 rows, hidden 512,
  4 scale packs, ept 24, 8192 tokens.  Each replay draws Zipf(1.1) indices
  with 5% padding and empties each layer with probability 1/4 inside the
  graph, calls the hooks in reverse order on another stream and overlaps a
  bf16 8192x4096x4096 GEMM on a third stream.  ``3h`` adds the hot-prefix
  replica (``ENGRAM_HOT_ROWS=262144``).  The same graph without the GEMM and
  the GEMM alone are timed too.
* ``4``  the scaling sweep: FP8 hidden 256, ept 24, 2 x 524288 rows; tokens
  256 / 1024 / 4096 / 16384; uniform (deduplication ``auto``) and Zipf(1.1)
  (deduplication on); ours and the NCCL all_to_all baseline on the same
  points.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from engram_rdma_lab_b200 import EngramBuffer, TorchEngramBuffer, _native  # noqa: E402
from engram_rdma_lab_b200.models import (  # noqa: E402
    expected_random_init,
    make_indices,
    normal_bf16_shard,
    quantized_fp8_shard,
)
from engram_rdma_lab_b200.utils.timing import ClockSampler, L2Flusher, percentile  # noqa: E402


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--configs", default="1,2,3,3h,4")
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--sweep-tokens", default="256,1024,4096,16384")
    return p.parse_args()


class Ctx:
    def __init__(self, args):
        self.args = args
        self.rank, self.world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        self.local = int(os.environ.get("LOCAL_RANK", self.rank))
        torch.cuda.set_device(self.local)
        from engram_rdma_lab_b200.utils.numa import bind_to_device_numa

        self.numa = bind_to_device_numa(self.local)  # pinned shards on this GPU's socket
        dist.init_process_group("nccl", rank=self.rank, world_size=self.world,
                                device_id=torch.device("cuda", self.local), timeout=datetime.timedelta(seconds=600))
        self.flush = L2Flusher()
        visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu_index = int(visible[self.local]) if visible and visible[self.local].isdigit() else self.local

    def emit(self, line):
        if self.rank == 0:
            print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- helpers
def build(cls, entries, hidden, tokens, ept, dtype, packs, env, probe=None):
    """A configured, written buffer; ``env`` is applied while it is built."""
    saved = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    C = _native.load()
    original = C.Runtime.probe_routes
    if probe is not None:
        C.Runtime.probe_routes = lambda rt, peers, cand: original(rt, probe(peers), cand)
    try:
        group = dist.group.WORLD
        sizes = cls.get_storage_size_hint(group, entries, hidden, tokens, ept, dtype, packs)
        cfg = cls.get_theoretical_config(group, len(entries), tokens, ept)
        buf = cls(group, *sizes, True, *cfg, num_gpu_timeout_secs=60, explicitly_destroy=True)
        buf.set_config(entries, hidden, tokens, ept, dtype, packs)
    finally:
        C.Runtime.probe_routes = original
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    rank, world = buf.rank_idx, buf.num_ranks
    if packs:
        storages, scales = quantized_fp8_shard(rank, world, entries, hidden, packs, "cuda")
    else:
        storages, scales = normal_bf16_shard(rank, world, entries, hidden, "cuda"), None
    buf.write(storages, scales)
    del storages, scales
    torch.cuda.empty_cache()
    return buf


def verify(outs, idx, entries, hidden, dtype, packs, world):
    want = expected_random_init(idx, entries, hidden, dtype, packs, world)
    T = idx.shape[1]
    bad = 0
    for layer, out in enumerate(outs):
        data, sf = out if packs else (out, None)
        bad += int(data.view(torch.uint8).reshape(T, -1).ne(want[layer][0]).sum())
        if packs:
            bad += int(sf.ne(want[layer][1]).sum())
    everyone = [None] * world
    dist.all_gather_object(everyone, bad)
    if any(everyone):
        raise SystemExit(f"verification failed: values differing per rank {everyone}")
    return True


def timed(ctx, step, align):
    """Aligned, flushed, event-timed steps; returns (mean, p50, p99) ms of the per-step max over ranks."""
    a = ctx.args
    for k in range(a.warmup):
        align()
        step(k)
    torch.cuda.synchronize()
    dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(a.steps)]
    for k in range(a.steps):
        ctx.flush()
        align()
        starts[k].record()
        step(k)
        ends[k].record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) for s, e in zip(starts, ends)], dtype=torch.float64, device="cuda")
    everyone = [torch.zeros_like(ms) for _ in range(ctx.world)]
    dist.all_gather(everyone, ms)
    per_step = torch.stack(everyone).max(dim=0).values.tolist()
    return sum(per_step) / len(per_step), percentile(per_step, 0.5), percentile(per_step, 0.99)


def clocks(ctx, sampler):
    mine = sampler.summary()
    everyone = [None] * ctx.world
    dist.all_gather_object(everyone, mine)
    return {"sm_mhz": [c.get("sm_mhz") for c in everyone], "sm_max_mhz": mine.get("sm_max_mhz"),
            "reasons": sorted({r for c in everyone for r in (c.get("reasons") or [])})}


def point(ctx, config, impl, buf, step, nbytes, verified, extra=None):
    align = buf.device_barrier
    with ClockSampler(gpu_index=ctx.gpu_index) as sampler:
        mean, p50, p99 = timed(ctx, step, align)
    line = {"config": config, "impl": impl, "gpus": ctx.world, "verified": verified,
            "per_requester_gbs": round(nbytes / (mean * 1e-3) / 1e9, 2), "mean_us": round(mean * 1e3, 1),
            "p50_us": round(p50 * 1e3, 1), "p99_us": round(p99 * 1e3, 1), "bytes_per_requester": nbytes,
            "clocks": clocks(ctx, sampler)}
    line.update(extra or {})
    ctx.emit(line)
    return mean


def pcie_envelope(ctx):
    """SM zero-copy read rate of 48 MiB of pinned host memory, every rank at once (GB/s per GPU)."""
    C = _native.load()
    src = torch.empty(48 << 20, dtype=torch.uint8).pin_memory()
    dst = torch.empty(48 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        C.host_read(src, dst, 2368)
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(5):
        C.host_read(src, dst, 2368)
    b.record()
    b.synchronize()
    gbs = torch.tensor([5 * (48 << 20) / (a.elapsed_time(b) * 1e-3) / 1e9], device="cuda")
    dist.all_reduce(gbs, op=dist.ReduceOp.MIN)
    return float(gbs)


def fetch_step(buf, pool):
    return lambda k: buf.fetch_all(pool[k % len(pool)])


# ----------------------------------------------------------------------------- configs
def config1(ctx):
    entries, hidden, tokens, ept = (524288, 524309), 256, 4096, 24
    envelope = pcie_envelope(ctx)
    buf = build(EngramBuffer, entries, hidden, tokens, ept, torch.bfloat16, 0, {"ENGRAM_EGM_ENABLE": "0"})
    pool = [make_indices(ctx.rank, ctx.world, entries, tokens, ept, epoch=e + 1, padding=0.02, device="cuda")
            for e in range(4)]
    ok = verify(buf.fetch_all(pool[0]), pool[0], entries, hidden, torch.bfloat16, 0, ctx.world)
    nbytes = len(entries) * tokens * ept * hidden * 2
    mean = point(ctx, "1_bf16_host_push", "ours", buf, fetch_step(buf, pool), nbytes, ok)
    # Uniform requests: each owner reads 1/world of every requester's rows from its host shard.
    host_bytes = nbytes * 0.98
    ctx.emit({"config": "1_bf16_host_push", "roofline": {
        "owner_host_read_bytes_per_step": int(host_bytes), "pcie_sm_read_envelope_gbs": round(envelope, 1),
        "owner_host_read_gbs": round(host_bytes / (mean * 1e-3) / 1e9, 1),
        "fraction_of_pcie_envelope": round(host_bytes / (mean * 1e-3) / 1e9 / envelope, 3)}})
    buf.destroy()


def config2_mixed(ctx):
    entries, hidden, tokens, ept, packs = (524288, 524309), 256, 4096, 24, 2
    rank = ctx.rank

    def probe(peers):
        altered = [dict(p) for p in peers]
        for owner in range(len(altered)):
            if owner != rank and (owner + rank) % 2 == 1:
                altered[owner]["mirror_bytes"] = 0  # this pair falls back to the host route
        return altered

    buf = build(EngramBuffer, entries, hidden, tokens, ept, torch.float8_e4m3fn, packs, {"ENGRAM_EGM_ENABLE": "1"},
                probe)
    routes = buf.get_route_info()["owner_routes"]
    pool = [make_indices(ctx.rank, ctx.world, entries, tokens, ept, epoch=e + 1, device="cuda") for e in range(4)]
    ok = verify(buf.fetch_all(pool[0]), pool[0], entries, hidden, torch.float8_e4m3fn, packs, ctx.world)
    nbytes = len(entries) * tokens * ept * hidden
    point(ctx, "2_fp8_mixed_routes", "ours", buf, fetch_step(buf, pool), nbytes, ok,
          {"rank0_routes": routes if ctx.rank == 0 else None})
    buf.destroy()


class ZipfProducer:
    """Capturable per-replay indices: Zipf(s) ids, padding, and layers emptied at random."""

    def __init__(self, entries, world, tokens, ept, s=1.1, padding=0.05, empty=0.25):
        total = entries[0] * world
        assert all(n == entries[0] for n in entries)
        ranks = torch.arange(1, total + 1, dtype=torch.float64, device="cuda")
        cdf = torch.cumsum(ranks.pow(-s), 0)
        self.cdf, self.total = cdf / cdf[-1], total
        self.idx = torch.empty(len(entries), tokens, ept, dtype=torch.int32, device="cuda")
        self.padding, self.empty = padding, empty

    def __call__(self):
        L, T, E = self.idx.shape
        u = torch.rand(L * T * E, dtype=torch.float64, device="cuda")
        x = torch.searchsorted(self.cdf, u).clamp_max(self.total - 1).view(L, T, E)
        drop = (torch.rand(L, T, E, device="cuda") < self.padding) | (torch.rand(L, 1, 1, device="cuda") < self.empty)
        self.idx.copy_(torch.where(drop, torch.full_like(x, -1), x))


def config3(ctx, hot):
    entries, hidden, tokens, ept, packs = (2097143,) * 4, 512, 8192, 24, 4
    env = {"ENGRAM_EGM_ENABLE": "1"}
    if hot:
        env["ENGRAM_HOT_ROWS"] = "262144"
    buf = build(EngramBuffer, entries, hidden, tokens, ept, torch.float8_e4m3fn, packs, env)
    produce = ZipfProducer(entries, ctx.world, tokens, ept)
    a_mat = torch.randn(8192, 4096, device="cuda", dtype=torch.bfloat16)
    b_mat = torch.randn(4096, 4096, device="cuda", dtype=torch.bfloat16)
    gemm_stream, hook_stream = torch.cuda.Stream(), torch.cuda.Stream()
    outs = [None] * len(entries)

    def forward(with_gemm):
        produce()
        hooks = buf.fetch(produce.idx)
        main = torch.cuda.current_stream()
        if with_gemm:
            gemm_stream.wait_stream(main)
            with torch.cuda.stream(gemm_stream):
                torch.mm(a_mat, b_mat)
        hook_stream.wait_stream(main)
        with torch.cuda.stream(hook_stream):
            for layer in reversed(range(len(hooks))):
                outs[layer] = hooks[layer]()
        main.wait_stream(hook_stream)
        if with_gemm:
            main.wait_stream(gemm_stream)

    graphs = {}
    for with_gemm in (True, False):
        for _ in range(2):
            forward(with_gemm)
        torch.cuda.synchronize()
        dist.barrier()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            forward(with_gemm)
        graphs[with_gemm] = g
    graphs[True].replay()
    torch.cuda.synchronize()
    ok = verify(outs, produce.idx, entries, hidden, torch.float8_e4m3fn, packs, ctx.world)
    nbytes = len(entries) * tokens * ept * hidden
    name = "3_fp8_graph_zipf" + ("_hot_rows" if hot else "")
    extra = {"hot_rows": buf.hot_rows, "note": "per replay: Zipf(1.1) draw + fetch + reverse cross-stream hooks"}
    point(ctx, name, "ours", buf, lambda k: graphs[True].replay(), nbytes, ok,
          dict(extra, gemm_overlapped="bf16 8192x4096x4096"))
    point(ctx, name, "ours", buf, lambda k: graphs[False].replay(), nbytes, ok, dict(extra, gemm_overlapped=None))
    gemm_ms = []
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.mm(a_mat, b_mat)
        e.record()
        e.synchronize()
        gemm_ms.append(s.elapsed_time(e))
    ctx.emit({"config": name, "gemm_alone_us": round(statistics.median(gemm_ms) * 1e3, 1),
              "dedup_last_unique_ratio": buf.memory_usage()["dedup_last_unique_ratio"]})
    del graphs
    buf.destroy()


def config4(ctx):
    """Scaling sweep.  Each (implementation, distribution) gets its own buffer:
    ``ENGRAM_DEDUP=auto`` decides from the fetches it has seen and re-measures
    only every 256 fetches once it is off, so a buffer that served uniform
    requests first would keep deduplication off for the few Zipf fetches here.
    Zipf points run with ``ENGRAM_DEDUP=1``, what ``auto`` picks on a steady
    Zipf stream from its first fetch."""
    entries, hidden, ept, packs = (524288, 524288), 256, 24, 2
    token_list = [int(t) for t in ctx.args.sweep_tokens.split(",")]
    cap = max(token_list)
    for impl, cls in (("ours", EngramBuffer), ("nccl_all_to_all", TorchEngramBuffer)):
        for dist_name in ("uniform", "zipf"):
            env = {"ENGRAM_EGM_ENABLE": "1", "ENGRAM_DEDUP": "1" if dist_name == "zipf" else "auto"}
            buf = build(cls, entries, hidden, cap, ept, torch.float8_e4m3fn, packs, env)
            for tokens in token_list:
                pool = [make_indices(ctx.rank, ctx.world, entries, tokens, ept, epoch=e + 1, distribution=dist_name,
                                     device="cuda") for e in range(4)]
                ok = verify(buf.fetch_all(pool[0]), pool[0], entries, hidden, torch.float8_e4m3fn, packs, ctx.world)
                nbytes = len(entries) * tokens * ept * hidden
                extra = {"tokens": tokens, "distribution": dist_name}
                if impl == "ours":
                    extra["dedup"] = env["ENGRAM_DEDUP"]
                point(ctx, "4_scaling_sweep", impl, buf, fetch_step(buf, pool), nbytes, ok, extra)
                if impl != "ours":
                    ctx.emit({"config": "4_scaling_sweep", "impl": impl, "tokens": tokens,
                              "distribution": dist_name, "phases_last_step": buf.phase_ms()})
            dist.barrier()
            buf.destroy()


def main():
    ctx = Ctx(parse())
    for name in ctx.args.configs.split(","):
        if name == "1":
            config1(ctx)
        elif name == "2":
            config2_mixed(ctx)
        elif name in ("3", "3h"):
            config3(ctx, hot=name == "3h")
        elif name == "4":
            config4(ctx)
        else:
            raise SystemExit(f"unknown config {name!r}")
        dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
