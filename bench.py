"""Headline benchmark: Engram fetch GB/s per requester and fetch->hook latency.

Workload (the reference's headline shape, ``README.md:123,130`` and
``benchmarks/test_read.py:19-20,288-291``): FP8 e4m3 rows of hidden=256 with
two 128-column fp32 scale packs, 2 layers of 524288 / 524309 rows per rank,
4096 tokens x 24 entries per token per requester, uniform requests over all
``world * n`` global rows, random-init weights (N(0,1) e4m3 codes with
power-of-two scales).  Every rank is a requester and an owner ("all-to-all"
traffic).

One step = ``fetch(indices)`` plus every layer hook, i.e. the full lookup
(issue + transfer + scales) as the reference times it.  Each timed step uses a
fresh index tensor and the L2 is flushed (256 MiB write) between steps outside
the timed events.  Before each step's start event a device barrier across all
ranks (the buffer's own NVLink barrier; an NCCL all-reduce for the baseline)
lines the GPUs up, so every rank's step runs against every other rank's
traffic.  Times are CUDA events on the launching stream; the reported step
time is the maximum over ranks.  The same steps without the barrier
("free-running") are reported beside it.  Before timing, one fetch is checked
bit-exactly against the random-init tables of every owner.

Run: ``python bench.py [--gpus N --steps K --warmup W]``; for N > 1 under
``torchrun --nproc-per-node N``.  ``--impl nccl`` times the torch
``all_to_all`` baseline; ``--impl reference`` reports the reference build.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MIN_WARMUP = 3
BASELINE_GBS_PER_REQUESTER = 180.0  # upper end of the reference's published 175-180 GB/s/requester
METRIC = "Engram fetch GB/s/requester and p50 fetch→hook latency, 8×B200, 4096 tok"


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "nccl", "reference"], default="ours")
    p.add_argument("--config", default="fp8", help="table set from engram_rdma_lab_b200.models.CONFIGS")
    p.add_argument("--tokens", type=int, default=None)
    p.add_argument("--route", choices=["peer_hbm", "host"], default="peer_hbm",
                   help="peer_hbm: ENGRAM_EGM_ENABLE=1 (HBM mirror, NVLink pull); host: owner push from host shards")
    p.add_argument("--distribution", default=None)
    p.add_argument("--graph", action="store_true", help="replay fetch+hooks from a CUDA graph")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-numa-bind", action="store_true",
                   help="leave the CPU affinity alone (default: pin to the GPU's local CPUs before pinned allocations)")
    p.add_argument("--e2e-input", choices=["copy", "staged", "pinned"], default="staged",
                   help="end-to-end input path: a copy-engine H2D one step ahead on a side stream, the runtime's own "
                        "staging of pinned host indices, or pinned host indices read in place by the kernels")
    p.add_argument("--e2e-host-memory", choices=["pinned", "write-combined"], default="pinned",
                   help="end-to-end index buffers: torch pinned memory, or EngramBuffer.pinned_indices "
                        "(pinned, write-combined: the GPU reads it without snooping the CPU's caches)")
    p.add_argument("--no-clocks", action="store_true")
    p.add_argument("--no-verify", action="store_true",
                   help="skip the bit-exact check of one fetch against the random-init tables (outside the timing)")
    args = p.parse_args()
    # Timed numbers need at least 3 warm-up steps; the JSON line reports the count that ran.
    args.warmup_requested = args.warmup
    args.warmup = max(args.warmup, MIN_WARMUP)
    return args


def unavailable_reference():
    reason = (
        "reference cannot be built or run on this box: deep_ep needs an NCCL with the GIN/GDAKI device API "
        "(NCCL 2.28.9 here) and fails to compile against CUDA 12.9; engram_sge_write needs NCCL_ROOT with GIN "
        "plus ibverbs/mlx5 HCAs; both need 2 nodes x 4 GPUs with RDMA NICs"
    )
    print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)


NUMA = None
NUMA_OFF = "--no-numa-bind" in sys.argv


def init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    global NUMA
    if not NUMA_OFF:
        from engram_rdma_lab_b200.utils.numa import bind_to_device_numa

        NUMA = bind_to_device_numa(local)  # pinned inputs on this GPU's socket
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if world == 1:
            import socket

            with socket.socket() as s:
                s.bind(("127.0.0.1", 0))
                os.environ.setdefault("MASTER_PORT", str(s.getsockname()[1]))
        import datetime

        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def build_buffer(args, spec, rank, world):
    from engram_rdma_lab_b200 import EngramBuffer, TorchEngramBuffer
    from engram_rdma_lab_b200.models import quantized_fp8_shard, normal_bf16_shard

    os.environ["ENGRAM_EGM_ENABLE"] = "1" if args.route == "peer_hbm" else "0"
    os.environ.setdefault("ENGRAM_WRITE_LOCAL_SF", "1")
    if not args.no_e2e:
        # The runtime's staging copies pinned indices on its own side stream
        # ("staged"); the other two paths hand the kernels device indices or
        # pinned indices to read in place.
        os.environ["ENGRAM_INDEX_STAGING"] = "1" if args.e2e_input == "staged" else "0"
    cls = EngramBuffer if args.impl == "ours" else TorchEngramBuffer
    group = dist.group.WORLD
    sizes = cls.get_storage_size_hint(group, spec.entries, spec.hidden, spec.max_tokens, spec.ept, spec.dtype,
                                      spec.num_sf_packs)
    cfg = cls.get_theoretical_config(group, spec.layers, spec.max_tokens, spec.ept)
    buf = cls(group, *sizes, True, *cfg, num_gpu_timeout_secs=60, explicitly_destroy=True)
    buf.set_config(spec.entries, spec.hidden, spec.max_tokens, spec.ept, spec.dtype, spec.num_sf_packs)
    if spec.num_sf_packs:
        storages, scales = quantized_fp8_shard(rank, world, spec.entries, spec.hidden, spec.num_sf_packs, "cuda")
    else:
        storages, scales = normal_bf16_shard(rank, world, spec.entries, spec.hidden, "cuda"), None
    buf.write(storages, scales)
    del storages, scales
    torch.cuda.empty_cache()
    return buf


def verify_once(buf, spec, idx, world):
    """One fetch + hooks, checked bit-exactly against every owner's random-init rows."""
    from engram_rdma_lab_b200.models import expected_random_init

    outs = [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    want = expected_random_init(idx, spec.entries, spec.hidden, spec.dtype, spec.num_sf_packs, world)
    bad = 0
    T = idx.shape[1]
    for layer, out in enumerate(outs):
        data, sf = out if spec.num_sf_packs else (out, None)
        bad += int(data.view(torch.uint8).reshape(T, -1).ne(want[layer][0]).sum())
        if spec.num_sf_packs:
            bad += int(sf.ne(want[layer][1]).sum())
    everyone = [None] * world
    dist.all_gather_object(everyone, bad)  # every rank stops together on a mismatch
    if any(everyone):
        raise SystemExit(f"verification failed: values differing per rank {everyone}")
    return True


def timed_steps(args, steps, run, flush, align, stream, host_split):
    """``steps`` steps, each bracketed by CUDA events; returns per-step ms on this rank."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for k in range(steps):
        flush()
        if align is not None:
            align()
        starts[k].record(stream)
        run(k, host_split)
        ends[k].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def summarize(step_ms, steps, bytes_req):
    from engram_rdma_lab_b200.parallel import gather_floats
    from engram_rdma_lab_b200.utils.timing import percentile

    all_ms = gather_floats(step_ms)
    per_step_max = [max(r[k] for r in all_ms) for k in range(steps)]
    ms_per_step = max(sum(r) for r in all_ms) / steps
    return dict(ms_per_step=ms_per_step, per_requester_gbs=bytes_req / (ms_per_step * 1e-3) / 1e9,
                p50_us=statistics.median(per_step_max) * 1e3, p99_us=percentile(per_step_max, 0.99) * 1e3)


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            unavailable_reference()
        return
    rank, world, local = init()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    from engram_rdma_lab_b200.models import CONFIGS, make_indices
    from engram_rdma_lab_b200.utils.env import describe_knobs
    from engram_rdma_lab_b200.utils.timing import ClockSampler, L2Flusher

    spec = CONFIGS[args.config]
    if args.tokens:
        spec = spec.with_(tokens=args.tokens, max_tokens=max(spec.max_tokens, args.tokens))
    if args.distribution:
        spec = spec.with_(distribution=args.distribution)
    T = spec.tokens
    buf = build_buffer(args, spec, rank, world)
    pool_size = max(2, min(args.steps, 16))
    pool = [make_indices(rank, world, spec.entries, T, spec.ept, epoch=e + 1, distribution=spec.distribution,
                         padding=spec.padding, device="cuda") for e in range(pool_size)]
    flush = L2Flusher()
    stream = torch.cuda.current_stream()
    native = args.impl == "ours"
    verified = None if args.no_verify else verify_once(buf, spec, pool[0], world)
    if native:
        align = buf.device_barrier
    else:
        token = torch.zeros(1, device="cuda")
        align = lambda: dist.all_reduce(token)  # noqa: E731 - an NCCL kernel every rank must reach

    def step(idx, host_split=None):
        t0 = time.perf_counter()
        hooks = buf.fetch(idx)
        t1 = time.perf_counter()
        outs = [h() for h in hooks]
        if host_split is not None:
            host_split[0].append(t1 - t0)
            host_split[1].append(time.perf_counter() - t1)
        return outs

    graph, graph_idx = None, None
    if args.graph:
        graph_idx = pool[0].clone()
        for _ in range(2):
            step(graph_idx)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        before = buf.runtime.memory_usage()["kernel_launches"] if native else 0
        with torch.cuda.graph(graph):
            step(graph_idx)
        graph_launches = (buf.runtime.memory_usage()["kernel_launches"] - before) if native else 0

    def run(k, host_split=None):
        if graph is None:
            return step(pool[k % pool_size], host_split)
        graph_idx.copy_(pool[k % pool_size])
        graph.replay()
        return None

    for k in range(args.warmup):
        align()
        run(k)
    torch.cuda.synchronize()
    dist.barrier()

    launches_before = buf.runtime.memory_usage()["kernel_launches"] if native else 0
    sampler = ClockSampler(gpu_index=_physical_index(local)) if not args.no_clocks else None
    if sampler:
        sampler.__enter__()
    dist.barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    host_split = ([], [])
    aligned_ms = timed_steps(args, args.steps, run, flush, align, stream, host_split)
    wall = time.perf_counter() - wall0
    launches = (buf.runtime.memory_usage()["kernel_launches"] - launches_before) if native else 0
    dist.barrier()
    torch.cuda.synchronize()
    free_ms = timed_steps(args, args.steps, run, flush, None, stream, None)
    dist.barrier()
    if sampler:
        sampler.__exit__(None, None, None)
    if graph is not None:
        # Kernels replayed from the captured graph, plus one barrier per step.
        launches = (graph_launches + 1) * args.steps
    phases = buf.phase_ms() if not native and hasattr(buf, "phase_ms") else None
    bytes_req = spec.bytes_per_fetch(T)
    aligned = summarize(aligned_ms, args.steps, bytes_req)
    free = summarize(free_ms, args.steps, bytes_req)

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(buf, spec, pool, flush, args, rank, world, graph is not None)

    clocks = sampler.summary() if sampler else {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["not sampled"]}
    all_clocks = [None] * world
    dist.all_gather_object(all_clocks, clocks)
    host = [None] * world
    med = (lambda v: round(statistics.median(v) * 1e6, 2) if v else None)  # noqa: E731
    dist.all_gather_object(host, (med(host_split[0]), med(host_split[1])))
    if rank == 0:
        per_req_gbs = aligned["per_requester_gbs"]
        reasons = sorted({r for c in all_clocks for r in (c.get("reasons") or [])})
        line = {
            "metric": METRIC,
            "value": round(per_req_gbs * world, 3),
            "unit": "GB/s (sum over requesters)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            **({"warmup_requested": args.warmup_requested} if args.warmup_requested != args.warmup else {}),
            "ms_per_step": round(aligned["ms_per_step"], 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": round(per_req_gbs / BASELINE_GBS_PER_REQUESTER, 3),
            "dtype": "fp8_e4m3" if spec.num_sf_packs else "bf16",
            "data": f"synthetic (random-init tables, seeded {spec.distribution} indices)",
            "impl": "ours" if native else "nccl_all_to_all_baseline",
            "verified": verified,
            "per_requester_gbs": round(per_req_gbs, 3),
            "p50_fetch_to_hook_us": round(aligned["p50_us"], 2),
            "p99_fetch_to_hook_us": round(aligned["p99_us"], 2),
            "free_running": {"per_requester_gbs": round(free["per_requester_gbs"], 3),
                             "ms_per_step": round(free["ms_per_step"], 5), "p50_fetch_to_hook_us": round(free["p50_us"], 2),
                             "note": "same steps without the device barrier before each start event"},
            "host_us_p50": {"fetch_call": [h[0] for h in host], "hooks_calls": [h[1] for h in host]},
            "gpu_launches": int(launches),
            "wall_s_timed_loop": round(wall, 3),
            "e2e": e2e,
            "clocks": {"sm_mhz": clocks.get("sm_mhz"), "sm_max_mhz": clocks.get("sm_max_mhz"), "reasons": reasons,
                       "per_rank_sm_mhz": [c.get("sm_mhz") for c in all_clocks]},
            "config": {
                "model": f"engram {spec.name}: {spec.layers} layers x {list(spec.entries)} rows/rank, hidden "
                         f"{spec.hidden}, ept {spec.ept}, {spec.num_sf_packs} scale packs",
                "global_batch": T * world,
                "seq_len": T,
                "tokens_per_requester": T,
                "bytes_per_requester_per_step": bytes_req,
                "parallelism": f"vocab-sharded x{world} (every rank requester and owner)",
                "numa": NUMA,
                "hot_rows": getattr(buf, "hot_rows", None),
                "knobs": describe_knobs(),
                "route": args.route if native else "all_to_all",
                "graph": bool(args.graph),
                "distribution": spec.distribution,
                "l2": "flushed between timed steps (256 MiB write + read-back outside the events); fresh indices per step",
                "timing": "CUDA events per step on the launching stream, ranks aligned by a device barrier before "
                          "each start event, max over ranks",
                "baseline_gbs_per_requester": BASELINE_GBS_PER_REQUESTER,
            },
        }
        if phases is not None:
            line["baseline_phases_last_step"] = phases
        print(json.dumps(line), flush=True)
    buf.destroy()
    del graph
    dist.barrier()
    dist.destroy_process_group()


def measure_e2e(buf, spec, pool, flush, args, rank, world, use_graph):
    """Same metric through the public API, with every step's input H2D and result D2H.

    Every step hands ``fetch_all`` (fetch plus every layer's wait, one native
    call) the step's indices from pinned host memory, then reads token 0's rows
    of the last layer back into pinned host memory with SM stores through its
    device mapping (one native call on the compute stream, no copy engine), so
    the result never queues behind the next step's index copy.  Input paths
    (``--e2e-input``):

    * ``copy``: step k+1's indices are copied by the copy engine into one of
      two device buffers on a side stream while step k runs;
    * ``staged``: ``fetch_all`` gets the pinned tensor and the runtime copies
      it on its own side stream into one of two device slots
      (``ENGRAM_INDEX_STAGING=1``, the default; measured fastest: 25.2 µs per
      step at 1 GPU against 31.8 and 40.8 for the other two paths);
    * ``pinned``: ``fetch_all`` gets the pinned tensor and the lookup kernels
      read it in place over PCIe (``ENGRAM_INDEX_STAGING=0``).

    The host pool has 32 separate pinned index tensors (25 MB), cycled, so a
    step never finds its indices in a cache.  The time is one CUDA-event
    interval around all steps (max over ranks); no L2 flush runs inside it, and
    every step reads fresh random rows from a table larger than the L2.  The
    host time per step and the time of one index H2D alone are reported beside
    it, to show which of them bounds the loop.
    """
    compute = torch.cuda.current_stream()
    base = [p.cpu() for p in pool]
    if args.e2e_host_memory == "write-combined" and hasattr(buf, "pinned_indices"):
        host_pool = []
        for i in range(32):
            t = buf.pinned_indices(base[0].shape[1])
            t.copy_(base[i % len(base)])
            host_pool.append(t)
    else:
        host_pool = [base[i % len(base)].clone().pin_memory() for i in range(32)]
    row = spec.ept * spec.row_bytes
    out_host = torch.empty(row, dtype=torch.uint8).pin_memory()
    packs = spec.num_sf_packs
    mode = args.e2e_input
    copier = torch.cuda.Stream()
    dev = [torch.empty_like(pool[0]), torch.empty_like(pool[0])]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    consumed = [torch.cuda.Event(), torch.cuda.Event()]
    from engram_rdma_lab_b200 import _native

    host_write = _native.load().host_write
    readback = {}

    def read_back(outs):
        # Each step's result goes to the host with one native call: SM stores
        # into the pinned buffer's device mapping, ordered on the compute
        # stream, so it never queues behind the copy engine's index copies.
        key = id(outs[-1])
        if readback.get("key") != key:
            data = outs[-1][0] if packs else outs[-1]
            readback.update(key=key, src=data[0].view(torch.uint8) if data.shape[0] else None)
        if readback["src"] is not None:
            host_write(readback["src"], out_host, 1)

    def run_host(steps):
        for k in range(steps):
            read_back(buf.fetch_all(host_pool[k % len(host_pool)]))

    def run_copy(steps):
        with torch.cuda.stream(copier):
            dev[0].copy_(host_pool[0], non_blocking=True)
            ready[0].record(copier)
        for k in range(steps):
            slot, nxt = k % 2, (k + 1) % 2
            if k + 1 < steps:
                with torch.cuda.stream(copier):
                    if k >= 1:
                        copier.wait_event(consumed[nxt])  # step k-1 finished reading that buffer
                    dev[nxt].copy_(host_pool[(k + 1) % len(host_pool)], non_blocking=True)
                    ready[nxt].record(copier)
            compute.wait_event(ready[slot])
            outs = buf.fetch_all(dev[slot])
            consumed[slot].record(compute)
            read_back(outs)

    run = run_copy if mode == "copy" else run_host
    run(args.warmup)
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record(compute)
    run(args.steps)
    end.record(compute)
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    from engram_rdma_lab_b200.parallel import max_over_ranks

    ms_per_step = max_over_ranks(start.elapsed_time(end) / args.steps)
    host_us = max_over_ranks(host_s / args.steps * 1e6)
    # One index H2D alone, on an idle stream (the copy engine's share of a step).
    h2d = []
    for k in range(5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(compute)
        dev[0].copy_(host_pool[k], non_blocking=True)
        b.record(compute)
        torch.cuda.synchronize()
        h2d.append(a.elapsed_time(b) * 1e3)
    h2d_us = max_over_ranks(statistics.median(h2d))
    bytes_req = spec.bytes_per_fetch(pool[0].shape[1])
    per_req = bytes_req / (ms_per_step * 1e-3) / 1e9
    how = {"copy": "pinned H2D of the indices by the copy engine, double-buffered on a side stream",
           "staged": "fetch_all(pinned host indices): the runtime copies them to a device slot on its side stream",
           "pinned": "fetch_all(pinned host indices): the lookup kernels read them in place over PCIe"}[mode]
    return {
        "value": round(per_req * world, 3),
        "unit": "GB/s (sum over requesters)",
        "per_requester_gbs": round(per_req, 3),
        "ms_per_step": round(ms_per_step, 5),
        "h2d_bytes_per_step": int(pool[0].numel() * pool[0].element_size()),
        "d2h_bytes_per_step": int(out_host.numel()),
        "input_path": mode,
        "host_memory": args.e2e_host_memory,
        "host_us_per_step": round(host_us, 2),
        "index_h2d_alone_us": round(h2d_us, 2),
        "path": f"per step: {how} -> fetch_all (fetch + every layer's wait) -> D2H of the last layer's token-0 "
                f"rows (SM stores into pinned host memory, engram _C.host_write); eager public API",
        "l2": "not flushed inside the interval; 32 separate pinned index tensors cycled; fresh random rows "
              "from a table larger than L2 every step",
    }


def _physical_index(local):
    visible = os.environ.get("CUDA_VISIBLE_DEVICES")
    if visible:
        items = [v.strip() for v in visible.split(",") if v.strip()]
        if local < len(items) and items[local].isdigit():
            return int(items[local])
        return None
    return local


if __name__ == "__main__":
    main()
