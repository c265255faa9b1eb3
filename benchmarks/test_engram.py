"""Integration test and benchmark entry for the B200 EngramBuffer (one process per GPU).

Run with ``python -m torch.distributed.run --nnodes 1 --nproc-per-node N
--master-addr 127.0.0.1 benchmarks/test_engram.py [options] --output-dir DIR``,
or plainly (``python benchmarks/test_engram.py --local-ranks N ...``) to have
it spawn N local workers itself.

Scenarios mirror the reference's two entries (``benchmarks/test_read.py``,
``benchmarks/test_write.py``): all-to-all, single-owner and single-requester
traffic (idle ranks never call fetch); eager or CUDA-Graph fetches; reverse
and cross-stream hooks; row-major scales; padding; varying token counts
(including 0); a GPU-side locality cycle (self, remote, mixed, empty layer,
all padding) replayed inside one graph; CPU-side writes and weight rewrites;
API-misuse checks; back-to-back forwards verified on the GPU without host
syncs; a torch.profiler trace; MT19937-matched inputs; host-side probe fault
injection (``--egm-fail-pair``) so chosen pairs fall back to the host route;
and a bf16 GEMM overlapped on another stream.

Every output is checked bit-exactly against the pattern oracle outside the
timed region.  Each rank writes ``engram-r{rank}.json`` with its metadata and
per-round samples (``e2e_ms``, ``gbps`` = bytes returned / latency).
"""

from __future__ import annotations

import argparse
import contextlib
import datetime
import hashlib
import json
import os
import sys
import time
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from engram_rdma_lab_b200 import EngramBuffer, TorchEngramBuffer, _native  # noqa: E402
from engram_rdma_lab_b200.models import expected_outputs, make_indices, pattern_shard  # noqa: E402


def parse_pair(value):
    try:
        requester, owner = map(int, value.split(":"))
    except ValueError as error:
        raise argparse.ArgumentTypeError("expected requester:owner") from error
    if min(requester, owner) < 0 or requester == owner:
        raise argparse.ArgumentTypeError("expected distinct nonnegative ranks")
    return requester, owner


def parse():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--impl", choices=["native", "torch"], default="native")
    p.add_argument("--route", choices=["peer_hbm", "host"], default="peer_hbm")
    p.add_argument("--tokens", type=int, default=4096)
    p.add_argument("--capacity", type=int, default=0)
    p.add_argument("--entries", default="524288,524309")
    p.add_argument("--hidden", type=int, default=256)
    p.add_argument("--ept", type=int, default=24)
    p.add_argument("--dtype", choices=["fp8", "bf16"], default="fp8")
    p.add_argument("--sf-packs", type=int, default=2)
    p.add_argument("--qps", type=int, default=0)
    p.add_argument("--qp-depth", type=int, default=0, help="0 uses the buffer's recommendation")
    p.add_argument("--local-ranks", type=int, default=2,
                   help="workers to spawn on this node when not launched by torchrun")
    p.add_argument("--traffic", choices=["all-to-all", "single", "single-requester"], default="all-to-all")
    p.add_argument("--requester-rank", type=int, default=0)
    p.add_argument("--owner-rank", type=int, default=1)
    p.add_argument("--rounds", type=int, default=20)
    p.add_argument("--warmups", type=int, default=3)
    p.add_argument("--distribution", choices=["uniform", "stratified", "zipf", "matched"], default="uniform")
    p.add_argument("--hook-order", choices=["forward", "reverse"], default="forward")
    p.add_argument("--row-major-sf", action="store_true")
    p.add_argument("--cross-stream", action="store_true")
    p.add_argument("--padding", type=float, default=0.0, help="fraction of slots set to -1")
    p.add_argument("--vary-tokens", action="store_true")
    p.add_argument("--locality-cycle", action="store_true")
    p.add_argument("--cpu-write", action="store_true")
    p.add_argument("--rewrite", action="store_true")
    p.add_argument("--check-errors", action="store_true")
    p.add_argument("--cuda-graph", action="store_true")
    p.add_argument("--async-check", action="store_true")
    p.add_argument("--async-eager", action="store_true")
    p.add_argument("--overlap-gemm", default="", help="M,N,K of a bf16 GEMM overlapped on another stream (empty = off)")
    p.add_argument("--pinned-indices", action="store_true",
                   help="hand fetch a pinned host copy of each round's indices (eager rounds only)")
    p.add_argument("--profile", action="store_true")
    p.add_argument("--profile-rank", type=int, default=0)
    p.add_argument("--egm-fail-pair", type=parse_pair, action="append", default=[])
    p.add_argument("--verify-every", type=int, default=1, help="check every K-th timed round (0 = never)")
    p.add_argument("--timeout", type=float, default=60.0, help="bounded GPU wait per hook, seconds")
    p.add_argument("--output-dir", required=True)
    a = p.parse_args()
    if a.tokens < 0 or a.rounds < 1 or (a.capacity and a.capacity < max(1, a.tokens)):
        p.error("invalid tokens/capacity/rounds")
    if a.vary_tokens and (a.cuda_graph or a.async_check):
        p.error("--vary-tokens needs ordinary fetches (graph replay has a fixed shape)")
    if a.async_eager and (not a.async_check or a.cuda_graph):
        p.error("--async-eager needs --async-check and excludes --cuda-graph")
    if a.traffic != "all-to-all" and (a.async_check or a.profile or a.check_errors or a.locality_cycle):
        p.error("single-requester traffic runs the ordinary or graph benchmark only")
    if a.pinned_indices and (a.cuda_graph or a.async_check or a.profile or a.impl != "native"):
        p.error("--pinned-indices runs eager rounds of the native buffer only")
    return a


def inject_probe_failures(rank, pairs):
    """Test-only: corrupt one direction's mirror metadata so the pair degrades to the host route."""
    if not pairs:
        return
    C = _native.load()
    original = C.Runtime.probe_routes

    def probe(runtime, peers, candidates):
        altered = [dict(peer) for peer in peers]
        for requester, owner in pairs:
            if requester == rank:
                altered[owner]["mirror_bytes"] = 0
        return original(runtime, altered, candidates)

    C.Runtime.probe_routes = probe


def main():
    args = parse()
    if "RANK" not in os.environ:
        # Not under torchrun: spawn --local-ranks workers on this node, like
        # the reference's entries do (test_write.py:599-600).
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        torch.multiprocessing.spawn(_local_worker, args=(args, port), nprocs=args.local_ranks)
        return
    run(args)


def _local_worker(local_rank, args, port):
    os.environ.update(RANK=str(local_rank), LOCAL_RANK=str(local_rank), WORLD_SIZE=str(args.local_ranks),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    run(args)


def run(args):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl" if args.impl == "torch" else "gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=180),
                            **({"device_id": torch.device("cuda", local)} if args.impl == "torch" else {}))
    control = dist.new_group(backend="gloo")
    os.environ["ENGRAM_EGM_ENABLE"] = "1" if args.route == "peer_hbm" else "0"
    if any(max(p) >= world for p in args.egm_fail_pair):
        raise ValueError("--egm-fail-pair names a rank outside the group")
    if args.egm_fail_pair and args.route != "peer_hbm":
        raise ValueError("--egm-fail-pair needs --route peer_hbm")
    if not (0 <= args.requester_rank < world and 0 <= args.owner_rank < world):
        raise ValueError("requester/owner rank outside the group")
    inject_probe_failures(rank, args.egm_fail_pair)

    active = args.traffic == "all-to-all" or rank == args.requester_rank
    owner = args.owner_rank if args.traffic == "single" else None
    entries = [int(n) for n in args.entries.split(",")]
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float8_e4m3fn
    packs = 0 if args.dtype == "bf16" else args.sf_packs
    capacity = args.capacity or max(1, args.tokens)
    cls = EngramBuffer if args.impl == "native" else TorchEngramBuffer
    group = dist.group.WORLD
    sizes = cls.get_storage_size_hint(group, entries, args.hidden, capacity, args.ept, dtype, packs)
    qps, depth, restrict = cls.get_theoretical_config(group, len(entries), capacity, args.ept)
    depth = args.qp_depth or depth
    buffer = cls(group, *sizes, True, qps, depth, restrict, num_gpu_timeout_secs=args.timeout,
                 explicitly_destroy=True)
    buffer.set_config(entries, args.hidden, capacity, args.ept, dtype, packs)

    def load_weights(salt):
        storages, scales = pattern_shard(rank, world, entries, args.hidden, dtype, packs, "cuda", salt)
        if args.cpu_write:
            storages = [s.cpu() for s in storages]
            scales = [s.cpu() for s in scales] if scales else None
        buffer.write(storages, scales)

    t_phase = time.perf_counter()

    def mark(name):
        nonlocal t_phase
        now = time.perf_counter()
        meta.setdefault("phase_s", {})[name] = round(now - t_phase, 3)
        t_phase = now

    meta = {}
    mark("init")
    salt = 0
    load_weights(salt)
    mark("write")
    order = list(range(len(entries)))[:: -1 if args.hook_order == "reverse" else 1]
    consume = torch.cuda.Stream() if args.cross_stream else None
    scratch = torch.zeros(64, device="cuda")
    phase = torch.zeros((), dtype=torch.int32, device="cuda")
    gemm = None
    if args.overlap_gemm:
        m, n, k = (int(v) for v in args.overlap_gemm.split(","))
        gemm = (torch.randn(m, k, device="cuda", dtype=torch.bfloat16),
                torch.randn(k, n, device="cuda", dtype=torch.bfloat16), torch.cuda.Stream())

    def advance_locality(indices):
        # GPU-side phase: 0 self, 1 layer0 padding + others remote, 2 all padding,
        # 3 all remote, 4 mixed owners per slot, 5 layer0 remote + others self.
        phase.add_(1)
        ph = phase.remainder(6)
        remote = (rank + 1) % world
        mixed = torch.arange(args.ept, device="cuda", dtype=torch.int32).remainder(world)
        for layer, n in enumerate(entries):
            use_remote = (ph == 3) | ((ph == 1) & (layer > 0)) | ((ph == 5) & (layer == 0))
            target = torch.where(ph == 4, mixed, torch.where(use_remote, torch.full_like(mixed, remote),
                                                              torch.full_like(mixed, rank)))
            indices[layer].add_(1).remainder_(n).add_(target * n)
            indices[layer].masked_fill_((ph == 2) | ((ph == 1) & (layer == 0)), -1)

    def forward(indices):
        if args.locality_cycle:
            advance_locality(indices)
        hooks = buffer.fetch(indices, num_qps=args.qps, use_tma_aligned_col_major_sf=not args.row_major_sf)
        scratch.add_(1)  # unrelated work between fetch and hooks
        if gemm is not None:
            gemm[2].wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(gemm[2]):
                torch.matmul(gemm[0], gemm[1])
        outputs = [None] * len(entries)
        with torch.cuda.stream(consume) if consume is not None else contextlib.nullcontext():
            if consume is not None:
                consume.wait_stream(torch.cuda.current_stream())
            for layer in order:
                outputs[layer] = hooks[layer]()
        if consume is not None:
            torch.cuda.current_stream().wait_stream(consume)
        if gemm is not None:
            torch.cuda.current_stream().wait_stream(gemm[2])
        return outputs

    def verify(outputs, indices, on_gpu=False):
        exp = expected_outputs(indices if on_gpu else indices.cpu(), entries, args.hidden, dtype, packs, salt)
        bad = torch.zeros((), dtype=torch.int64, device="cuda" if on_gpu else "cpu")
        T = indices.shape[1]
        for layer, out in enumerate(outputs):
            data, sf = out if packs else (out, None)
            got = data.view(torch.uint8).reshape(T, args.ept * args.hidden * dtype.itemsize)
            bad = bad + (got if on_gpu else got.cpu()).ne(exp[layer][0]).sum()
            if packs:
                want = (args.ept * packs, 1) if args.row_major_sf else (1, (T + 3) // 4 * 4)
                assert sf.stride() == want, (sf.stride(), want)
                bad = bad + (sf if on_gpu else sf.cpu()).ne(exp[layer][1]).sum()
        return bad

    def draw(epoch, tokens=None):
        t = args.tokens if tokens is None else tokens
        if not active:
            return torch.empty(len(entries), 0, args.ept, dtype=torch.int32, device="cuda")
        return make_indices(rank, world, entries, t, args.ept, epoch=epoch, distribution=args.distribution,
                            padding=args.padding, owner=owner, device="cuda")

    indices = draw(1)
    submissions = 0
    for _ in range(2 if active else 0):
        outputs = forward(indices)
        submissions += 1
    torch.cuda.synchronize()
    if active:
        assert int(verify(outputs, indices, on_gpu=True)) == 0, "warm-up outputs differ from the oracle"

    if args.check_errors and active:
        hooks = buffer.fetch(indices)
        try:
            buffer.fetch(indices)
            raise AssertionError("a second fetch overwrote pending hooks")
        except RuntimeError:
            pass
        for hook in hooks:
            hook()
        newer = buffer.fetch(indices)
        try:
            hooks[0]()
            raise AssertionError("a stale hook was accepted")
        except RuntimeError:
            pass
        for hook in newer:
            hook()
        submissions += 2
    if args.rewrite:
        salt = 17
        load_weights(salt)

    graph = None
    if active and (args.cuda_graph or (args.async_check and not args.async_eager)):
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        limit = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None] * world
        with torch.cuda.graph(graph):
            if not args.locality_cycle and owner is None and args.distribution != "matched":
                indices.add_(1).remainder_(limit)  # the producer is part of the graph
            outputs = forward(indices)
        graph.replay()
        torch.cuda.synchronize()
        submissions += 1

    mark("warmup_graph")
    records = []
    if args.profile:
        selected = rank == args.profile_rank
        prof = (torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU,
                                                   torch.profiler.ProfilerActivity.CUDA], record_shapes=True)
                if selected else contextlib.nullcontext())
        scope = torch.profiler.record_function if selected else (lambda name: contextlib.nullcontext())
        dist.barrier(group=control)
        torch.cuda.synchronize()
        with prof:
            for frame in range(args.rounds):
                with scope(f"ENGRAM/forward_{frame}"):
                    if graph is not None:
                        with scope("ENGRAM/graph_replay"):
                            graph.replay()
                    else:
                        with scope("ENGRAM/fetch_and_hooks"):
                            outputs = forward(indices)
                submissions += 1
            torch.cuda.synchronize()
        trace = Path(args.output_dir) / f"engram-r{rank}.trace.json"
        if selected:
            Path(args.output_dir).mkdir(parents=True, exist_ok=True)
            prof.export_chrome_trace(str(trace))
        if active:
            assert int(verify(outputs, indices)) == 0
        meta.update(profile=True, trace=str(trace) if selected else None)
        dist.barrier(group=control)
    elif args.async_check and active:
        verdict = torch.zeros(args.rounds, dtype=torch.int64, device="cuda")
        dist.barrier(group=control)
        limit = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None] * world
        for frame in range(args.rounds):
            start = time.perf_counter_ns()
            if graph is None:
                if not args.locality_cycle:
                    indices.add_(1).remainder_(limit)
                outputs = forward(indices)
            else:
                graph.replay()
            records.append(dict(rank=rank, round=frame, enqueue_us=(time.perf_counter_ns() - start) / 1e3))
            verdict[frame] = verify(outputs, indices, on_gpu=True)  # no host sync inside the loop
            submissions += 1
        pending = not torch.cuda.current_stream().query()
        t_sync = time.perf_counter_ns()
        torch.cuda.synchronize()
        meta.update(final_sync_ms=(time.perf_counter_ns() - t_sync) / 1e6)
        assert int(verdict.sum()) == 0, f"GPU verdicts: {verdict.tolist()}"
        meta.update(async_check=True, per_forward_host_syncs=0, pending_after_enqueue=pending)
    else:
        for it in range(-args.warmups, args.rounds):
            epoch = it + args.warmups + 2
            if graph is None and active:
                tokens = [args.tokens, args.tokens // 2, 0][it % 3] if args.vary_tokens else args.tokens
                indices = draw(epoch, tokens)
            elif graph is not None and args.distribution == "matched":
                indices.copy_(draw(epoch))
            dist.barrier(group=control)
            torch.cuda.synchronize()
            if not active:
                records.append(dict(rank=rank, round=it, warmup=it < 0, requester_active=False, bytes=0,
                                    e2e_ms=None, gbps=None))
                dist.barrier(group=control)
                continue
            # --pinned-indices: the fetch reads a pinned host copy in place
            # (its PCIe transfer is inside the timed region).
            source = indices.cpu().pin_memory() if args.pinned_indices else indices
            start = time.perf_counter_ns()
            if graph is None:
                outputs = forward(source)
            else:
                graph.replay()
            torch.cuda.synchronize()
            elapsed = (time.perf_counter_ns() - start) / 1e6
            submissions += 1
            checked = args.verify_every > 0 and (it < 0 or it % args.verify_every == 0)
            if checked:
                assert int(verify(outputs, indices, on_gpu=True)) == 0, f"round {it}: outputs differ from the oracle"
            nbytes = len(entries) * indices.shape[1] * args.ept * args.hidden * dtype.itemsize
            records.append(dict(rank=rank, round=it, warmup=it < 0, requester_active=True, bytes=nbytes,
                                e2e_ms=elapsed, gbps=nbytes / elapsed / 1e6 if elapsed else None,
                                indices_sha256=hashlib.sha256(indices.cpu().numpy().tobytes()).hexdigest(),
                                data_ok=True if checked else None, scale_ok=True if checked else None))
            dist.barrier(group=control)
    mark("measure")
    if args.impl == "native":
        meta.update(error_state=buffer.error_state())
    meta.update(
        impl=args.impl, route=args.route, routing=buffer.get_route_info(), dtype=args.dtype, entries=entries,
        tokens=args.tokens, capacity=capacity, hook_order=args.hook_order, cross_stream=args.cross_stream,
        col_major_sf=not args.row_major_sf, traffic=args.traffic, requester_active=active, owner_rank=owner,
        cuda_graph=graph is not None, injected_probe_failures=args.egm_fail_pair, forward_submissions=submissions,
        locality_cycle=args.locality_cycle, rewrite=args.rewrite, cpu_write=args.cpu_write,
        pinned_indices=args.pinned_indices, hot_rows=getattr(buffer, "hot_rows", None),
    )
    root = Path(args.output_dir)
    root.mkdir(parents=True, exist_ok=True)
    (root / f"engram-r{rank}.json").write_text(json.dumps(dict(metadata=meta, samples=records), indent=2,
                                                           default=str))
    print(f"rank {rank}: phases {meta['phase_s']}", flush=True)
    timed = [r["e2e_ms"] for r in records if r.get("e2e_ms") and not r.get("warmup")]
    if timed:
        timed.sort()
        print(f"rank {rank}: p50 {timed[len(timed) // 2]:.4f} ms over {len(timed)} rounds, routes "
              f"{meta['routing']['owner_routes']}", flush=True)
    dist.barrier(group=control)
    del graph
    buffer.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
