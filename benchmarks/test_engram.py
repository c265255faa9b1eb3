"""Integration test and benchmark entry for the B200 EngramBuffer (one process per GPU).

Run with ``python -m torch.distributed.run --nnodes 1 --nproc-per-node N
--master-addr 127.0.0.1 benchmarks/test_engram.py [options] --output-dir DIR``,
or plainly (``python benchmarks/test_engram.py --local-ranks N ...``) to have
it spawn N local workers itself.

It covers the scenarios of the reference's two entries
(``benchmarks/test_read.py``, ``benchmarks/test_write.py:519-573``) with its own
structure:

* a :class:`Requests` source per run: random draws (uniform, stratified,
  Zipf, single owner, MT19937-matched), a locality plan cycled on the GPU, or
  nothing for ranks that only serve;
* a :class:`Forward` that submits ``fetch``, optional unrelated work (a scratch
  update, a bf16 GEMM on another stream) and the hooks in the chosen order on
  the chosen stream;
* one of three run modes, picked from :data:`MODES`: ``rounds`` (host-timed
  rounds with issue / hooks / synchronize / device splits), ``async``
  (back-to-back forwards judged on the GPU, one host sync at the end), or
  either of them replayed from a CUDA graph;
* optional API-misuse checks (:data:`MISUSE`), weight rewrites, CPU writes,
  pinned host indices, a torch.profiler trace and host-side probe fault
  injection (``--egm-fail-pair``).

Every output is checked bit-exactly against the pattern oracle outside the
timed region.  Each rank writes ``engram-r{rank}.json``: metadata (placement,
CPU affinity, GPU UUID, sha256 of the kernel sources and of the loaded
extension, routes) and per-round samples.
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

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from engram_rdma_lab_b200 import EngramBuffer, TorchEngramBuffer, _native  # noqa: E402
from engram_rdma_lab_b200.models import expected_outputs, make_indices, pattern_shard  # noqa: E402


# ----------------------------------------------------------------------------- options
def parse_pair(value):
    try:
        requester, owner = map(int, value.split(":"))
    except ValueError as error:
        raise argparse.ArgumentTypeError("expected requester:owner") from error
    if min(requester, owner) < 0 or requester == owner:
        raise argparse.ArgumentTypeError("expected distinct nonnegative ranks")
    return requester, owner


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add = p.add_argument
    add("--impl", choices=["native", "torch"], default="native")
    add("--route", choices=["peer_hbm", "host"], default="peer_hbm")
    add("--tokens", type=int, default=4096)
    add("--capacity", type=int, default=0)
    add("--entries", default="524288,524309")
    add("--hidden", type=int, default=256)
    add("--ept", type=int, default=24)
    add("--dtype", choices=["fp8", "bf16"], default="fp8")
    add("--sf-packs", type=int, default=2)
    add("--qps", type=int, default=0)
    add("--qp-depth", type=int, default=0, help="0 uses the buffer's recommendation")
    add("--local-ranks", type=int, default=2, help="workers to spawn on this node when not launched by torchrun")
    add("--traffic", choices=["all-to-all", "single", "single-requester"], default="all-to-all")
    add("--requester-rank", type=int, default=0)
    add("--owner-rank", type=int, default=1)
    add("--rounds", type=int, default=20)
    add("--warmups", type=int, default=3)
    add("--distribution", choices=["uniform", "stratified", "zipf", "matched"], default="uniform")
    add("--hook-order", choices=["forward", "reverse"], default="forward")
    add("--row-major-sf", action="store_true")
    add("--cross-stream", action="store_true")
    add("--padding", type=float, default=0.0, help="fraction of slots set to -1")
    add("--vary-tokens", action="store_true", help="eager rounds cycle through T, T/2, 0 and T-1 tokens")
    add("--locality-cycle", action="store_true")
    add("--cpu-write", action="store_true")
    add("--rewrite", action="store_true")
    add("--check-errors", action="store_true")
    add("--cuda-graph", action="store_true")
    add("--async-check", action="store_true")
    add("--async-eager", action="store_true")
    add("--overlap-gemm", default="", help="M,N,K of a bf16 GEMM overlapped on another stream (empty = off)")
    add("--pinned-indices", action="store_true",
        help="hand fetch a pinned host copy of each round's indices (eager rounds only)")
    add("--profile", action="store_true")
    add("--profile-rank", type=int, default=0)
    add("--egm-fail-pair", type=parse_pair, action="append", default=[])
    add("--verify-every", type=int, default=1, help="check every K-th timed round (0 = never)")
    add("--timeout", type=float, default=60.0, help="bounded GPU wait per hook, seconds")
    add("--output-dir", required=True)
    a = p.parse_args(argv)
    problems = [
        (a.tokens < 0 or a.rounds < 1 or (a.capacity and a.capacity < max(1, a.tokens)),
         "invalid tokens/capacity/rounds"),
        (a.vary_tokens and (a.cuda_graph or a.async_check), "--vary-tokens needs eager rounds (a graph has one shape)"),
        (a.async_eager and (not a.async_check or a.cuda_graph), "--async-eager needs --async-check, not --cuda-graph"),
        (a.traffic != "all-to-all" and (a.async_check or a.profile or a.check_errors or a.locality_cycle),
         "single-owner / single-requester traffic runs plain or graph rounds only"),
        (a.pinned_indices and (a.cuda_graph or a.async_check or a.profile or a.impl != "native"),
         "--pinned-indices runs eager rounds of the native buffer only"),
    ]
    for bad, message in problems:
        if bad:
            p.error(message)
    return a


# ----------------------------------------------------------------------------- requests
class Requests:
    """Index source of one rank: fresh draws per round, or nothing when idle."""

    def __init__(self, args, rank, world, entries):
        self.args, self.rank, self.world, self.entries = args, rank, world, entries
        self.active = args.traffic == "all-to-all" or rank == args.requester_rank
        self.owner = args.owner_rank if args.traffic == "single" else None
        # Global ids per layer, made before any capture (a host-to-device copy
        # cannot be captured).
        self.limit = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None] * world

    def draw(self, epoch, tokens=None):
        a = self.args
        t = a.tokens if tokens is None else tokens
        if not self.active:
            t = 0
        return make_indices(self.rank, self.world, self.entries, t, a.ept, epoch=epoch, distribution=a.distribution,
                            padding=a.padding, owner=self.owner, device="cuda")

    def next_round(self, indices, epoch, tokens):
        """Indices of an eager timed round: a fresh draw."""
        return self.draw(epoch, tokens)

    def advance(self, indices):
        """Graph-capturable producer step: every non-padding id moves to the next global id (wrapping)."""
        if self.owner is None and self.args.distribution != "matched":
            indices.copy_(torch.where(indices >= 0, (indices + 1).remainder(self.limit), indices))


class LocalityPlan(Requests):
    """Locality changes driven by the GPU, so one captured graph replays them all.

    ``plan[p, l, s]`` names the owner of entry slot ``s`` of layer ``l`` in
    phase ``p`` (-1 = padding).  A device counter selects the phase; each step
    also moves every slot to a fresh local row, so no two phases repeat rows.
    Phases: rows owned by every rank in turn across slots; this rank's own
    rows; the first layer empty and the rest from the next rank; everything
    from the next rank; only padding; the first layer from the next rank and
    the rest local.
    """

    def __init__(self, args, rank, world, entries):
        super().__init__(args, rank, world, entries)
        L, E = len(entries), args.ept
        nxt = (rank + 1) % world
        spread = [(rank + s) % world for s in range(E)]
        phases = [
            [spread] * L,
            [[rank] * E] * L,
            [[-1] * E] + [[nxt] * E] * (L - 1),
            [[nxt] * E] * L,
            [[-1] * E] * L,
            [[nxt] * E] + [[rank] * E] * (L - 1),
        ]
        self.plan = torch.tensor(phases, dtype=torch.int32, device="cuda").unsqueeze(2)  # [P, L, 1, E]
        self.rows = torch.tensor(entries, dtype=torch.int32, device="cuda")[:, None, None]
        self.counter = torch.zeros(1, dtype=torch.int64, device="cuda")
        gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
        self.local = (torch.rand(L, max(args.tokens, 1), E, device="cuda", generator=gen) * self.rows).to(torch.int32)

    def next_round(self, indices, epoch, tokens):
        self.advance(indices)  # the next phase, in place
        return indices

    def advance(self, indices):
        self.counter.add_(1)
        owners = self.plan.index_select(0, self.counter.remainder(self.plan.shape[0])).squeeze(0)
        self.local.add_(5).remainder_(self.rows)
        T = indices.shape[1]
        ids = torch.where(owners < 0, torch.full_like(owners, -1), owners * self.rows + self.local[:, :T])
        indices.copy_(ids)


# ----------------------------------------------------------------------------- forward
class Forward:
    """fetch -> unrelated work -> hooks, with the chosen hook order and stream."""

    def __init__(self, args, buffer, layers):
        self.args, self.buffer = args, buffer
        self.order = list(range(layers))[::-1] if args.hook_order == "reverse" else list(range(layers))
        self.hook_stream = torch.cuda.Stream() if args.cross_stream else None
        self.scratch = torch.zeros(64, device="cuda")
        self.gemm = None
        if args.overlap_gemm:
            m, n, k = (int(v) for v in args.overlap_gemm.split(","))
            self.gemm = (torch.randn(m, k, device="cuda", dtype=torch.bfloat16),
                         torch.randn(k, n, device="cuda", dtype=torch.bfloat16), torch.cuda.Stream())
        self.issue_s = self.hooks_s = 0.0

    def __call__(self, indices):
        a = self.args
        t0 = time.perf_counter()
        hooks = self.buffer.fetch(indices, num_qps=a.qps, use_tma_aligned_col_major_sf=not a.row_major_sf)
        t1 = time.perf_counter()
        self.scratch.mul_(0.5).add_(1)  # unrelated work between fetch and hooks
        main = torch.cuda.current_stream()
        if self.gemm is not None:
            x, w, side = self.gemm
            side.wait_stream(main)
            with torch.cuda.stream(side):
                torch.mm(x, w)
        outputs = [None] * len(hooks)
        t2 = time.perf_counter()
        if self.hook_stream is not None:
            self.hook_stream.wait_stream(main)
        with torch.cuda.stream(self.hook_stream) if self.hook_stream is not None else contextlib.nullcontext():
            for layer in self.order:
                outputs[layer] = hooks[layer]()
        if self.hook_stream is not None:
            main.wait_stream(self.hook_stream)
        if self.gemm is not None:
            main.wait_stream(self.gemm[2])
        t3 = time.perf_counter()
        self.issue_s, self.hooks_s = t1 - t0, t3 - t2
        return outputs


# ----------------------------------------------------------------------------- oracle
class Oracle:
    def __init__(self, args, entries, dtype, packs):
        self.args, self.entries, self.dtype, self.packs = args, entries, dtype, packs
        self.row_width = args.ept * args.hidden * torch.empty((), dtype=dtype).element_size()
        self.salt = 0

    def mismatches(self, outputs, indices, on_gpu):
        """Differing bytes and scale words (a device scalar when ``on_gpu``)."""
        a = self.args
        source = indices if on_gpu else indices.cpu()
        want = expected_outputs(source, self.entries, a.hidden, self.dtype, self.packs, self.salt)
        T = indices.shape[1]
        total = torch.zeros((), dtype=torch.int64, device=source.device)
        sf_stride = (a.ept * self.packs, 1) if a.row_major_sf else (1, (T + 3) // 4 * 4)
        for layer, out in enumerate(outputs):
            data, sf = out if self.packs else (out, None)
            got = data.view(torch.uint8).reshape(T, self.row_width)
            total = total + (got if on_gpu else got.cpu()).ne(want[layer][0]).sum()
            if self.packs:
                if T and sf.stride() != sf_stride:
                    raise AssertionError(f"scale strides {sf.stride()} != {sf_stride}")
                total = total + (sf if on_gpu else sf.cpu()).ne(want[layer][1]).sum()
        return total


# ----------------------------------------------------------------------------- misuse checks
def _expect(error, call):
    try:
        call()
    except error:
        return True
    return False


def _pending_fetch_refused(b, x, s):
    s["first"] = b.fetch(x)
    return _expect(RuntimeError, lambda: b.fetch(x))


def _pending_destroy_refused(b, x, s):
    return _expect(RuntimeError, b.destroy)  # refused before any collective step


def _second_hook_call_refused(b, x, s):
    for hook in s["first"]:
        hook()
    return _expect(RuntimeError, s["first"][0])


def _superseded_hook_refused(b, x, s):
    newer = b.fetch(x)
    refused = _expect(RuntimeError, s["first"][-1])
    for hook in newer:
        hook()
    return refused


def _wrong_dtype_refused(b, x, s):
    return _expect(ValueError, lambda: b.fetch(x.long()))


def _over_capacity_refused(b, x, s):
    big = torch.zeros(x.shape[0], b._config.max_tokens + 1, x.shape[2], dtype=torch.int32, device=x.device)
    return _expect(ValueError, lambda: b.fetch(big))


# Run in order on one buffer; each returns True when the misuse was refused.
# The sequence leaves no hook outstanding.
MISUSE = [
    ("second fetch while hooks are pending", _pending_fetch_refused),
    ("destroy while hooks are pending", _pending_destroy_refused),
    ("hook called twice", _second_hook_call_refused),
    ("hook of a superseded fetch", _superseded_hook_refused),
    ("indices of the wrong dtype", _wrong_dtype_refused),
    ("more tokens than the capacity", _over_capacity_refused),
]


def run_misuse_checks(buffer, indices):
    state = {}
    failed = [name for name, action in MISUSE if not action(buffer, indices, state)]
    if failed:
        raise AssertionError(f"API misuse accepted: {failed}")
    return [name for name, _ in MISUSE]


# ----------------------------------------------------------------------------- run modes
class Run:
    """Shared state of one harness run on one rank."""

    def __init__(self, args, rank, world, control, buffer, requests, forward, oracle):
        self.args, self.rank, self.world, self.control = args, rank, world, control
        self.buffer, self.requests, self.forward, self.oracle = buffer, requests, forward, oracle
        self.indices = requests.draw(1)
        self.outputs = None
        self.graph = None
        self.samples = []
        self.submissions = 0
        self.meta = {}

    def step(self):
        """One forward (a replay when a graph was captured); returns host seconds of the call."""
        t0 = time.perf_counter()
        if self.graph is not None:
            self.graph.replay()
        else:
            if self.args.locality_cycle or self.args.async_check:
                self.requests.advance(self.indices)
            self.outputs = self.forward(self.indices)
        self.submissions += 1
        return time.perf_counter() - t0

    def capture(self):
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.requests.advance(self.indices)  # the producer is part of the graph
            self.outputs = self.forward(self.indices)
        self.graph.replay()
        self.submissions += 1
        torch.cuda.synchronize()

    def check(self, where):
        bad = int(self.oracle.mismatches(self.outputs, self.indices, on_gpu=True))
        if bad:
            raise AssertionError(f"{where}: {bad} values differ from the oracle")


def mode_rounds(run):
    """Host-timed rounds: barrier, then fetch + hooks + synchronize, with timing splits."""
    a, req = run.args, run.requests
    token_cycle = [a.tokens, a.tokens // 2, 0, max(a.tokens - 1, 0)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for it in range(-a.warmups, a.rounds):
        if run.graph is None and req.active:
            tokens = token_cycle[it % len(token_cycle)] if a.vary_tokens else a.tokens
            run.indices = req.next_round(run.indices, it + a.warmups + 2, tokens)
        elif run.graph is not None and a.distribution == "matched":
            run.indices.copy_(req.draw(it + a.warmups + 2))
        dist.barrier(group=run.control)
        torch.cuda.synchronize()
        if not req.active:
            run.samples.append(dict(rank=run.rank, round=it, warmup=it < 0, requester_active=False))
            dist.barrier(group=run.control)
            continue
        source = run.indices.cpu().pin_memory() if a.pinned_indices else run.indices
        t0 = time.perf_counter()
        start.record()
        if run.graph is None:
            run.outputs = run.forward(source)
            run.submissions += 1
            issue_s, hooks_s = run.forward.issue_s, run.forward.hooks_s
        else:
            issue_s, hooks_s = run.step(), 0.0
        end.record()
        t_sync = time.perf_counter()
        torch.cuda.synchronize()
        t_end = time.perf_counter()
        elapsed_ms = (t_end - t0) * 1e3
        checked = a.verify_every > 0 and (it < 0 or it % a.verify_every == 0)
        if checked:
            run.check(f"round {it}")
        nbytes = len(req.entries) * run.indices.shape[1] * run.oracle.row_width
        run.samples.append(dict(
            rank=run.rank, round=it, warmup=it < 0, requester_active=True, tokens=int(run.indices.shape[1]),
            bytes=nbytes, e2e_ms=elapsed_ms, device_ms=start.elapsed_time(end),
            python_issue_ms=issue_s * 1e3, python_hooks_ms=hooks_s * 1e3, synchronize_ms=(t_end - t_sync) * 1e3,
            gbps=nbytes / elapsed_ms / 1e6 if elapsed_ms else None,
            indices_sha256=hashlib.sha256(run.indices.cpu().numpy().tobytes()).hexdigest(),
            verified=checked))
        dist.barrier(group=run.control)


def mode_async(run):
    """Back-to-back forwards judged on the GPU: no host sync until the end."""
    a = run.args
    mismatches = torch.zeros((), dtype=torch.int64, device="cuda")
    bad_rounds = torch.zeros((), dtype=torch.int64, device="cuda")
    dist.barrier(group=run.control)
    for it in range(a.rounds):
        host_s = run.step()
        wrong = run.oracle.mismatches(run.outputs, run.indices, on_gpu=True)
        mismatches += wrong
        bad_rounds += (wrong > 0).long()
        run.samples.append(dict(rank=run.rank, round=it, enqueue_us=host_s * 1e6))
    busy = not torch.cuda.current_stream().query()
    t0 = time.perf_counter()
    torch.cuda.synchronize()
    run.meta.update(closing_sync_ms=(time.perf_counter() - t0) * 1e3, stream_busy_after_enqueue=busy,
                    host_syncs_per_round=0, async_check=True)
    if int(mismatches):
        raise AssertionError(f"{int(bad_rounds)} of {a.rounds} rounds differ ({int(mismatches)} values)")


MODES = {"rounds": mode_rounds, "async": mode_async}


@contextlib.contextmanager
def profiled(run):
    """torch.profiler (CPU + CUDA) around the measured rounds on the chosen rank."""
    a = run.args
    if not a.profile or run.rank != a.profile_rank:
        yield
        return
    activities = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=activities, record_shapes=True) as prof:
        with torch.profiler.record_function("engram.measured_rounds"):
            yield
        torch.cuda.synchronize()
    out = Path(a.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    trace = out / f"engram-r{run.rank}.trace.json"
    prof.export_chrome_trace(str(trace))
    run.meta.update(profile=True, trace=str(trace))


# ----------------------------------------------------------------------------- metadata
def _sha256_files(paths):
    h = hashlib.sha256()
    for path in sorted(paths):
        h.update(path.relative_to(ROOT).as_posix().encode())
        h.update(path.read_bytes())
    return h.hexdigest()


def run_metadata(buffer, local_rank):
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    sources = [p for ext in ("*.cu", "*.cuh", "*.h", "*.cpp") for p in (ROOT / "csrc").rglob(ext)]
    meta = dict(
        gpu_uuid=str(props.uuid), gpu_name=props.name, local_rank=local_rank, cuda_visible_devices=visible,
        cpu_affinity=sorted(os.sched_getaffinity(0)), hostname=os.uname().nodename,
        kernel_sources_sha256=_sha256_files(sources),
    )
    if isinstance(buffer, EngramBuffer):
        so = Path(_native.load().__file__)
        meta.update(extension=so.name, extension_sha256=hashlib.sha256(so.read_bytes()).hexdigest())
    return meta


# ----------------------------------------------------------------------------- setup
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


def make_buffer(args, world, entries, dtype, packs, capacity):
    cls = EngramBuffer if args.impl == "native" else TorchEngramBuffer
    group = dist.group.WORLD
    sizes = cls.get_storage_size_hint(group, entries, args.hidden, capacity, args.ept, dtype, packs)
    qps, depth, restrict = cls.get_theoretical_config(group, len(entries), capacity, args.ept)
    buffer = cls(group, *sizes, True, qps, args.qp_depth or depth, restrict, num_gpu_timeout_secs=args.timeout,
                 explicitly_destroy=True)
    buffer.set_config(entries, args.hidden, capacity, args.ept, dtype, packs)
    return buffer


def main():
    args = parse()
    if "RANK" not in os.environ:
        # Not under torchrun: spawn --local-ranks workers on this node.
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        torch.multiprocessing.spawn(_local_worker, args=(args, port), nprocs=args.local_ranks)
        return
    run_rank(args)


def _local_worker(local_rank, args, port):
    os.environ.update(RANK=str(local_rank), LOCAL_RANK=str(local_rank), WORLD_SIZE=str(args.local_ranks),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    run_rank(args)


def run_rank(args):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    extra = {"device_id": torch.device("cuda", local)} if args.impl == "torch" else {}
    dist.init_process_group("nccl" if args.impl == "torch" else "gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=180), **extra)
    control = dist.new_group(backend="gloo")
    os.environ["ENGRAM_EGM_ENABLE"] = "1" if args.route == "peer_hbm" else "0"
    if any(max(p) >= world for p in args.egm_fail_pair):
        raise ValueError("--egm-fail-pair names a rank outside the group")
    if args.egm_fail_pair and args.route != "peer_hbm":
        raise ValueError("--egm-fail-pair needs --route peer_hbm")
    # The requester and owner ranks matter only for the traffic that names them.
    if args.traffic != "all-to-all" and not 0 <= args.requester_rank < world:
        raise ValueError("--requester-rank outside the group")
    if args.traffic == "single" and not 0 <= args.owner_rank < world:
        raise ValueError("--owner-rank outside the group")
    inject_probe_failures(rank, args.egm_fail_pair)

    entries = [int(n) for n in args.entries.split(",")]
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float8_e4m3fn
    packs = 0 if args.dtype == "bf16" else args.sf_packs
    capacity = args.capacity or max(1, args.tokens)
    phases, t_phase = {}, time.perf_counter()

    def phase(name):
        nonlocal t_phase
        now = time.perf_counter()
        phases[name] = round(now - t_phase, 3)
        t_phase = now

    buffer = make_buffer(args, world, entries, dtype, packs, capacity)
    phase("init")
    oracle = Oracle(args, entries, dtype, packs)

    def load_weights(salt):
        oracle.salt = salt
        storages, scales = pattern_shard(rank, world, entries, args.hidden, dtype, packs, "cuda", salt)
        if args.cpu_write:
            storages = [s.cpu() for s in storages]
            scales = [s.cpu() for s in scales] if scales else None
        buffer.write(storages, scales)

    load_weights(0)
    phase("write")
    requests = (LocalityPlan if args.locality_cycle else Requests)(args, rank, world, entries)
    run = Run(args, rank, world, control, buffer, requests, Forward(args, buffer, len(entries)), oracle)
    if requests.active:
        for _ in range(2):
            run.step()
        torch.cuda.synchronize()
        run.check("warm-up")
    if args.check_errors and requests.active:
        run.meta["misuse_checks"] = run_misuse_checks(buffer, run.indices)
    if args.rewrite:
        load_weights(17)
    if requests.active and (args.cuda_graph or (args.async_check and not args.async_eager)):
        run.capture()
    phase("warmup_graph")
    with profiled(run):
        MODES["async" if args.async_check and requests.active else "rounds"](run)
    phase("measure")

    meta = dict(run.meta, phase_s=phases, **run_metadata(buffer, local))
    if args.impl == "native":
        meta.update(error_state=buffer.error_state())
    meta.update(
        impl=args.impl, route=args.route, routing=buffer.get_route_info(), dtype=args.dtype, entries=entries,
        tokens=args.tokens, capacity=capacity, world=world, hook_order=args.hook_order,
        cross_stream=args.cross_stream, col_major_sf=not args.row_major_sf, traffic=args.traffic,
        requester_active=requests.active, owner_rank=requests.owner, cuda_graph=run.graph is not None,
        injected_probe_failures=args.egm_fail_pair, forward_submissions=run.submissions,
        locality_cycle=args.locality_cycle, rewrite=args.rewrite, cpu_write=args.cpu_write,
        pinned_indices=args.pinned_indices, hot_rows=getattr(buffer, "hot_rows", None),
    )
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    (out / f"engram-r{rank}.json").write_text(json.dumps(dict(metadata=meta, samples=run.samples), indent=2,
                                                         default=str))
    timed = sorted(s["e2e_ms"] for s in run.samples if s.get("e2e_ms") and not s.get("warmup"))
    if timed:
        device = sorted(s["device_ms"] for s in run.samples if s.get("device_ms") and not s.get("warmup"))
        print(f"rank {rank}: p50 {timed[len(timed) // 2]:.4f} ms host / {device[len(device) // 2]:.4f} ms device "
              f"over {len(timed)} rounds, routes {meta['routing']['owner_routes']}", flush=True)
    print(f"rank {rank}: phases {phases}", flush=True)
    dist.barrier(group=control)
    run.graph = None
    buffer.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
