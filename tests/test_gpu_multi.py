"""EngramBuffer across several GPUs of one node (one process per GPU).

Needs at least two GPUs; uses every visible GPU, up to eight (the node size).  The control plane is a gloo group
(the data plane never touches a process group).  NVLS is not used anywhere:
peers are reached with plain peer loads and stores.
"""

import os

import pytest
import torch
import torch.distributed as dist

from .conftest import cuda_device_count
from ._spawn import run_ranks

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(cuda_device_count() < 2, reason="needs at least two GPUs"),
]


def _world():
    return min(8, cuda_device_count())


def _buffer(entries, hidden, max_tokens, ept, dtype, packs, egm, local_sf=True, timeout=30, qps=None):
    from engram_rdma_lab_b200 import EngramBuffer

    os.environ["ENGRAM_EGM_ENABLE"] = "1" if egm else "0"
    os.environ["ENGRAM_WRITE_LOCAL_SF"] = "1" if local_sf else "0"
    group = dist.group.WORLD
    sizes = EngramBuffer.get_storage_size_hint(group, entries, hidden, max_tokens, ept, dtype, packs)
    cfg = list(EngramBuffer.get_theoretical_config(group, len(entries), max_tokens, ept))
    if qps:
        cfg[0] = qps
    buf = EngramBuffer(group, *sizes, True, *cfg, num_gpu_timeout_secs=timeout, explicitly_destroy=True)
    buf.set_config(entries, hidden, max_tokens, ept, dtype, packs)
    return buf


def _check(outputs, indices, entries, hidden, dtype, packs, salt=0, col_major=True):
    from engram_rdma_lab_b200.models import expected_outputs

    exp = expected_outputs(indices.cpu(), entries, hidden, dtype, packs, salt)
    T = indices.shape[1]
    for layer, out in enumerate(outputs):
        data, sf = out if packs else (out, None)
        got = data.view(torch.uint8).reshape(T, -1).cpu()
        bad = (got != exp[layer][0]).any(dim=1).nonzero().flatten().tolist()
        assert not bad, f"layer {layer}: {len(bad)} wrong token rows, first {bad[:4]}"
        if packs:
            assert torch.equal(sf.cpu(), exp[layer][1]), f"layer {layer} scales"


def _setup(rank):
    torch.cuda.set_device(rank)


def _peer_hbm(rank, world):
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    entries, hidden, ept, dtype, packs = (20011, 20021), 256, 24, torch.float8_e4m3fn, 2
    # The default kernel (SIMT, 32-byte vectors), the SIMT kernel with 16-byte
    # vectors, and the opted-in TMA ring, each with both scale layouts.
    # The last pass moves the peers' rows by owner push from their mirrors.
    passes = [("auto", "auto", False, "pull"), ("simt", "16", True, "pull"), ("bulk", "32", True, "pull"),
              ("auto", "auto", True, "pull"), ("auto", "auto", True, "push")]
    for kernel, vector, local_sf, transport in passes:
        os.environ["ENGRAM_GATHER_KERNEL"] = kernel
        os.environ["ENGRAM_GATHER_VECTOR"] = vector
        os.environ["ENGRAM_PEER_TRANSPORT"] = transport
        buf = _buffer(entries, hidden, 512, ept, dtype, packs, egm=True, local_sf=local_sf)
        mem = buf.memory_usage()
        assert mem["gather_kernel"] == ("tma_bulk" if kernel == "bulk" else "simt"), mem
        pulled = transport == "pull" and world > 1
        assert mem["gather_vector_bytes"] == ((32 if pulled else 16) if vector == "auto" else int(vector)), mem
        assert mem["peer_transport"] == transport and mem["has_host_routes"] == (transport == "push"), mem
        info = buf.get_route_info()
        assert info["owner_routes"] == ["peer_hbm"] * world, info
        storages, scales = pattern_shard(rank, world, entries, hidden, dtype, packs, "cuda")
        buf.write(storages, scales)
        dist.barrier()
        for epoch in range(5):
            dist_name = "zipf" if epoch == 3 else "uniform"  # skewed requests exercise deduplication
            idx = make_indices(rank, world, entries, 512, ept, epoch=epoch, padding=0.02, distribution=dist_name,
                               device="cuda")
            if epoch == 4:  # pinned host indices, read in place by the kernels
                idx = idx.cpu().pin_memory()
            outs = [h() for h in buf.fetch(idx, use_tma_aligned_col_major_sf=epoch != 1)]
            torch.cuda.synchronize()
            _check(outs, idx, entries, hidden, dtype, packs, col_major=epoch != 1)
        # Graph capture with the producer inside the graph.
        idx = make_indices(rank, world, entries, 512, ept, epoch=9, device="cuda")
        graph = torch.cuda.CUDAGraph()
        limit = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None] * world
        with torch.cuda.graph(graph):
            idx.add_(3).remainder_(limit)
            outs = [h() for h in reversed(buf.fetch(idx))][::-1]
        for _ in range(2):
            graph.replay()
            torch.cuda.synchronize()
            _check(outs, idx, entries, hidden, dtype, packs)
        del graph
        dist.barrier()
        buf.destroy()
    for knob in ("ENGRAM_GATHER_KERNEL", "ENGRAM_GATHER_VECTOR", "ENGRAM_PEER_TRANSPORT"):
        os.environ.pop(knob, None)


def _host_route(rank, world):
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    entries, hidden, ept, dtype = (30011, 30013), 256, 8, torch.bfloat16
    buf = _buffer(entries, hidden, 1024, ept, dtype, 0, egm=False, local_sf=False)
    info = buf.get_route_info()
    assert info["owner_routes"] == ["host"] * world
    assert info["memory"]["owner_threads"] == 1
    storages, _ = pattern_shard(rank, world, entries, hidden, dtype, 0, "cuda")
    buf.write(storages)
    for epoch, tokens in enumerate([1024, 257, 1024]):
        idx = make_indices(rank, world, entries, tokens, ept, epoch=epoch, padding=0.03, device="cuda")
        if epoch == 1:  # pinned host indices: dispatch and gather read them over PCIe
            idx = idx.cpu().pin_memory()
        hooks = buf.fetch(idx)
        outs = [None, None]
        outs[1], outs[0] = hooks[1](), hooks[0]()
        torch.cuda.synchronize()
        _check(outs, idx, entries, hidden, dtype, 0)
    state = buf.runtime.debug_state()
    epochs_before = list(state["epochs"])
    # Layer 0 empty (all padding): its epochs must not advance.
    idx = make_indices(rank, world, entries, 64, ept, epoch=5, device="cuda")
    idx[0].fill_(-1)
    outs = [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    _check(outs, idx, entries, hidden, dtype, 0)
    state = buf.runtime.debug_state()
    assert state["epochs"][:world] == epochs_before[:world]
    # Single-owner traffic: every row from the next rank.
    owner = (rank + 1) % world
    idx = make_indices(rank, world, entries, 512, ept, epoch=6, owner=owner, device="cuda")
    outs = [h() for h in buf.fetch(idx, num_qps=1)]
    torch.cuda.synchronize()
    _check(outs, idx, entries, hidden, dtype, 0)
    # Empty fetch.
    outs = [h() for h in buf.fetch(torch.empty(2, 0, ept, dtype=torch.int32, device="cuda"))]
    dist.barrier()
    mem = buf.memory_usage()
    assert mem["served_requests"] > 0 and mem["served_rows"] > 0
    buf.destroy()


def _host_route_graph(rank, world):
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    entries, hidden, ept, dtype, packs = (10007, 10009), 256, 24, torch.float8_e4m3fn, 2
    buf = _buffer(entries, hidden, 256, ept, dtype, packs, egm=False, local_sf=False)
    storages, scales = pattern_shard(rank, world, entries, hidden, dtype, packs, "cuda")
    buf.write(storages, scales)
    idx = make_indices(rank, world, entries, 256, ept, epoch=2, device="cuda")
    for _ in range(2):
        [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    dist.barrier()
    graph = torch.cuda.CUDAGraph()
    limit = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None] * world
    side = torch.cuda.Stream()
    with torch.cuda.graph(graph):
        idx.add_(1).remainder_(limit)
        hooks = buf.fetch(idx)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            outs = [None, None]
            outs[1], outs[0] = hooks[1](), hooks[0]()
        torch.cuda.current_stream().wait_stream(side)
    for _ in range(4):
        graph.replay()
        torch.cuda.synchronize()
        _check(outs, idx, entries, hidden, dtype, packs)
    del graph
    dist.barrier()
    buf.destroy()


def _mixed_routes(rank, world):
    from engram_rdma_lab_b200 import _native
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    C = _native.load()
    original = C.Runtime.probe_routes
    broken = (0, 1)  # rank 0 cannot map owner 1's mirror

    def probe(runtime, peers, candidates):
        altered = [dict(p) for p in peers]
        if rank == broken[0]:
            altered[broken[1]]["mirror_bytes"] = 0
        return original(runtime, altered, candidates)

    C.Runtime.probe_routes = probe
    try:
        entries, hidden, ept, dtype, packs = (8191, 8209), 256, 24, torch.float8_e4m3fn, 2
        buf = _buffer(entries, hidden, 512, ept, dtype, packs, egm=True, local_sf=True)
    finally:
        C.Runtime.probe_routes = original
    info = buf.get_route_info()
    expected = ["peer_hbm"] * world
    if rank in broken:
        expected[broken[1] if rank == broken[0] else broken[0]] = "host"
        other = broken[1] if rank == broken[0] else broken[0]
        assert "0->1" in info["owner_fallback_reasons"][other]
    assert info["owner_routes"] == expected, info
    storages, scales = pattern_shard(rank, world, entries, hidden, dtype, packs, "cuda")
    buf.write(storages, scales)
    for epoch in range(3):
        idx = make_indices(rank, world, entries, 512, ept, epoch=epoch, padding=0.01, device="cuda")
        outs = [h() for h in buf.fetch(idx)]
        torch.cuda.synchronize()
        _check(outs, idx, entries, hidden, dtype, packs)
    dist.barrier()
    buf.destroy()


def _idle_requesters(rank, world):
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    entries, hidden, ept, dtype = (4099, 4111), 128, 7, torch.bfloat16
    buf = _buffer(entries, hidden, 8192, ept, dtype, 0, egm=False)
    storages, _ = pattern_shard(rank, world, entries, hidden, dtype, 0, "cuda")
    buf.write(storages)
    for epoch in range(3):
        dist.barrier()
        if rank == 0:  # only rank 0 queries; the others only serve
            idx = make_indices(0, world, entries, 8192, ept, epoch=epoch, padding=0.05, device="cuda")
            outs = [h() for h in buf.fetch(idx)]
            torch.cuda.synchronize()
            _check(outs, idx, entries, hidden, dtype, 0)
        dist.barrier()
    buf.destroy()


def _dead_owner_times_out(rank, world):
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    entries, hidden, ept, dtype = (1024, 1024), 128, 4, torch.bfloat16
    buf = _buffer(entries, hidden, 64, ept, dtype, 0, egm=False, timeout=1.0)
    storages, _ = pattern_shard(rank, world, entries, hidden, dtype, 0, "cuda")
    buf.write(storages)
    if rank == 1:
        buf.runtime.debug_stop_service()  # owner 1 stops serving, as if its service died
    dist.barrier()
    if rank == 0:
        idx = make_indices(0, world, entries, 64, ept, owner=1, device="cuda")
        outs = [h() for h in buf.fetch(idx)]
        torch.cuda.synchronize()  # the bounded wait returns after ~1 s
        state = buf.error_state()
        assert state["status"] == 1 and state["owner"] == 1, state
        with pytest.raises(RuntimeError, match="timed out"):
            buf.fetch(idx)
    dist.barrier()
    buf.destroy()


def _hot_replica(rank, world):
    from engram_rdma_lab_b200.models import make_indices, pattern_shard

    _setup(rank)
    entries, hidden, ept, dtype, packs = (20011, 20021), 256, 24, torch.float8_e4m3fn, 2
    os.environ["ENGRAM_HOT_ROWS"] = "30000"  # spans owners 0 and 1
    try:
        for egm in (True, False):  # the replica fills through either route
            buf = _buffer(entries, hidden, 512, ept, dtype, packs, egm=egm, local_sf=True)
            assert buf.hot_rows == [30000, 30000]
            for salt in (0, 3):
                storages, scales = pattern_shard(rank, world, entries, hidden, dtype, packs, "cuda", salt=salt)
                buf.write(storages, scales)
                for epoch in range(3):
                    idx = make_indices(rank, world, entries, 512, ept, epoch=epoch, padding=0.02,
                                       distribution="zipf" if epoch else "uniform", device="cuda")
                    outs = [h() for h in buf.fetch(idx)]
                    torch.cuda.synchronize()
                    _check(outs, idx, entries, hidden, dtype, packs, salt=salt)
            dist.barrier()
            buf.destroy()
    finally:
        os.environ.pop("ENGRAM_HOT_ROWS", None)


def test_hot_prefix_replica(port):
    run_ranks(_hot_replica, _world(), port)


def _litmus(rank, world):
    _setup(rank)
    buf = _buffer((4099, 4111), 256, 512, 24, torch.bfloat16, 0, egm=True)
    rt = buf.runtime
    for producer, words, epochs, weak in ((0, 64, 4000, False), (1, 65536, 1000, False), (0, 4096, 2000, True)):
        consumer = 1 - producer
        rt.debug_litmus_reset()
        dist.barrier()
        if rank == producer:
            r = rt.debug_litmus(consumer, "producer", epochs, words, ctas=16, weak_loads=weak, timeout_ms=5000.0)
            assert r["status"] == 0, r
        elif rank == consumer:
            r = rt.debug_litmus(producer, "consumer", epochs, words, ctas=16, weak_loads=weak, timeout_ms=5000.0)
            assert r["status"] == 0 and r["mismatches"] == 0 and r["epochs_done"] == epochs, r
        dist.barrier()
    # A consumer whose producer never runs gives up after its bounded wait.
    rt.debug_litmus_reset()
    dist.barrier()
    if rank == 1:
        r = rt.debug_litmus(0, "consumer", 10, 64, ctas=2, timeout_ms=200.0)
        assert r["status"] == 2 and r["epoch"] == 1 and r["epochs_done"] == 0, r
    dist.barrier()
    buf.destroy()


def _device_barrier(rank, world):
    _setup(rank)
    buf = _buffer((4099, 4111), 256, 64, 4, torch.bfloat16, 0, egm=True, timeout=1.0)
    for _ in range(200):  # back to back: the counts stay in step without resets
        buf.device_barrier()
    state = buf.runtime.barrier_state()
    assert state["count"] == 200 and state["slots"] == [200] * world, state
    # A late rank holds everyone: rank 0 sleeps on its stream before arriving.
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if rank == 0:
        torch.cuda._sleep(100_000_000)  # ~50 ms of GPU cycles
    start.record()
    buf.device_barrier()
    end.record()
    torch.cuda.synchronize()
    if rank != 0:
        assert start.elapsed_time(end) > 10.0, start.elapsed_time(end)
    # Captured into a graph: each replay advances the counts.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        buf.device_barrier()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    del graph
    assert buf.runtime.barrier_state()["count"] == 204
    assert buf.error_state()["status"] == 0
    # A rank whose peers never arrive gives up after the bounded wait.
    dist.barrier()
    if rank == 0:
        buf.device_barrier()
        torch.cuda.synchronize()
        state = buf.error_state()
        assert state["status"] == 6 and state["expected"] == 205, state
        with pytest.raises(RuntimeError, match="barrier"):
            buf.device_barrier()
    dist.barrier()
    buf.destroy()


def test_device_barrier(port):
    run_ranks(_device_barrier, _world(), port)


def test_flag_protocol_litmus_two_gpus(port):
    run_ranks(_litmus, 2, port)


def test_peer_hbm_route(port):
    run_ranks(_peer_hbm, _world(), port)


def test_host_route(port):
    run_ranks(_host_route, _world(), port)


def test_host_route_graph(port):
    run_ranks(_host_route_graph, _world(), port)


def test_mixed_routes_after_probe_failure(port):
    run_ranks(_mixed_routes, _world(), port)


def test_idle_requesters_still_served(port):
    run_ranks(_idle_requesters, _world(), port)


def test_dead_owner_bounded_timeout(port):
    run_ranks(_dead_owner_times_out, 2, port)
