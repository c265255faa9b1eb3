"""EngramBuffer on one B200 (world_size=1): the gather kernel end to end.

Every output is compared bit-exactly with the pattern oracle or with plain
torch indexing of the written tables.
"""

import os

import pytest
import torch
import torch.distributed as dist

from engram_rdma_lab_b200 import EngramBuffer
from engram_rdma_lab_b200.models import expected_outputs, make_indices, pattern_shard

from .conftest import free_port

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def world1():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    if not dist.is_initialized():
        dist.init_process_group("gloo", rank=0, world_size=1, init_method=f"tcp://127.0.0.1:{free_port()}")
    yield
    # Leave the group for the rest of the session.


def make_buffer(entries, hidden, max_tokens, ept, dtype, packs, egm, local_sf=None, timeout=20):
    os.environ["ENGRAM_EGM_ENABLE"] = "1" if egm else "0"
    if local_sf is None:
        os.environ.pop("ENGRAM_WRITE_LOCAL_SF", None)
    else:
        os.environ["ENGRAM_WRITE_LOCAL_SF"] = "1" if local_sf else "0"
    group = dist.group.WORLD
    sizes = EngramBuffer.get_storage_size_hint(group, entries, hidden, max_tokens, ept, dtype, packs)
    cfg = EngramBuffer.get_theoretical_config(group, len(entries), max_tokens, ept)
    buf = EngramBuffer(group, *sizes, True, *cfg, num_gpu_timeout_secs=timeout, explicitly_destroy=True)
    buf.set_config(entries, hidden, max_tokens, ept, dtype, packs)
    return buf


def check(outputs, indices, entries, hidden, dtype, packs, salt=0, col_major=True):
    exp = expected_outputs(indices.cpu(), entries, hidden, dtype, packs, salt)
    T, E = indices.shape[1], indices.shape[2]
    for layer, out in enumerate(outputs):
        data, sf = out if packs else (out, None)
        assert data.shape == (T, E * hidden) and data.dtype == dtype and data.is_cuda
        assert torch.equal(data.view(torch.uint8).reshape(T, -1).cpu(), exp[layer][0]), f"layer {layer} data"
        if packs:
            assert sf.shape == (T, E * packs)
            assert sf.stride() == ((1, (T + 3) // 4 * 4) if col_major else (E * packs, 1))
            assert torch.equal(sf.cpu(), exp[layer][1]), f"layer {layer} scales"


@pytest.mark.parametrize("egm", [True, False])
def test_bf16_gather(egm):
    entries, hidden, ept = (5000, 7001), 256, 8
    buf = make_buffer(entries, hidden, 1024, ept, torch.bfloat16, 0, egm)
    storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda")
    buf.write(storages)
    for epoch, tokens in enumerate([1024, 333, 1]):
        idx = make_indices(0, 1, entries, tokens, ept, epoch=epoch, padding=0.05, device="cuda")
        hooks = buf.fetch(idx)
        outs = [None, None]
        outs[1], outs[0] = hooks[1](), hooks[0]()  # reverse order
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, torch.bfloat16, 0)
    info = buf.get_route_info()
    assert info["owner_routes"] == ["peer_hbm" if egm else "host"]
    mem = info["memory"]
    assert mem["hbm_mirror_bytes"] == (sum(entries) * hidden * 2 if egm else 0)
    assert mem["kernel_launches"] >= 3
    buf.destroy()


@pytest.mark.parametrize("local_sf", [True, False])
@pytest.mark.parametrize("hidden,packs", [(256, 2), (512, 4), (128, 1)])
def test_fp8_gather_and_scales(local_sf, hidden, packs):
    entries, ept = (3001, 4099), 24
    buf = make_buffer(entries, hidden, 512, ept, torch.float8_e4m3fn, packs, True, local_sf)
    storages, scales = pattern_shard(0, 1, entries, hidden, torch.float8_e4m3fn, packs, "cuda")
    buf.write(storages, scales)
    for col_major in (True, False):
        idx = make_indices(0, 1, entries, 509, ept, epoch=7, padding=0.03, device="cuda")
        outs = [h() for h in buf.fetch(idx, use_tma_aligned_col_major_sf=col_major)]
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, torch.float8_e4m3fn, packs, col_major=col_major)
    buf.destroy()


def test_matches_plain_torch_indexing_with_cpu_weights():
    entries, hidden, ept = (4096, 4100), 64, 4
    buf = make_buffer(entries, hidden, 256, ept, torch.bfloat16, 0, False)
    g = torch.Generator().manual_seed(3)
    tables = [(torch.randn(n, hidden, generator=g) * 0.02).to(torch.bfloat16) for n in entries]
    buf.write(tables)  # CPU tensors
    idx = make_indices(0, 1, entries, 256, ept, padding=0.1, device="cuda")
    outs = [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    for layer, table in enumerate(tables):
        x = idx[layer].cpu().long()
        ref = table.float()[x.clamp_min(0)] * (x >= 0)[..., None]
        assert torch.equal(outs[layer].cpu().float().reshape(256, ept, hidden), ref)
    buf.destroy()


def test_zero_tokens_and_capacity_checks():
    entries, hidden, ept = (100, 200), 64, 3
    buf = make_buffer(entries, hidden, 16, ept, torch.bfloat16, 0, True)
    storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda")
    buf.write(storages)
    outs = [h() for h in buf.fetch(torch.empty(2, 0, ept, dtype=torch.int32, device="cuda"))]
    assert all(o.shape == (0, ept * hidden) for o in outs)
    with pytest.raises(ValueError):
        buf.fetch(torch.zeros(2, 17, ept, dtype=torch.int32, device="cuda"))  # over capacity
    with pytest.raises(ValueError):
        buf.fetch(torch.zeros(2, 4, ept, dtype=torch.int32))  # CPU indices
    buf.destroy()


def test_cuda_graph_replay_and_cross_stream_hooks():
    entries, hidden, ept = (9000, 9001), 256, 24
    buf = make_buffer(entries, hidden, 256, ept, torch.float8_e4m3fn, 2, True)
    storages, scales = pattern_shard(0, 1, entries, hidden, torch.float8_e4m3fn, 2, "cuda")
    buf.write(storages, scales)
    idx = make_indices(0, 1, entries, 256, ept, padding=0.02, device="cuda")
    side = torch.cuda.Stream()
    for _ in range(2):  # warm up outside the graph
        outs = [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None]
    with torch.cuda.graph(graph):
        idx.add_(7).remainder_(n)  # the producer is part of the graph
        hooks = buf.fetch(idx)
        outs = [None, None]
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            outs[1] = hooks[1]()
            outs[0] = hooks[0]()
        torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, torch.float8_e4m3fn, 2)
    # Eager fetch after the graph still works and waits for the graph's layers.
    more = [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    check(more, idx, entries, hidden, torch.float8_e4m3fn, 2)
    del graph
    buf.destroy()


def test_out_of_range_index_reports_error():
    entries, hidden, ept = (64, 64), 64, 2
    buf = make_buffer(entries, hidden, 8, ept, torch.bfloat16, 0, True)
    storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda")
    buf.write(storages)
    idx = torch.zeros(2, 8, ept, dtype=torch.int32, device="cuda")
    idx[1, 3, 1] = 64 * 5  # beyond the single rank's vocabulary
    hooks = buf.fetch(idx)
    torch.cuda.synchronize()  # the kernel has reported by now
    state = buf.error_state()
    assert state["status"] == 2 and state["layer"] == 1 and state["owner"] == 5
    with pytest.raises(RuntimeError, match="outside the vocabulary"):
        hooks[0]()  # hooks re-raise the latched device error
    buf._pending = set()  # a raising hook leaves its layer pending
    with pytest.raises(RuntimeError, match="outside the vocabulary"):
        buf.fetch(idx)
    buf._pending = set()
    buf.destroy()


def test_bounded_wait_times_out_without_fault():
    entries, hidden, ept = (64,), 64, 2
    buf = make_buffer(entries, hidden, 8, ept, torch.bfloat16, 0, True)
    result = buf.runtime.run_wait_probe(200.0)
    assert result["status"] == 1  # timeout reported
    assert result["elapsed_ms"] >= 150
    # The context is still usable.
    storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda")
    buf.write(storages)
    idx = make_indices(0, 1, entries, 8, ept, device="cuda")
    outs = [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    check(outs, idx, entries, hidden, torch.bfloat16, 0)
    buf.destroy()


def test_native_extension_is_in_tree():
    from engram_rdma_lab_b200 import _native

    mod = _native.load()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    assert os.path.realpath(mod.__file__).startswith(os.path.realpath(root))


@pytest.mark.parametrize("kernel", ["simt", "bulk"])
@pytest.mark.parametrize("mode", ["1", "auto"])
def test_dedup_on_skewed_requests(kernel, mode, monkeypatch):
    monkeypatch.setenv("ENGRAM_DEDUP", mode)
    monkeypatch.setenv("ENGRAM_GATHER_KERNEL", kernel)
    entries, hidden, ept, dtype, packs = (20011, 20021), 256, 24, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 1024, ept, dtype, packs, True)
    storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda")
    buf.write(storages, scales)
    for epoch in range(4):
        idx = make_indices(0, 1, entries, 1024 - 100 * epoch, ept, epoch=epoch, distribution="zipf", padding=0.03,
                           device="cuda")
        outs = [h() for h in buf.fetch(idx)]
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, dtype, packs)
    idx = make_indices(0, 1, entries, 1024, ept, epoch=9, distribution="zipf", device="cuda")
    [h() for h in buf.fetch(idx)]
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    n = torch.tensor(entries, device="cuda", dtype=torch.int32)[:, None, None]
    with torch.cuda.graph(graph):
        idx.add_(1).remainder_(n)
        outs = [h() for h in buf.fetch(idx)]
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, dtype, packs)
    del graph
    mem = buf.memory_usage()
    assert mem["dedup_fetches"] >= 4
    assert 0 < mem["dedup_last_unique_ratio"] < 0.75
    buf.destroy()


def test_dedup_auto_turns_off_for_uniform_requests(monkeypatch):
    monkeypatch.setenv("ENGRAM_DEDUP", "auto")
    entries, hidden, ept = (200003, 200009), 128, 8
    buf = make_buffer(entries, hidden, 512, ept, torch.bfloat16, 0, True)
    storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda")
    buf.write(storages)
    for epoch in range(10):
        idx = make_indices(0, 1, entries, 512, ept, epoch=epoch, device="cuda")
        outs = [h() for h in buf.fetch(idx)]
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, torch.bfloat16, 0)
    mem = buf.memory_usage()
    assert mem["dedup_last_unique_ratio"] > 0.9
    assert mem["dedup_fetches"] <= 2  # measured once, then off until the next probe
    buf.destroy()


def _pinned_view(idx, offset):
    """``idx`` copied into a pinned block at an element offset (not 16-byte aligned for odd offsets)."""
    block = torch.full((idx.numel() + offset,), -7, dtype=torch.int32).pin_memory()
    host = block[offset:].view(idx.shape)
    host.copy_(idx)
    assert host.is_pinned() and host.is_contiguous()
    return host


@pytest.mark.parametrize("kernel", ["simt", "bulk"])
@pytest.mark.parametrize("dedup", ["0", "1"])
@pytest.mark.parametrize("staging", ["0", "1"])
def test_pinned_host_indices_read_in_place(kernel, dedup, staging, monkeypatch):
    monkeypatch.setenv("ENGRAM_GATHER_KERNEL", kernel)
    monkeypatch.setenv("ENGRAM_DEDUP", dedup)
    monkeypatch.setenv("ENGRAM_INDEX_STAGING", staging)
    entries, hidden, ept, dtype, packs = (5003, 5009), 256, 24, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 512, ept, dtype, packs, True)
    try:
        storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda")
        buf.write(storages, scales)
        for epoch, (tokens, col_major, offset) in enumerate([(300, True, 1001), (512, False, 0), (77, True, 3)]):
            idx = make_indices(0, 1, entries, tokens, ept, epoch=epoch, padding=0.05,
                               distribution="zipf" if dedup == "1" else "uniform")
            host = _pinned_view(idx, offset)
            outs = [h() for h in buf.fetch(host, use_tma_aligned_col_major_sf=col_major)]
            torch.cuda.synchronize()
            check(outs, idx, entries, hidden, dtype, packs, col_major=col_major)
        with pytest.raises(ValueError, match="pinned host"):
            buf.fetch(idx.clone())  # pageable host memory is refused before any launch
        assert buf.memory_usage()["index_staging"] == (staging == "1")
        # Back-to-back fetches from rotating pinned tensors, checked after the last.
        pool = [_pinned_view(make_indices(0, 1, entries, 512, ept, epoch=10 + k), 0) for k in range(3)]
        for k in range(7):
            outs = [h() for h in buf.fetch(pool[k % 3])]
        torch.cuda.synchronize()
        check(outs, pool[6 % 3], entries, hidden, dtype, packs)
    finally:
        buf.destroy()


@pytest.mark.parametrize("staging", ["0", "1"])
def test_write_combined_pinned_indices(staging, monkeypatch):
    """EngramBuffer.pinned_indices: write-combined pinned memory as fetch input, staged or read in place."""
    monkeypatch.setenv("ENGRAM_INDEX_STAGING", staging)
    entries, hidden, ept, dtype, packs = (5003, 5009), 256, 24, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 512, ept, dtype, packs, True)
    try:
        storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda")
        buf.write(storages, scales)
        pool = [buf.pinned_indices(tokens) for tokens in (512, 300, 512)]
        assert all(t.is_pinned() for t in pool)
        with pytest.raises(ValueError):
            buf.pinned_indices(513)
        for k in range(6):
            idx = make_indices(0, 1, entries, pool[k % 3].shape[1], ept, epoch=20 + k, padding=0.05)
            torch.cuda.synchronize()  # the fetch that read this buffer three steps ago is done
            pool[k % 3].copy_(idx)
            outs = buf.fetch_all(pool[k % 3])
            torch.cuda.synchronize()
            check(outs, idx, entries, hidden, dtype, packs)
        plain = buf.pinned_indices(64, write_combined=False)
        assert plain.is_pinned() and plain.shape == (2, 64, ept)
    finally:
        buf.destroy()


def test_pinned_host_indices_under_graph_capture():
    entries, hidden, ept = (4099, 4111), 128, 8
    buf = make_buffer(entries, hidden, 256, ept, torch.bfloat16, 0, True)
    try:
        storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda")
        buf.write(storages)
        idx = make_indices(0, 1, entries, 256, ept, epoch=1)
        host = _pinned_view(idx, 0)
        [h() for h in buf.fetch(host)]
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = [h() for h in buf.fetch(host)]
        for epoch in range(2, 4):  # the graph reads whatever the host buffer holds at replay
            idx = make_indices(0, 1, entries, 256, ept, epoch=epoch)
            host.copy_(idx)
            graph.replay()
            torch.cuda.synchronize()
            check(outs, idx, entries, hidden, torch.bfloat16, 0)
        del graph
    finally:
        buf.destroy()


@pytest.mark.parametrize("weak_loads", [False, True])
def test_flag_protocol_litmus_one_gpu(weak_loads):
    """Producer and consumer CTAs of one cooperative launch run the release/acquire protocol for many epochs."""
    buf = make_buffer((4099, 4111), 256, 512, 24, torch.bfloat16, 0, True)
    try:
        rt = buf.runtime
        for words, epochs in ((64, 4000), (65536, 1000)):
            rt.debug_litmus_reset()
            r = rt.debug_litmus(0, "both", epochs, words, ctas=16, weak_loads=weak_loads, timeout_ms=2000.0)
            assert r["status"] == 0, r
            assert r["mismatches"] == 0 and r["first_bad_epoch"] == -1, r
            assert r["epochs_done"] == epochs, r
        with pytest.raises(RuntimeError, match="alone"):
            rt.debug_litmus(0, "producer", 1, 64)
    finally:
        buf.destroy()


@pytest.mark.parametrize("kernel", ["simt", "bulk"])
def test_hot_prefix_replica_follows_rewrites(kernel, monkeypatch):
    monkeypatch.setenv("ENGRAM_GATHER_KERNEL", kernel)
    monkeypatch.setenv("ENGRAM_HOT_ROWS", "3000,700")
    entries, hidden, ept, dtype, packs = (5003, 5009), 256, 24, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 256, ept, dtype, packs, True)
    try:
        assert buf.hot_rows == [3000, 700]
        mem = buf.memory_usage()
        assert mem["hot_replica_bytes"] == 3700 * 256 and not mem["hot_replica_active"]
        for salt in (0, 5):  # a rewrite must refresh the replica
            storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda", salt=salt)
            buf.write(storages, scales)
            assert buf.memory_usage()["hot_replica_active"]
            for epoch in range(3):
                idx = make_indices(0, 1, entries, 256, ept, epoch=epoch, distribution="zipf", padding=0.02,
                                   device="cuda")
                assert int((idx[0] < 3000).sum()) > 0
                outs = [h() for h in buf.fetch(idx)]
                torch.cuda.synchronize()
                check(outs, idx, entries, hidden, dtype, packs, salt=salt)
    finally:
        buf.destroy()


@pytest.mark.parametrize("local_sf", [False, True])
def test_state_dict_roundtrip_native(local_sf):
    import io

    entries, hidden, ept, dtype, packs = (3001, 3011), 256, 8, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 128, ept, dtype, packs, True, local_sf=local_sf)
    storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda", salt=11)
    buf.write(storages, scales)
    blob = io.BytesIO()
    torch.save(buf.state_dict(), blob)
    buf.destroy()
    fresh = make_buffer(entries, hidden, 128, ept, dtype, packs, True, local_sf=local_sf)
    try:
        state = torch.load(io.BytesIO(blob.getvalue()))
        for layer in range(2):
            assert torch.equal(state["storages"][layer].view(torch.uint8), storages[layer].cpu().view(torch.uint8))
            assert torch.equal(state["sfs"][layer], scales[layer].cpu())
        fresh.load_state_dict(state)
        idx = make_indices(0, 1, entries, 128, ept, epoch=3, padding=0.05, device="cuda")
        outs = [h() for h in fresh.fetch(idx)]
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, dtype, packs, salt=11)
    finally:
        fresh.destroy()


def test_device_barrier_one_rank_and_probe():
    """The device barrier on one rank (its own slot only), and the random-row probe on the local mirror."""
    buf = make_buffer((4099, 4111), 256, 64, 4, torch.bfloat16, 0, True)
    try:
        for _ in range(10):
            buf.device_barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            buf.device_barrier()
        graph.replay()
        torch.cuda.synchronize()
        del graph
        assert buf.runtime.barrier_state() == {"count": 11, "slots": [11]}
        for mode in range(10):  # every ProbeMode, local rows only at world size 1
            us = buf.runtime.debug_peer_probe(mode, mode, 4096, 148)
            assert us > 0
        assert buf.error_state()["status"] == 0
    finally:
        buf.destroy()


@pytest.mark.parametrize("egm", [False, True])
def test_host_route_serving_on_one_gpu(egm):
    """The push kernel and a serving hook move a request of this rank to itself, bit-exactly, epoch after epoch."""
    entries, hidden = (5003, 5009), 256
    buf = make_buffer(entries, hidden, 512, 8, torch.bfloat16, 0, egm)
    try:
        storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda", salt=3)
        buf.write(storages)
        for rows, worker, blocks in ((4096, "push", 8), (4096, "hook", 8), (777, "push", 148), (1, "hook", 8)):
            r = buf.runtime.debug_serve_local(rows, worker, blocks)
            assert r["mismatched_rows"] == 0 and r["done_epoch"] == r["expected_epoch"], r
        assert buf.error_state()["status"] == 0
    finally:
        buf.destroy()


@pytest.mark.parametrize("egm", [False, True])
def test_serving_with_small_chunks_many_claims(egm, monkeypatch):
    """64-row chunks: a 4096-row request is 64 claims raced by up to 296 CTAs (and the control warps' early
    claims of the next chunk), epoch after epoch, including a request that ends in a partial chunk."""
    monkeypatch.setenv("ENGRAM_SERVE_CHUNK_ROWS", "64")
    entries, hidden = (5003, 5009), 256
    buf = make_buffer(entries, hidden, 512, 8, torch.bfloat16, 0, egm)
    try:
        assert buf.memory_usage()["serve_chunk_rows"] == 64
        storages, _ = pattern_shard(0, 1, entries, hidden, torch.bfloat16, 0, "cuda", salt=5)
        buf.write(storages)
        for rows, worker, blocks in ((4096, "push", 296), (4096, "hook", 8), (4033, "push", 148), (65, "hook", 8),
                                     (4096, "push", 16)):
            r = buf.runtime.debug_serve_local(rows, worker, blocks)
            assert r["mismatched_rows"] == 0 and r["done_epoch"] == r["expected_epoch"], r
        assert buf.error_state()["status"] == 0
    finally:
        buf.destroy()


def test_fetch_all_matches_hooks_and_supersedes_them():
    entries, hidden, ept, dtype, packs = (4099, 4111), 256, 24, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 256, ept, dtype, packs, True)
    try:
        storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda", salt=2)
        buf.write(storages, scales)
        idx = make_indices(0, 1, entries, 256, ept, epoch=7, padding=0.05, device="cuda")
        hooks = buf.fetch(idx)
        for hook in hooks:
            hook()
        outs = buf.fetch_all(idx)
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, dtype, packs, salt=2)
        with pytest.raises(RuntimeError, match="superseded"):
            hooks[0]()
        # Pinned host indices and graph capture take the same path.
        host = idx.cpu().pin_memory()
        outs = buf.fetch_all(host)
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, dtype, packs, salt=2)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            outs = buf.fetch_all(idx)
        idx.copy_(make_indices(0, 1, entries, 256, ept, epoch=8, device="cuda"))
        graph.replay()
        torch.cuda.synchronize()
        check(outs, idx, entries, hidden, dtype, packs, salt=2)
        del graph
    finally:
        buf.destroy()


@pytest.mark.parametrize("l2_prefetch", ["0", "1"])
def test_simt_gather_256_bit_vectors(l2_prefetch, monkeypatch):
    """256-bit loads and stores, with and without the 256-byte L2 prefetch-size hint, bit-exact."""
    monkeypatch.setenv("ENGRAM_GATHER_VECTOR", "32")
    monkeypatch.setenv("ENGRAM_GATHER_L2_PREFETCH", l2_prefetch)
    entries, hidden, ept, dtype, packs = (8191, 8209), 256, 24, torch.float8_e4m3fn, 2
    buf = make_buffer(entries, hidden, 512, ept, dtype, packs, True)
    try:
        mem = buf.memory_usage()
        assert mem["gather_vector_bytes"] == 32 and mem["gather_l2_prefetch"] == (l2_prefetch == "1")
        storages, scales = pattern_shard(0, 1, entries, hidden, dtype, packs, "cuda", salt=4)
        buf.write(storages, scales)
        for tokens in (512, 37, 1):
            idx = make_indices(0, 1, entries, tokens, ept, epoch=tokens, padding=0.03, device="cuda")
            outs = buf.fetch_all(idx)
            torch.cuda.synchronize()
            check(outs, idx, entries, hidden, dtype, packs, salt=4)
    finally:
        buf.destroy()
