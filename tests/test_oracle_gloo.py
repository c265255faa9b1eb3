"""The pure-torch EngramBuffer over gloo with world_size=2 (no GPU).

Covers the oracle configuration: 2 layers, per-rank entries [2048, 2050],
hidden 64, ept 4, 128 tokens, BF16, 10% padding, plus FP8 with both scale
layouts, out-of-order hooks, stale/pending hook errors, empty fetches and a
weight rewrite.
"""

import pytest
import torch
import torch.distributed as dist

from engram_rdma_lab_b200 import TorchEngramBuffer
from engram_rdma_lab_b200.models import CONFIGS, expected_outputs, make_indices, pattern_shard

from ._spawn import run_ranks


def _make(world, spec, dtype, packs, local_sf="1"):
    import os

    os.environ["ENGRAM_EGM_ENABLE"] = "0"
    os.environ["ENGRAM_WRITE_LOCAL_SF"] = local_sf
    group = dist.group.WORLD
    sizes = TorchEngramBuffer.get_storage_size_hint(group, spec.entries, spec.hidden, spec.max_tokens, spec.ept,
                                                    dtype, packs)
    cfg = TorchEngramBuffer.get_theoretical_config(group, len(spec.entries), spec.max_tokens, spec.ept)
    buf = TorchEngramBuffer(group, *sizes, True, *cfg, explicitly_destroy=True)
    buf.set_config(spec.entries, spec.hidden, spec.max_tokens, spec.ept, dtype, packs)
    return buf


def _check(outputs, indices, spec, dtype, packs, salt=0, col_major=True):
    exp = expected_outputs(indices, spec.entries, spec.hidden, dtype, packs, salt)
    T, E = indices.shape[1], indices.shape[2]
    for layer, out in enumerate(outputs):
        data, sf = out if packs else (out, None)
        assert data.shape == (T, E * spec.hidden) and data.dtype == dtype
        assert torch.equal(data.contiguous().view(torch.uint8).reshape(T, -1), exp[layer][0])
        if packs:
            assert sf.shape == (T, E * packs) and sf.dtype == torch.float32
            want = (1, (T + 3) // 4 * 4) if col_major else (E * packs, 1)
            assert sf.stride() == want
            assert torch.equal(sf, exp[layer][1])


def _oracle_bf16(rank, world):
    spec = CONFIGS["oracle"]
    buf = _make(world, spec, torch.bfloat16, 0)
    storages, _ = pattern_shard(rank, world, spec.entries, spec.hidden, torch.bfloat16, 0, "cpu")
    with pytest.raises(RuntimeError):
        buf.fetch(make_indices(rank, world, spec.entries, spec.tokens, spec.ept))  # before write
    buf.write(storages)
    idx = make_indices(rank, world, spec.entries, spec.tokens, spec.ept, padding=spec.padding)
    hooks = buf.fetch(idx)
    with pytest.raises(RuntimeError):
        buf.fetch(idx)  # pending hooks
    outs = [None, None]
    outs[1] = hooks[1]()  # out of order
    outs[0] = hooks[0]()
    assert outs[0].shape == (128, 256)
    _check(outs, idx, spec, torch.bfloat16, 0)
    with pytest.raises(RuntimeError):
        hooks[0]()  # already called
    newer = buf.fetch(idx)
    with pytest.raises(RuntimeError):
        hooks[1]()  # superseded
    for h in newer:
        h()
    # Empty fetch.
    empty = torch.empty(2, 0, spec.ept, dtype=torch.int32)
    outs = [h() for h in buf.fetch(empty)]
    assert all(o.shape == (0, spec.ept * spec.hidden) for o in outs)
    # Bad shapes.
    with pytest.raises(ValueError):
        buf.fetch(idx[:, :, :2].contiguous())
    with pytest.raises(ValueError):
        buf.fetch(idx.to(torch.int64))
    info = buf.get_route_info()
    assert set(info) >= {"egm_enabled", "owner_routes", "owner_fallback_reasons", "memory"}
    assert len(info["owner_routes"]) == world
    buf.destroy()
    with pytest.raises(RuntimeError):
        buf.fetch(idx)


def _oracle_fp8(rank, world, local_sf):
    spec = CONFIGS["oracle"].with_(hidden=256, tokens=37, max_tokens=64)
    dtype, packs = torch.float8_e4m3fn, 2
    buf = _make(world, spec, dtype, packs, local_sf)
    storages, scales = pattern_shard(rank, world, spec.entries, spec.hidden, dtype, packs, "cpu")
    buf.write(storages, scales)
    for col_major in (True, False):
        idx = make_indices(rank, world, spec.entries, spec.tokens, spec.ept, padding=0.1, epoch=3)
        outs = [h() for h in buf.fetch(idx, use_tma_aligned_col_major_sf=col_major)]
        _check(outs, idx, spec, dtype, packs, col_major=col_major)
    # Rewrite with new weights (weight update) and fetch again.
    storages, scales = pattern_shard(rank, world, spec.entries, spec.hidden, dtype, packs, "cpu", salt=17)
    buf.write(storages, scales)
    idx = make_indices(rank, world, spec.entries, spec.tokens, spec.ept, epoch=4)
    outs = [h() for h in buf.fetch(idx)]
    _check(outs, idx, spec, dtype, packs, salt=17)
    with pytest.raises(ValueError):
        buf.write(storages, None)  # FP8 needs scales
    hooks = buf.fetch(idx)
    with pytest.raises(RuntimeError):
        buf.destroy()  # outstanding hooks
    for h in hooks:
        h()
    buf.destroy()


def test_oracle_bf16_world2(port):
    run_ranks(_oracle_bf16, 2, port)


@pytest.mark.parametrize("local_sf", ["0", "1"])
def test_oracle_fp8_world2(port, local_sf):
    run_ranks(_oracle_fp8, 2, port, args=(local_sf,))


def _config_errors(rank, world):
    spec = CONFIGS["oracle"]
    group = dist.group.WORLD
    sizes = TorchEngramBuffer.get_storage_size_hint(group, spec.entries, spec.hidden, spec.max_tokens, spec.ept,
                                                    torch.bfloat16, 0)
    small = TorchEngramBuffer(group, sizes[0] // 4, sizes[1], True, 1, 1024, explicitly_destroy=True)
    with pytest.raises(ValueError):
        small.set_config(spec.entries, spec.hidden, spec.max_tokens, spec.ept, torch.bfloat16, 0)
    with pytest.raises(ValueError):
        TorchEngramBuffer(group, *sizes, True, 17, 1024)
    implicit = TorchEngramBuffer(group, *sizes, True, 1, 1024)
    with pytest.raises(RuntimeError):
        implicit.destroy()  # explicitly_destroy=False
    import os

    os.environ["ENGRAM_EGM_ENABLE"] = "1"
    with pytest.raises(ValueError, match="allow_hybrid_mode"):
        TorchEngramBuffer(group, *sizes, True, 1, 1024, allow_hybrid_mode=False)
    os.environ["ENGRAM_EGM_ENABLE"] = "0"
    TorchEngramBuffer(group, *sizes, True, 1, 1024, allow_hybrid_mode=False, explicitly_destroy=True).destroy()


def test_oracle_config_errors(port):
    run_ranks(_config_errors, 2, port)


def _state_roundtrip(rank, world, local_sf):
    import io

    spec = CONFIGS["oracle"]
    dtype, packs = torch.float8_e4m3fn, 2
    buf = _make(world, spec, dtype, packs, local_sf)
    storages, scales = pattern_shard(rank, world, spec.entries, spec.hidden, dtype, packs, "cpu", salt=7)
    buf.write(storages, scales)
    blob = io.BytesIO()
    torch.save(buf.state_dict(), blob)
    buf.destroy()
    fresh = _make(world, spec, dtype, packs, local_sf)
    state = torch.load(io.BytesIO(blob.getvalue()))
    for layer in range(len(spec.entries)):
        assert torch.equal(state["storages"][layer].view(torch.uint8), storages[layer].view(torch.uint8))
        n = spec.entries[layer]
        mine = slice(rank * n, (rank + 1) * n)
        assert torch.equal(state["sfs"][layer][mine], scales[layer][mine])
        if local_sf == "1":
            assert torch.equal(state["sfs"][layer], scales[layer])
    bad = dict(state, rank=1 - rank)
    with pytest.raises(ValueError):
        fresh.load_state_dict(bad)
    fresh.load_state_dict(state)
    idx = make_indices(rank, world, spec.entries, spec.tokens, spec.ept, padding=spec.padding)
    _check([h() for h in fresh.fetch(idx)], idx, spec, dtype, packs, salt=7)
    fresh.destroy()


@pytest.mark.parametrize("local_sf", ["0", "1"])
def test_state_dict_roundtrip_world2(port, local_sf):
    run_ranks(_state_roundtrip, 2, port, args=(local_sf,))


def _fetch_all_and_barrier(rank, world):
    spec = CONFIGS["oracle"]
    buf = _make(world, spec, torch.bfloat16, 0)
    storages, _ = pattern_shard(rank, world, spec.entries, spec.hidden, torch.bfloat16, 0, "cpu")
    buf.write(storages)
    idx = make_indices(rank, world, spec.entries, spec.tokens, spec.ept, epoch=3, padding=spec.padding)
    hooks = buf.fetch(idx)
    for hook in hooks:
        hook()
    outs = buf.fetch_all(idx)  # fetch and every hook, in layer order
    _check(outs, idx, spec, torch.bfloat16, 0)
    with pytest.raises(RuntimeError):
        hooks[0]()  # superseded by fetch_all
    buf.device_barrier()  # on this group: a one-word all-reduce
    host = buf.pinned_indices(spec.tokens)
    assert host.shape == idx.shape and host.dtype == torch.int32
    host.copy_(idx)
    _check(buf.fetch_all(host), idx, spec, torch.bfloat16, 0)
    with pytest.raises(ValueError):
        buf.pinned_indices(spec.max_tokens + 1)
    buf.destroy()


def test_fetch_all_and_device_barrier_gloo(port):
    run_ranks(_fetch_all_and_barrier, 2, port)
