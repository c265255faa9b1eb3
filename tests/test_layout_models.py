"""Configuration checks, memory plan, synthetic tables and index streams (host only)."""

import pytest
import torch

from engram_rdma_lab_b200.buffer import theoretical_config
from engram_rdma_lab_b200.layout import (
    ALLOC_ALIGN,
    REGION_ALIGN,
    plan_memory,
    sf_strides,
    storage_size_hint,
    validate_config,
)
from engram_rdma_lab_b200.models import (
    CONFIGS,
    expected_outputs,
    make_indices,
    pattern_scales,
    pattern_shard,
    row_pattern,
)
from engram_rdma_lab_b200.ops import dequantize_fp8_blockwise, quantize_fp8_blockwise


def test_validate_config_rules():
    validate_config([10, 11], 64, 8, 2, torch.bfloat16, 0, world=2)
    with pytest.raises(ValueError):
        validate_config([10], 64, 8, 2, torch.bfloat16, 2)  # BF16 takes no scales
    with pytest.raises(ValueError):
        validate_config([10], 64, 8, 2, torch.float8_e4m3fn, 0)  # FP8 needs scales
    with pytest.raises(ValueError):
        validate_config([10], 12, 8, 2, torch.float8_e4m3fn, 1)  # 12 B rows
    with pytest.raises(ValueError):
        validate_config([10], 64, 8, 2, torch.float32, 0)
    with pytest.raises(ValueError):
        validate_config([], 64, 8, 2, torch.bfloat16, 0)
    with pytest.raises(ValueError):
        validate_config([0], 64, 8, 2, torch.bfloat16, 0)
    with pytest.raises(ValueError):
        validate_config([2**30], 64, 8, 2, torch.bfloat16, 0, world=4)  # global ids overflow int32
    with pytest.raises(ValueError):
        validate_config([1] * 33, 64, 8, 2, torch.bfloat16, 0)


@pytest.mark.parametrize("mirror", [False, True])
@pytest.mark.parametrize("local_sf", [False, True])
def test_plan_regions_disjoint_and_aligned(mirror, local_sf):
    cfg = validate_config([524288, 524309], 256, 4096, 24, torch.float8_e4m3fn, 2, world=8)
    plan = plan_memory(cfg, 8, mirror, local_sf)
    spans = sorted((off, off + size) for off, size in plan.device.values())
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert all(off % REGION_ALIGN == 0 for off, _ in plan.device.values())
    assert plan.device_bytes % ALLOC_ALIGN == 0 and plan.host_bytes % ALLOC_ALIGN == 0
    assert plan.device["mirror"][1] == (cfg.table_rows * 256 if mirror else 0)
    assert plan.device["output"][1] == 2 * 4096 * 24 * 256
    assert plan.host["table"][1] == cfg.table_rows * 256
    assert plan.host_bytes == plan.table_bytes + plan.mailbox_bytes and plan.mailbox_bytes < (4 << 20)
    sf_rows = sum(n * (8 if local_sf else 1) for n in cfg.entries)
    assert plan.device["sf_table"][1] == sf_rows * 2 * 4
    assert storage_size_hint([524288, 524309], 256, 4096, 24, torch.float8_e4m3fn, 2, 8, mirror, local_sf) == (
        plan.device_bytes, plan.host_bytes)


def test_sf_strides():
    assert sf_strides(5, 3, 2, True) == (1, 8, 8 * 6)
    assert sf_strides(5, 3, 2, False) == (6, 1, 30)
    assert sf_strides(0, 3, 2, True) == (1, 0, 0)


def test_theoretical_config():
    ch, depth, restrict = theoretical_config(8, 2, 4096, 24)
    assert 1 <= ch <= 16 and depth >= 1024 and restrict is False
    with pytest.raises(ValueError):
        theoretical_config(8, 0, 4096, 24)


def test_row_pattern_deterministic_and_distinct():
    rows = torch.arange(64)
    a = row_pattern(rows, 0, 256)
    assert a.shape == (64, 256) and a.dtype == torch.uint8
    assert torch.equal(a, row_pattern(rows, 0, 256))
    assert not torch.equal(a, row_pattern(rows, 1, 256))
    assert len({bytes(r.tolist()) for r in a}) == 64


def test_pattern_shard_matches_expected():
    world, entries, hidden = 3, (7, 9), 16
    shards = [pattern_shard(r, world, entries, hidden, torch.float8_e4m3fn, 2, "cpu") for r in range(world)]
    idx = torch.tensor([[[0, 20, -1], [5, 13, 2]], [[26, 0, 9], [-1, -1, 17]]], dtype=torch.int32)
    exp = expected_outputs(idx, entries, hidden, torch.float8_e4m3fn, 2)
    for layer, n in enumerate(entries):
        flat = idx[layer].reshape(-1)
        for i, x in enumerate(flat.tolist()):
            got = exp[layer][0].reshape(-1, hidden)[i]
            sf = exp[layer][1].reshape(-1, 2)[i]
            if x < 0:
                assert got.sum() == 0 and sf.sum() == 0
            else:
                owner, local = divmod(x, n)
                assert torch.equal(got, shards[owner][0][layer][local].view(torch.uint8))
                assert torch.equal(sf, shards[owner][1][layer][x])
    sc = pattern_scales(torch.arange(1000), 0, 2)
    assert float(sc.min()) >= 2**-8 and float(sc.max()) <= 1.0
    assert torch.all(torch.log2(sc) == torch.round(torch.log2(sc)))


def test_make_indices_distributions():
    world, entries = 4, (100, 103)
    u = make_indices(0, world, entries, 64, 6, distribution="uniform")
    assert u.shape == (2, 64, 6) and u.dtype == torch.int32
    assert int(u[0].max()) < world * 100 and int(u[1].max()) < world * 103 and int(u.min()) >= 0
    o = make_indices(1, world, entries, 64, 6, owner=2)
    for layer, n in enumerate(entries):
        assert torch.all(o[layer] // n == 2)
    s = make_indices(0, world, entries, 64, 6, distribution="stratified")
    interval = world * 100 // 6
    assert torch.all(s[0] // interval == torch.arange(6))
    p = make_indices(0, world, entries, 512, 6, padding=0.1)
    frac = float((p < 0).float().mean())
    assert 0.05 < frac < 0.15
    z = make_indices(0, world, entries, 2048, 6, distribution="zipf")
    owners = (z[0].long() // 100).flatten()
    counts = torch.bincount(owners, minlength=world)
    assert counts[0] > counts[-1]  # low ids are hot
    m1 = make_indices(3, world, entries, 16, 6, distribution="matched", epoch=2)
    m2 = make_indices(3, world, entries, 16, 6, distribution="matched", epoch=2)
    assert torch.equal(m1, m2)
    assert not torch.equal(m1, make_indices(3, world, entries, 16, 6, distribution="matched", epoch=3))


def test_configs_shapes():
    assert CONFIGS["fp8"].bytes_per_fetch() == 2 * 4096 * 24 * 256
    assert CONFIGS["fp8_graph"].row_bytes == 512
    assert CONFIGS["oracle"].layers == 2


def test_fp8_roundtrip():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(32, 256, generator=g)
    codes, scales = quantize_fp8_blockwise(x)
    assert codes.dtype == torch.float8_e4m3fn and scales.shape == (32, 2)
    back = dequantize_fp8_blockwise(codes, scales, dtype=torch.float32)
    rel = (back - x).abs().max() / x.abs().max()
    assert rel < 0.07  # e4m3 has a 3-bit mantissa
    codes2, scales2 = quantize_fp8_blockwise(x, power_of_two=True)
    assert torch.all(torch.log2(scales2) == torch.round(torch.log2(scales2)))


def test_l2_flusher_and_percentile_on_cpu():
    from engram_rdma_lab_b200.utils.timing import L2Flusher, percentile

    f = L2Flusher(nbytes=4096, device="cpu")
    f()
    assert int(f.sink) == 1024 and int(f.buffer[0]) == 1
    f()
    assert int(f.sink) == 0
    assert percentile([1.0, 2.0, 3.0, 4.0], 0.5) == 2.5
    assert percentile([5.0], 0.99) == 5.0


def test_numa_locality_from_fake_sysfs(tmp_path):
    import os

    from engram_rdma_lab_b200.utils.numa import bind_to_device_numa, device_locality, parse_cpulist

    assert parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert parse_cpulist("") == set()
    dev = tmp_path / "0000:1b:00.0"
    dev.mkdir()
    allowed = sorted(os.sched_getaffinity(0))
    (dev / "numa_node").write_text("1\n")
    (dev / "local_cpulist").write_text(f"{allowed[0]}\n")
    assert device_locality("0000:1B:00.0", str(tmp_path)) == (1, {allowed[0]})
    assert device_locality("0000:99:00.0", str(tmp_path)) == (-1, set())
    before = os.sched_getaffinity(0)
    try:
        info = bind_to_device_numa(sysfs=str(tmp_path), address="0000:1b:00.0")
        assert info["numa_node"] == 1
        assert os.sched_getaffinity(0) == {allowed[0]}
        assert info["bound"] == (len(before) > 1)
        # Unknown slot: nothing changes.
        info = bind_to_device_numa(sysfs=str(tmp_path), address="0000:99:00.0")
        assert not info["bound"] and os.sched_getaffinity(0) == {allowed[0]}
    finally:
        os.sched_setaffinity(0, before)


def test_hot_rows_spec_and_replica_region():
    from engram_rdma_lab_b200.layout import hot_rows_for

    cfg = validate_config([100, 200], 64, 8, 2, torch.bfloat16, 0, world=4)
    assert hot_rows_for(cfg, 4, "") == [0, 0]
    assert hot_rows_for(cfg, 4, "50") == [50, 50]
    assert hot_rows_for(cfg, 4, "1000,30") == [400, 30]  # clamped to world * n
    assert hot_rows_for(cfg, 4, [5, 6]) == [5, 6]
    with pytest.raises(ValueError):
        hot_rows_for(cfg, 4, "1,2,3")
    plan = plan_memory(cfg, 4, True, False, hot_rows=[400, 30])
    assert plan.device["replica"][1] == 430 * 128
    spans = sorted((off, off + size) for off, size in plan.device.values())
    assert all(a1 <= b0 for (a0, a1), (b0, b1) in zip(spans, spans[1:]))
    assert storage_size_hint([100, 200], 64, 8, 2, torch.bfloat16, 0, 4, True, False, hot_rows="400,30")[0] == (
        plan.device_bytes)


def test_replica_fill_plan_covers_every_hot_id_once():
    from engram_rdma_lab_b200.layout import replica_chunks

    assert replica_chunks([0, 0], 100) == []
    plan = replica_chunks([250, 30, 0], 100)
    assert [start for start, _ in plan] == [0, 100, 200]
    assert plan[0][1] == [100, 30, 0] and plan[1][1] == [100, 0, 0] and plan[2][1] == [50, 0, 0]
    for layer, hot in enumerate([250, 30, 0]):
        covered = [start + i for start, counts in plan for i in range(counts[layer])]
        assert covered == list(range(hot))


def test_knob_table_covers_every_env_read():
    import pathlib
    import re

    from engram_rdma_lab_b200.utils import KNOBS, describe_knobs

    pkg = pathlib.Path(__file__).resolve().parents[1] / "engram_rdma_lab_b200"
    used = set()
    for path in pkg.rglob("*.py"):
        used |= set(re.findall(r'"(ENGRAM_[A-Z_]+)"', path.read_text()))
    assert used <= set(KNOBS), used - set(KNOBS)
    got = describe_knobs({"ENGRAM_DEDUP": "0"})
    assert got["ENGRAM_DEDUP"] == "0" and got["ENGRAM_HOT_ROWS"] == "default:"


def test_random_init_tables():
    from engram_rdma_lab_b200.models import normal_bf16_shard, quantized_fp8_shard

    bf = normal_bf16_shard(1, 4, (300, 301), 64, "cpu")
    assert [t.shape for t in bf] == [(300, 64), (301, 64)] and bf[0].dtype == torch.bfloat16
    assert 0.015 < float(bf[0].float().std()) < 0.025
    assert torch.equal(bf[0], normal_bf16_shard(1, 4, (300, 301), 64, "cpu")[0])
    assert not torch.equal(bf[0], normal_bf16_shard(2, 4, (300, 301), 64, "cpu")[0])
    codes0, scales0 = quantized_fp8_shard(0, 4, (300, 301), 256, 2, "cpu")
    codes1, scales1 = quantized_fp8_shard(1, 4, (300, 301), 256, 2, "cpu")
    assert codes0[0].dtype == torch.float8_e4m3fn and codes0[0].shape == (300, 256)
    assert scales0[0].shape == (4 * 300, 2) and torch.equal(scales0[1], scales1[1])  # global table, same everywhere
    assert not torch.equal(codes0[0].view(torch.uint8), codes1[0].view(torch.uint8))
    sc = scales0[0]
    assert float(sc.min()) >= 2**-8 and float(sc.max()) <= 1.0 and torch.all(torch.log2(sc) == torch.round(torch.log2(sc)))


@pytest.mark.parametrize("packs", [0, 2])
def test_expected_random_init_matches_the_owners_tables(packs):
    from engram_rdma_lab_b200.models import (expected_random_init, make_indices, normal_bf16_shard,
                                             quantized_fp8_shard)

    world, entries, hidden, ept, tokens = 3, (101, 67), 256, 5, 9
    dtype = torch.float8_e4m3fn if packs else torch.bfloat16
    idx = make_indices(1, world, entries, tokens, ept, epoch=4, padding=0.2)
    got = expected_random_init(idx, entries, hidden, dtype, packs, world)
    for layer, n in enumerate(entries):
        want_rows, want_sf = [], []
        for x in idx[layer].reshape(-1).tolist():
            if x < 0:
                want_rows.append(torch.zeros(hidden * dtype.itemsize, dtype=torch.uint8))
                want_sf.append(torch.zeros(packs))
                continue
            owner = x // n
            if packs:
                storages, sf = quantized_fp8_shard(owner, world, entries, hidden, packs, "cpu")
                want_sf.append(sf[layer][x])
            else:
                storages = normal_bf16_shard(owner, world, entries, hidden, "cpu")
            want_rows.append(storages[layer][x - owner * n].view(torch.uint8))
        assert torch.equal(got[layer][0], torch.stack(want_rows).reshape(tokens, -1))
        if packs:
            assert torch.equal(got[layer][1], torch.stack(want_sf).reshape(tokens, ept * packs))
        else:
            assert got[layer][1] is None


def test_serve_chunk_rows_knob(monkeypatch):
    from engram_rdma_lab_b200.buffer import _serve_chunk_rows

    monkeypatch.delenv("ENGRAM_SERVE_CHUNK_ROWS", raising=False)
    assert _serve_chunk_rows() == 512
    monkeypatch.setenv("ENGRAM_SERVE_CHUNK_ROWS", "256")
    assert _serve_chunk_rows() == 256
    for bad in ("8", "520", "1024", "100"):
        monkeypatch.setenv("ENGRAM_SERVE_CHUNK_ROWS", bad)
        with pytest.raises(ValueError):
            _serve_chunk_rows()


def test_serve_chunk_limits_match_the_kernels():
    """The Python check of ENGRAM_SERVE_CHUNK_ROWS and the CUDA limits agree."""
    import os
    import re

    from engram_rdma_lab_b200.buffer import _serve_chunk_rows

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    text = open(os.path.join(root, "csrc", "kernels", "params.h")).read()
    max_rows = int(re.search(r"kMaxServeChunkRows = (\d+);", text).group(1))
    base, shift = re.search(r"kMaxServeChunks = (\d+)u? << (\d+);", text).groups()
    max_chunks = int(base) << int(shift)
    assert max_chunks <= 1 << 15  # 16-bit limit and count in the claim word, with headroom
    os.environ["ENGRAM_SERVE_CHUNK_ROWS"] = str(max_rows)
    try:
        assert _serve_chunk_rows() == max_rows
        os.environ["ENGRAM_SERVE_CHUNK_ROWS"] = str(max_rows + 16)
        with pytest.raises(ValueError):
            _serve_chunk_rows()
    finally:
        del os.environ["ENGRAM_SERVE_CHUNK_ROWS"]
