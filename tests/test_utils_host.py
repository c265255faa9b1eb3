"""Host-side helpers: numeric utilities, scoped env overrides, the event helper's
error paths and the process-group helpers (gloo, world size 2)."""

import os

import pytest
import torch

from engram_rdma_lab_b200.utils import EnvOverride, EventOverlap
from engram_rdma_lab_b200.ops import calc_diff, dequantize_fp8_blockwise, quantize_fp8_blockwise
from engram_rdma_lab_b200.utils.math import align, ceil_div

from ._spawn import run_ranks


def test_math_helpers():
    assert ceil_div(7, 2) == 4 and ceil_div(8, 2) == 4 and align(5, 4) == 8 and align(8, 4) == 8
    x = torch.randn(64, generator=torch.Generator().manual_seed(0))
    assert calc_diff(x, x) == pytest.approx(0.0, abs=1e-12)
    assert calc_diff(x, -x) > 0.1
    # The FP8 round trip of N(0, 1) rows is close to its source by this measure.
    table = torch.randn(32, 256, generator=torch.Generator().manual_seed(1))
    codes, scales = quantize_fp8_blockwise(table)
    assert calc_diff(dequantize_fp8_blockwise(codes, scales, dtype=torch.float32), table) < 1e-3


def test_env_override_restores_previous_values():
    os.environ["ENGRAM_TEST_A"] = "old"
    os.environ.pop("ENGRAM_TEST_B", None)
    with EnvOverride([("ENGRAM_TEST_A", "new", True), ("ENGRAM_TEST_B", "set", True), ("ENGRAM_TEST_C", "x", False)]):
        assert os.environ["ENGRAM_TEST_A"] == "new" and os.environ["ENGRAM_TEST_B"] == "set"
        assert "ENGRAM_TEST_C" not in os.environ
    assert os.environ["ENGRAM_TEST_A"] == "old" and "ENGRAM_TEST_B" not in os.environ
    os.environ.pop("ENGRAM_TEST_A")


def test_event_overlap_misuse_is_refused():
    empty = EventOverlap()
    with pytest.raises(RuntimeError):
        empty.current_stream_wait()
    with empty:  # leaving a context without an event waits for nothing
        pass
    empty.register_hook_after_wait(lambda: 1)
    with pytest.raises(RuntimeError):
        empty.register_hook_after_wait(lambda: 2)


def _dist_helpers(rank, world):
    from engram_rdma_lab_b200.parallel import gather_floats, max_over_ranks
    from engram_rdma_lab_b200.parallel.dist import init_dist

    assert init_dist(backend="gloo") == (rank, world, rank)  # already initialised: returns the placement
    assert max_over_ranks(float(rank) * 2.5) == 2.5
    assert gather_floats([rank, rank + 0.5]) == [[0, 0.5], [1, 1.5]]


def test_process_group_helpers_over_gloo(port):
    run_ranks(_dist_helpers, 2, port)


def test_single_process_helpers_without_a_group():
    from engram_rdma_lab_b200.parallel import gather_floats, max_over_ranks

    assert max_over_ranks(3.0) == 3.0
    assert gather_floats([1.0, 2.0]) == [[1.0, 2.0]]


def test_doctor_reports_without_a_gpu(capsys):
    import json

    from engram_rdma_lab_b200 import doctor

    assert doctor.main(["--json"]) == 0  # the extension is built in-tree
    r = json.loads(capsys.readouterr().out)
    assert r["extension"]["loaded"] and "gather_simt_kernel" in r["extension"]["kernels"]
    assert set(r["knobs"]) >= {"ENGRAM_EGM_ENABLE", "ENGRAM_HOT_ROWS"}
    assert doctor.main([]) == 0
    assert "knobs:" in capsys.readouterr().out


def test_bench_reference_arm_prints_one_unavailable_line():
    """``bench.py --impl reference`` (the driver's reference arm) exits 0 with one JSON line on rank 0 only."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, os.path.join(root, "bench.py"), "--impl", "reference", "--gpus", "1", "--steps", "2",
           "--warmup", "3"]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    out = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [line for line in out.stdout.splitlines() if line.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unavailable"]
    env["RANK"] = "1"
    out = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and not out.stdout.strip()


def test_bench_defaults_and_minimum_warmup(monkeypatch):
    import importlib
    import os
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    monkeypatch.syspath_prepend(root)
    bench = importlib.import_module("bench")
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    args = bench.parse()
    assert args.gpus == 1 and args.steps >= 1 and args.warmup >= 3 and args.impl == "ours"
    monkeypatch.setattr(sys, "argv", ["bench.py", "--warmup", "1", "--steps", "2"])
    args = bench.parse()
    assert args.warmup == 3 and args.warmup_requested == 1
