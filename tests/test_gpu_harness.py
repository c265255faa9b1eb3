"""Drive benchmarks/test_engram.py through torchrun (scenario coverage).

Most scenarios run on two GPUs; the full-node scenarios run on every visible
GPU (up to eight), where every output is still checked bit-exactly.
"""

import json
import os
import subprocess
import sys

import pytest

from .conftest import cuda_device_count, free_port

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(cuda_device_count() < 2, reason="needs two GPUs")]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SMALL = ["--entries", "4099,4111", "--hidden", "128", "--ept", "7", "--tokens", "512", "--rounds", "4",
         "--warmups", "1"]

SCENARIOS = {
    "graph_reverse_cross_stream": SMALL + ["--dtype", "fp8", "--sf-packs", "1", "--cuda-graph", "--hook-order",
                                           "reverse", "--cross-stream", "--padding", "0.1"],
    "locality_cycle_async": SMALL + ["--dtype", "bf16", "--locality-cycle", "--async-check", "--rounds", "12"],
    "host_route_misc": SMALL + ["--dtype", "bf16", "--route", "host", "--vary-tokens", "--check-errors",
                                "--rewrite", "--cpu-write", "--row-major-sf"],
    "host_route_graph_locality": SMALL + ["--dtype", "fp8", "--sf-packs", "1", "--route", "host", "--cuda-graph",
                                          "--locality-cycle", "--async-check", "--rounds", "12"],
    "probe_fault_fallback": SMALL + ["--dtype", "fp8", "--sf-packs", "1", "--egm-fail-pair", "0:1"],
    "single_owner_traffic": SMALL + ["--dtype", "bf16", "--traffic", "single", "--requester-rank", "0",
                                     "--owner-rank", "1", "--distribution", "matched"],
    "torch_baseline": SMALL + ["--dtype", "fp8", "--sf-packs", "1", "--impl", "torch", "--padding", "0.05"],
    "pinned_indices_zipf": SMALL + ["--dtype", "fp8", "--sf-packs", "1", "--pinned-indices", "--distribution",
                                    "zipf", "--padding", "0.05"],
}


# Full-node scenarios: the headline shape on every GPU, the host route, and
# graph replays with cross-stream hooks, all verified every round.
FULL_NODE = {
    "full_node_headline": ["--entries", "524288,524309", "--tokens", "4096", "--dtype", "fp8", "--sf-packs", "2",
                           "--rounds", "4", "--warmups", "1", "--padding", "0.02"],
    "full_node_host_route": SMALL + ["--dtype", "bf16", "--route", "host", "--padding", "0.02"],
    "full_node_graph_locality": SMALL + ["--dtype", "fp8", "--sf-packs", "1", "--cuda-graph", "--locality-cycle",
                                         "--async-check", "--rounds", "12", "--cross-stream", "--hook-order",
                                         "reverse"],
}


def _run_harness(args, world, out):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(world),
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "benchmarks", "test_engram.py"), *args, "--output-dir", str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    return [json.loads((out / f"engram-r{r}.json").read_text()) for r in range(world)]


@pytest.mark.parametrize("name", sorted(FULL_NODE))
def test_harness_full_node(name, tmp_path):
    world = min(8, cuda_device_count())
    reports = _run_harness(FULL_NODE[name], world, tmp_path / name)
    for report in reports:
        meta = report["metadata"]
        assert meta["world"] == world and meta["error_state"]["status"] == 0
        assert meta["extension_sha256"] and meta["kernel_sources_sha256"] and meta["gpu_uuid"]
        timed = [s for s in report["samples"] if "e2e_ms" in s]
        assert all(s["verified"] for s in timed)
    assert len({r["metadata"]["gpu_uuid"] for r in reports}) == world


@pytest.mark.parametrize("name", sorted(SCENARIOS))
def test_harness_scenario(name, tmp_path):
    out = tmp_path / name
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(ROOT, "benchmarks", "test_engram.py"), *SCENARIOS[name], "--output-dir", str(out)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    meta = json.loads((out / "engram-r0.json").read_text())["metadata"]
    if name == "host_route_misc":
        assert len(meta["misuse_checks"]) >= 5
        timed = [s for s in json.loads((out / "engram-r0.json").read_text())["samples"] if "device_ms" in s]
        assert timed and all(s["python_issue_ms"] >= 0 and s["synchronize_ms"] >= 0 for s in timed)
    if name == "pinned_indices_zipf":
        assert meta["pinned_indices"] is True
    if name == "probe_fault_fallback":
        assert meta["routing"]["owner_routes"] == ["peer_hbm", "host"]
        assert "0->1" in meta["routing"]["owner_fallback_reasons"][1]


def test_harness_spawns_local_ranks_without_torchrun(tmp_path):
    out = tmp_path / "spawned"
    cmd = [sys.executable, os.path.join(ROOT, "benchmarks", "test_engram.py"), *SMALL, "--dtype", "bf16",
           "--local-ranks", "2", "--qp-depth", "512", "--output-dir", str(out)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    env["NCCL_NVLS_ENABLE"] = "0"
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    for rank in range(2):
        assert (out / f"engram-r{rank}.json").exists()
