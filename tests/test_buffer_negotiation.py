"""EngramBuffer's collective set_config on CPU ranks with a fake native runtime.

The Python orchestration (bootstrap exchange -> route probe -> agreement ->
commit -> connect) must end the same way on every rank: when one rank's step
fails, all ranks raise and release their runtime, and nobody waits forever in
a later collective.  Failures are injected on the host into a stand-in for
``_C.Runtime``; no GPU is used (gloo, world size 2).  The same stand-in,
answering fetches from the pattern oracle, checks the order of the hot-prefix
replica fill (off, capacity-sized fetches, health check, on) and its content.
"""

import contextlib
import types

import pytest
import torch

from ._spawn import run_ranks

PHASES = ("init", "bootstrap", "probe", "prepare", "connect")


calls = []  # data-path calls of the fake runtime in this process


def _install_fakes(rank, world, fail_phase, fail_rank, closed, probe_errors=None):
    """Patch torch.cuda and the native loader for a CPU-only rank."""
    from engram_rdma_lab_b200 import _native

    def maybe_fail(phase):
        if phase == fail_phase and rank == fail_rank:
            raise RuntimeError(f"injected {phase} failure")

    class FakeRuntime:
        def __init__(self, cfg):
            maybe_fail("init")
            self.cfg = cfg
            self.routes = None

        def bootstrap(self):
            maybe_fail("bootstrap")
            c = self.cfg
            return dict(socket=f"fake-{rank}", mirror=c["egm"], mirror_bytes=0, mirror_offset=0,
                        config=(c["world"], c["entries"], c["hidden"], c["max_tokens"], c["ept"], c["packs"]))

        def probe_routes(self, peers, candidates):
            maybe_fail("probe")
            errors = [""] * world
            routes = list(candidates)
            for owner in (probe_errors or {}).get(rank, ()):
                routes[owner], errors[owner] = 0, "injected mapping failure"
            return {"routes": routes, "errors": errors}

        def prepare_routes(self, routes):
            maybe_fail("prepare")
            self.routes = routes

        def connect(self):
            maybe_fail("connect")

        def close(self):
            closed.append(rank)

        def memory_usage(self):
            return {"fake": True}

        # Data path stand-ins for the replica-fill test: a "fetch" returns the
        # pattern oracle's rows, like the kernels would.
        def write(self, layer, storage, scales):
            pass

        def fetch(self, indices, qps, col_major):
            from engram_rdma_lab_b200.models import expected_outputs

            c = self.cfg
            dtype = torch.bfloat16 if c["packs"] == 0 else torch.float8_e4m3fn
            exp = expected_outputs(indices, c["entries"], c["hidden"], dtype, c["packs"])
            calls.append(("fetch", int((indices >= 0).sum())))
            return [e[0].view(dtype).reshape(indices.shape[1], -1) for e in exp]

        def wait_layer(self, layer):
            pass

        def check_health(self):
            calls.append(("health",))

        def replica_view(self):
            if not hasattr(self, "_replica"):
                rows = sum(self.cfg["hot_rows"])
                self._replica = torch.zeros(rows, self.cfg["hidden"] * self.cfg["element_bytes"], dtype=torch.uint8)
            return self._replica

        def set_hot_active(self, on):
            calls.append(("hot", bool(on)))

    _native._C = types.SimpleNamespace(Runtime=FakeRuntime)
    torch.cuda.is_available = lambda: True
    torch.cuda.current_device = lambda: 0
    torch.cuda.get_device_properties = lambda device: types.SimpleNamespace(uuid=f"GPU-fake-{rank}")
    torch.cuda.device = lambda device: contextlib.nullcontext()
    torch.cuda.synchronize = lambda *args, **kwargs: None


def _make(world):
    import torch.distributed as dist

    from engram_rdma_lab_b200 import EngramBuffer

    group = dist.group.WORLD
    entries, hidden, tokens, ept = (64, 64), 64, 16, 4
    sizes = EngramBuffer.get_storage_size_hint(group, entries, hidden, tokens, ept, torch.bfloat16, 0)
    buf = EngramBuffer(group, *sizes, True, 2, 64, explicitly_destroy=True)
    return buf, (entries, hidden, tokens, ept, torch.bfloat16, 0)


def _negotiate(rank, world, fail_phase, egm):
    import os

    os.environ["ENGRAM_EGM_ENABLE"] = "1" if egm else "0"
    os.environ.pop("ENGRAM_WRITE_LOCAL_SF", None)
    closed = []
    _install_fakes(rank, world, fail_phase, 1, closed)
    buf, args = _make(world)
    if fail_phase is None:
        buf.set_config(*args)
        want = ["peer_hbm" if egm else "host"] * world
        info = buf.get_route_info()
        assert info["owner_routes"] == want and info["memory"] == {"fake": True}
        assert buf.runtime.routes == [1 if egm else 0] * world
        return
    with pytest.raises(RuntimeError, match=f"injected {fail_phase} failure"):
        buf.set_config(*args)
    # Every rank that built a runtime released it; nobody is left configured.
    built = not (fail_phase == "init" and rank == 1)
    assert closed == ([rank] if built else [])
    assert buf.runtime is None
    with pytest.raises(RuntimeError):
        buf.fetch(torch.zeros(2, 4, 4, dtype=torch.int32))


@pytest.mark.parametrize("fail_phase", [None, *PHASES])
def test_set_config_fails_on_every_rank(port, fail_phase):
    run_ranks(_negotiate, 2, port, args=(fail_phase, True))


def test_set_config_host_routes_without_the_switch(port):
    run_ranks(_negotiate, 2, port, args=(None, False))


def _one_direction_fails(rank, world):
    import os

    os.environ["ENGRAM_EGM_ENABLE"] = "1"
    closed = []
    # Rank 0 cannot map owner 1's mirror: both directions of the pair fall back.
    _install_fakes(rank, world, None, None, closed, probe_errors={0: (1,)})
    buf, args = _make(world)
    buf.set_config(*args)
    info = buf.get_route_info()
    other = 1 - rank
    expected = ["peer_hbm", "peer_hbm"]
    expected[other] = "host"
    assert info["owner_routes"] == expected
    assert "0->1" in info["owner_fallback_reasons"][other]
    assert info["owner_fallback_reasons"][rank] == ""


def test_probe_failure_downgrades_only_that_pair(port):
    run_ranks(_one_direction_fails, 2, port)


def _replica_fill(rank, world):
    import os

    from engram_rdma_lab_b200.base import EngramBufferBase
    from engram_rdma_lab_b200.models import pattern_shard, row_pattern

    os.environ["ENGRAM_EGM_ENABLE"] = "1"
    os.environ["ENGRAM_HOT_ROWS"] = "100,37"
    closed = []
    _install_fakes(rank, world, None, None, closed)
    buf, args = _make(world)  # capacity 16 tokens x 4 = 64 rows per fetch
    buf.set_config(*args)
    assert buf.hot_rows == [100, 37]
    # The CPU stand-in returns CPU views; relax only the device check.
    check = EngramBufferBase._check_fetch_args
    buf._check_fetch_args = lambda idx, dev, **kw: check(buf, idx, None, require_cuda=False)
    storages, _ = pattern_shard(rank, world, args[0], args[1], torch.bfloat16, 0, "cpu")
    buf.write(storages)
    # Off during the fill, two capacity-sized fetches (ids 0-63, 64-99 / 0-36), health check, then on.
    assert [c for c in calls if c[0] != "fetch"] == [("hot", False), ("health",), ("hot", True)]
    assert [c[1] for c in calls if c[0] == "fetch"] == [64 + 37, 36]
    replica = buf.runtime.replica_view()
    # Replica row hot_base[l] + x holds global id x of layer l (pattern rows are keyed by global id).
    want = [row_pattern(torch.arange(hot), layer, 128) for layer, hot in enumerate(buf.hot_rows)]
    assert torch.equal(replica, torch.cat(want))
    os.environ.pop("ENGRAM_HOT_ROWS", None)


def test_hot_replica_fill_orchestration(port):
    run_ranks(_replica_fill, 2, port)
