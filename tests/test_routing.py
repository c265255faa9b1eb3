"""Route negotiation and topology helpers (host only)."""


import pytest

from engram_rdma_lab_b200.routing import (
    EgmConfig,
    OwnerRoute,
    agree_owner_routes,
    env_flag,
    env_int,
    fabric_identity,
    legacy_route_names,
    local_control_domain,
    node_layout,
    owner_routes,
    route_names,
)


def test_env_flag_strict(monkeypatch):
    monkeypatch.delenv("ENGRAM_EGM_ENABLE", raising=False)
    assert env_flag("ENGRAM_EGM_ENABLE") is False
    assert env_flag("ENGRAM_EGM_ENABLE", True) is True
    monkeypatch.setenv("ENGRAM_EGM_ENABLE", "1")
    assert EgmConfig.from_env().enabled
    for bad in ("true", "2", "", "yes"):
        monkeypatch.setenv("ENGRAM_EGM_ENABLE", bad)
        with pytest.raises(ValueError):
            env_flag("ENGRAM_EGM_ENABLE")


def test_env_int(monkeypatch):
    monkeypatch.setenv("ENGRAM_X", "7")
    assert env_int("ENGRAM_X", 1) == 7
    monkeypatch.setenv("ENGRAM_X", "abc")
    with pytest.raises(ValueError):
        env_int("ENGRAM_X", 1)
    monkeypatch.setenv("ENGRAM_X", "0")
    with pytest.raises(ValueError):
        env_int("ENGRAM_X", 1, minimum=1)


def test_route_aliases():
    assert OwnerRoute.RDMA is OwnerRoute.HOST
    assert OwnerRoute.EGM is OwnerRoute.PEER_HBM
    assert route_names([0, 1]) == ["host", "peer_hbm"]
    assert legacy_route_names([0, 1]) == ["rdma", "egm"]


def test_node_layout():
    assert node_layout(["a"] * 8, 5) == (5, 8)
    assert node_layout(["a", "a", "b", "b"], 3) == (1, 2)
    with pytest.raises(ValueError):
        node_layout(["a", "b", "a", "b"], 0)  # not contiguous
    with pytest.raises(ValueError):
        node_layout(["a", "a", "a", "b"], 0)  # unequal


def _peers(nodes, domains=None, fabric=None):
    out = []
    for i, n in enumerate(nodes):
        out.append(dict(node=n, fabric_domain=(domains or [None] * len(nodes))[i],
                        mirror_fabric=(fabric or [b""] * len(nodes))[i]))
    return out


def test_owner_routes_same_node():
    peers = _peers(["a"] * 4)
    assert owner_routes(peers, 1, EgmConfig(True)) == [OwnerRoute.PEER_HBM] * 4
    assert owner_routes(peers, 1, EgmConfig(False)) == [OwnerRoute.HOST] * 4


def test_owner_routes_cross_node_needs_shared_fabric():
    peers = _peers(["a", "a", "b", "b"], domains=[("x", 1)] * 2 + [("y", 1)] * 2, fabric=[b"h"] * 4)
    r = owner_routes(peers, 0, EgmConfig(True))
    assert r == [OwnerRoute.PEER_HBM, OwnerRoute.PEER_HBM, OwnerRoute.HOST, OwnerRoute.HOST]
    peers = _peers(["a", "a", "b", "b"], domains=[("x", 1)] * 4, fabric=[b"h", b"h", b"", b"h"])
    r = owner_routes(peers, 0, EgmConfig(True))
    assert r == [OwnerRoute.PEER_HBM, OwnerRoute.PEER_HBM, OwnerRoute.HOST, OwnerRoute.PEER_HBM]


def test_agree_intersects_directions():
    ok = {"routes": [1, 1, 1], "errors": ["", "", ""]}
    bad0 = {"routes": [1, 1, 0], "errors": ["", "", "map failed"]}
    reports = [bad0, ok, ok]
    routes0, reasons0 = agree_owner_routes(reports, 0)
    assert routes0 == [OwnerRoute.PEER_HBM, OwnerRoute.PEER_HBM, OwnerRoute.HOST]
    assert reasons0 == ["", "", "0->2: map failed"]
    routes2, reasons2 = agree_owner_routes(reports, 2)
    # The reverse direction degrades too, and reports the failing direction.
    assert routes2 == [OwnerRoute.HOST, OwnerRoute.PEER_HBM, OwnerRoute.PEER_HBM]
    assert reasons2[0] == "0->2: map failed"
    routes1, _ = agree_owner_routes(reports, 1)
    assert routes1 == [OwnerRoute.PEER_HBM] * 3


def test_agree_rejects_malformed():
    with pytest.raises(ValueError):
        agree_owner_routes([{"routes": [1], "errors": [""]}, {"routes": [1, 1], "errors": ["", ""]}], 0)
    with pytest.raises(ValueError):
        agree_owner_routes([{"routes": [3], "errors": [""]}], 0)
    with pytest.raises(ValueError):
        agree_owner_routes([{"routes": [1], "errors": [""]}], 1)


class _FakeNvml:
    """Stands in for libnvidia-ml: returns a configurable fabric record."""

    def __init__(self, state=3, status=0, cluster=b"\x01" * 16, clique=7, init_rc=0):
        self.state, self.status, self.cluster, self.clique, self.init_rc = state, status, cluster, clique, init_rc
        self.shutdown = False

    def nvmlInit_v2(self):
        return self.init_rc

    def nvmlDeviceGetHandleByUUID(self, uuid, handle):
        return 0

    def nvmlDeviceGetGpuFabricInfo(self, handle, info_ref):
        info = info_ref._obj
        for i, b in enumerate(self.cluster):
            info.cluster[i] = b
        info.state, info.status, info.clique = self.state, self.status, self.clique
        return 0

    def nvmlShutdown(self):
        self.shutdown = True


def test_fabric_identity_with_fake_nvml():
    assert fabric_identity("GPU-x", False) == (None, "disabled")
    fake = _FakeNvml()
    domain, err = fabric_identity("GPU-x", True, nvml=fake)
    assert err is None and domain == ((b"\x01" * 16).hex(), 7) and fake.shutdown
    domain, err = fabric_identity("GPU-x", True, nvml=_FakeNvml(state=1))
    assert domain is None and "fabric unavailable" in err
    domain, err = fabric_identity("GPU-x", True, nvml=_FakeNvml(cluster=b"\x00" * 16))
    assert domain is None
    domain, err = fabric_identity("GPU-x", True, nvml=_FakeNvml(init_rc=9))
    assert domain is None and "init" in err


def test_local_control_domain_restores(monkeypatch):
    monkeypatch.delenv("NCCL_MNNVL_ENABLE", raising=False)
    import os

    with local_control_domain():
        assert os.environ["NCCL_MNNVL_ENABLE"] == "0"
    assert "NCCL_MNNVL_ENABLE" not in os.environ
