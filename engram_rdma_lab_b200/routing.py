"""Topology discovery and per-(requester, owner) route negotiation.

Runs only at initialisation. The hot path never calls into this module.

Route values (``OwnerRoute``) keep the reference's integer encoding so a route
table written by either side means the same thing:

* ``HOST`` (0): rows stay in the owner's host-pinned shard.  The owner GPU reads
  them zero-copy and pushes them with peer stores into the requester's output
  (the analog of the reference's RDMA / SGE-WRITE route, legacy name ``rdma``).
* ``PEER_HBM`` (1): the requester's SMs load rows directly from the owner's
  HBM mirror through NVLink / NVSwitch (the analog of the reference's EGM direct
  read, legacy name ``egm``).

Parity: ``deepep/deep_ep/utils/engram_routing.py:11-156`` and the byte-identical
``sge_write/engram_sge_write/routing.py``.  Negotiation keeps the reference's
rules: candidates are proposed per owner, each direction is probed, and a pair
only uses ``PEER_HBM`` when both directions succeeded; a failed pair degrades
alone and its reasons are reported per owner.
"""

from __future__ import annotations

import ctypes
import os
from contextlib import contextmanager
from dataclasses import dataclass
from enum import IntEnum
from pathlib import Path

__all__ = [
    "env_flag",
    "env_int",
    "EgmConfig",
    "OwnerRoute",
    "node_identity",
    "fabric_identity",
    "node_layout",
    "owner_routes",
    "agree_owner_routes",
    "route_names",
    "legacy_route_names",
    "local_control_domain",
]


def env_flag(name: str, default: bool = False) -> bool:
    """Read a strict 0/1 switch; anything else is a configuration error."""
    raw = os.environ.get(name)
    if raw is None:
        return default
    if raw not in ("0", "1"):
        raise ValueError(f"{name} must be 0 or 1, got {raw!r}")
    return raw == "1"


def env_int(name: str, default: int, minimum: int | None = None) -> int:
    """Read an integer knob with an optional lower bound."""
    raw = os.environ.get(name)
    if raw is None or raw == "":
        return default
    try:
        value = int(raw)
    except ValueError as error:
        raise ValueError(f"{name} must be an integer, got {raw!r}") from error
    if minimum is not None and value < minimum:
        raise ValueError(f"{name} must be >= {minimum}, got {value}")
    return value


@dataclass(frozen=True)
class EgmConfig:
    """The direct-route switch, fixed for a buffer's lifetime.

    ``ENGRAM_EGM_ENABLE=1`` asks every same-node pair to try the peer-HBM
    direct route (and cross-node pairs when a shared NVLink fabric domain and
    exportable fabric handles exist).  ``0`` keeps every remote owner on the
    host route.
    """

    enabled: bool = False

    @classmethod
    def from_env(cls) -> "EgmConfig":
        return cls(env_flag("ENGRAM_EGM_ENABLE", False))


class OwnerRoute(IntEnum):
    HOST = 0
    PEER_HBM = 1

    # Reference spellings; same integer values.
    RDMA = 0
    EGM = 1


_ROUTE_NAMES = {OwnerRoute.HOST: "host", OwnerRoute.PEER_HBM: "peer_hbm"}
_LEGACY_NAMES = {OwnerRoute.HOST: "rdma", OwnerRoute.PEER_HBM: "egm"}


def node_identity() -> str:
    """Identify the physical host by its kernel boot id.

    Container hostnames can differ on one machine or repeat across machines;
    the boot id does neither.
    """
    try:
        return Path("/proc/sys/kernel/random/boot_id").read_text().strip()
    except OSError:
        return os.uname().nodename


class _FabricInfo(ctypes.Structure):
    # nvmlGpuFabricInfo_t: clusterUuid[16], status, cliqueId, state.
    _fields_ = [
        ("cluster", ctypes.c_ubyte * 16),
        ("status", ctypes.c_int),
        ("clique", ctypes.c_uint),
        ("state", ctypes.c_ubyte),
    ]


_NVML_FABRIC_STATE_COMPLETED = 3


def fabric_identity(cuda_uuid, enabled: bool, nvml=None):
    """Return ``((cluster_uuid_hex, clique), None)`` or ``(None, reason)``.

    Looks the device up by UUID (a CUDA ordinal is not a physical index once
    ``CUDA_VISIBLE_DEVICES`` reorders devices).  A fabric counts only if its
    registration completed, its status is success and its cluster UUID is
    non-zero.  ``nvml`` may be an object exposing the three NVML calls used
    here; tests pass a fake.
    """
    if not enabled:
        return None, "disabled"
    lib = nvml
    initialised = False
    try:
        if lib is None:
            lib = ctypes.CDLL("libnvidia-ml.so.1")
        rc = lib.nvmlInit_v2()
        if rc:
            raise RuntimeError(f"NVML init error {rc}")
        initialised = True
        handle = ctypes.c_void_p()
        rc = lib.nvmlDeviceGetHandleByUUID(str(cuda_uuid).encode(), ctypes.byref(handle))
        if rc:
            raise RuntimeError(f"NVML UUID lookup error {rc}")
        info = _FabricInfo()
        rc = lib.nvmlDeviceGetGpuFabricInfo(handle, ctypes.byref(info))
        if rc or info.state != _NVML_FABRIC_STATE_COMPLETED or info.status != 0 or not any(info.cluster):
            raise RuntimeError(f"fabric unavailable: rc={rc}, state={info.state}, status={info.status}")
        return (bytes(info.cluster).hex(), int(info.clique)), None
    except (OSError, AttributeError, RuntimeError) as error:
        return None, str(error)
    finally:
        if initialised:
            try:
                lib.nvmlShutdown()
            except Exception:  # pragma: no cover - shutdown failures are not actionable
                pass


def node_layout(nodes, rank: int):
    """Check ranks are grouped contiguously per node with equal counts.

    Returns ``(local_rank, ranks_per_node)``.
    """
    world = len(nodes)
    if not 0 <= rank < world:
        raise ValueError("rank outside the node list")
    local = nodes.count(nodes[rank])
    if local == 0 or world % local:
        raise ValueError("Every physical node must contribute the same number of ranks")
    for i, node in enumerate(nodes):
        if node != nodes[(i // local) * local]:
            raise ValueError("Ranks must be grouped contiguously by physical node")
    if any(nodes.count(node) != local for node in set(nodes)):
        raise ValueError("Every physical node must contribute the same number of ranks")
    return rank % local, local


def owner_routes(peers, rank: int, config: EgmConfig):
    """Propose a route for every owner from this requester's point of view.

    Same node: ``PEER_HBM`` when the switch is on.  Other node: ``PEER_HBM`` only
    if both sides report the same fabric domain and both exported a fabric
    handle for their mirror.
    """
    me = peers[rank]
    routes = []
    for peer in peers:
        if not config.enabled:
            direct = False
        elif peer["node"] == me["node"]:
            direct = True
        else:
            domain = me.get("fabric_domain")
            direct = (
                domain is not None
                and peer.get("fabric_domain") == domain
                and bool(me.get("mirror_fabric"))
                and bool(peer.get("mirror_fabric"))
            )
        routes.append(OwnerRoute.PEER_HBM if direct else OwnerRoute.HOST)
    return routes


def agree_owner_routes(reports, rank: int):
    """Intersect both directions of every probe.

    ``reports[r]`` is rank r's probe result: ``{"routes": [...], "errors": [...]}``
    indexed by owner.  A pair is direct only when r→p and p→r both succeeded, so
    the owner service on one side always matches the requester on the other.
    Returns ``(routes, reasons)`` for ``rank``; ``reasons[p]`` is empty for direct
    pairs and lists the failing direction(s) otherwise.
    """
    world = len(reports)
    if not 0 <= rank < world:
        raise ValueError("Invalid route negotiation rank")
    for report in reports:
        routes, errors = report.get("routes"), report.get("errors")
        if routes is None or errors is None or len(routes) != world or len(errors) != world:
            raise ValueError("Invalid route probe report")
        if any(int(r) not in (OwnerRoute.HOST, OwnerRoute.PEER_HBM) for r in routes):
            raise ValueError("Invalid route probe report")
    routes, reasons = [], []
    for peer in range(world):
        direct = int(reports[rank]["routes"][peer]) == int(reports[peer]["routes"][rank]) == OwnerRoute.PEER_HBM
        routes.append(OwnerRoute.PEER_HBM if direct else OwnerRoute.HOST)
        if direct:
            reasons.append("")
            continue
        failures = []
        seen = set()
        for requester, owner in ((rank, peer), (peer, rank)):
            if (requester, owner) in seen:
                continue
            seen.add((requester, owner))
            error = reports[requester]["errors"][owner]
            if error:
                failures.append(f"{requester}->{owner}: {error}")
        reasons.append("; ".join(failures))
    return routes, reasons


def route_names(routes):
    return [_ROUTE_NAMES[OwnerRoute(int(r))] for r in routes]


def legacy_route_names(routes):
    return [_LEGACY_NAMES[OwnerRoute(int(r))] for r in routes]


@contextmanager
def local_control_domain():
    """Keep any NCCL communicator created inside on the node-local domain.

    The data plane never goes through NCCL; the baseline and bootstrap
    communicators must not silently span a multi-node NVLink domain.
    """
    keys = {"NCCL_MNNVL_ENABLE": "0"}
    previous = {key: os.environ.get(key) for key in keys}
    os.environ.update(keys)
    try:
        yield
    finally:
        for key, value in previous.items():
            if value is None:
                os.environ.pop(key, None)
            else:
                os.environ[key] = value
