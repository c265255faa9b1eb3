"""Place a rank's host threads and pinned memory on its GPU's NUMA node.

Pinned host memory that the GPU reads (index tensors handed to ``fetch``,
host shards, H2D staging) crosses the socket interconnect when its pages sit
on the other socket, which costs PCIe read throughput: on a two-socket B200
host the same 786 KB index read ran at about half speed from the remote node.
``cudaHostAlloc`` places pages on the node of the CPU that allocates them, so
pinning the process to the GPU's local CPUs before allocating pinned memory
keeps those reads local.  Nothing here changes a device setting.
"""

from __future__ import annotations

import os

SYSFS_PCI = "/sys/bus/pci/devices"


def parse_cpulist(text: str) -> set[int]:
    """Parse a sysfs CPU list such as ``"0-3,8,10-11"``."""
    cpus: set[int] = set()
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-", 1)
            cpus.update(range(int(lo), int(hi) + 1))
        else:
            cpus.add(int(part))
    return cpus


def pci_address(device) -> str:
    """Sysfs name (``dddd:bb:dd.0``) of a CUDA device's PCI function."""
    import torch

    p = torch.cuda.get_device_properties(device)
    return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"


def device_locality(address: str, sysfs: str = SYSFS_PCI) -> tuple[int, set[int]]:
    """``(numa_node, local_cpus)`` of a PCI function; ``(-1, set())`` when unknown."""
    base = os.path.join(sysfs, address.lower())
    node, cpus = -1, set()
    try:
        with open(os.path.join(base, "numa_node")) as f:
            node = int(f.read().strip())
    except (OSError, ValueError):
        pass
    try:
        with open(os.path.join(base, "local_cpulist")) as f:
            cpus = parse_cpulist(f.read())
    except (OSError, ValueError):
        pass
    return node, cpus


def bind_to_device_numa(device=None, sysfs: str = SYSFS_PCI, address: str | None = None) -> dict:
    """Restrict this process's CPUs to those local to ``device``'s PCI slot.

    Keeps the CPUs the process may already use (container cpusets); does
    nothing when that leaves none or sysfs does not say.  Call it before
    allocating pinned memory.  Returns what was done.
    """
    if address is None:
        import torch

        address = pci_address(torch.cuda.current_device() if device is None else device)
    node, local = device_locality(address, sysfs)
    allowed = os.sched_getaffinity(0)
    chosen = local & allowed
    info = {"pci": address, "numa_node": node, "local_cpus": len(local), "bound": False}
    if chosen and chosen != allowed:
        os.sched_setaffinity(0, chosen)
        info["bound"] = True
    info["cpus"] = len(os.sched_getaffinity(0))
    return info
