"""Environment report for the Engram buffer: ``python -m engram_rdma_lab_b200.doctor [--json]``.

Answers the questions behind most setup problems before a job starts: is the
in-tree extension built and loadable, which GPUs are visible and can each pair
reach the other's memory (the peer-HBM route needs it), which ENGRAM_* knobs
are set, and which CPUs and NUMA node sit next to each GPU (pinned host
indices and host shards should live there).  Read-only: it changes no device
or process setting.
"""

from __future__ import annotations

import argparse
import json
import os
import sys


def extension_report() -> dict:
    from . import _native

    try:
        mod = _native.load()
    except ImportError as error:
        return {"loaded": False, "error": str(error)}
    return {"loaded": True, "path": getattr(mod, "__file__", None), "kernels": list(getattr(mod, "KERNELS", ())),
            "max_ranks": getattr(mod, "MAX_RANKS", None), "max_layers": getattr(mod, "MAX_LAYERS", None)}


def gpu_report() -> dict:
    import torch

    if not torch.cuda.is_available():
        return {"available": False, "count": 0, "devices": [], "peer_access": []}
    from .utils.numa import device_locality, pci_address

    devices = []
    count = torch.cuda.device_count()
    for i in range(count):
        p = torch.cuda.get_device_properties(i)
        entry = {"index": i, "name": p.name, "sm": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
                 "memory_gb": round(p.total_memory / 1e9, 1), "uuid": str(p.uuid)}
        try:
            address = pci_address(i)
            node, cpus = device_locality(address)
            entry.update(pci=address, numa_node=node, local_cpus=len(cpus))
        except Exception as error:  # noqa: BLE001 - a report, not a check
            entry["pci_error"] = str(error)
        devices.append(entry)
    peer = [[i == j or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(count)] for i in range(count)]
    return {"available": True, "count": count, "devices": devices, "peer_access": peer,
            "all_pairs_peer": all(all(row) for row in peer)}


def report() -> dict:
    import torch

    from .utils.env import describe_knobs

    return {
        "python": sys.version.split()[0],
        "torch": torch.__version__,
        "torch_cuda": torch.version.cuda,
        "extension": extension_report(),
        "gpus": gpu_report(),
        "knobs": describe_knobs(),
        "process_cpus": len(os.sched_getaffinity(0)),
    }


def _print_text(r: dict) -> None:
    ext = r["extension"]
    print(f"python {r['python']}  torch {r['torch']} (CUDA {r['torch_cuda']})")
    print("extension: " + (f"loaded from {ext['path']}" if ext["loaded"] else f"NOT loaded: {ext['error']}"))
    g = r["gpus"]
    if not g["available"]:
        print("GPUs: none visible (the native buffer needs one; TorchEngramBuffer runs on the CPU)")
    else:
        for d in g["devices"]:
            where = f"numa {d.get('numa_node', '?')}, {d.get('local_cpus', '?')} local CPUs"
            print(f"GPU {d['index']}: {d['name']} sm_{d['sm'].replace('.', '')}, {d['sms']} SMs, "
                  f"{d['memory_gb']} GB, {where}")
        print("peer access between every pair: " + ("yes" if g["all_pairs_peer"] else "NO (peer_hbm will fall back)"))
    print("knobs:")
    for name, value in r["knobs"].items():
        print(f"  {name}={value}")


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--json", action="store_true", help="print one JSON object")
    args = p.parse_args(argv)
    r = report()
    if args.json:
        print(json.dumps(r))
    else:
        _print_text(r)
    return 0 if r["extension"]["loaded"] else 1


if __name__ == "__main__":
    sys.exit(main())
