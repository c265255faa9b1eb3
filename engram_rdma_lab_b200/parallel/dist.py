"""Process-group bootstrap and GPU placement for one-process-per-GPU jobs.

* :func:`init_dist` reads ``RANK`` / ``LOCAL_RANK`` / ``WORLD_SIZE`` /
  ``MASTER_ADDR`` / ``MASTER_PORT`` (as set by ``torchrun``), binds the rank to
  its GPU and creates the default group with a short timeout so that ranks that
  wait on a dead peer fail instead of hanging.
* :func:`assigned_devices` / :func:`bind_rank` mirror the reference's
  fresh-process placement helpers (``benchmarks/rank_startup.py:13-71``): the
  parent resolves GPU UUIDs, and a spawned worker can put its own GPU first in
  ``CUDA_VISIBLE_DEVICES`` before the CUDA driver initialises, verifying the
  UUID afterwards.
"""

from __future__ import annotations

import datetime
import os
import subprocess

import torch
import torch.distributed as dist


def init_dist(backend: str | None = None, timeout_s: float = 120.0, device_id: bool = True):
    """Initialise the default process group from torchrun-style env vars.

    Returns ``(rank, world_size, local_rank)``.  With ``backend=None`` the NCCL
    backend is used when CUDA is available, gloo otherwise.  When the default
    group exists already, its own rank and size are returned.
    """
    if dist.is_initialized():
        rank, world = dist.get_rank(), dist.get_world_size()
        return rank, world, int(os.environ.get("LOCAL_RANK", str(rank)))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kwargs = dict(backend=backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        torch.cuda.set_device(local_rank)
        if device_id:
            kwargs["device_id"] = torch.device("cuda", local_rank)
    dist.init_process_group(**kwargs)
    return rank, world, local_rank


def assigned_devices(local_ranks: int):
    """UUID and physical index of every visible GPU, resolved in the parent."""
    count = torch.cuda.device_count()
    if count < local_ranks:
        raise ValueError(f"Need {local_ranks} GPUs, found {count}")
    physical = {}
    try:
        rows = subprocess.check_output(["nvidia-smi", "--query-gpu=uuid,index", "--format=csv,noheader"], text=True)
        for row in rows.splitlines():
            uuid, index = row.split(",")
            physical[uuid.strip()] = int(index)
    except (OSError, subprocess.CalledProcessError, ValueError):
        pass
    devices = []
    for ordinal in range(count):
        uuid = str(torch.cuda.get_device_properties(ordinal).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        devices.append({"uuid": uuid, "physical_index": physical.get(uuid)})
    if len({d["uuid"] for d in devices}) != count:
        raise ValueError("Assigned GPU UUIDs must be unique")
    return devices


def bind_rank(local_rank: int, devices, own_gpu_first: bool = False):
    """Select this worker's GPU; optionally list it first in CUDA_VISIBLE_DEVICES.

    Must run before the process initialises CUDA.  Returns
    ``(cuda_ordinal, placement_dict)``.
    """
    if torch.cuda.is_initialized():
        raise RuntimeError("Bind the rank before its first CUDA initialization")
    if not 0 <= local_rank < len(devices):
        raise ValueError("Invalid local rank")
    if own_gpu_first:
        order = [local_rank] + [i for i in range(len(devices)) if i != local_rank]
        os.environ["CUDA_VISIBLE_DEVICES"] = ",".join(devices[i]["uuid"] for i in order)
    ordinal = 0 if own_gpu_first else local_rank
    torch.cuda.set_device(ordinal)
    actual = str(torch.cuda.get_device_properties(ordinal).uuid).removeprefix("GPU-")
    if actual != devices[local_rank]["uuid"].removeprefix("GPU-"):
        raise RuntimeError("GPU enumeration changed the rank's physical GPU assignment")
    return ordinal, {
        "own_gpu_first": own_gpu_first,
        "logical_local_rank": local_rank,
        "cuda_ordinal": ordinal,
        "physical_gpu_uuid": devices[local_rank]["uuid"],
        "physical_gpu_index": devices[local_rank]["physical_index"],
        "cuda_visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES"),
    }


def max_over_ranks(value: float, group=None) -> float:
    """Maximum of a host scalar over the group (device tensor for NCCL)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    device = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def gather_floats(values, group=None):
    """All-gather equal-length float lists; returns ``[rank][i]``."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [list(values)]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, list(values), group=group)
    return out
