"""Run a function on N local ranks (one process each) and collect failures."""

import datetime
import os
import sys
import traceback

import torch.distributed as dist
import torch.multiprocessing as mp


def _entry(rank, world, port, backend, fn, args, errors):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        if backend == "nccl":
            import torch

            torch.cuda.set_device(rank)
        dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        try:
            fn(rank, world, *args)
            dist.barrier()  # no rank tears its connections down while a peer still uses them
        finally:
            dist.destroy_process_group()
    except BaseException:  # noqa: BLE001 - report everything to the parent
        errors.put((rank, traceback.format_exc()))
        raise
    # Success: leave without interpreter finalisation.  Process-group
    # destructors that run at exit while the peer process is exiting too
    # have aborted a finished rank (SIGABRT) now and then.
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(0)


def run_ranks(fn, world, port, backend="gloo", args=(), timeout=300):
    ctx = mp.get_context("spawn")
    errors = ctx.SimpleQueue()
    procs = [ctx.Process(target=_entry, args=(r, world, port, backend, fn, args, errors)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    messages = []
    while not errors.empty():
        messages.append(errors.get())
    if messages:
        rank, text = messages[0]
        raise AssertionError(f"rank {rank} failed:\n{text}")
    if alive:
        raise AssertionError(f"{len(alive)} rank(s) timed out")
    bad = [p.exitcode for p in procs if p.exitcode != 0]
    if bad:
        raise AssertionError(f"rank exit codes {bad}")
