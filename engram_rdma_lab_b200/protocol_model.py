"""Executable model of the host route's serving protocol, for randomized interleaving checks.

The protocol (``csrc/kernels/exchange.cu``, ``csrc/owner_service.cpp``) for one
(requester, layer) slot at one owner:

* the requester's dispatch publishes epoch ``e`` in the mailbox header
  (``header.ready = e`` with ``rows``), and only after its hook saw
  ``done == e - 1`` (every owner released the previous epoch);
* ``claim`` and ``finish`` hold ``(e - 1) << 32 | count``: a worker claims the
  next 512-row chunk with a CAS that succeeds only while ``claim`` is armed for
  ``e - 1`` and ``count < chunks`` (``claim_chunk``), copies it, then adds one
  to ``finish``; the worker whose addition completes the epoch re-arms both
  words to ``e << 32`` and releases ``done = e`` (``serve_request``);
* workers are push kernels that the owner's CPU service launches for epochs it
  sees in the mailbox (``OwnerService::loop``), and the owner's own hook
  kernels, which copy the header into a board and serve whatever is armed
  while they wait (``refresh_board`` / ``hook_kernel``).

:func:`run` drives that model with a seeded random scheduler in which every
atomic step of every actor is one scheduling point, and checks the protocol's
invariants: each chunk of each epoch is copied exactly once, ``done`` is
released only after every chunk was copied, workers never copy for an epoch
that is not the armed one, and the service never reports an error on a legal
run.  ``strict_service=True`` restores a service that demands consecutive
epochs; the model finds runs where hooks finished epochs the service never
saw, which is why the service accepts forward jumps.
"""

from __future__ import annotations

import random
from dataclasses import dataclass, field


class ProtocolViolation(AssertionError):
    pass


@dataclass
class Slot:
    """Shared words of one (requester, layer) slot."""

    header_epoch: int = 0
    header_chunks: int = 0
    board_epoch: int = 0
    board_chunks: int = 0
    claim: tuple = (0, 0)   # (armed epoch - 1, chunks claimed)
    finish: tuple = (0, 0)  # (armed epoch - 1, chunks finished)
    done: int = 0
    copies: dict = field(default_factory=dict)  # (epoch, chunk) -> times copied


def _worker(slot: Slot, epoch: int, chunks: int, log):
    """A serving worker (push kernel or hook CTA) as a generator of atomic steps."""
    while True:
        yield "claim"
        armed, count = slot.claim
        if armed != epoch - 1 or count >= chunks:
            return
        slot.claim = (armed, count + 1)  # the CAS succeeded
        chunk = count
        yield "copy"
        if slot.done >= epoch:
            raise ProtocolViolation(f"chunk {chunk} of epoch {epoch} copied after done")
        slot.copies[(epoch, chunk)] = slot.copies.get((epoch, chunk), 0) + 1
        yield "finish"
        f_armed, f_count = slot.finish
        if f_armed != epoch - 1:
            raise ProtocolViolation(f"finish word armed for {f_armed + 1} while epoch {epoch} finishes")
        slot.finish = (f_armed, f_count + 1)
        if f_count + 1 == chunks:
            yield "rearm"
            slot.claim = (epoch, 0)
            slot.finish = (epoch, 0)
            yield "release"
            missing = [c for c in range(chunks) if slot.copies.get((epoch, c), 0) != 1]
            if missing:
                raise ProtocolViolation(f"epoch {epoch} released with chunks {missing} not copied once")
            slot.done = epoch
            log.append(("done", epoch))


def _requester(slot: Slot, epochs: list, log):
    """Publishes each epoch once the previous one is done (the hook saw it)."""
    for epoch, chunks in enumerate(epochs, start=1):
        while slot.done != epoch - 1:
            yield "wait_done"
        yield "write_rows"  # relaxed stores of the header fields ...
        slot.header_chunks = chunks
        yield "release_ready"  # ... then the releasing store of the epoch
        slot.header_epoch = epoch
        log.append(("publish", epoch))
    while slot.done != len(epochs):
        yield "wait_done"


def _service(slot: Slot, spawn, strict: bool, stop):
    """The owner's CPU thread: polls the header and launches push workers."""
    completed = 0
    while not stop():
        yield "poll_ready"  # acquire load of the epoch ...
        epoch = slot.header_epoch
        yield "poll_rows"  # ... then the rows, which may already belong to a later epoch
        chunks = slot.header_chunks
        if epoch == completed:
            continue
        if epoch < completed or (strict and epoch != completed + 1):
            raise ProtocolViolation(f"service saw epoch {epoch} after {completed}")
        completed = epoch
        spawn(_worker(slot, epoch, chunks, []), "push")


def _hook(slot: Slot, spawn, stop):
    """The owner's hook kernel: refreshes the board and serves armed requests."""
    while not stop():
        yield "refresh_ready"
        epoch = slot.header_epoch
        yield "refresh_rows"
        slot.board_epoch, slot.board_chunks = epoch, slot.header_chunks  # one 64-bit board store
        yield "look"
        epoch, chunks = slot.board_epoch, slot.board_chunks
        armed, count = slot.claim
        if epoch and armed == epoch - 1 and count < chunks:
            yield from _worker(slot, epoch, chunks, [])


def run(seed: int, epochs: int = 6, max_chunks: int = 4, hooks: int = 2, strict_service: bool = False,
        service_stall: float = 0.0, max_steps: int = 200000) -> dict:
    """One randomized run; raises :class:`ProtocolViolation` on a broken invariant.

    ``service_stall`` is the probability that the service is skipped when it
    is picked (a CPU thread that is descheduled now and then).
    """
    rng = random.Random(seed)
    slot = Slot()
    plan = [rng.randint(1, max_chunks) for _ in range(epochs)]
    log = []
    actors = []  # [name, generator]

    def finished():
        return slot.done == epochs

    def spawn(gen, name):
        actors.append([name, gen])

    actors.append(["requester", _requester(slot, plan, log)])
    actors.append(["service", _service(slot, spawn, strict_service, finished)])
    for h in range(hooks):
        actors.append([f"hook{h}", _hook(slot, spawn, finished)])
    steps = 0
    while actors:
        steps += 1
        if steps > max_steps:
            raise ProtocolViolation(f"no progress after {max_steps} steps (done={slot.done}, plan={plan})")
        i = rng.randrange(len(actors))
        name, gen = actors[i]
        if name == "service" and rng.random() < service_stall:
            continue
        try:
            next(gen)
        except StopIteration:
            actors.pop(i)
    for epoch, chunks in enumerate(plan, start=1):
        for chunk in range(chunks):
            if slot.copies.get((epoch, chunk), 0) != 1:
                raise ProtocolViolation(f"chunk {chunk} of epoch {epoch} copied {slot.copies.get((epoch, chunk), 0)}x")
    return {"plan": plan, "steps": steps, "done": slot.done}
