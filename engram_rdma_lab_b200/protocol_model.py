"""Executable model of the host route's serving protocol, for randomized interleaving checks.

The protocol (``csrc/kernels/exchange.cu``, ``csrc/owner_service.cpp``) for one
(requester, layer) slot at one owner:

* the requester's dispatch publishes epoch ``e`` in the mailbox header
  (``header.ready = e`` with ``rows``), and only after its hook saw
  ``done == e - 1`` (every owner released the previous epoch);
* the claim word holds ``(armed epoch, chunk limit, chunks claimed)``.  A
  worker that knows epoch ``e`` is published and finds the word armed for an
  earlier epoch arms it for ``e`` by CAS (limit = ``e``'s chunk count, count
  0); every claim is then one fetch-and-add (``claim_chunk``), which never
  retries, so the claims of many CTAs pipeline in the L2 instead of queueing
  behind one another's CAS;
* a fetch-and-add can land after the epoch the worker meant was finished and
  the word re-armed for the next one; it then holds a chunk of that later
  epoch, which is already published (arming needs the header), so it serves
  it, reading the rows from the header.  Only a worker's first claim can land
  like that: it claims each further chunk while it still holds an unfinished
  one (a CTA's control warp finishes the previous chunk and claims the next
  while the other warps copy the current one), so that epoch cannot complete.
  Re-arming at the last finish instead (``claim="add_eager"``) lets such a
  late addition take a chunk of an epoch that is not published yet, and the
  model finds runs that lose it;
* ``finish`` holds ``(e - 1, count)``; a worker adds one per copied chunk, and
  the one that completes the epoch resets it to ``(e, 0)`` and releases
  ``done = e`` (``serve_request``);
* workers are push kernels that the owner's CPU service launches for epochs it
  sees in the mailbox (``OwnerService::loop``), and the owner's own hook
  kernels, which copy the header into a board and serve whatever is armed
  while they wait (``refresh_board`` / ``hook_kernel``).

``claim="cas"`` restores the earlier scheme: ``claim`` held
``(e - 1, count)``, every claim was a CAS, and the last finisher re-armed it.

:func:`run` drives that model with a seeded random scheduler in which every
atomic step of every actor is one scheduling point, and checks the protocol's
invariants: each chunk of each epoch is copied exactly once, ``done`` is
released only after every chunk was copied, workers never copy for an epoch
that is not published, and the service never reports an error on a legal
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
    claim: tuple = (0, 0, 0)  # "add": (armed epoch, chunk limit, chunks claimed); "cas": (epoch - 1, count, 0)
    finish: tuple = (0, 0)    # (armed epoch - 1, chunks finished)
    done: int = 0
    copies: dict = field(default_factory=dict)  # (epoch, chunk) -> times copied
    late_claims: int = 0  # fetch-and-adds that landed on a later epoch and served it


def _copy(slot: Slot, epoch: int, chunk: int):
    yield "copy"
    if slot.done >= epoch:
        raise ProtocolViolation(f"chunk {chunk} of epoch {epoch} copied after done")
    if slot.header_epoch != epoch:
        raise ProtocolViolation(f"chunk {chunk} of epoch {epoch} copied while the header shows {slot.header_epoch}")
    slot.copies[(epoch, chunk)] = slot.copies.get((epoch, chunk), 0) + 1


def _finish(slot: Slot, epoch: int, chunks: int, rearm_claim: bool):
    """Counts one copied chunk; the last finisher releases ``done``."""
    yield "finish"
    f_armed, f_count = slot.finish
    if f_armed != epoch - 1:
        raise ProtocolViolation(f"finish word armed for {f_armed + 1} while epoch {epoch} finishes")
    slot.finish = (f_armed, f_count + 1)
    if f_count + 1 == chunks:
        yield "rearm"
        if rearm_claim:
            slot.claim = (epoch, 0, 0)
        slot.finish = (epoch, 0)
        yield "release"
        missing = [c for c in range(chunks) if slot.copies.get((epoch, c), 0) != 1]
        if missing:
            raise ProtocolViolation(f"epoch {epoch} released with chunks {missing} not copied once")
        slot.done = epoch


def _copy_and_finish(slot: Slot, epoch: int, chunk: int, chunks: int, rearm_claim: bool):
    yield from _copy(slot, epoch, chunk)
    yield from _finish(slot, epoch, chunks, rearm_claim)


def _worker_cas(slot: Slot, epoch: int, chunks: int):
    """The CAS scheme: claim while armed for ``epoch`` (tag ``epoch - 1``)."""
    while True:
        yield "claim"
        armed, count, _ = slot.claim
        if armed != epoch - 1 or count >= chunks:
            return
        slot.claim = (armed, count + 1, 0)  # the CAS succeeded
        yield from _copy_and_finish(slot, epoch, count, chunks, rearm_claim=True)


def _worker_add_eager(slot: Slot, epoch: int, chunks: int):
    """Fetch-and-add on a word the last finisher re-arms (unsafe: see the module doc)."""
    while True:
        yield "claim_add"
        armed, count, _ = slot.claim
        slot.claim = (armed, count + 1, 0)
        if armed != epoch - 1 or count >= chunks:
            return  # an addition to a word armed for another epoch is lost
        yield from _copy_and_finish(slot, epoch, count, chunks, rearm_claim=True)


def _claim_add(slot: Slot, epoch: int, chunks: int):
    """``claim_chunk``: arm for ``epoch`` if behind, then one fetch-and-add.

    Returns ``(epoch', chunk, limit, chunks')`` or None; ``epoch'`` can be a
    later epoch than ``epoch`` (a late addition), whose chunk count comes
    from the header.
    """
    while True:
        yield "arm_read"
        armed, limit, count = slot.claim
        if armed > epoch:
            return None
        if armed == epoch:
            if count >= limit:
                return None  # every chunk taken: leave without adding
            break
        yield "arm_cas"
        if slot.claim == (armed, limit, count):
            slot.claim = (epoch, chunks, 0)
            break
    yield "claim_add"
    armed, limit, count = slot.claim
    slot.claim = (armed, limit, count + 1)
    if armed < epoch:
        raise ProtocolViolation(f"claim word armed for {armed} after epoch {epoch} armed it")
    if count >= limit:
        return None
    if armed == epoch:
        return armed, count, limit, chunks
    yield "late_ready"  # a chunk of a later epoch: its rows come from the header
    seen = slot.header_epoch
    yield "late_rows"
    rows = slot.header_chunks
    if seen != armed:
        raise ProtocolViolation(f"late claim of epoch {armed} while the header shows {seen}")
    slot.late_claims += 1
    return armed, count, limit, rows


def _worker_add(slot: Slot, epoch: int, chunks: int):
    """``serve_request``: the first claim may arm the word or land on a later
    epoch; while a chunk is copied, the control warp finishes the previously
    copied chunk and claims the next one with a plain fetch-and-add, which
    cannot land on another epoch because the chunk in hand is unfinished."""
    got = yield from _claim_add(slot, epoch, chunks)
    if got is None:
        return
    epoch, chunk, limit, chunks = got
    if chunks != limit:
        raise ProtocolViolation(f"epoch {epoch}: {chunks} chunks from the worker's source, limit {limit}")
    copied = False
    while True:
        if copied:
            yield from _finish(slot, epoch, limit, rearm_claim=False)
        yield "claim_add"
        armed, lim, count = slot.claim
        slot.claim = (armed, lim, count + 1)
        if armed != epoch:
            raise ProtocolViolation(f"next claim of epoch {epoch} landed on epoch {armed}")
        yield from _copy(slot, epoch, chunk)
        copied = True
        if count >= lim:
            break
        chunk = count
    yield from _finish(slot, epoch, limit, rearm_claim=False)


WORKERS = {"add": _worker_add, "add_eager": _worker_add_eager, "cas": _worker_cas}


def _worth_serving(slot: Slot, epoch: int, chunks: int, claim: str) -> bool:
    """The hook's look at the board and the claim word before it serves."""
    if not epoch:
        return False
    if claim == "add":
        armed, limit, count = slot.claim
        return armed < epoch or (armed == epoch and count < limit)
    armed, count, _ = slot.claim
    return armed == epoch - 1 and count < chunks


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


def _service(slot: Slot, spawn, strict: bool, stop, worker):
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
        spawn(worker(slot, epoch, chunks), "push")


def _hook(slot: Slot, stop, claim: str):
    """The owner's hook kernel: refreshes the board and serves armed requests."""
    while not stop():
        yield "refresh_ready"
        epoch = slot.header_epoch
        yield "refresh_rows"
        slot.board_epoch, slot.board_chunks = epoch, slot.header_chunks  # one 64-bit board store
        yield "look"
        epoch, chunks = slot.board_epoch, slot.board_chunks
        if _worth_serving(slot, epoch, chunks, claim):
            yield from WORKERS[claim](slot, epoch, chunks)


def run(seed: int, epochs: int = 6, max_chunks: int = 4, hooks: int = 2, strict_service: bool = False,
        service_stall: float = 0.0, max_steps: int = 200000, claim: str = "add", add_stall: float = 0.0) -> dict:
    """One randomized run; raises :class:`ProtocolViolation` on a broken invariant.

    ``service_stall`` is the probability that the service is skipped when it
    is picked (a CPU thread that is descheduled now and then).  ``add_stall``
    is the same for a worker whose next step is its claim's fetch-and-add (an
    atomic that is slow to reach the L2), which is what makes additions land
    on a later epoch.  ``claim`` picks the claim scheme: ``add`` (the
    kernels'), ``cas`` or ``add_eager``.
    """
    worker = WORKERS[claim]
    rng = random.Random(seed)
    slot = Slot()
    plan = [rng.randint(1, max_chunks) for _ in range(epochs)]
    log = []
    actors = []  # [name, generator, the step it performs when next resumed]

    def finished():
        return slot.done == epochs

    def spawn(gen, name):
        actors.append([name, gen, None])

    actors.append(["requester", _requester(slot, plan, log), None])
    actors.append(["service", _service(slot, spawn, strict_service, finished, worker), None])
    for h in range(hooks):
        actors.append([f"hook{h}", _hook(slot, finished, claim), None])
    steps = 0
    while actors:
        steps += 1
        if steps > max_steps:
            raise ProtocolViolation(f"no progress after {max_steps} steps (done={slot.done}, plan={plan})")
        i = rng.randrange(len(actors))
        name, gen, pending = actors[i]
        if name == "service" and rng.random() < service_stall:
            continue
        if pending == "claim_add" and rng.random() < add_stall:
            continue
        try:
            actors[i][2] = next(gen)
        except StopIteration:
            actors.pop(i)
    for epoch, chunks in enumerate(plan, start=1):
        for chunk in range(chunks):
            if slot.copies.get((epoch, chunk), 0) != 1:
                raise ProtocolViolation(f"chunk {chunk} of epoch {epoch} copied {slot.copies.get((epoch, chunk), 0)}x")
    return {"plan": plan, "steps": steps, "done": slot.done, "late_claims": slot.late_claims}
