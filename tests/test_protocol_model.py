"""Randomized interleavings of the host route's serving protocol (model in
``engram_rdma_lab_b200/protocol_model.py``; no GPU)."""

import pytest

from engram_rdma_lab_b200.protocol_model import ProtocolViolation, run


@pytest.mark.parametrize("claim", ["add", "cas"])
@pytest.mark.parametrize("hooks", [0, 1, 3])
@pytest.mark.parametrize("add_stall", [0.0, 0.95])
def test_every_chunk_copied_once_under_random_interleavings(hooks, claim, add_stall):
    late = 0
    for seed in range(400):
        result = run(seed, epochs=6, max_chunks=4, hooks=hooks, service_stall=0.5, claim=claim, add_stall=add_stall)
        assert result["done"] == 6
        late += result["late_claims"]
    if claim == "add" and hooks and add_stall:
        # Fetch-and-adds that landed on the next epoch and served it were exercised.
        assert late > 0


def test_fetch_and_add_claims_need_arming_at_publication():
    """Claiming by fetch-and-add on a word that the last finisher re-arms lets
    a worker's final (failing) addition take chunk 0 of an epoch that is not
    published yet; nobody serves it and the epoch never completes."""
    failures = 0
    for seed in range(100):
        try:
            run(seed, hooks=1, service_stall=0.5, claim="add_eager", max_steps=20000)
        except ProtocolViolation as error:
            assert "no progress" in str(error)
            failures += 1
    assert failures > 0


def test_hooks_alone_serve_everything_when_the_service_stalls():
    for seed in range(200):
        assert run(seed, hooks=2, service_stall=0.99)["done"] == 6


def test_a_strict_service_breaks_on_epochs_the_hooks_finished():
    """The service once demanded consecutive epochs; hooks that serve while
    they wait can finish an epoch before the CPU thread looks, so that rule
    failed on real GPUs (mailbox sequence skipped).  The model finds it too."""
    failures = 0
    for seed in range(400):
        try:
            run(seed, hooks=2, strict_service=True, service_stall=0.9)
        except ProtocolViolation as error:
            assert "service saw epoch" in str(error)
            failures += 1
    assert failures > 0
