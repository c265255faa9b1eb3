"""Randomized interleavings of the host route's serving protocol (model in
``engram_rdma_lab_b200/protocol_model.py``; no GPU)."""

import pytest

from engram_rdma_lab_b200.protocol_model import ProtocolViolation, run


@pytest.mark.parametrize("hooks", [0, 1, 3])
def test_every_chunk_copied_once_under_random_interleavings(hooks):
    for seed in range(400):
        result = run(seed, epochs=6, max_chunks=4, hooks=hooks, service_stall=0.5)
        assert result["done"] == 6


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
