"""Native host components without a GPU: owner service and descriptor passing.

Failure detection is exercised on the host: a requester that skips an epoch,
a mailbox with out-of-range bounds, a launcher that fails, and an importer
asking for a descriptor that does not exist.
"""

import time

import pytest
import torch  # noqa: F401  (loads libc10 before the extension)

from engram_rdma_lab_b200 import _native

C = _native.load()

from ._spawn import run_ranks  # noqa: E402


def _wait(pred, timeout=5.0):
    deadline = time.time() + timeout
    while time.time() < deadline:
        if pred():
            return True
        time.sleep(0.005)
    return pred()


def test_owner_service_serves_in_sequence():
    h = C.OwnerServiceHarness(4, 2, 4096, [1, 1, 0, 1])
    h.start()
    h.publish(1, 0, 1, 100, 4)
    h.publish(3, 1, 1, 7, 2)
    assert _wait(lambda: len(h.launched()) == 2)
    h.publish(1, 0, 2, 50, 1)
    assert _wait(lambda: len(h.launched()) == 3)
    launched = sorted(h.launched())
    assert (1, 0, 100, 1, 4) in launched and (3, 1, 7, 1, 2) in launched and (1, 0, 50, 2, 1) in launched
    # Requester 2 is not served (it reads directly); its mailbox is ignored.
    h.publish(2, 0, 1, 10, 1)
    time.sleep(0.05)
    assert len(h.launched()) == 3
    assert h.running
    h.stop()
    assert h.error() == ""


def test_owner_service_accepts_forward_jumps_and_latches_backward_sequence():
    h = C.OwnerServiceHarness(2, 1, 64, [0, 1])
    h.start()
    h.publish(1, 0, 1, 5, 1)
    assert _wait(lambda: len(h.launched()) == 1)
    # Epochs 2-3 were finished by the owner's hooks before the thread looked.
    h.publish(1, 0, 4, 6, 1)
    assert _wait(lambda: len(h.launched()) == 2)
    assert (1, 0, 6, 4, 1) in h.launched() and h.error() == ""
    h.publish(1, 0, 2, 5, 1)  # backwards
    assert _wait(lambda: h.error() != "")
    assert "backwards" in h.error()
    assert not h.running
    with pytest.raises(RuntimeError):
        h.check()
    h.stop()


def test_owner_service_latches_bounds_error():
    h = C.OwnerServiceHarness(2, 1, 64, [0, 1])
    h.start()
    h.publish(1, 0, 1, 65, 1)  # more rows than the slot holds
    assert _wait(lambda: "bounds" in h.error())
    h.stop()


def test_owner_service_launch_failure():
    h = C.OwnerServiceHarness(2, 2, 64, [0, 1])
    h.start(fail_after=1)
    h.publish(1, 0, 1, 5, 1)
    assert _wait(lambda: len(h.launched()) == 1)
    h.publish(1, 1, 1, 5, 1)
    assert _wait(lambda: "injected" in h.error())
    h.stop()


def test_fd_server_same_process():
    fd = C.memfd_with_bytes(b"engram shard bytes")
    server = C.FdServer("engram-test-local", [fd, -1])
    got = C.fetch_fd("engram-test-local", 0, 5.0)
    assert C.read_fd_bytes(got, 18) == b"engram shard bytes"
    with pytest.raises(RuntimeError):
        C.fetch_fd("engram-test-local", 1, 2.0)  # not exported
    with pytest.raises(RuntimeError):
        C.fetch_fd("engram-test-local", 5, 2.0)  # out of range
    server.stop()
    with pytest.raises(RuntimeError):
        C.fetch_fd("engram-test-local", 0, 0.2)  # server gone


def test_fd_server_refuses_other_users():
    import os
    import subprocess
    import sys

    if os.geteuid() != 0:
        pytest.skip("switching to another user needs root")
    fd = C.memfd_with_bytes(b"private")
    server = C.FdServer("engram-test-uid", [fd])
    code = (
        "import os, socket, struct\n"
        "s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)\n"
        "os.setgid(65534); os.setuid(65534)\n"
        "s.connect('\\0engram-test-uid')\n"
        "s.sendall(struct.pack('i', 0))\n"
        "s.settimeout(5)\n"
        "try:\n"
        "    print('refused' if not s.recv(16) else 'served')\n"
        "except ConnectionResetError:\n"
        "    print('refused')\n"
    )
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "refused"  # closed (or reset) without a byte or a descriptor
    assert server.rejected == 1 and server.served == 0
    assert C.read_fd_bytes(C.fetch_fd("engram-test-uid", 0, 5.0), 7) == b"private"  # same user still served
    server.stop()


def _fd_exchange(rank, world, token):
    import torch.distributed as dist

    fd = C.memfd_with_bytes(f"rank-{rank}-payload".encode())
    server = C.FdServer(f"engram-test-{token}-{rank}", [fd])
    dist.barrier()
    for peer in range(world):
        got = C.fetch_fd(f"engram-test-{token}-{peer}", 0, 10.0)
        want = f"rank-{peer}-payload".encode()
        assert C.read_fd_bytes(got, len(want)) == want
    dist.barrier()
    server.stop()


def test_fd_exchange_across_processes(port):
    run_ranks(_fd_exchange, 3, port, args=(str(port),))


def test_nvtx_ranges_toggle_and_run_without_a_profiler():
    assert C.nvtx_enabled() is False
    C.set_nvtx(True)
    try:
        assert C.nvtx_enabled() is True
        h = C.OwnerServiceHarness(2, 1, 64, [0, 1])  # launches run inside an NVTX range
        h.start()
        h.publish(1, 0, 1, 5, 1)
        assert _wait(lambda: len(h.launched()) == 1)
        h.stop()
        assert h.error() == ""
    finally:
        C.set_nvtx(False)
