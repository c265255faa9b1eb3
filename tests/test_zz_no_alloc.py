"""The allocation-free pack entry point, called through its exported C symbol.

`engram_route_pack_noalloc` serves callers that cannot allocate GPU memory
themselves (code inside CUDA Graph stream capture, plugins whose host framework
owns all device memory, C callers without torch's allocator): its scratch is a
fixed device array inside the library.  This test calls the symbol through
ctypes on two calls in a row and checks each result against the torch-facing
`route_pack` op, which takes caller-allocated scratch.  It lives in its own
file, collected last, so a failure here cannot hide the other tests.
"""

import ctypes

import pytest
import torch

from engram_rdma_lab_b200 import _native
from engram_rdma_lab_b200.models import make_indices
from engram_rdma_lab_b200.ops import route_pack

pytestmark = pytest.mark.gpu


def _symbol():
    lib = ctypes.CDLL(_native.load().__file__)
    fn = lib.engram_route_pack_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,  # indices, layers, tokens, ept
        ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint8),  # entries, world, owners
        ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,  # packed, capacity, counts
        ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t,  # stream, err, err_len
    ]
    return fn


def _call(fn, idx, entries, world, owners, packed, counts):
    L, T, E = idx.shape
    ent = (ctypes.c_uint32 * L)(*entries)
    own = (ctypes.c_uint8 * world)(*owners)
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(idx.data_ptr(), L, T, E, ent, world, own, packed.data_ptr(), packed.shape[2], counts.data_ptr(),
            ctypes.c_void_p(stream), err, len(err))
    return rc, err.value.decode()


def _canonical(packed, counts):
    world, layers = packed.shape[0], packed.shape[1]
    return {
        (o, l): torch.sort(packed[o, l, : int(counts[l, o])].cpu()).values
        for o in range(world)
        for l in range(layers)
    }


def test_noalloc_entry_point_matches_route_pack():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    fn = _symbol()
    entries, world, ept = (4099, 4111), 8, 24
    owners = [1, 1, 0, 1, 1, 1, 0, 1]
    for call, tokens in enumerate([1024, 777]):  # two calls in a row share the scratch array
        idx = make_indices(0, world, entries, tokens, ept, epoch=call + 1, padding=0.03, device="cuda")
        packed = torch.zeros(world, len(entries), tokens * ept, dtype=torch.int64, device="cuda")
        counts = torch.full((len(entries), world), -1, dtype=torch.int32, device="cuda")
        rc, msg = _call(fn, idx, entries, world, owners, packed, counts)
        assert rc == 0, msg
        want_packed, want_counts = route_pack(idx, entries, world, owners)
        torch.cuda.synchronize()
        assert torch.equal(counts.cpu(), want_counts.cpu())
        got, want = _canonical(packed, counts), _canonical(want_packed, want_counts)
        for key in want:
            assert torch.equal(got[key], want[key]), (call, key)


def test_noalloc_entry_point_rejects_oversized_requests():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    fn = _symbol()
    idx = torch.zeros(33, 2, 2, dtype=torch.int32, device="cuda")
    packed = torch.zeros(1, 33, 4, dtype=torch.int64, device="cuda")
    counts = torch.zeros(33, 1, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, idx, [10] * 33, 1, [1], packed, counts)
    assert rc != 0 and "layers" in msg
    idx = torch.zeros(1, 2, 2, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, idx, [10], 65, [1] * 65, torch.zeros(65, 1, 4, dtype=torch.int64, device="cuda"),
                    torch.zeros(1, 65, dtype=torch.int32, device="cuda"))
    assert rc != 0 and "world" in msg
