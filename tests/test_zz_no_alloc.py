"""The allocation-free pack entry point, called through its exported C symbol.

`engram_route_pack_noalloc` serves callers that cannot allocate GPU memory
themselves: code inside CUDA Graph stream capture (cudaMalloc is not allowed
there), plugins whose host framework owns all device memory, and C callers
without torch's allocator.  Its scratch is a fixed device array inside the
library.  This test reads the C prototype from `csrc/engram_noalloc.h` (so the
header is the one statement of the signature), calls the symbol through ctypes
on consecutive calls, and checks each result against `route_pack_reference`,
the plain torch oracle of the pack.  It lives in its own file, collected last,
so a failure here cannot hide the other tests.
"""

import ctypes
import os
import re

import pytest
import torch

from engram_rdma_lab_b200 import _native
from engram_rdma_lab_b200.models import make_indices
from engram_rdma_lab_b200.ops.pack import route_pack_reference

pytestmark = pytest.mark.gpu

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc", "engram_noalloc.h")
C_TYPES = {"uint32_t": ctypes.c_uint32, "size_t": ctypes.c_size_t, "cudaStream_t": ctypes.c_void_p}


def _prototype():
    """(argtypes, codes) parsed from the header's declaration and #defines."""
    text = open(HEADER).read()
    decl = re.search(r"int\s+engram_route_pack_noalloc\s*\(([^)]*)\)\s*;", text)
    assert decl, "engram_noalloc.h declares engram_route_pack_noalloc"
    argtypes = []
    for param in decl.group(1).split(","):
        words = param.replace("*", " * ").split()
        if "*" in words:
            argtypes.append(ctypes.c_char_p if words[0] == "char" else ctypes.c_void_p)
        else:
            argtypes.append(C_TYPES[words[-2]])
    codes = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define ENGRAM_NOALLOC_(\w+) (\d+)", text)}
    return argtypes, codes


def _symbol():
    argtypes, codes = _prototype()
    fn = ctypes.CDLL(_native.load().__file__).engram_route_pack_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = argtypes
    return fn, codes


def _call(fn, idx, entries, world, owners, packed, counts):
    L, T, E = idx.shape
    ent = (ctypes.c_uint32 * L)(*entries)
    own = (ctypes.c_uint8 * world)(*owners)
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(idx.data_ptr(), L, T, E, ctypes.cast(ent, ctypes.c_void_p), world, ctypes.cast(own, ctypes.c_void_p),
            packed.data_ptr(), packed.shape[2], counts.data_ptr(), stream, err, len(err))
    return rc, err.value.decode()


def _check_against_oracle(idx, entries, world, owners, packed, counts):
    want, want_counts = route_pack_reference(idx, entries, world, owners)
    got_counts = counts.cpu()
    assert torch.equal(got_counts, want_counts), (got_counts, want_counts)
    for (o, layer), entry in want.items():
        got = torch.sort(packed[o, layer, : int(got_counts[layer, o])].cpu()).values
        assert torch.equal(got, torch.sort(entry).values), (o, layer)


def test_noalloc_entry_point_matches_torch_oracle():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    fn, _ = _symbol()
    entries, world, ept = (4099, 4111), 8, 24
    owners = [1, 1, 0, 1, 1, 1, 0, 1]
    for call, tokens in enumerate([1024, 777, 1024]):  # consecutive calls share the scratch array
        idx = make_indices(0, world, entries, tokens, ept, epoch=call + 1, padding=0.03, device="cuda")
        if call == 1:
            # An id beyond the vocabulary is skipped: it is in no list and no count.
            idx[0, 3, 5] = entries[0] * world + 11
            idx[1, 0, 0] = entries[1] * world
        packed = torch.zeros(world, len(entries), tokens * ept, dtype=torch.int64, device="cuda")
        counts = torch.full((len(entries), world), -1, dtype=torch.int32, device="cuda")
        rc, msg = _call(fn, idx, entries, world, owners, packed, counts)
        assert rc == 0, msg
        torch.cuda.synchronize()
        _check_against_oracle(idx, entries, world, owners, packed, counts)


def test_noalloc_entry_point_empty_request_clears_counts():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    fn, _ = _symbol()
    entries, world = (4099, 4111), 4
    idx = torch.empty(2, 0, 24, dtype=torch.int32, device="cuda")
    packed = torch.zeros(world, 2, 1, dtype=torch.int64, device="cuda")
    counts = torch.full((2, world), -1, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, idx, entries, world, [1] * world, packed, counts)
    assert rc == 0, msg
    torch.cuda.synchronize()
    assert torch.equal(counts.cpu(), torch.zeros(2, world, dtype=torch.int32))


def test_noalloc_entry_point_rejects_oversized_requests():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)
    fn, codes = _symbol()
    idx = torch.zeros(33, 2, 2, dtype=torch.int32, device="cuda")
    packed = torch.zeros(1, 33, 4, dtype=torch.int64, device="cuda")
    counts = torch.zeros(33, 1, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, idx, [10] * 33, 1, [1], packed, counts)
    assert rc == codes["BAD_SHAPE"] and "layers" in msg
    idx = torch.zeros(1, 2, 2, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, idx, [10], 65, [1] * 65, torch.zeros(65, 1, 4, dtype=torch.int64, device="cuda"),
                    torch.zeros(1, 65, dtype=torch.int32, device="cuda"))
    assert rc == codes["BAD_SHAPE"] and "world" in msg
    # Three layers of 2^31 - 1 rows each: the running table base would pass 2^32.
    idx = torch.zeros(3, 2, 2, dtype=torch.int32, device="cuda")
    rc, msg = _call(fn, idx, [2**31 - 1] * 3, 1, [1], torch.zeros(1, 3, 4, dtype=torch.int64, device="cuda"),
                    torch.zeros(3, 1, dtype=torch.int32, device="cuda"))
    assert rc == codes["BAD_ENTRIES"] and "2^32" in msg
