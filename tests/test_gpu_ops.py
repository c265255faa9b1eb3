"""Single-GPU ops: per-owner request packing vs. a plain torch reference, and the zero-copy host read and write."""

import pytest
import torch

from engram_rdma_lab_b200.models import make_indices
from engram_rdma_lab_b200.ops import route_pack, route_pack_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    torch.cuda.set_device(0)


def canonical(packed, counts, world, layers):
    out = {}
    for o in range(world):
        for layer in range(layers):
            n = int(counts[layer, o])
            out[(o, layer)] = torch.sort(packed[o, layer, :n].cpu()).values
    return out


@pytest.mark.parametrize("world,tokens,ept", [(8, 4096, 24), (3, 1000, 7), (64, 33, 5), (1, 5, 1)])
def test_route_pack_matches_reference(world, tokens, ept):
    entries = (1031, 997)
    idx = make_indices(0, world, entries, tokens, ept, padding=0.05, device="cuda")
    owners = [1 if o % 3 != 1 else 0 for o in range(world)]
    packed, counts = route_pack(idx, entries, world, owners)
    torch.cuda.synchronize()
    ref, ref_counts = route_pack_reference(idx, entries, world, owners)
    assert torch.equal(counts.cpu(), ref_counts)
    got = canonical(packed, counts, world, len(entries))
    for key, want in ref.items():
        assert torch.equal(got[key], torch.sort(want).values), key


def test_route_pack_empty_and_padding_only():
    entries = (100,)
    idx = torch.full((1, 16, 4), -1, dtype=torch.int32, device="cuda")
    packed, counts = route_pack(idx, entries, 4)
    assert int(counts.sum()) == 0
    empty = torch.empty(1, 0, 4, dtype=torch.int32, device="cuda")
    packed, counts = route_pack(empty, entries, 4)
    assert int(counts.sum()) == 0


def test_host_read_streams_pinned_memory_into_the_gpu():
    from engram_rdma_lab_b200 import _native

    C = _native.load()
    src = torch.randint(0, 255, (3 * 65536 + 48,), dtype=torch.uint8).pin_memory()
    dst = torch.zeros(src.numel(), dtype=torch.uint8, device="cuda")
    C.host_read(src, dst, 37)
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu(), src)
    with pytest.raises(RuntimeError, match="pinned"):
        C.host_read(src.clone(), dst, 8)  # pageable memory is refused


def test_host_write_streams_a_gpu_tensor_into_pinned_memory():
    from engram_rdma_lab_b200 import _native

    C = _native.load()
    for size in (16, 6144, 1 << 20):
        src = torch.randint(0, 255, (size,), dtype=torch.uint8, device="cuda")
        dst = torch.zeros(size, dtype=torch.uint8).pin_memory()
        C.host_write(src, dst, 1 if size < 8192 else 64)
        torch.cuda.synchronize()
        assert torch.equal(dst, src.cpu())
    with pytest.raises(RuntimeError):
        C.host_write(src, torch.zeros(1 << 20, dtype=torch.uint8), 8)  # pageable memory is refused
