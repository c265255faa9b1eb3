"""Per-owner request packing on one GPU (the dispatch kernel as an op).

``route_pack(indices, entries, world)`` buckets every non-padding request of
``indices [layers, tokens, ept]`` by owner (``x // entries[l]``) and returns

* ``packed [world, layers, capacity]`` int64: for owner ``o`` and layer ``l``,
  the first ``counts[l, o]`` entries are ``(position << 32) | local_row`` where
  ``position`` is the flat ``token * ept + slot`` index and ``local_row`` is the
  row inside the owner's shard (``table_base[l] + x % entries[l]``);
* ``counts [layers, world]`` int32.

The order of entries within one owner is not specified (slots are reserved
with warp-aggregated atomics).  This is the requester half of the host route,
exposed for callers who run their own transport; parity with the reference's
``route_counts`` / ``route_prefix`` / ``route_pack`` kernels
(``sge_write/csrc/gpu_request.cu:8-115``), which produce a stable order.
"""

from __future__ import annotations

import torch

from .. import _native


def route_pack(indices: torch.Tensor, entries, world: int, owners=None, capacity: int | None = None):
    C = _native.load()
    L, T, E = indices.shape
    cap = capacity or max(1, T * E)
    owners = [1] * world if owners is None else [1 if o else 0 for o in owners]
    packed = torch.zeros(world, L, cap, dtype=torch.int64, device=indices.device)
    counts = torch.empty(L, world, dtype=torch.int32, device=indices.device)
    scratch = torch.zeros(L * world * 4 + L, dtype=torch.int32, device=indices.device)
    C.route_pack(indices, [int(n) for n in entries], int(world), owners, packed, counts, scratch)
    return packed, counts


def route_pack_reference(indices: torch.Tensor, entries, world: int, owners=None):
    """Plain torch version with a stable (ascending position) order."""
    L, T, E = indices.shape
    owners = [1] * world if owners is None else owners
    bases, at = [], 0
    for n in entries:
        bases.append(at)
        at += n
    out, counts = {}, torch.zeros(L, world, dtype=torch.int32)
    for layer, n in enumerate(entries):
        x = indices[layer].reshape(-1).to(torch.int64).cpu()
        pos = torch.arange(x.numel())
        for o in range(world):
            if not owners[o]:
                continue
            sel = (x >= 0) & (x // n == o)
            entry = (pos[sel] << 32) | (bases[layer] + x[sel] % n)
            out[(o, layer)] = entry
            counts[layer, o] = int(sel.sum())
    return out, counts
