"""Engram table sets: shapes, synthetic weights and request distributions.

An "Engram model" here is a set of per-layer embedding tables sharded by row
over the ranks of one NVLink node, plus the index stream a model emits per
forward (``[layers, tokens, entries_per_token]`` int32, ``-1`` = padding).

* :data:`CONFIGS` names the benchmark shapes (the table sets of the project's
  benchmark configurations 0-4).
* :func:`row_pattern` gives every global row a deterministic byte pattern, so a
  fetched output can be checked bit-exactly from the indices alone (the
  reference's tests use the same idea with their own hash,
  ``benchmarks/test_write.py:20-58``; the hash below is splitmix64, not theirs).
* :func:`normal_bf16_shard` / :func:`quantized_fp8_shard` give random-init
  weights of the named distributions.
* :func:`make_indices` draws uniform, stratified, single-owner, Zipf or
  MT19937-matched request streams.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np
import torch


_MASK63 = (1 << 63) - 1
_GOLDEN = 0x9E3779B97F4A7C15 - (1 << 64)
_MIX1 = 0xBF58476D1CE4E5B9 - (1 << 64)
_MIX2 = 0x94D049BB133111EB - (1 << 64)


@dataclass(frozen=True)
class TableSpec:
    """One benchmark table set.  ``entries`` are rows per rank per layer."""

    name: str
    entries: tuple
    hidden: int
    ept: int
    max_tokens: int
    tokens: int
    dtype: torch.dtype
    num_sf_packs: int
    distribution: str = "uniform"
    padding: float = 0.0
    weights: str = "pattern"

    @property
    def layers(self) -> int:
        return len(self.entries)

    @property
    def row_bytes(self) -> int:
        return self.hidden * torch.empty((), dtype=self.dtype).element_size()

    def bytes_per_fetch(self, tokens: int | None = None) -> int:
        """Embedding bytes returned to one requester per fetch."""
        t = self.tokens if tokens is None else tokens
        return self.layers * t * self.ept * self.row_bytes

    def with_(self, **kw) -> "TableSpec":
        return replace(self, **kw)


CONFIGS = {
    # 0: CPU/gloo oracle shape.
    "oracle": TableSpec("oracle", (4096 // 2, 4099 // 2 + 1), 64, 4, 128, 128, torch.bfloat16, 0,
                        padding=0.10, weights="normal"),
    # 1: BF16, host shards, owner-push route.
    "bf16_host": TableSpec("bf16_host", (524288, 524309), 256, 24, 4096, 4096, torch.bfloat16, 0,
                           padding=0.02, weights="normal"),
    # 2: FP8 e4m3 with two 128-column scale packs (the headline shape).
    "fp8": TableSpec("fp8", (524288, 524309), 256, 24, 4096, 4096, torch.float8_e4m3fn, 2,
                     weights="quantized"),
    # 3: FP8 CUDA-Graph replay, 4 layers, prime-sized entries, Zipf skew.
    "fp8_graph": TableSpec("fp8_graph", (2097143, 2097143, 2097143, 2097143), 512, 24, 8192, 8192,
                           torch.float8_e4m3fn, 4, distribution="zipf", padding=0.05, weights="quantized"),
    # 4: scaling sweep base shape (tokens varied by the sweep).
    "scaling": TableSpec("scaling", (524288, 524288), 256, 24, 16384, 4096, torch.float8_e4m3fn, 2),
}


def _splitmix(z: torch.Tensor) -> torch.Tensor:
    """splitmix64 finaliser on int64 tensors (wrapping arithmetic)."""

    def lshr(v, s):
        return (v >> s) & ((1 << (64 - s)) - 1)

    z = z * _GOLDEN
    z = (z ^ lshr(z, 30)) * _MIX1
    z = (z ^ lshr(z, 27)) * _MIX2
    return z ^ lshr(z, 31)


def row_pattern(global_rows: torch.Tensor, layer: int, row_bytes: int, salt: int = 0) -> torch.Tensor:
    """Deterministic bytes ``[N, row_bytes]`` for global rows of ``layer``."""
    if row_bytes % 8:
        raise ValueError("row_bytes must be a multiple of 8")
    words = row_bytes // 8
    key = (global_rows.to(torch.int64) * 64 + layer) * 1024 + salt
    w = torch.arange(words, dtype=torch.int64, device=global_rows.device)
    mixed = _splitmix(key[:, None] * words + w[None, :] + 1)
    return mixed.contiguous().view(torch.uint8).reshape(-1, row_bytes)


def pattern_scales(global_rows: torch.Tensor, layer: int, packs: int, salt: int = 0) -> torch.Tensor:
    """Deterministic power-of-two fp32 scales in ``[2^-8, 2^0]``, ``[N, packs]``."""
    key = (global_rows.to(torch.int64) * 64 + layer) * 1024 + salt + 7
    p = torch.arange(packs, dtype=torch.int64, device=global_rows.device)
    h = _splitmix(key[:, None] * 131 + p[None, :])
    exponent = (h & 0xFF) % 9
    return torch.pow(2.0, -exponent.to(torch.float32))


def pattern_shard(rank: int, world: int, spec_entries, hidden: int, dtype, packs: int, device, salt: int = 0):
    """This rank's tables and the global scale tables in the pattern scheme."""
    esize = torch.empty((), dtype=dtype).element_size()
    storages, scales = [], []
    for layer, n in enumerate(spec_entries):
        rows = torch.arange(n, dtype=torch.int64, device=device) + rank * n
        storages.append(row_pattern(rows, layer, hidden * esize, salt).view(dtype).reshape(n, hidden))
        if packs:
            scales.append(pattern_scales(torch.arange(world * n, device=device), layer, packs, salt))
    return storages, (scales if packs else None)


def expected_outputs(indices: torch.Tensor, spec_entries, hidden: int, dtype, packs: int, salt: int = 0):
    """What a fetch of ``indices`` must return under the pattern scheme.

    Returns per layer ``(bytes [tokens, ept*row_bytes], scales [tokens, ept*packs] | None)``.
    """
    esize = torch.empty((), dtype=dtype).element_size()
    row_bytes = hidden * esize
    L, T, E = indices.shape
    out = []
    for layer, n in enumerate(spec_entries):
        x = indices[layer].reshape(-1).to(torch.int64)
        valid = x >= 0
        safe = x.clamp_min(0)
        data = row_pattern(safe, layer, row_bytes, salt) * valid[:, None].to(torch.uint8)
        sf = None
        if packs:
            sf = pattern_scales(safe, layer, packs, salt) * valid[:, None].to(torch.float32)
            sf = sf.reshape(T, E * packs)
        out.append((data.reshape(T, E * row_bytes), sf))
    return out


def normal_bf16_shard(rank: int, world: int, entries, hidden: int, device, std: float = 0.02, seed: int = 1):
    """Random-init BF16 tables ~ N(0, std) for this rank's rows."""
    g = torch.Generator(device=device).manual_seed(seed * 7919 + rank)
    return [
        (torch.randn(n, hidden, generator=g, device=device, dtype=torch.float32) * std).to(torch.bfloat16)
        for n in entries
    ]


def quantized_fp8_shard(rank: int, world: int, entries, hidden: int, packs: int, device, seed: int = 1):
    """FP8 e4m3 tables whose dequantised values are ``N(0, 1) * scale``.

    Every 128-column block of global row ``x`` has a power-of-two scale in
    ``[2^-8, 2^0]`` drawn from a per-layer seed, so the global scale table
    ``[world * n, packs]`` is identical on every rank.  The stored codes are
    ``e4m3(value / scale)``, i.e. standard-normal draws rounded to e4m3.
    """
    storages, scales = [], []
    for layer, n in enumerate(entries):
        g = torch.Generator(device=device).manual_seed((seed * 104729 + layer) * 8191 + rank)
        codes = torch.randn(n, hidden, generator=g, device=device, dtype=torch.float32)
        storages.append(codes.clamp(-448.0, 448.0).to(torch.float8_e4m3fn))
        gs = torch.Generator(device=device).manual_seed(seed * 15485863 + layer)
        exponent = torch.randint(0, 9, (world * n, packs), generator=gs, device=device)
        scales.append(torch.pow(2.0, -exponent.to(torch.float32)))
    return storages, scales


def expected_random_init(indices: torch.Tensor, spec_entries, hidden: int, dtype, packs: int, world: int,
                         seed: int = 1):
    """What a fetch of ``indices`` must return when every rank wrote the random-init tables.

    The tables are :func:`quantized_fp8_shard` (``packs > 0``) or
    :func:`normal_bf16_shard` with ``seed``; each owner's rows are regenerated
    here from its rank (one owner at a time, so memory stays at one shard), and
    the requested rows are gathered from them.  Returns per layer
    ``(bytes [tokens, ept*row_bytes], scales [tokens, ept*packs] | None)`` on
    the indices' device, like :func:`expected_outputs`.
    """
    device = indices.device
    L, T, E = indices.shape
    esize = torch.empty((), dtype=dtype).element_size()
    row_bytes = hidden * esize
    x = indices.reshape(L, T * E).to(torch.int64)
    data = [torch.zeros(T * E, row_bytes, dtype=torch.uint8, device=device) for _ in range(L)]
    scales = [None] * L
    for owner in range(world):
        if packs:
            storages, sf = quantized_fp8_shard(owner, world, spec_entries, hidden, packs, device, seed)
        else:
            storages, sf = normal_bf16_shard(owner, world, spec_entries, hidden, device, seed=seed), None
        for layer, n in enumerate(spec_entries):
            mine = ((x[layer] >= 0) & (x[layer] // n == owner)).nonzero().flatten()
            rows = storages[layer].view(torch.uint8).reshape(n, row_bytes)
            data[layer].index_copy_(0, mine, rows.index_select(0, x[layer].index_select(0, mine) - owner * n))
            if packs and scales[layer] is None:
                valid = (x[layer] >= 0)[:, None].to(torch.float32)
                scales[layer] = (sf[layer].index_select(0, x[layer].clamp_min(0)) * valid).reshape(T, E * packs)
        del storages, sf
    return [(d.reshape(T, E * row_bytes), scales[layer]) for layer, d in enumerate(data)]


def _zipf_cdf(size: int, s: float, device) -> torch.Tensor:
    ranks = torch.arange(1, size + 1, dtype=torch.float64, device=device)
    w = ranks.pow(-s)
    cdf = torch.cumsum(w, 0)
    return cdf / cdf[-1]


_ZIPF_CACHE: dict = {}


def make_indices(
    rank: int,
    world: int,
    entries,
    tokens: int,
    ept: int,
    epoch: int = 1,
    distribution: str = "uniform",
    padding: float = 0.0,
    owner: int | None = None,
    zipf_s: float = 1.1,
    device="cpu",
) -> torch.Tensor:
    """Draw one ``[layers, tokens, ept]`` int32 request tensor.

    ``distribution``: ``uniform`` over all ``world * n`` global rows;
    ``stratified`` (entry slot ``e`` draws from its own ``1/ept`` interval);
    ``zipf`` (rank-``k`` row has weight ``k^-s``; low global ids, hence low
    owners, are hot); ``matched`` (numpy MT19937 raw uint32 draws reduced
    modulo the range, seeded like the reference's matched-read inputs so both
    benchmarks see identical requests).  ``owner`` restricts every row to one
    owner.  ``padding`` is the fraction of slots set to ``-1``.
    """
    seed = 12345 + rank * 1009 + epoch * 97
    layers = []
    if distribution == "matched":
        rng = np.random.RandomState(seed)
        raw = rng.randint(0, 1 << 32, size=(len(entries), tokens, ept), dtype=np.uint32)
        for layer, n in enumerate(entries):
            if owner is not None:
                raw[layer] %= n
                raw[layer] += owner * n
            else:
                raw[layer] %= world * n
        out = torch.from_numpy(raw.view(np.int32).copy()).to(device)
    else:
        g = torch.Generator(device=device).manual_seed(seed)
        for layer, n in enumerate(entries):
            total = world * n
            if owner is not None:
                x = torch.randint(0, n, (tokens, ept), generator=g, device=device, dtype=torch.int64) + owner * n
            elif distribution == "uniform":
                x = torch.randint(0, total, (tokens, ept), generator=g, device=device, dtype=torch.int64)
            elif distribution == "stratified":
                interval = total // ept
                x = torch.randint(0, interval, (tokens, ept), generator=g, device=device, dtype=torch.int64)
                x = x + torch.arange(ept, device=device, dtype=torch.int64) * interval
            elif distribution == "zipf":
                key = (total, zipf_s, str(device))
                if key not in _ZIPF_CACHE:
                    _ZIPF_CACHE.clear()
                    _ZIPF_CACHE[key] = _zipf_cdf(total, zipf_s, device)
                u = torch.rand(tokens * ept, generator=g, device=device, dtype=torch.float64)
                x = torch.searchsorted(_ZIPF_CACHE[key], u).clamp_max(total - 1).reshape(tokens, ept)
            else:
                raise ValueError(f"unknown distribution {distribution!r}")
            layers.append(x.to(torch.int32))
        out = torch.stack(layers) if layers else torch.empty(0, tokens, ept, dtype=torch.int32, device=device)
    if padding > 0 and tokens:
        gp = torch.Generator(device=device).manual_seed(seed + 1)
        mask = torch.rand(out.shape, generator=gp, device=device) < padding
        out = out.masked_fill(mask, -1)
    return out.contiguous()
