"""Per-rank memory plan shared by the native runtime and the torch oracle.

Every rank owns three allocations (the mailbox and the arena are exported):

* a **host shard** (pinned host memory, CUDA-VMM ``HOST_NUMA`` when the driver
  supports it): the vocabulary rows of every layer back to back, read only by
  this rank's GPU;
* a small **host mailbox**: the request headers that requesters' GPUs write
  and this rank's owner service polls (the only host memory peers map);
* a **device arena** (one CUDA-VMM ``DEVICE`` allocation): the optional HBM
  mirror of the vocabulary, the FP8 scale table, the per-layer output region,
  the scale output, the per-(layer, owner) done flags, the request inbox that
  requesters fill, and small scratch words.

Row ``x`` of layer ``l`` is owned by rank ``x // n_l`` and stored there as local
row ``x % n_l`` at ``table_bases[l] + x % n_l`` (reference:
``sge_write/csrc/gpu_request.cu:20,103,187-188``, ``runtime.cpp:137-148``).
Output rows of layer ``l`` live at ``output + (l * capacity + at) * row_bytes``
with ``capacity = max_tokens * ept`` (reference ``runtime.cpp:151-156, 519-522``).
"""

from __future__ import annotations

from .utils.math import align

from dataclasses import dataclass, field

import torch

REGION_ALIGN = 4096
ALLOC_ALIGN = 2 << 20
HEADER_BYTES = 64
MAX_RANKS = 64
MAX_LAYERS = 32




@dataclass(frozen=True)
class EngramConfig:
    entries: tuple  # per-rank rows per layer
    hidden: int
    max_tokens: int
    ept: int
    dtype: torch.dtype
    num_sf_packs: int

    @property
    def layers(self) -> int:
        return len(self.entries)

    @property
    def element_bytes(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    @property
    def row_bytes(self) -> int:
        return self.hidden * self.element_bytes

    @property
    def capacity(self) -> int:
        return self.max_tokens * self.ept

    @property
    def table_rows(self) -> int:
        return int(sum(self.entries))

    def table_bases(self):
        out, at = [], 0
        for n in self.entries:
            out.append(at)
            at += n
        return out


def validate_config(entries, hidden, max_tokens, ept, dtype, num_sf_packs, world=None):
    """Check a configuration and return it as an :class:`EngramConfig`.

    Rules follow the reference's WRITE backend (``buffer.py:111-119,151-156``,
    ``runtime.cpp:117-145``): BF16 rows take no scales, FP8 e4m3 rows need at
    least one scale pack, rows are whole 16-byte vectors, and every global row id
    and flat output position fits the 32-bit indices the kernels use.
    """
    entries = tuple(int(n) for n in entries)
    if not entries or min(entries) < 1 or hidden < 1 or max_tokens < 1 or ept < 1:
        raise ValueError("Storage dimensions must be positive")
    if len(entries) > MAX_LAYERS:
        raise ValueError(f"At most {MAX_LAYERS} layers are supported")
    if dtype not in (torch.bfloat16, torch.float8_e4m3fn):
        raise ValueError("Supported vocabulary dtypes: bfloat16 and float8_e4m3fn")
    if (dtype == torch.float8_e4m3fn) != (num_sf_packs > 0):
        raise ValueError("FP8 requires scales; BF16 requires num_sf_packs=0")
    cfg = EngramConfig(entries, int(hidden), int(max_tokens), int(ept), dtype, int(num_sf_packs))
    if cfg.row_bytes % 16:
        raise ValueError("A vocabulary row must be a multiple of 16 bytes")
    if cfg.capacity * cfg.layers >= 2**32:
        raise ValueError("max_tokens * ept * layers must fit in 32 bits")
    if cfg.table_rows >= 2**32:
        raise ValueError("Local vocabulary exceeds 2^32 rows")
    if world is not None:
        if not 1 <= world <= MAX_RANKS:
            raise ValueError(f"World size must be in [1, {MAX_RANKS}]")
        if any(n * world > 2**31 - 1 for n in entries):
            raise ValueError("Global row ids must fit in int32")
    return cfg


@dataclass
class MemoryPlan:
    """Byte offsets of every region, for one rank of a ``world``-rank buffer."""

    config: EngramConfig
    world: int
    mirror: bool
    local_sf: bool
    device: dict = field(default_factory=dict)
    host: dict = field(default_factory=dict)
    device_bytes: int = 0
    host_bytes: int = 0
    table_bytes: int = 0
    mailbox_bytes: int = 0
    sf_bases: list = field(default_factory=list)
    sf_rows_per_layer: list = field(default_factory=list)

    def as_native(self) -> dict:
        """Flat dict handed to the C++ runtime (all ints)."""
        out = {f"dev_{k}": int(v[0]) for k, v in self.device.items()}
        out.update({f"dev_{k}_bytes": int(v[1]) for k, v in self.device.items()})
        out.update({f"host_{k}": int(v[0]) for k, v in self.host.items()})
        out.update({f"host_{k}_bytes": int(v[1]) for k, v in self.host.items()})
        out["device_bytes"] = int(self.device_bytes)
        out["host_bytes"] = int(self.host_bytes)
        out["table_bytes"] = int(self.table_bytes)
        out["mailbox_bytes"] = int(self.mailbox_bytes)
        return out


def dedup_table_slots(config: EngramConfig) -> int:
    """Slots of the request-deduplication table: a power of two >= 2x the requests."""
    need = max(1024, 2 * config.layers * config.capacity)
    return 1 << (need - 1).bit_length()


def plan_memory(config: EngramConfig, world: int, mirror: bool, local_sf: bool, dedup: bool = True,
                hot_rows=None) -> MemoryPlan:
    """Lay out one rank's host shard and device arena.

    ``mirror``: keep an HBM copy of the vocabulary for the peer-HBM route.
    ``hot_rows``: per-layer counts of the global-id prefix replicated on
    every rank (a ``replica`` region of ``sum(hot_rows)`` rows).
    ``local_sf``: every rank holds the full global FP8 scale table
    (``ENGRAM_WRITE_LOCAL_SF=1``); otherwise each rank holds the scales of its own
    rows only (on one NVLink node that is the node-local shard of the reference,
    ``runtime.cpp:114-121``).
    """
    c = config
    L, W, P = c.layers, world, c.num_sf_packs
    plan = MemoryPlan(config=c, world=W, mirror=mirror, local_sf=local_sf)

    sf_rows_per_layer = [n * (W if local_sf else 1) for n in c.entries]
    sf_bases, at = [], 0
    for rows in sf_rows_per_layer:
        sf_bases.append(at)
        at += rows * P
    plan.sf_bases, plan.sf_rows_per_layer = sf_bases, sf_rows_per_layer
    sf_floats = at

    regions = [
        ("mirror", c.table_rows * c.row_bytes if mirror else 0),
        ("sf_table", sf_floats * 4),
        ("output", L * c.capacity * c.row_bytes),
        ("sf_output", L * align(c.max_tokens, 4) * c.ept * P * 4),
        ("done", L * W * 8),
        ("inbox", W * L * c.capacity * 8),
        # dedup: keys[H] u64 + vals[H] u64 + slots[L * capacity] u32
        ("dedup", (dedup_table_slots(c) * 16 + L * c.capacity * 4) if dedup else 0),
        # scratch: epochs[L*W] u64, totals[L*W] u32, cursors[L*W] u32, layer_arrivals[L] u32,
        # serve claim/finish/board [W*L] u64 each, device error record, dedup state,
        # device barrier count u64 + slots[W] u64, alignment slack
        ("scratch", L * W * 8 + L * W * 4 + L * W * 4 + L * 4 + 3 * W * L * 8 + 16 + 8 + W * 8 + 256),
        ("replica", sum(hot_rows or ()) * c.row_bytes),
    ]
    off = 0
    for name, size in regions:
        plan.device[name] = (off, size)
        off = align(off + max(size, 0), REGION_ALIGN)
    plan.device_bytes = align(max(off, REGION_ALIGN), ALLOC_ALIGN)

    # Host memory: the vocabulary shard (read only by this rank's GPU) and, in a
    # separate small allocation that every peer maps, the mailbox headers.
    plan.host["table"] = (0, c.table_rows * c.row_bytes)
    plan.host["headers"] = (0, W * L * HEADER_BYTES)
    plan.table_bytes = align(max(c.table_rows * c.row_bytes, 1), ALLOC_ALIGN)
    plan.mailbox_bytes = align(W * L * HEADER_BYTES, ALLOC_ALIGN)
    plan.host_bytes = plan.table_bytes + plan.mailbox_bytes
    return plan


def hot_rows_for(config: EngramConfig, world: int, spec) -> list:
    """Per-layer replicated prefix lengths from ``ENGRAM_HOT_ROWS``-style input.

    ``spec``: ``None``/``""``/``0`` (off), one count for every layer, or one
    count per layer (comma-separated string or sequence).  Each count is
    clamped to the layer's ``world * n_l`` global rows.
    """
    if spec is None or spec == "":
        values = [0] * config.layers
    elif isinstance(spec, str):
        parts = [int(v) for v in spec.split(",") if v.strip()]
        values = parts * config.layers if len(parts) == 1 else parts
    elif isinstance(spec, int):
        values = [spec] * config.layers
    else:
        values = [int(v) for v in spec]
    if len(values) != config.layers or min(values) < 0:
        raise ValueError("hot rows: give one non-negative count, or one per layer")
    return [min(v, n * world) for v, n in zip(values, config.entries)]


def replica_chunks(hot_rows, capacity: int):
    """Fetch plan that fills a hot-prefix replica: one entry per fetch.

    Each entry is ``(start, counts)``: that fetch requests global ids
    ``[start, start + counts[l])`` of layer ``l`` in its first output rows
    (the rest padding), and those rows go to replica rows ``hot_base[l] +
    start`` onward.
    """
    plan = []
    for start in range(0, max(hot_rows, default=0), capacity):
        plan.append((start, [max(0, min(capacity, hot - start)) for hot in hot_rows]))
    return plan


def storage_size_hint(entries, hidden, max_tokens, ept, dtype, num_sf_packs, world, mirror, local_sf, dedup=True,
                      hot_rows=None):
    cfg = validate_config(entries, hidden, max_tokens, ept, dtype, num_sf_packs, world)
    plan = plan_memory(cfg, world, mirror, local_sf, dedup, hot_rows_for(cfg, world, hot_rows))
    return plan.device_bytes, plan.host_bytes


def sf_strides(tokens: int, ept: int, packs: int, col_major: bool):
    """Strides of one layer's scale output ``[tokens, ept * packs]`` (fp32 units).

    Column-major is TMA aligned: token stride 1, column stride ``align(tokens, 4)``
    (reference ``runtime.cpp:430-432``).  Returns
    ``(token_stride, column_stride, layer_stride)``.
    """
    if col_major:
        hs = align(tokens, 4)
        return 1, hs, hs * ept * packs
    return ept * packs, 1, tokens * ept * packs
