"""The B200 EngramBuffer: sharded embedding-row lookups over NVLink 5 / NVSwitch.

Public API (kept from both reference backends, ``deepep/deep_ep/buffers/engram.py``
and ``sge_write/engram_sge_write/buffer.py``)::

    sizes = EngramBuffer.get_storage_size_hint(group, entries, hidden, max_tokens, ept, dtype, packs)
    config = EngramBuffer.get_theoretical_config(group, len(entries), max_tokens, ept)
    buffer = EngramBuffer(group, *sizes, True, *config, explicitly_destroy=True)
    buffer.set_config(entries, hidden, max_tokens, ept, dtype, packs)   # collective init
    buffer.write(storages, sfs)            # this rank's rows per layer + global FP8 scales
    hooks = buffer.fetch(indices)          # int32 [layers, tokens, ept] on this GPU
    data, scales = hooks[0]()              # FP8: (data, scales); BF16: data
    buffer.destroy()                       # collective

Transport, per (requester, owner) pair, negotiated once at ``set_config``:

* ``peer_hbm`` (``ENGRAM_EGM_ENABLE=1``): every rank keeps an HBM mirror of its
  shard; requesters' SMs load rows from the owner's mirror through NVLink and
  store them at their final output positions in the same kernel that fills
  padding with zeros and gathers the FP8 scales.  Hooks only add stream
  dependencies.
* ``host`` (``ENGRAM_EGM_ENABLE=0`` or a failed probe): rows stay in the
  owner's host-pinned shard.  The requester's dispatch kernel writes
  (row, position) pairs into the owner's HBM inbox and publishes a mailbox
  header in the owner's host memory; the owner's service thread launches a push
  kernel that reads the rows zero-copy and stores them through NVLink into the
  requester's output, then releases a per-(layer, owner) done flag that the
  hook's bounded wait kernel checks.

No NCCL call and no host synchronisation happens in ``fetch`` or the hooks;
``torch.distributed`` is used only for bootstrap and barriers.
"""

from __future__ import annotations

import math
import os
import secrets

import torch
import torch.distributed as dist

from . import _native
from .base import EngramBufferBase, accept_legacy_storage_size
from .layout import hot_rows_for, plan_memory, replica_chunks, storage_size_hint
from .routing import (
    EgmConfig,
    OwnerRoute,
    agree_owner_routes,
    env_flag,
    env_int,
    fabric_identity,
    legacy_route_names,
    node_identity,
    node_layout,
    owner_routes,
    route_names,
)
from .utils.env import describe_knobs

__all__ = ["EngramBuffer", "theoretical_config"]


def theoretical_config(world, num_layers, num_max_tokens, num_entries_per_token, num_max_read_requests_per_qp=16):
    """Recommended ``(channels, depth, restrict)`` for this transport.

    ``channels`` (the reference's ``num_qps``) is the number of 16-CTA groups an
    owner's push kernel may use per request.  A host-route owner reads rows from
    host memory over PCIe: sustaining ~55 GB/s at ~2 us latency needs ~110 KB in
    flight, i.e. ~8 CTAs of 256 threads each holding 4 rows of 256 B per 16
    lanes, so one channel per ~512 KB of expected rows per (requester, owner,
    layer) request, clamped to [1, 16].  ``depth`` bounds the rows of one
    request slot; ``restrict`` is kept for signature compatibility.
    """
    if min(num_layers, num_max_tokens, num_entries_per_token, num_max_read_requests_per_qp) < 1:
        raise ValueError("config dimensions must be positive")
    rows_per_request = num_max_tokens * num_entries_per_token / max(1, world)
    channels = max(1, min(16, math.ceil(rows_per_request * 256 / (512 * 1024))))
    depth = 1024
    while depth < min(32768, num_max_tokens * num_entries_per_token):
        depth *= 2
    return channels, depth, False


def _hot_rows_env() -> str:
    """``ENGRAM_HOT_ROWS``: replicate global ids ``[0, H)`` of each layer on
    every rank (one count, or one per layer, comma-separated; default off).
    Skewed traffic whose hot ids are a low prefix (frequency-ordered
    vocabularies, Zipf over ids) then reads them from local HBM instead of
    the hot owner's NVLink.
    """
    return os.environ.get("ENGRAM_HOT_ROWS", "")


def _gather_kernel() -> str:
    """``ENGRAM_GATHER_KERNEL``: ``auto`` (default), ``simt`` or ``bulk``.

    ``auto`` and ``simt`` run the SIMT gather: every row, local or from a
    peer's HBM mirror, is moved with per-thread vector loads and stores.
    ``bulk`` runs the TMA ring instead, one ``cp.async.bulk`` per row into
    shared memory; for rows on the peer-HBM route those bulk copies read the
    peer's memory, which the default path never does, so it is an opt-in for
    comparison.
    """
    value = os.environ.get("ENGRAM_GATHER_KERNEL", "auto")
    if value not in ("auto", "bulk", "simt"):
        raise ValueError("ENGRAM_GATHER_KERNEL must be 'auto', 'bulk' or 'simt'")
    return value


def _gather_vector() -> int:
    """``ENGRAM_GATHER_VECTOR``: bytes per SIMT load and store, ``auto`` (default), ``32`` or ``16``.

    ``auto`` picks 32-byte (256-bit) accesses when rows come over NVLink and
    16-byte ones when every row is local.  32-byte accesses need rows of 256
    bytes or more in multiples of 32; other row sizes use 16 bytes whatever
    the setting.  Returns 0 for ``auto``.
    """
    value = os.environ.get("ENGRAM_GATHER_VECTOR", "auto")
    if value not in ("auto", "16", "32"):
        raise ValueError("ENGRAM_GATHER_VECTOR must be 'auto', '16' or '32'")
    return 0 if value == "auto" else int(value)


def _peer_transport() -> str:
    """``ENGRAM_PEER_TRANSPORT``: how rows of peer-HBM pairs move, ``pull`` (default) or ``push``.

    ``pull``: the requester's gather loads them from the owner's HBM mirror.
    ``push``: the requester dispatches ``(row, position)`` requests to the
    owner, whose GPU reads its HBM mirror and stores the rows into the
    requester's output (the host route's serving code, with the mirror as the
    source).  Every rank must use the same value.
    """
    value = os.environ.get("ENGRAM_PEER_TRANSPORT", "pull")
    if value not in ("pull", "push"):
        raise ValueError("ENGRAM_PEER_TRANSPORT must be 'pull' or 'push'")
    return value


def _serve_chunk_rows() -> int:
    """``ENGRAM_SERVE_CHUNK_ROWS``: rows per claimed chunk when an owner serves a request (default 512).

    Host-route and pushed requests are split into chunks that the owner's push
    kernels and serving hooks claim one at a time; larger chunks mean fewer
    claims on the request's claim word.  The serving code stages a chunk's
    inbox entries in shared memory, so the value is a multiple of 16 in
    [16, 512].
    """
    value = env_int("ENGRAM_SERVE_CHUNK_ROWS", 512, minimum=16)
    if value > 512 or value % 16:
        raise ValueError("ENGRAM_SERVE_CHUNK_ROWS must be a multiple of 16 in [16, 512]")
    return value


def _dedup_mode() -> int:
    """``ENGRAM_DEDUP``: ``auto`` (default), ``1`` or ``0``.

    Deduplication moves each distinct requested row once per fetch and copies
    repeats locally; ``auto`` enables it while the last measured distinct ratio
    is below 0.75 and re-measures periodically.
    """
    value = os.environ.get("ENGRAM_DEDUP", "auto")
    if value not in ("auto", "0", "1"):
        raise ValueError("ENGRAM_DEDUP must be 'auto', '0' or '1'")
    return {"0": 0, "1": 1, "auto": 2}[value]


class EngramBuffer(EngramBufferBase):
    """Native B200 EngramBuffer (peer-HBM and host-push routes)."""

    impl_name = "native"

    @accept_legacy_storage_size
    def __init__(
        self,
        group,
        num_gpu_bytes,
        num_rdma_storage_bytes,
        use_cpu_rdma_storage=True,
        num_allocated_qps=4,
        qp_depth=1024,
        restrict_rd_atomic=False,
        allow_hybrid_mode=True,
        sl_idx=None,
        num_gpu_timeout_secs=100,
        explicitly_destroy=False,
        **legacy,
    ):
        if legacy:
            raise TypeError(f"Unknown arguments: {', '.join(legacy)}")
        super().__init__(group, explicitly_destroy)
        if not 1 <= num_allocated_qps <= 16 or qp_depth < 32:
            raise ValueError("num_allocated_qps must be in [1, 16] and qp_depth >= 32")
        if num_gpu_timeout_secs <= 0:
            raise ValueError("num_gpu_timeout_secs must be positive")
        if not torch.cuda.is_available():
            raise RuntimeError("EngramBuffer needs a CUDA device; use TorchEngramBuffer on CPU")
        self._C = _native.load()
        self.use_cpu_rdma_storage = bool(use_cpu_rdma_storage)
        # Every rank of a buffer shares one NVLink node here, so "hybrid"
        # (NVLink + RDMA) and pure modes move data the same way; only the
        # reference's rule for the direct route is kept
        # (deepep/deep_ep/buffers/engram.py:87-88).
        self.allow_hybrid_mode = bool(allow_hybrid_mode)
        self.egm = EgmConfig(True) if not self.use_cpu_rdma_storage else EgmConfig.from_env()
        if self.egm.enabled and not self.allow_hybrid_mode:
            raise ValueError("The peer-HBM (EGM) route requires allow_hybrid_mode=True")
        self.local_sf = env_flag("ENGRAM_WRITE_LOCAL_SF", self.egm.enabled)
        self.device = torch.cuda.current_device()
        self.num_gpu_bytes, self.num_rdma_storage_bytes = int(num_gpu_bytes), int(num_rdma_storage_bytes)
        self.num_allocated_qps, self.qp_depth = int(num_allocated_qps), int(qp_depth)
        self.restrict_rd_atomic, self.sl_idx = restrict_rd_atomic, sl_idx
        self.num_gpu_timeout_secs = float(num_gpu_timeout_secs)
        self.runtime = self.context = None
        self.routes = [OwnerRoute.HOST] * self.num_ranks
        self.hot_rows = []  # per-layer replicated id prefixes (ENGRAM_HOT_ROWS), set by set_config
        self.owner_fallback_reasons = [""] * self.num_ranks

        nodes = [None] * self.num_ranks
        self.node_id = node_identity()
        dist.all_gather_object(nodes, self.node_id, group=group)
        self.scaleup_rank_idx, self.num_scaleup_ranks = node_layout(nodes, self.rank_idx)
        self.num_scaleout_ranks = self.num_ranks // self.num_scaleup_ranks
        self.scaleout_rank_idx = self.rank_idx // self.num_scaleup_ranks
        self.num_nvlink_ranks, self.num_rdma_ranks = self.num_scaleup_ranks, self.num_scaleout_ranks
        uuid = torch.cuda.get_device_properties(self.device).uuid
        self.fabric_domain, self.fabric_error = fabric_identity(uuid, self.egm.enabled and self.num_scaleout_ranks > 1)
        self.peer_transport = _peer_transport()
        options = (self.egm.enabled, self.local_sf, self.use_cpu_rdma_storage, self.num_gpu_bytes,
                   self.num_rdma_storage_bytes, self.num_allocated_qps, self.qp_depth, self.peer_transport)
        everyone = [None] * self.num_ranks
        dist.all_gather_object(everyone, options, group=group)
        if any(o != options for o in everyone):
            raise ValueError("All ranks must use identical EngramBuffer options")
        if self.num_scaleout_ranks > 1:
            raise NotImplementedError(
                "the ranks span several nodes; this transport serves one NVLink/NVSwitch node per buffer"
            )

    # ------------------------------------------------------------ static helpers
    @staticmethod
    def get_storage_size_hint(group, num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token,
                              dtype=torch.bfloat16, num_sf_packs=0):
        """``(device_bytes, host_bytes)`` this rank needs for the configuration.

        Depends on ``ENGRAM_EGM_ENABLE`` (an HBM mirror of the shard is added),
        ``ENGRAM_WRITE_LOCAL_SF`` (full vs. own-rows scale table) and
        ``ENGRAM_HOT_ROWS`` (a replica of each layer's hot id prefix).
        """
        egm = EgmConfig.from_env().enabled
        return storage_size_hint(num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token, dtype,
                                 num_sf_packs, group.size(), egm, env_flag("ENGRAM_WRITE_LOCAL_SF", egm),
                                 _dedup_mode() != 0, _hot_rows_env())

    @staticmethod
    def get_theoretical_config(group, num_layers, num_max_tokens, num_entries_per_token,
                               num_max_read_requests_per_qp=16):
        return theoretical_config(group.size(), num_layers, num_max_tokens, num_entries_per_token,
                                  num_max_read_requests_per_qp)

    # ------------------------------------------------------------------ config
    def set_config(self, num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token,
                   dtype=torch.bfloat16, num_sf_packs=0):
        """Collective initialisation: allocate, exchange, probe, agree, commit."""
        if self._destroyed:
            raise RuntimeError("Buffer is destroyed")
        cfg = self._check_config_args(num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token, dtype,
                                      num_sf_packs)
        self.hot_rows = hot_rows_for(cfg, self.num_ranks, _hot_rows_env())
        plan = plan_memory(cfg, self.num_ranks, self.egm.enabled, self.local_sf, _dedup_mode() != 0, self.hot_rows)
        if plan.device_bytes > self.num_gpu_bytes or plan.host_bytes > self.num_rdma_storage_bytes:
            raise ValueError("Insufficient capacity: use EngramBuffer.get_storage_size_hint")
        tokens = [None] * self.num_ranks
        dist.all_gather_object(tokens, secrets.token_hex(8), group=self.group)
        native_cfg = dict(
            rank=self.rank_idx, world=self.num_ranks, local_rank=self.scaleup_rank_idx,
            local_size=self.num_scaleup_ranks, device=self.device, entries=list(cfg.entries), hidden=cfg.hidden,
            element_bytes=cfg.element_bytes, max_tokens=cfg.max_tokens, ept=cfg.ept, packs=cfg.num_sf_packs,
            channels=self.num_allocated_qps, egm=self.egm.enabled, local_sf=self.local_sf,
            timeout_s=self.num_gpu_timeout_secs, token=tokens[0],
            allow_host_vmm=env_flag("ENGRAM_HOST_VMM", True), plan=plan.as_native(),
            gather_kernel=_gather_kernel(),
            gather_ctas_per_sm=env_int("ENGRAM_GATHER_CTAS_PER_SM", 0, minimum=0),
            gather_unroll=env_int("ENGRAM_GATHER_UNROLL", 0, minimum=0),
            gather_strided=env_int("ENGRAM_GATHER_STRIDED", 0, minimum=0),
            gather_vector=_gather_vector(),
            peer_transport=self.peer_transport,
            gather_l2_prefetch=env_flag("ENGRAM_GATHER_L2_PREFETCH", False),
            serve_chunk_rows=_serve_chunk_rows(),
            dedup=_dedup_mode(),
            nvtx=env_flag("ENGRAM_NVTX", False),
            hot_rows=list(self.hot_rows),
            index_staging=env_flag("ENGRAM_INDEX_STAGING", True),
        )
        native = None
        with torch.cuda.device(self.device):
            try:
                native = self._C.Runtime(native_cfg)
                boot = dict(native.bootstrap(), node=self.node_id, fabric_domain=self.fabric_domain,
                            fabric_probe_error=self.fabric_error)
            except Exception as error:  # reported collectively below
                boot = {"error": str(error)}
            peers = [None] * self.num_ranks
            dist.all_gather_object(peers, boot, group=self.group)
            failures = [f"rank {r}: {p['error']}" for r, p in enumerate(peers) if "error" in p]
            if failures:
                if native is not None:
                    native.close()
                raise RuntimeError(f"EngramBuffer initialization failed: {failures[0]}")
            if any(p["config"] != boot["config"] for p in peers):
                native.close()
                raise ValueError("All ranks must use identical EngramBuffer configurations")
            try:
                candidates = owner_routes(peers, self.rank_idx, self.egm)
                try:
                    report = dict(native.probe_routes(peers, [int(c) for c in candidates]))
                except Exception as error:
                    report = {"error": str(error)}
                reports = self._exchange(report, "probe")
                routes, reasons = agree_owner_routes(reports, self.rank_idx)
                try:
                    if not self.use_cpu_rdma_storage and any(
                        int(r) == OwnerRoute.HOST for p, r in enumerate(routes) if p != self.rank_idx
                    ):
                        raise RuntimeError("HBM-resident vocabulary needs the peer_hbm route to every owner")
                    native.prepare_routes([int(r) for r in routes])
                    report = {}
                except Exception as error:
                    report = {"error": str(error)}
                self._exchange(report, "commit")
                try:
                    native.connect()
                    report = {}
                except Exception as error:
                    report = {"error": str(error)}
                self._exchange(report, "connect")  # every rank raises if one could not start serving
            except Exception:
                native.close()
                raise
            self.routes, self.owner_fallback_reasons = routes, reasons
            self.runtime = self.context = native
            self._config, self._plan = cfg, plan
            self._configured = True
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)

    def _exchange(self, report, phase):
        reports = [None] * self.num_ranks
        dist.all_gather_object(reports, report, group=self.group)
        failures = [f"rank {r}: {item['error']}" for r, item in enumerate(reports) if "error" in item]
        if failures:
            raise RuntimeError(f"EngramBuffer route {phase} failed: {failures[0]}")
        return reports

    # ------------------------------------------------------------------- write
    def write(self, storages, sfs=None):
        """Collective: load this rank's rows per layer and the global scales.

        ``storages[l]``: ``[n_l, hidden]`` (CPU or this GPU).  ``sfs[l]``:
        ``[world * n_l, num_sf_packs]`` fp32 for FP8 (identical on every rank).
        """
        self._check_write_args(storages, sfs, self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for layer, storage in enumerate(storages):
            sf = sfs[layer] if self._config.num_sf_packs else None
            self.runtime.write(layer, storage, sf)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._written = True
        if any(self.hot_rows):
            self._refresh_replica()
            dist.barrier(group=self.group)

    def _read_layer(self, layer):
        rows, scales = self.runtime.read_layer(layer)
        return rows, scales

    def _refresh_replica(self):
        """Fill this rank's replica of the hot id prefixes from the owners.

        The replica is switched off, then ids ``[0, hot_rows[l])`` are fetched
        through the ordinary routes in capacity-sized chunks and copied into
        the replica; then reads of those ids go local.  Runs inside write()
        (every rank at once), so the owners' data is final.
        """
        c = self._config
        rt = self.runtime
        rt.set_hot_active(False)
        replica = rt.replica_view()
        bases = [sum(self.hot_rows[:l]) for l in range(c.layers)]
        dev = replica.device  # the fill's requests live where the replica does
        with torch.cuda.device(self.device):
            for start, counts in replica_chunks(self.hot_rows, c.capacity):
                idx = torch.full((c.layers, c.max_tokens, c.ept), -1, dtype=torch.int32, device=dev)
                flat = idx.view(c.layers, -1)
                for layer, n in enumerate(counts):
                    if n:
                        flat[layer, :n] = torch.arange(start, start + n, dtype=torch.int32, device=dev)
                outs = [h() for h in self.fetch(idx)]
                for layer, n in enumerate(counts):
                    if n:
                        data = outs[layer][0] if c.num_sf_packs else outs[layer]
                        rows = data.view(torch.uint8).reshape(-1, c.row_bytes)[:n]
                        replica[bases[layer] + start: bases[layer] + start + n].copy_(rows)
            torch.cuda.synchronize()
        rt.check_health()  # a failed fill raises here instead of serving a broken replica
        rt.set_hot_active(True)

    # ------------------------------------------------------------------- fetch
    def fetch(self, indices, num_qps=0, use_tma_aligned_col_major_sf=True):
        """Submit every layer's lookup on the current stream; return one hook per layer.

        ``indices`` is int32 [layers, tokens, ept] on this GPU, or in pinned
        host memory: then the runtime copies it on its own side stream into
        one of two device slots, so the next step's copy overlaps this step's
        lookup (``ENGRAM_INDEX_STAGING=0``: the kernels read it in place over
        PCIe; under CUDA graph capture they always do), and the caller keeps it
        unchanged until the hooks' work is done, as with any non-blocking copy.
        ``num_qps`` selects how many push channels host-route owners may use
        (0 = all allocated).  ``use_tma_aligned_col_major_sf`` selects the
        column-major, 4-aligned scale layout (default) or row-major.
        """
        self._check_fetch_args(indices, self.device, require_cuda=True, allow_pinned=True)
        qps = num_qps or self.num_allocated_qps
        if not 1 <= qps <= self.num_allocated_qps:
            raise ValueError("num_qps exceeds the allocated channels")
        generation = self._begin_fetch()
        try:
            # The runtime records `indices` on the current stream for the allocator.
            outputs = self.runtime.fetch(indices, qps, bool(use_tma_aligned_col_major_sf))
        except Exception:
            self._pending = set()
            raise
        self._input = indices
        return self._make_hooks(generation, self.runtime.wait_layer, outputs)

    def fetch_all(self, indices, num_qps=0, use_tma_aligned_col_major_sf=True):
        """``fetch(indices)`` and every layer's hook in one native call.

        Returns the per-layer outputs (``data`` or ``(data, scales)``), ready
        on the current stream like the hooks' return values.  For callers that
        consume all layers at once it saves the host cost of one hook call per
        layer; no hook is left outstanding.
        """
        self._check_fetch_args(indices, self.device, require_cuda=True, allow_pinned=True)
        qps = num_qps or self.num_allocated_qps
        if not 1 <= qps <= self.num_allocated_qps:
            raise ValueError("num_qps exceeds the allocated channels")
        self._generation += 1  # hooks of earlier fetches are superseded
        outputs = self.runtime.fetch_all(indices, qps, bool(use_tma_aligned_col_major_sf))
        self._input = indices
        return list(outputs)

    def pinned_indices(self, tokens: int, write_combined: bool = True) -> torch.Tensor:
        """An int32 host tensor ``[layers, tokens, ept]`` for ``fetch`` / ``fetch_all`` inputs.

        Page-locked and mapped into the GPU's address space, so a fetch copies
        it (``ENGRAM_INDEX_STAGING=1``) or reads it in place without a bounce
        through pageable memory.  With ``write_combined`` (the default) the
        pages are write-combined: the host writes them without filling its
        caches and the GPU reads them over PCIe without snooping the CPU's
        caches, which suits indices the host writes every step.  Fill it with
        sequential writes (``copy_``, numpy assignment); reading it back on the
        CPU is slow (uncached).  The memory is freed with the tensor.
        """
        self._ready()
        cfg = self._config
        if not write_combined:
            return super().pinned_indices(tokens, False)
        if not 0 <= tokens <= cfg.max_tokens:
            raise ValueError(f"tokens must be in [0, {cfg.max_tokens}]")
        count = cfg.layers * tokens * cfg.ept
        raw = self._C.alloc_pinned(max(count, 1) * 4, True)
        return raw.view(torch.int32)[:count].view(cfg.layers, tokens, cfg.ept)

    def device_barrier(self):
        """Enqueue a device barrier over every rank of the group on the current stream.

        One warp per GPU stores its barrier count into every peer's arena and
        waits (bounded by ``num_gpu_timeout_secs``) until every peer's count
        arrived; work each rank enqueued before it is visible to every rank's
        work after it.  Every rank must call it the same number of times.  It
        can be captured into a CUDA graph (the counts live in device memory).
        A timeout is reported like any device error and leaves the barrier
        unusable until the buffer is rebuilt.  Reference: the NVLink barrier
        of ``deepep/deep_ep/include/deep_ep/comm/barrier.cuh:88-131``.
        """
        self._ready()
        self.runtime.barrier()

    # -------------------------------------------------------------- inspection
    def get_route_info(self):
        self._ready()
        return dict(
            egm_enabled=self.egm.enabled,
            owner_routes=route_names(self.routes),
            owner_routes_legacy=legacy_route_names(self.routes),
            owner_fallback_reasons=list(self.owner_fallback_reasons),
            fabric_domain=self.fabric_domain,
            fabric_probe_error=self.fabric_error,
            transport="nvlink peer loads / owner push",
            knobs=describe_knobs(),
            memory=self.runtime.memory_usage(),
        )

    def memory_usage(self):
        self._ready()
        return self.runtime.memory_usage()

    def print_memory_usage(self):
        self._ready()
        print(self.runtime.memory_usage(), flush=True)

    def error_state(self):
        self._ready()
        return self.runtime.error_state()

    def get_physical_domain_size(self):
        return self.num_rdma_ranks, self.num_nvlink_ranks

    def get_logical_domain_size(self):
        return self.num_scaleout_ranks, self.num_scaleup_ranks

    def destroy(self):
        """Collective teardown; every outstanding hook must have been called."""
        self._check_destroy()
        if self._destroyed:
            return
        if self.runtime is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.runtime.close()
            dist.barrier(group=self.group)
        self.runtime = self.context = None
        self._input = None
        self._destroyed = True
