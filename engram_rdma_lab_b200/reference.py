"""Pure-torch EngramBuffer: the correctness oracle and the NCCL baseline.

Same public API as :class:`engram_rdma_lab_b200.EngramBuffer`, built only from
torch tensor ops and ``torch.distributed`` collectives:

1. bucket every requested row by owner (``x // n_l``) with a counting
   placement, padding last;
2. ``all_to_all_single`` of per-owner counts, then of ``(layer, local_row)``
   requests;
3. each owner gathers the requested rows and FP8 scales from its shard into
   one payload per row;
4. one ``all_to_all_single`` of those payloads back;
5. scatter into the per-layer output region; padding rows and scales are zero.

On CPU with a ``gloo`` group it is the oracle of the unit tests.  On GPUs with
an ``nccl`` group it is the "NCCL all_to_all" baseline the fused kernels are
measured against.  The baseline has to read the counts back to the host to size
the exchange, so every fetch synchronises the host once (one read of the sent
and received counts); the native buffer never does.  Reference semantics reproduced: ``sge_write/engram_sge_write/buffer.py``
(API, validation, hook generations), ``sge_write/csrc/runtime.cpp:389-535``
(storage, scale sharding, output and scale layouts).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .base import EngramBufferBase, accept_legacy_storage_size
from .layout import plan_memory, sf_strides, storage_size_hint
from .routing import EgmConfig, env_flag, node_identity, node_layout, route_names, legacy_route_names, OwnerRoute


def _group_device(group, device):
    if device is not None:
        return torch.device(device)
    backend = dist.get_backend(group)
    if backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


class TorchEngramBuffer(EngramBufferBase):
    """EngramBuffer implemented with torch collectives (oracle / baseline)."""

    impl_name = "torch"

    @accept_legacy_storage_size
    def __init__(
        self,
        group,
        num_gpu_bytes,
        num_rdma_storage_bytes,
        use_cpu_rdma_storage=True,
        num_allocated_qps=1,
        qp_depth=1024,
        restrict_rd_atomic=False,
        allow_hybrid_mode=True,
        sl_idx=None,
        num_gpu_timeout_secs=100,
        explicitly_destroy=False,
        device=None,
    ):
        super().__init__(group, explicitly_destroy)
        if not 1 <= num_allocated_qps <= 16 or qp_depth < 32:
            raise ValueError("num_allocated_qps must be in [1, 16] and qp_depth >= 32")
        self.egm = EgmConfig.from_env()
        self.local_sf = env_flag("ENGRAM_WRITE_LOCAL_SF", self.egm.enabled)
        self.device = _group_device(group, device)
        self.num_gpu_bytes, self.num_rdma_storage_bytes = int(num_gpu_bytes), int(num_rdma_storage_bytes)
        self.use_cpu_rdma_storage = bool(use_cpu_rdma_storage)
        self.allow_hybrid_mode = bool(allow_hybrid_mode)
        if self.egm.enabled and not self.allow_hybrid_mode:
            raise ValueError("The peer-HBM (EGM) route requires allow_hybrid_mode=True")
        self.num_allocated_qps, self.qp_depth = int(num_allocated_qps), int(qp_depth)
        self.restrict_rd_atomic, self.sl_idx = restrict_rd_atomic, sl_idx
        self.num_gpu_timeout_secs = num_gpu_timeout_secs
        nodes = [None] * self.num_ranks
        dist.all_gather_object(nodes, node_identity(), group=group)
        self.scaleup_rank_idx, self.num_scaleup_ranks = node_layout(nodes, self.rank_idx)
        self.num_scaleout_ranks = self.num_ranks // self.num_scaleup_ranks
        self.scaleout_rank_idx = self.rank_idx // self.num_scaleup_ranks
        self.runtime = self

    # ------------------------------------------------------------ static helpers
    @staticmethod
    def get_storage_size_hint(
        group, num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token, dtype=torch.bfloat16,
        num_sf_packs=0,
    ):
        egm = EgmConfig.from_env().enabled
        return storage_size_hint(
            num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token, dtype, num_sf_packs,
            group.size(), egm, env_flag("ENGRAM_WRITE_LOCAL_SF", egm),
        )

    @staticmethod
    def get_theoretical_config(group, num_layers, num_max_tokens, num_entries_per_token,
                               num_max_read_requests_per_qp=16):
        from .buffer import theoretical_config

        return theoretical_config(group.size(), num_layers, num_max_tokens, num_entries_per_token,
                                  num_max_read_requests_per_qp)

    # ------------------------------------------------------------------ config
    def set_config(self, num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token,
                   dtype=torch.bfloat16, num_sf_packs=0):
        cfg = self._check_config_args(num_entries_per_layer, hidden, num_max_tokens, num_entries_per_token, dtype,
                                      num_sf_packs)
        plan = plan_memory(cfg, self.num_ranks, self.egm.enabled, self.local_sf)
        if plan.device_bytes > self.num_gpu_bytes or plan.host_bytes > self.num_rdma_storage_bytes:
            raise ValueError("Insufficient capacity: use get_storage_size_hint")
        mine = (tuple(cfg.entries), cfg.hidden, cfg.max_tokens, cfg.ept, str(cfg.dtype), cfg.num_sf_packs,
                self.egm.enabled, self.local_sf)
        everyone = [None] * self.num_ranks
        dist.all_gather_object(everyone, mine, group=self.group)
        if any(other != mine for other in everyone):
            raise ValueError("All ranks must use identical configurations")
        self._config, self._plan = cfg, plan
        dev = self.device
        self._table = torch.zeros(cfg.table_rows, cfg.row_bytes, dtype=torch.uint8, device=dev)
        self._table_bases = torch.tensor(cfg.table_bases(), dtype=torch.int64, device=dev)
        self._entries_t = torch.tensor(cfg.entries, dtype=torch.int64, device=dev)
        P = cfg.num_sf_packs
        total_sf = sum(plan.sf_rows_per_layer)
        self._sf_table = torch.zeros(max(total_sf, 1), max(P, 1), dtype=torch.float32, device=dev)
        self._sf_bases = torch.tensor([b // max(P, 1) for b in plan.sf_bases], dtype=torch.int64, device=dev)
        self._output = torch.zeros(cfg.layers, cfg.capacity, cfg.row_bytes, dtype=torch.uint8, device=dev)
        self._sf_output = torch.zeros(max(plan.device["sf_output"][1] // 4, 1), dtype=torch.float32, device=dev)
        self.routes = [OwnerRoute.PEER_HBM if self.egm.enabled else OwnerRoute.HOST] * self.num_ranks
        self.owner_fallback_reasons = [""] * self.num_ranks
        self._marks = [torch.cuda.Event(enable_timing=True) for _ in range(6)] if dev.type == "cuda" else None
        self._last_exchange = None
        self._configured = True
        dist.barrier(group=self.group)

    def write(self, storages, sfs=None):
        dev_index = self.device.index if self.device.type == "cuda" else None
        self._check_write_args(storages, sfs, dev_index)
        c = self._config
        dist.barrier(group=self.group)
        bases = c.table_bases()
        for layer, n in enumerate(c.entries):
            src = storages[layer].reshape(n, c.hidden).view(torch.uint8).reshape(n, c.row_bytes)
            self._table[bases[layer]:bases[layer] + n].copy_(src)
            if c.num_sf_packs:
                sf = sfs[layer]
                rows = self._plan.sf_rows_per_layer[layer]
                start = 0 if self.local_sf else self.rank_idx * n
                base = self._plan.sf_bases[layer] // c.num_sf_packs
                self._sf_table[base:base + rows].copy_(sf[start:start + rows])
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._written = True

    def _read_layer(self, layer):
        c = self._config
        base, n = c.table_bases()[layer], c.entries[layer]
        rows = self._table[base:base + n].cpu()
        if not c.num_sf_packs:
            return rows, None
        sf_base = self._plan.sf_bases[layer] // c.num_sf_packs
        return rows, self._sf_table[sf_base:sf_base + self._plan.sf_rows_per_layer[layer]].cpu()

    # ------------------------------------------------------------------- fetch
    def fetch(self, indices, num_qps=0, use_tma_aligned_col_major_sf=True):
        """Exchange requests and rows with all_to_all; returns one hook per layer.

        On a CUDA device, pinned host indices are accepted like the native
        buffer accepts them; here they are copied to the device without
        blocking (a copy-engine H2D on the current stream).
        """
        on_cuda = self.device.type == "cuda"
        dev_index = self.device.index if on_cuda else None
        self._check_fetch_args(indices, dev_index, require_cuda=on_cuda, allow_pinned=on_cuda)
        if not on_cuda and indices.device.type != "cpu":
            raise ValueError("indices must live on the buffer's device")
        if on_cuda and indices.device.type == "cpu":
            indices = indices.to(self.device, non_blocking=True)
        qps = num_qps or self.num_allocated_qps
        if not 1 <= qps <= self.num_allocated_qps:
            raise ValueError("num_qps exceeds the allocated channels")
        generation = self._begin_fetch()
        self._input = indices
        outputs = self._exchange(indices, use_tma_aligned_col_major_sf)
        return self._make_hooks(generation, lambda layer: None, outputs)

    def _exchange(self, indices, col_major):
        """One fetch as three ``all_to_all_single`` calls with a single host sync.

        1. Bucket the requests by owner with a counting placement: a running
           count per owner gives each request its slot inside its owner's
           bucket, so no sort runs.
        2. Exchange the per-owner counts (device), then read sent and received
           counts back together: the only host sync, needed to size the
           variable splits.
        3. Exchange the ``(layer << 32) | local_row`` requests.
        4. Each owner gathers rows (``index_select``) and appends the FP8
           scale words to each row, so one exchange returns both.
        5. The requester scatters rows and scales to their positions with
           ``index_copy_``; padding stays zero.

        On a CUDA device every phase is bracketed by events; ``phase_ms()``
        reads them (it synchronises) to separate the row exchange from the
        bookkeeping around it.
        """
        c, W, dev = self._config, self.num_ranks, self.device
        L, T, E = indices.shape
        P, R = c.num_sf_packs, c.row_bytes
        rows = T * E
        N = L * rows
        marks = self._marks if dev.type == "cuda" else None
        if marks is not None:
            marks[0].record()
        x = indices.reshape(N).to(torch.int64)
        layer = torch.arange(N, device=dev, dtype=torch.int64) // max(rows, 1)
        n = self._entries_t.index_select(0, layer)
        valid = x >= 0
        owner = torch.where(valid, torch.div(x.clamp_min(0), n, rounding_mode="floor"), torch.full_like(x, W))
        bad = (owner > W) | (valid & (owner >= W))
        owner = owner.clamp_max(W)  # padding (and ids past the vocabulary) go to bucket W, never sent
        counts = torch.bincount(owner, minlength=W + 1)
        offsets = torch.cumsum(counts, 0) - counts
        # Running count of each owner along the requests: one row per owner,
        # scanned along its innermost dimension (a scan down the outer one
        # would run one thread per owner).
        hits = owner[None, :] == torch.arange(W + 1, device=dev, dtype=torch.int64)[:, None]
        running = hits.cumsum(1, dtype=torch.int32)
        slot = offsets.index_select(0, owner) + running.gather(0, owner[None, :]).squeeze(0).to(torch.int64) - 1
        request = torch.empty(N, dtype=torch.int64, device=dev)
        request.index_copy_(0, slot, (layer << 32) | torch.where(valid, x.clamp_min(0) % n, torch.zeros_like(x)))
        position_of_slot = torch.empty(N, dtype=torch.int64, device=dev)
        position_of_slot.index_copy_(0, slot, torch.arange(N, device=dev, dtype=torch.int64))
        send_counts = counts[:W].contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        meta = torch.cat([send_counts, recv_counts, bad.sum().view(1)]).tolist()  # the one host sync
        send_split, recv_split = meta[:W], meta[W:2 * W]
        if meta[-1]:
            raise ValueError("index outside the global vocabulary")
        total = sum(send_split)
        if marks is not None:
            marks[1].record()
        incoming = torch.empty(sum(recv_split), dtype=torch.int64, device=dev)
        dist.all_to_all_single(incoming, request[:total], recv_split, send_split, group=self.group)
        if marks is not None:
            marks[2].record()

        # Owner side: rows (and scale words) of this rank's shard, one payload per request.
        in_layer, in_row = incoming >> 32, incoming & 0xFFFFFFFF
        served = self._table.index_select(0, self._table_bases.index_select(0, in_layer) + in_row)
        if P:
            sf_off = self._entries_t.index_select(0, in_layer) * self.rank_idx if self.local_sf else 0
            sf_at = self._sf_bases.index_select(0, in_layer) + sf_off + in_row
            served_sf = self._sf_table.index_select(0, sf_at)[:, :P].contiguous().view(torch.uint8)
            served = torch.cat([served, served_sf], dim=1)
        answer = torch.empty(total, served.shape[1], dtype=torch.uint8, device=dev)
        if marks is not None:
            marks[3].record()
        dist.all_to_all_single(answer, served, send_split, recv_split, group=self.group)
        if marks is not None:
            marks[4].record()

        # Requester side: scatter into the output region; padding stays zero.
        positions = position_of_slot[:total]
        dst = (positions // max(rows, 1)) * c.capacity + positions % max(rows, 1)
        self._output[:, :rows].zero_()
        self._output.view(L * c.capacity, R).index_copy_(0, dst, answer[:, :R])
        results = []
        if P:
            ts, hs, ls = sf_strides(T, E, P, col_major)
            sf_rows = torch.zeros(N, P, dtype=torch.float32, device=dev)
            sf_rows.index_copy_(0, positions, answer[:, R:].contiguous().view(torch.float32))
            for lyr in range(L):
                view = self._sf_output.as_strided((T, E * P), (ts, hs), lyr * ls)
                view.copy_(sf_rows[lyr * rows:(lyr + 1) * rows].reshape(T, E * P))
        for lyr in range(L):
            data = self._output[lyr, :rows].view(c.dtype).reshape(T, E * c.hidden)
            if P:
                ts, hs, ls = sf_strides(T, E, P, col_major)
                results.append((data, self._sf_output.as_strided((T, E * P), (ts, hs), lyr * ls)))
            else:
                results.append(data)
        if marks is not None:
            marks[5].record()
            self._last_exchange = dict(rows_sent=total, payload_bytes=int(served.shape[1]))
        return results

    def phase_ms(self):
        """Device time of the last fetch's phases (CUDA only; synchronises).

        ``bookkeeping_ms``: bucketing, the count exchange and its host read;
        ``requests_ms``: the request exchange; ``serve_ms``: the owner's row
        and scale gather; ``rows_all_to_all_ms``: the row + scale exchange;
        ``scatter_ms``: placing rows and scales at their positions.
        ``rows_all_to_all_gbs``: payload bytes this rank received over that
        exchange's time.
        """
        if self.device.type != "cuda" or self._last_exchange is None:
            return None
        m = self._marks
        m[5].synchronize()
        spans = [m[i].elapsed_time(m[i + 1]) for i in range(5)]
        names = ["bookkeeping_ms", "requests_ms", "serve_ms", "rows_all_to_all_ms", "scatter_ms"]
        out = {k: round(v, 4) for k, v in zip(names, spans)}
        received = self._last_exchange["rows_sent"] * self._last_exchange["payload_bytes"]
        out["rows_all_to_all_gbs"] = round(received / (spans[3] * 1e-3) / 1e9, 2) if spans[3] > 0 else None
        out["payload_bytes_per_row"] = self._last_exchange["payload_bytes"]
        return out

    def device_barrier(self):
        """A barrier ordered on the current stream: an all-reduce of one word over the group."""
        self._ready()
        token = torch.zeros(1, device=self.device)
        dist.all_reduce(token, group=self.group)

    # -------------------------------------------------------------- inspection
    def get_route_info(self):
        self._ready()
        return dict(
            egm_enabled=self.egm.enabled,
            owner_routes=route_names(self.routes),
            owner_routes_legacy=legacy_route_names(self.routes),
            owner_fallback_reasons=list(self.owner_fallback_reasons),
            fabric_domain=None,
            fabric_probe_error="disabled",
            transport="torch.distributed all_to_all",
            memory=self.memory_usage(),
        )

    def memory_usage(self):
        c = self._config
        return dict(
            rank=self.rank_idx,
            impl=self.impl_name,
            device_bytes=self._plan.device_bytes,
            host_bytes=self._plan.host_bytes,
            cpu_vocabulary_bytes=c.table_rows * c.row_bytes,
            local_sf=self.local_sf,
            egm_enabled=self.egm.enabled,
        )

    def print_memory_usage(self):
        self._ready()
        print(self.memory_usage(), flush=True)

    def get_physical_domain_size(self):
        return self.num_scaleout_ranks, self.num_scaleup_ranks

    def get_logical_domain_size(self):
        return self.num_scaleout_ranks, self.num_scaleup_ranks

    def destroy(self):
        self._check_destroy()
        if self._destroyed:
            return
        if self._configured:
            if self.device.type == "cuda":
                torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
        self._destroyed = True
        self._input = None
        self._table = self._output = self._sf_table = self._sf_output = None
