"""Lifecycle and argument checks shared by every EngramBuffer implementation.

The public contract (reference ``sge_write/engram_sge_write/buffer.py:39-352``
and ``deepep/deep_ep/buffers/engram.py:42-297``):

* construction, ``set_config``, ``write`` and ``destroy`` are collective over the
  group;
* ``fetch(indices)`` submits every layer's lookup on the current CUDA stream and
  returns one hook per layer; a hook submits that layer's wait on the stream
  current at hook time and returns the layer's output view (``data`` for BF16,
  ``(data, scales)`` for FP8);
* one fetch is outstanding at a time: a second ``fetch`` before every hook was
  called raises, and a hook of a superseded fetch raises;
* ``destroy`` requires ``explicitly_destroy=True`` and no outstanding hooks.
"""

from __future__ import annotations

import functools
import warnings
from abc import ABC, abstractmethod

import torch
import torch.distributed as dist

from .layout import EngramConfig, validate_config


def accept_legacy_storage_size(init):
    """Accept the reference's older ``num_rdma_storage_size`` keyword."""

    @functools.wraps(init)
    def wrapped(self, *args, **kwargs):
        if "num_rdma_storage_size" in kwargs:
            if "num_rdma_storage_bytes" in kwargs:
                raise TypeError("Specify only one of num_rdma_storage_bytes and num_rdma_storage_size")
            kwargs["num_rdma_storage_bytes"] = kwargs.pop("num_rdma_storage_size")
        return init(self, *args, **kwargs)

    return wrapped


class EngramBufferBase(ABC):
    """Host-side state machine common to the native and the torch buffers."""

    impl_name = "base"

    def __init__(self, group, explicitly_destroy: bool):
        self.group = group
        self.rank_idx = group.rank()
        self.num_ranks = group.size()
        self.explicitly_destroy = explicitly_destroy
        self._config: EngramConfig | None = None
        self._configured = False
        self._written = False
        self._generation = 0
        self._pending: set = set()
        self._input = None
        self._destroyed = False

    # -------------------------------------------------------------- checkpoint
    STATE_FORMAT = 1

    @abstractmethod
    def _read_layer(self, layer: int):
        """``(rows uint8 [n_l, row_bytes], stored scales fp32 [rows, packs] | None)`` on the CPU."""

    def state_dict(self) -> dict:
        """This rank's vocabulary shard and scales, on the CPU, for a checkpoint.

        Not collective.  ``storages[l]`` is ``[n_l, hidden]`` in the table
        dtype and ``sfs[l]`` the global-shaped ``[world * n_l, packs]`` scale
        table ``write()`` takes (rows this rank does not store are zero when
        ``ENGRAM_WRITE_LOCAL_SF=0``).  The reference has no checkpoint path;
        ``write()`` is its only loader, and ``load_state_dict`` calls it.
        """
        self._ready()
        if not self._written:
            raise RuntimeError("write() must initialize the vocabulary before state_dict()")
        if self._pending:
            raise RuntimeError("Call all outstanding hooks before state_dict()")
        c = self._config
        storages, sfs = [], []
        for layer, n in enumerate(c.entries):
            rows, stored = self._read_layer(layer)
            storages.append(rows.reshape(n, c.row_bytes).view(c.dtype).reshape(n, c.hidden))
            if c.num_sf_packs:
                if stored.shape[0] == self.num_ranks * n:
                    sfs.append(stored.reshape(self.num_ranks * n, c.num_sf_packs))
                else:
                    full = torch.zeros(self.num_ranks * n, c.num_sf_packs, dtype=torch.float32)
                    full[self.rank_idx * n:(self.rank_idx + 1) * n] = stored.reshape(n, c.num_sf_packs)
                    sfs.append(full)
        return dict(
            format=self.STATE_FORMAT, rank=self.rank_idx, world=self.num_ranks,
            config=dict(entries=list(c.entries), hidden=c.hidden, dtype=str(c.dtype), num_sf_packs=c.num_sf_packs),
            storages=storages, sfs=sfs if c.num_sf_packs else None,
        )

    def load_state_dict(self, state: dict):
        """Collective: restore a ``state_dict()`` of the same rank and table shape via ``write()``."""
        self._ready()
        c = self._config
        want = dict(entries=list(c.entries), hidden=c.hidden, dtype=str(c.dtype), num_sf_packs=c.num_sf_packs)
        if state.get("format") != self.STATE_FORMAT:
            raise ValueError("Unknown Engram state format")
        if state.get("rank") != self.rank_idx or state.get("world") != self.num_ranks:
            raise ValueError("State belongs to another rank or world size")
        if state.get("config") != want:
            raise ValueError(f"State table shape {state.get('config')} does not match {want}")
        self.write(state["storages"], state["sfs"])

    # ------------------------------------------------------------------ checks
    def _ready(self):
        if self._destroyed or not self._configured:
            raise RuntimeError("Buffer is unconfigured or destroyed")

    def _check_config_args(self, entries, hidden, max_tokens, ept, dtype, num_sf_packs) -> EngramConfig:
        if self._configured:
            raise RuntimeError("set_config is initialization-only; create a new Buffer to reconfigure")
        return validate_config(entries, hidden, max_tokens, ept, dtype, num_sf_packs, self.num_ranks)

    def _check_write_args(self, storages, sfs, device_index):
        self._ready()
        if self._pending:
            raise RuntimeError("Call all outstanding hooks before replacing vocabulary contents")
        c = self._config
        if len(storages) != c.layers or (c.num_sf_packs and (sfs is None or len(sfs) != c.layers)):
            raise ValueError("One storage/scales tensor is required per layer")
        for layer, (storage, n) in enumerate(zip(storages, c.entries)):
            if tuple(storage.shape) != (n, c.hidden) or storage.dtype != c.dtype or not storage.is_contiguous():
                raise ValueError(f"Invalid vocabulary tensor for layer {layer}")
            if storage.is_cuda and device_index is not None and storage.device.index != device_index:
                raise ValueError("Vocabulary CUDA tensor is on the wrong device")
            if c.num_sf_packs:
                sf = sfs[layer]
                if (
                    tuple(sf.shape) != (self.num_ranks * n, c.num_sf_packs)
                    or sf.dtype != torch.float32
                    or not sf.is_contiguous()
                ):
                    raise ValueError(f"Invalid global scale tensor for layer {layer}")
                if sf.is_cuda and device_index is not None and sf.device.index != device_index:
                    raise ValueError("Scale CUDA tensor is on the wrong device")

    def _check_fetch_args(self, indices, device_index, require_cuda: bool, allow_pinned: bool = False):
        self._ready()
        if not self._written:
            raise RuntimeError("write() must initialize the vocabulary before fetch()")
        if self._pending:
            raise RuntimeError("Call every previous layer hook before the next fetch")
        # Runs on every fetch: few tensor property reads (each costs a call
        # into torch), one get_device() for both the device and its index.
        c = self._config
        ok = isinstance(indices, torch.Tensor) and indices.dim() == 3
        if ok:
            layers, tokens, ept = indices.shape
            ok = (
                layers == len(c.entries)
                and ept == c.ept
                and tokens <= c.max_tokens
                and indices.dtype is torch.int32
                and indices.is_contiguous()
            )
        if ok and require_cuda:
            device = indices.get_device()  # -1 on the CPU
            if device < 0:
                ok = allow_pinned and indices.device.type == "cpu" and indices.is_pinned()
            else:
                ok = indices.is_cuda and (device_index is None or device == device_index)
        if not ok:
            where = ("CUDA or pinned host " if allow_pinned else "CUDA ") if require_cuda else ""
            raise ValueError(
                f"indices must be contiguous {where}int32 [layers, tokens, entries_per_token] within capacity"
            )

    def _make_hooks(self, generation, wait_layer, outputs):
        def make(layer):
            def hook():
                self._ready()
                if generation != self._generation:
                    raise RuntimeError("This hook belongs to a superseded fetch")
                if layer not in self._pending:
                    raise RuntimeError("This layer hook was already called")
                wait_layer(layer)
                self._pending.discard(layer)
                return outputs[layer]

            return hook

        return [make(layer) for layer in range(self._config.layers)]

    def _begin_fetch(self):
        self._generation += 1
        self._pending = set(range(self._config.layers))
        return self._generation

    # ---------------------------------------------------------------- shared API
    def fetch_all(self, indices, num_qps=0, use_tma_aligned_col_major_sf=True):
        """``fetch`` plus every layer hook, in layer order; returns the per-layer outputs."""
        hooks = self.fetch(indices, num_qps=num_qps, use_tma_aligned_col_major_sf=use_tma_aligned_col_major_sf)
        return [hook() for hook in hooks]

    def pinned_indices(self, tokens: int, write_combined: bool = True) -> torch.Tensor:
        """An int32 host tensor ``[layers, tokens, ept]`` to pass to ``fetch`` / ``fetch_all``.

        Page-locked when CUDA is available, so a fetch can take it as it is.
        This version ignores ``write_combined``; the native buffer honours it.
        """
        self._ready()
        cfg = self._config
        if not 0 <= tokens <= cfg.max_tokens:
            raise ValueError(f"tokens must be in [0, {cfg.max_tokens}]")
        return torch.empty((cfg.layers, tokens, cfg.ept), dtype=torch.int32, pin_memory=torch.cuda.is_available())

    def barrier(self):
        """Host barrier over the group (not a stream operation; never capture it)."""
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def get_comm_stream(self):
        """The stream fetch/hooks submit to: the caller's current stream."""
        if torch.cuda.is_available():
            return torch.cuda.current_stream()
        return None

    @property
    def main_context(self):
        return getattr(self, "runtime", None)

    @abstractmethod
    def destroy(self):  # pragma: no cover - interface
        ...

    def _check_destroy(self):
        if not self.explicitly_destroy:
            raise RuntimeError("Set explicitly_destroy=True before calling destroy()")
        if self._pending and not self._destroyed:
            raise RuntimeError("Outstanding layer hooks must be called before destroy()")

    def __del__(self):
        if getattr(self, "explicitly_destroy", False) and not getattr(self, "_destroyed", True) and getattr(
            self, "_configured", False
        ):
            warnings.warn(
                f"{type(self).__name__} was not collectively destroyed before process shutdown", ResourceWarning
            )
