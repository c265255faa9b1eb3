"""B200-native Engram lookup buffer.

Sharded embedding-row lookups for per-layer "engram" tables over one NVLink 5 /
NVSwitch node, with the EngramBuffer API of yykzjh/engram-rdma-lab:

* :class:`EngramBuffer` - the native buffer (sm_100a kernels, C++ runtime);
* :class:`TorchEngramBuffer` - the same API on torch collectives (CPU/gloo
  oracle, NCCL ``all_to_all`` baseline);
* :mod:`.routing` - route negotiation (``ENGRAM_EGM_ENABLE``);
* :mod:`.models` - benchmark table sets, synthetic weights and index streams;
* :mod:`.ops` - FP8 block quantisation helpers;
* :mod:`.parallel` - process-group bootstrap and GPU placement;
* :mod:`.utils` - timing, events, environment helpers.
"""

from .base import EngramBufferBase
from .buffer import EngramBuffer, theoretical_config
from .layout import EngramConfig, plan_memory, sf_strides, storage_size_hint, validate_config
from .reference import TorchEngramBuffer
from .routing import EgmConfig, OwnerRoute

__version__ = "0.1.0"

__all__ = [
    "EgmConfig",
    "EngramBuffer",
    "EngramBufferBase",
    "EngramConfig",
    "OwnerRoute",
    "TorchEngramBuffer",
    "plan_memory",
    "sf_strides",
    "storage_size_hint",
    "theoretical_config",
    "validate_config",
]
