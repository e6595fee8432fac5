"""HBM tier: chunk objects kept in this GPU's memory, above the CPU tier.

A B200 has 180 GB of HBM; a serving instance that leaves some of it to the
cache keeps hot prefixes one device-to-device copy away from the paged KV
(TMA gather on store, TMA scatter on retrieve, several TB/s) instead of a
PCIe / host-memory transfer, and eight replicas of a box then stop sharing
one host memory system for every prefix hit.

* It is the allocator backend when enabled: stores gather straight into its
  device pages (``GPUMemoryAllocator``, one exportable cudaMalloc slab).
* LRU eviction writes the victim back to the CPU tier (a pinned page and one
  device-to-host copy) unless the CPU tier already holds the key, so the
  hierarchy stays inclusive of everything that was stored.
* The CPU tier does not keep device objects itself; it receives them only
  through this write-back.

Config: ``local_gpu`` (bool), ``max_local_gpu_size`` (GB).
"""

from __future__ import annotations

from typing import Optional

import torch

from ...config import LMCacheEngineConfig
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ..memory_management import GPUMemoryAllocator
from .local_cpu_backend import LocalCPUBackend

logger = init_logger(__name__)


class LocalGPUBackend(LocalCPUBackend):
    name = "LocalGPUBackend"

    def __init__(self, config: LMCacheEngineConfig, lower: Optional[LocalCPUBackend] = None,
                 device: Optional[torch.device] = None):
        dev = device or torch.device("cuda", torch.cuda.current_device())
        alloc = GPUMemoryAllocator(int(config.max_local_gpu_size * (1 << 30)), dev)
        super().__init__(config, allocator=alloc, store_objects=True)
        self.store_objects = True  # independent of local_cpu
        self.device = dev
        self.lower = lower
        self.writebacks = 0

    def batched_submit_put_task(self, keys, objs, transfer_spec=None):
        keep = [(k, o) for k, o in zip(keys, objs) if o.raw_data is not None and
                o.raw_data.is_cuda and o.raw_data.device == self.device]
        if keep:
            super().batched_submit_put_task([k for k, _ in keep], [o for _, o in keep],
                                            transfer_spec)
        return None

    def _write_back(self, key: CacheEngineKey, obj) -> None:
        low = self.lower
        if low is None or not low.store_objects or low.contains(key):
            return
        dst = low.allocate(obj.get_shape(), obj.get_dtype(), obj.get_memory_format())
        if dst is None:
            logger.warning("HBM tier: CPU tier full, %s dropped on eviction", key)
            return
        n = obj.get_size()
        dst.raw_data[:n].copy_(obj.raw_data[:n])  # D2H, ordered after the writes
        low.batched_submit_put_task([key], [dst])
        dst.ref_count_down()  # the CPU tier holds its own reference
        self.writebacks += 1
        self.stats.inc("hbm_writebacks")

    def _evict_one(self) -> bool:
        with self._lock:
            victim = None
            for k, o in self.hot_cache.items():
                if not o.is_pinned and o.get_ref_count() == 1:
                    victim = (k, o)
                    break
            if victim is None:
                return False
        self._write_back(*victim)
        self.remove(victim[0])
        self.stats.inc("evictions")
        return True
