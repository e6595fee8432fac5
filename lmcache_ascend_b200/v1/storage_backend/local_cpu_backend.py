"""Pinned-CPU (hot) backend with LRU eviction.

It is also the allocator backend: chunk objects for every store are
allocated here (pinned host memory the copy engines and zero-copy kernels
reach at full PCIe rate), as in upstream LMCache where ``LocalCPUBackend``
hands out memory for the other tiers.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from concurrent.futures import Future
from typing import Any, Callable, List, Optional, Sequence

import torch

from ...config import LMCacheEngineConfig
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ...utils.metrics import get_stats
from ..memory_management import (
    BaseAllocator,
    MemoryFormat,
    MemoryObj,
    PinnedMemoryAllocator,
    TensorMemoryAllocator,
)
from .abstract_backend import StorageBackendInterface

logger = init_logger(__name__)


class LocalCPUBackend(StorageBackendInterface):
    name = "LocalCPUBackend"

    def __init__(self, config: LMCacheEngineConfig,
                 allocator: Optional[BaseAllocator] = None,
                 store_objects: bool = True):
        self.config = config
        self.store_objects = store_objects and config.local_cpu
        if allocator is None:
            nbytes = int(config.max_local_cpu_size * (1 << 30))
            numa = config.numa_node
            if numa == -2:  # auto: the current GPU's node, when the host reports one
                import torch

                from ...utils.system_detection import resolve_numa_node

                dev = torch.cuda.current_device() if torch.cuda.is_available() else None
                numa = resolve_numa_node(numa, dev)
            if config.shared_cpu_cache and config.shared_cpu_cache_name:
                allocator = PinnedMemoryAllocator(nbytes, numa,
                                                  shm_name=config.shared_cpu_cache_name)
            else:
                allocator = PinnedMemoryAllocator(nbytes, numa)
        self.allocator = allocator
        self.hot_cache: "OrderedDict[CacheEngineKey, MemoryObj]" = OrderedDict()
        self._lock = threading.RLock()
        self.evict_listeners: List[Callable[[CacheEngineKey], None]] = []
        self.stats = get_stats()

    # ------------------------------------------------------------- queries
    def contains(self, key: CacheEngineKey, pin: bool = False) -> bool:
        with self._lock:
            obj = self.hot_cache.get(key)
            if obj is None:
                return False
            if pin:
                obj.pin()
            return True

    def keys(self) -> List[CacheEngineKey]:
        with self._lock:
            return list(self.hot_cache.keys())

    def __len__(self) -> int:
        return len(self.hot_cache)

    # --------------------------------------------------------------- puts
    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey],
                                objs: Sequence[MemoryObj],
                                transfer_spec: Any = None) -> Optional[List[Future]]:
        if not self.store_objects:
            return None
        if type(self) is LocalCPUBackend:
            # device chunks belong to the HBM tier; they reach this tier only
            # through its eviction write-back
            pairs = [(k, o) for k, o in zip(keys, objs)
                     if o.raw_data is None or not o.raw_data.is_cuda]
            keys, objs = [k for k, _ in pairs], [o for _, o in pairs]
        with self._lock:
            for k, o in zip(keys, objs):
                old = self.hot_cache.pop(k, None)
                if old is not None:
                    old.ref_count_down()
                o.ref_count_up()
                self.hot_cache[k] = o
        return None

    # --------------------------------------------------------------- gets
    def get_blocking(self, key: CacheEngineKey) -> Optional[MemoryObj]:
        with self._lock:
            obj = self.hot_cache.get(key)
            if obj is None:
                return None
            self.hot_cache.move_to_end(key)
            obj.ref_count_up()  # caller owns one reference
            return obj

    def batched_get_blocking(self, keys: Sequence[CacheEngineKey]) -> List[Optional[MemoryObj]]:
        """One lock acquisition for the whole batch (a layerwise 16k-token
        request asks for thousands of per-layer chunks)."""
        with self._lock:
            hc = self.hot_cache
            get, touch = hc.get, hc.move_to_end
            out: List[Optional[MemoryObj]] = [get(k) for k in keys]
            for key, obj in zip(keys, out):
                if obj is not None:
                    touch(key)
                    obj.ref_count_up()
        return out

    def pin(self, key: CacheEngineKey) -> bool:
        with self._lock:
            obj = self.hot_cache.get(key)
            return obj.pin() if obj is not None else False

    def unpin(self, key: CacheEngineKey) -> bool:
        with self._lock:
            obj = self.hot_cache.get(key)
            return obj.unpin() if obj is not None else False

    def remove(self, key: CacheEngineKey, force: bool = True) -> bool:
        with self._lock:
            obj = self.hot_cache.get(key)
            if obj is None:
                return False
            if obj.is_pinned and not force:
                return False
            del self.hot_cache[key]
        obj.ref_count_down()
        for cb in self.evict_listeners:
            cb(key)
        return True

    # ---------------------------------------------------------- allocation
    def _evict_one(self) -> bool:
        with self._lock:
            for k, o in self.hot_cache.items():
                if not o.is_pinned and o.get_ref_count() == 1:
                    victim = k
                    break
            else:
                return False
        self.remove(victim)
        self.stats.inc("evictions")
        return True

    def allocate(self, shape, dtype, fmt: MemoryFormat = MemoryFormat.KV_2LTD,
                 eviction: bool = True) -> Optional[MemoryObj]:
        while True:
            obj = self.allocator.allocate(shape, dtype, fmt)
            if obj is not None or not eviction:
                return obj
            if not self._evict_one():
                return None

    def batched_allocate(self, shape, dtype, batch_size: int,
                         fmt: MemoryFormat = MemoryFormat.KV_2LTD,
                         eviction: bool = True) -> Optional[List[MemoryObj]]:
        out = []
        for _ in range(batch_size):
            o = self.allocate(shape, dtype, fmt, eviction)
            if o is None:
                for p in out:
                    p.ref_count_down()
                return None
            out.append(o)
        return out

    def get_allocator_backend(self):
        return self

    @property
    def used_bytes(self) -> int:
        a = self.allocator
        return getattr(a, "used_bytes", 0)

    def close(self) -> None:
        with self._lock:
            objs = list(self.hot_cache.values())
            self.hot_cache.clear()
        for o in objs:
            o.ref_count_down()
        close = getattr(self.allocator, "close", None)
        if close is not None:
            close()
