"""Storage manager: ordered backend hierarchy.

Puts go to every backend (each decides whether to keep the object); gets and
contains walk the hierarchy in order (PD -> LocalCPU -> P2P -> LocalDisk ->
Remote, the order of reference lmcache_ascend/v1/storage_backend/
__init__.py:51-167).  A hit in a lower tier is promoted into the CPU tier so
the next retrieve of the same prefix is served from pinned memory.
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from ...config import LMCacheEngineConfig, LMCacheEngineMetadata
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ...utils.metrics import get_stats
from ..memory_management import MemoryFormat, MemoryObj
from .abstract_backend import StorageBackendInterface

logger = init_logger(__name__)


class StorageManager:
    def __init__(self, config: LMCacheEngineConfig,
                 metadata: Optional[LMCacheEngineMetadata] = None,
                 backends: Optional["OrderedDict[str, StorageBackendInterface]"] = None,
                 **kw):
        from . import CreateStorageBackends

        self.config = config
        self.metadata = metadata
        self.backends: "OrderedDict[str, StorageBackendInterface]" = (
            backends if backends is not None else CreateStorageBackends(config, metadata, **kw))
        self._lock = threading.Lock()
        self.stats = get_stats()

    # ---------------------------------------------------------- allocation
    @property
    def allocator_backend(self):
        """First backend that provides chunk memory (a PD sender's page pool
        becomes available only after post_init, so this is not cached)."""
        for b in self.backends.values():
            ab = b.get_allocator_backend()
            if ab is not None:
                return ab
        return None

    def allocate(self, shape, dtype, fmt: MemoryFormat = MemoryFormat.KV_2LTD,
                 eviction: bool = True) -> Optional[MemoryObj]:
        ab = self.allocator_backend
        if ab is None:
            raise RuntimeError("no backend provides an allocator")
        return ab.allocate(shape, dtype, fmt, eviction=eviction)

    def batched_allocate(self, shape, dtype, batch_size: int,
                         fmt: MemoryFormat = MemoryFormat.KV_2LTD,
                         eviction: bool = True) -> Optional[List[MemoryObj]]:
        return self.allocator_backend.batched_allocate(shape, dtype, batch_size, fmt,
                                                       eviction=eviction)

    # ---------------------------------------------------------------- puts
    def batched_put(self, keys: Sequence[CacheEngineKey], objs: Sequence[MemoryObj],
                    transfer_spec=None, location: Optional[str] = None) -> list:
        """Hand the chunks to every backend; returns the futures of the puts
        that complete asynchronously."""
        futs: list = []
        for name, b in self.backends.items():
            if location is not None and name != location:
                continue
            r = b.batched_submit_put_task(keys, objs, transfer_spec=transfer_spec)
            if r:
                futs.extend(f for f in r if f is not None)
        self.stats.inc("stored_chunks", len(keys))
        return futs

    def put(self, key: CacheEngineKey, obj: MemoryObj) -> None:
        self.batched_put([key], [obj])

    # ------------------------------------------------------------- lookups
    def contains(self, key: CacheEngineKey, search_range: Optional[List[str]] = None,
                 pin: bool = False) -> Optional[str]:
        for name, b in self.backends.items():
            if search_range is not None and name not in search_range:
                continue
            if b.contains(key, pin=pin):
                return name
        return None

    def batched_contains(self, keys: Sequence[CacheEngineKey], pin: bool = False) -> int:
        """Length of the prefix of ``keys`` present in some backend."""
        n = 0
        for k in keys:
            if self.contains(k, pin=pin) is None:
                break
            n += 1
        return n

    def unpin(self, key: CacheEngineKey) -> None:
        for b in self.backends.values():
            b.unpin(key)

    def remove(self, key: CacheEngineKey, locations: Optional[List[str]] = None) -> int:
        n = 0
        for name, b in self.backends.items():
            if locations is not None and name not in locations:
                continue
            n += int(b.remove(key))
        return n

    # ----------------------------------------------------------------- gets
    def get(self, key: CacheEngineKey, location: Optional[str] = None
            ) -> Optional[MemoryObj]:
        for name, b in self.backends.items():
            if location is not None and name != location:
                continue
            obj = b.get_blocking(key)
            if obj is None:
                continue
            self._promote(name, key, obj)
            return obj
        return None

    def batched_get(self, keys: Sequence[CacheEngineKey], location: Optional[str] = None
                    ) -> List[Optional[MemoryObj]]:
        out: List[Optional[MemoryObj]] = [None] * len(keys)
        todo = list(range(len(keys)))
        for name, b in self.backends.items():
            if not todo:
                break
            if location is not None and name != location:
                continue
            got = b.batched_get_blocking([keys[i] for i in todo])
            rest = []
            # hits of the CPU and HBM tiers are already where they belong
            promote = name not in ("LocalCPUBackend", "LocalGPUBackend")
            for i, obj in zip(todo, got):
                if obj is None:
                    rest.append(i)
                else:
                    out[i] = obj
                    if promote:
                        self._promote(name, keys[i], obj)
            todo = rest
        return out

    def _promote(self, name: str, key: CacheEngineKey, obj: MemoryObj) -> None:
        """A hit in a lower tier is kept in the tier its memory belongs to:
        host chunks in the CPU tier, device chunks (a peer's HBM chunk copied
        over NVLink) in the HBM tier."""
        if obj.raw_data is None or obj.meta.dtype is None:
            return
        tier = "LocalGPUBackend" if obj.raw_data.is_cuda else "LocalCPUBackend"
        dst = self.backends.get(tier)
        if dst is None or name == tier or not dst.store_objects:
            return
        dst.batched_submit_put_task([key], [obj])

    def close(self) -> None:
        for b in reversed(list(self.backends.values())):
            try:
                b.close()
            except Exception:  # pragma: no cover
                logger.exception("closing backend %s", b)
