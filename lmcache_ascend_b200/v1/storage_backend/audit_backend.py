"""Audit wrapper around a storage backend (``enable_audit``).

Wraps another backend and checks what flows through it: every put records a
checksum of the chunk bytes, every get verifies the returned object against
it and counts mismatches; removals are only forwarded when
``audit_actual_remove`` is set (so an audit run never loses data).  Mirrors
the optional audit layer of the reference's backend factory
(lmcache_ascend/v1/storage_backend/__init__.py:51-167).
"""

from __future__ import annotations

import threading
import zlib
from typing import Any, Dict, List, Optional, Sequence

from ...config import LMCacheEngineConfig
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ...utils.metrics import get_stats
from ..memory_management import MemoryObj
from .abstract_backend import StorageBackendInterface

logger = init_logger(__name__)


def _checksum(obj: MemoryObj) -> int:
    if obj.raw_data is None:
        return zlib.crc32(obj.byte_array)
    n = obj.get_size()
    return zlib.crc32(obj.raw_data[:n].cpu().numpy().tobytes())


class AuditBackend(StorageBackendInterface):
    def __init__(self, inner: StorageBackendInterface, config: LMCacheEngineConfig):
        self.inner = inner
        self.name = inner.name  # keeps the hierarchy's names stable
        self.config = config
        self._sums: Dict[CacheEngineKey, int] = {}
        self._lock = threading.Lock()
        self.stats = get_stats()
        self.mismatches = 0

    def contains(self, key, pin: bool = False) -> bool:
        return self.inner.contains(key, pin)

    def exists_in_put_tasks(self, key) -> bool:
        return self.inner.exists_in_put_tasks(key)

    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey], objs: Sequence[MemoryObj],
                                transfer_spec: Any = None):
        with self._lock:
            for k, o in zip(keys, objs):
                if o.raw_data is not None and not o.raw_data.is_cuda:
                    self._sums[k] = _checksum(o)
        self.stats.inc("audit_puts", len(keys))
        return self.inner.batched_submit_put_task(keys, objs, transfer_spec)

    def get_blocking(self, key) -> Optional[MemoryObj]:
        obj = self.inner.get_blocking(key)
        if obj is not None:
            with self._lock:
                want = self._sums.get(key)
            if want is not None and obj.raw_data is not None and not obj.raw_data.is_cuda:
                if _checksum(obj) != want:
                    self.mismatches += 1
                    self.stats.inc("audit_mismatches")
                    logger.error("audit: chunk %s changed between put and get", key)
            self.stats.inc("audit_gets")
        return obj

    def pin(self, key) -> bool:
        return self.inner.pin(key)

    def unpin(self, key) -> bool:
        return self.inner.unpin(key)

    def remove(self, key, force: bool = True) -> bool:
        self.stats.inc("audit_removes")
        if not self.config.audit_actual_remove:
            return False
        with self._lock:
            self._sums.pop(key, None)
        return self.inner.remove(key, force)

    def keys(self) -> List[CacheEngineKey]:
        return self.inner.keys()

    def get_allocator_backend(self):
        return self.inner.get_allocator_backend()

    def __getattr__(self, item):  # wait_for_writes, post_init, ... of the inner backend
        return getattr(self.inner, item)

    def close(self) -> None:
        self.inner.close()
