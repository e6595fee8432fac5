"""Storage backend interface.

Re-creates the upstream LMCache backend contract the reference's backends
implement (``contains``, ``batched_submit_put_task``, ``get_blocking``,
``batched_get_non_blocking``, ``pin``/``unpin``, ``remove``, ``close``; call
sites in reference lmcache_ascend/v1/storage_backend/pd/backend.py:285 and
p2p_backend.py:106-985).
"""

from __future__ import annotations

import abc
from concurrent.futures import Future
from typing import Any, List, Optional, Sequence

from ..memory_management import MemoryObj
from ...utils.keys import CacheEngineKey


class StorageBackendInterface(abc.ABC):
    name: str = "abstract"

    @abc.abstractmethod
    def contains(self, key: CacheEngineKey, pin: bool = False) -> bool: ...

    def exists_in_put_tasks(self, key: CacheEngineKey) -> bool:
        return False

    @abc.abstractmethod
    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey],
                                objs: Sequence[MemoryObj],
                                transfer_spec: Any = None) -> Optional[List[Future]]: ...

    def submit_put_task(self, key: CacheEngineKey, obj: MemoryObj) -> Optional[Future]:
        r = self.batched_submit_put_task([key], [obj])
        return r[0] if r else None

    @abc.abstractmethod
    def get_blocking(self, key: CacheEngineKey) -> Optional[MemoryObj]: ...

    def batched_get_blocking(self, keys: Sequence[CacheEngineKey]
                             ) -> List[Optional[MemoryObj]]:
        return [self.get_blocking(k) for k in keys]

    def batched_get_non_blocking(self, keys: Sequence[CacheEngineKey]) -> Future:
        f: Future = Future()
        try:
            f.set_result(self.batched_get_blocking(keys))
        except Exception as e:  # pragma: no cover
            f.set_exception(e)
        return f

    def pin(self, key: CacheEngineKey) -> bool:
        return False

    def unpin(self, key: CacheEngineKey) -> bool:
        return False

    def remove(self, key: CacheEngineKey, force: bool = True) -> bool:
        return False

    def batched_remove(self, keys: Sequence[CacheEngineKey], force: bool = True) -> int:
        return sum(1 for k in keys if self.remove(k, force))

    def get_allocator_backend(self):
        return None

    def keys(self) -> List[CacheEngineKey]:
        return []

    def close(self) -> None:
        pass
