"""Local-disk backend: one file per chunk, asynchronous writes, LRU by size.

Each file holds a small JSON header (shape, dtype, format) followed by the raw
chunk bytes.  Reads land directly in a pinned chunk object allocated from the
CPU tier (``readinto`` on the pinned buffer, no intermediate copy), so a disk
hit reaches the GPU through the same copy-engine path as a CPU hit.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct
import threading
from collections import OrderedDict
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any, List, Optional, Sequence

import torch

from ...config import LMCacheEngineConfig
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ..memory_management import MemoryFormat, MemoryObj
from .abstract_backend import StorageBackendInterface

logger = init_logger(__name__)

_MAGIC = b"LMCB"
_DTYPES = {str(d).removeprefix("torch."): d for d in
           (torch.float32, torch.float16, torch.bfloat16, torch.uint8, torch.int8,
            torch.float8_e4m3fn, torch.int32, torch.int64)}


class LocalDiskBackend(StorageBackendInterface):
    name = "LocalDiskBackend"

    def __init__(self, config: LMCacheEngineConfig, allocator_backend,
                 num_workers: int = 4):
        self.path = config.local_disk
        if self.path is None:
            raise ValueError("LocalDiskBackend needs config.local_disk")
        if self.path.startswith("file://"):
            self.path = self.path[len("file://"):]
        os.makedirs(self.path, exist_ok=True)
        self.capacity = int(config.max_local_disk_size * (1 << 30))
        self.allocator_backend = allocator_backend
        self.index: "OrderedDict[CacheEngineKey, int]" = OrderedDict()  # key -> bytes
        self.pinned: dict = {}
        self.used = 0
        self._lock = threading.RLock()
        self._pool = ThreadPoolExecutor(max_workers=num_workers,
                                        thread_name_prefix="lmc-disk")
        self._pending: dict = {}

    def _file(self, key: CacheEngineKey) -> str:
        h = hashlib.sha1(key.to_string().encode()).hexdigest()
        return os.path.join(self.path, h + ".kv")

    # ------------------------------------------------------------- queries
    def contains(self, key: CacheEngineKey, pin: bool = False) -> bool:
        with self._lock:
            ok = key in self.index
            if ok and pin:
                self.pinned[key] = self.pinned.get(key, 0) + 1
            return ok

    def exists_in_put_tasks(self, key: CacheEngineKey) -> bool:
        with self._lock:
            return key in self._pending

    def keys(self) -> List[CacheEngineKey]:
        with self._lock:
            return list(self.index.keys())

    def pin(self, key) -> bool:
        with self._lock:
            if key not in self.index:
                return False
            self.pinned[key] = self.pinned.get(key, 0) + 1
            return True

    def unpin(self, key) -> bool:
        with self._lock:
            n = self.pinned.get(key, 0)
            if n <= 1:
                self.pinned.pop(key, None)
            else:
                self.pinned[key] = n - 1
            return True

    # --------------------------------------------------------------- puts
    def _write(self, key: CacheEngineKey, obj: MemoryObj) -> None:
        try:
            t = obj.tensor
            header = json.dumps({
                "shape": list(obj.get_shape()),
                "dtype": str(obj.get_dtype()).removeprefix("torch."),
                "fmt": obj.get_memory_format().name,
            }).encode()
            size = obj.get_size()
            tmp = self._file(key) + ".tmp"
            with open(tmp, "wb") as f:
                f.write(_MAGIC + struct.pack("<I", len(header)) + header)
                f.write(memoryview(obj.raw_data[:size].numpy()))
            os.replace(tmp, self._file(key))
            with self._lock:
                self._pending.pop(key, None)
                if key not in self.index:
                    self.index[key] = size
                    self.used += size
                self._evict_if_needed()
        except Exception:
            logger.exception("disk write failed for %s", key)
            with self._lock:
                self._pending.pop(key, None)
        finally:
            obj.ref_count_down()

    def _evict_if_needed(self) -> None:
        if self.capacity <= 0:
            return
        while self.used > self.capacity and self.index:
            for k in self.index:
                if k not in self.pinned:
                    victim = k
                    break
            else:
                return
            self.used -= self.index.pop(victim)
            try:
                os.remove(self._file(victim))
            except FileNotFoundError:
                pass

    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey],
                                objs: Sequence[MemoryObj],
                                transfer_spec: Any = None) -> Optional[List[Future]]:
        futs = []
        for k, o in zip(keys, objs):
            with self._lock:
                if k in self.index or k in self._pending:
                    continue
                self._pending[k] = True
            o.ref_count_up()
            futs.append(self._pool.submit(self._write, k, o))
        return futs

    # --------------------------------------------------------------- gets
    def get_blocking(self, key: CacheEngineKey) -> Optional[MemoryObj]:
        with self._lock:
            if key not in self.index:
                return None
            self.index.move_to_end(key)
        path = self._file(key)
        try:
            with open(path, "rb") as f:
                magic = f.read(4)
                if magic != _MAGIC:
                    raise IOError(f"bad chunk file {path}")
                (hlen,) = struct.unpack("<I", f.read(4))
                hdr = json.loads(f.read(hlen))
                shape = torch.Size(hdr["shape"])
                dtype = _DTYPES[hdr["dtype"]]
                obj = self.allocator_backend.allocate(shape, dtype, MemoryFormat[hdr["fmt"]])
                if obj is None:
                    return None
                n = obj.get_size()
                got = f.readinto(memoryview(obj.raw_data[:n].numpy()))
                if got != n:
                    obj.ref_count_down()
                    raise IOError(f"short read {got}/{n} from {path}")
                return obj
        except FileNotFoundError:
            with self._lock:
                if key in self.index:
                    self.used -= self.index.pop(key)
            return None

    def batched_get_non_blocking(self, keys: Sequence[CacheEngineKey]) -> Future:
        return self._pool.submit(self.batched_get_blocking, keys)

    def remove(self, key: CacheEngineKey, force: bool = True) -> bool:
        with self._lock:
            if key not in self.index or (key in self.pinned and not force):
                return False
            self.used -= self.index.pop(key)
        try:
            os.remove(self._file(key))
        except FileNotFoundError:
            pass
        return True

    def wait_for_writes(self) -> None:
        import time

        while True:
            with self._lock:
                if not self._pending:
                    return
            time.sleep(0.001)

    def close(self) -> None:
        self.wait_for_writes()
        self._pool.shutdown(wait=True)
