"""Remote backend: serialized chunks on a remote KV server.

``remote_url`` forms: ``lm://host:port`` (``lmcache_ascend_b200.server``)
or ``mem://name`` (process-local store, for tests and single-process use).
Puts serialize (naive or CacheGen, ``remote_serde``) and send on a worker
thread; gets fetch and deserialize into a pinned chunk from the CPU tier's
allocator (upstream RemoteBackend semantics used by the reference's
storage-backend factory, lmcache_ascend/v1/storage_backend/__init__.py:51-167).
"""

from __future__ import annotations

import threading
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Any, Dict, List, Optional, Sequence

import msgpack
import zmq

from ...config import LMCacheEngineConfig
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ...utils.metrics import get_stats
from ..memory_management import MemoryObj
from .abstract_backend import StorageBackendInterface
from .serde import create_serde

logger = init_logger(__name__)

_MEM_STORES: Dict[str, Dict[str, bytes]] = {}
_MEM_LOCK = threading.Lock()


class RemoteConnector:
    def __init__(self, url: str, timeout_ms: int = 10000):
        self.url = url
        self._local = threading.local()
        self.timeout_ms = timeout_ms
        if url.startswith("mem://"):
            with _MEM_LOCK:
                self.mem = _MEM_STORES.setdefault(url, {})
        elif url.startswith("lm://"):
            self.mem = None
            self.endpoint = "tcp://" + url[len("lm://"):]
        else:
            raise ValueError(f"unsupported remote_url {url!r} (lm://host:port or mem://name)")

    def _sock(self) -> zmq.Socket:
        s = getattr(self._local, "sock", None)
        if s is None:
            s = zmq.Context.instance().socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
            s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
            s.connect(self.endpoint)
            self._local.sock = s
        return s

    def _rpc(self, op: str, key: str = "", payload: Any = None):
        if self.mem is not None:
            with _MEM_LOCK:
                if op == "put":
                    self.mem[key] = payload
                    return True
                if op == "get":
                    return self.mem.get(key)
                if op == "exists":
                    return key in self.mem
                if op == "remove":
                    return self.mem.pop(key, None) is not None
                if op == "list":
                    return list(self.mem)
            raise ValueError(op)
        s = self._sock()
        try:
            s.send(msgpack.packb([op, key, payload], use_bin_type=True))
            st, res = msgpack.unpackb(s.recv(), raw=False)
        except zmq.Again:
            s.close()
            self._local.sock = None
            raise TimeoutError(f"remote KV server {self.url} did not answer")
        if st != "ok":
            raise RuntimeError(f"remote KV server error: {res}")
        return res

    def put(self, key: str, data: bytes) -> None:
        self._rpc("put", key, data)

    def get(self, key: str) -> Optional[bytes]:
        return self._rpc("get", key)

    def exists(self, key: str) -> bool:
        return bool(self._rpc("exists", key))

    def remove(self, key: str) -> bool:
        return bool(self._rpc("remove", key))

    def list(self) -> List[str]:
        return self._rpc("list")


class RemoteBackend(StorageBackendInterface):
    name = "RemoteBackend"

    def __init__(self, config: LMCacheEngineConfig, metadata, allocator_backend,
                 num_workers: int = 2):
        self.config = config
        self.conn = RemoteConnector(config.remote_url,
                                    int(config.blocking_timeout_secs * 1000))
        self.serde = create_serde(config)
        self.allocator_backend = allocator_backend
        self._pool = ThreadPoolExecutor(max_workers=num_workers, thread_name_prefix="lmc-remote")
        self._inflight: Dict[str, Future] = {}
        self._lock = threading.Lock()
        self.stats = get_stats()

    def contains(self, key: CacheEngineKey, pin: bool = False) -> bool:
        try:
            return self.conn.exists(key.to_string())
        except (TimeoutError, RuntimeError) as e:
            logger.warning("remote contains failed: %s", e)
            return False

    def exists_in_put_tasks(self, key: CacheEngineKey) -> bool:
        with self._lock:
            return key.to_string() in self._inflight

    def _put(self, k: str, obj: MemoryObj) -> None:
        try:
            data = self.serde.serialize(obj)
            self.conn.put(k, data)
            self.stats.inc("remote_put_bytes", len(data))
            self.stats.inc("remote_put_raw_bytes", obj.get_size())
        except Exception:
            logger.exception("remote put failed for %s", k)
        finally:
            obj.ref_count_down()
            with self._lock:
                self._inflight.pop(k, None)

    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey],
                                objs: Sequence[MemoryObj], transfer_spec: Any = None):
        futs = []
        for key, o in zip(keys, objs):
            k = key.to_string()
            with self._lock:
                if k in self._inflight:
                    continue
                o.ref_count_up()
                f = self._pool.submit(self._put, k, o)
                self._inflight[k] = f
            futs.append(f)
        return futs

    def get_blocking(self, key: CacheEngineKey) -> Optional[MemoryObj]:
        try:
            data = self.conn.get(key.to_string())
        except (TimeoutError, RuntimeError) as e:
            logger.warning("remote get failed: %s", e)
            return None
        if data is None:
            return None
        self.stats.inc("remote_get_bytes", len(data))
        return self.serde.deserialize(data, self.allocator_backend)

    def remove(self, key: CacheEngineKey, force: bool = True) -> bool:
        return self.conn.remove(key.to_string())

    def keys(self) -> List[CacheEngineKey]:
        return [CacheEngineKey.from_string(k) for k in self.conn.list()]

    def wait_for_puts(self) -> None:
        with self._lock:
            fs = list(self._inflight.values())
        for f in fs:
            f.result()

    def close(self) -> None:
        self.wait_for_puts()
        self._pool.shutdown(wait=True)
