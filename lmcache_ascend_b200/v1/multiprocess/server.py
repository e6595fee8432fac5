"""Multiprocess cache server: one process owns the CPU tier for many workers.

Serving workers register their paged KV caches by IPC handle (no copy: the
server maps the worker's device allocations, or its shared-memory host
caches) and then ask the server to store, look up and retrieve token
prefixes; the server runs the transfer kernels on the mapped caches.  All
registered workers share the server's storage, so a prefix stored by one
worker is a hit for every other worker of the same model.  The reference
registers NPU caches with upstream LMCache's multiprocess cache engine
(lmcache_ascend/v1/multiprocess/server.py:10-42, where the NPU cache context
is still NotImplemented); this module is the server and client of that mode.

Wire protocol: ZMQ ROUTER/REQ, msgpack ``[op, instance_id, payload]`` ->
``["ok", result]`` or ``["err", message]``.  Tokens and slot mappings travel
as int64 byte strings.

``python -m lmcache_ascend_b200.v1.multiprocess.server --port 5555 --chunk-size 256 --cpu-buffer-size 20``
"""

from __future__ import annotations

import argparse
import threading
from typing import Dict, Optional, Sequence

import msgpack
import numpy as np
import torch
import zmq

from ...config import LMCacheEngineConfig, LMCacheEngineMetadata
from ...utils.logging import init_logger
from ..cache_engine import LMCacheEngine
from ..gpu_connector import VLLMPagedMemGPUConnector
from ..storage_backend.storage_manager import StorageManager
from .custom_types import unwrap_kv_caches, wrap_kv_caches

logger = init_logger(__name__)


def _ints(t) -> bytes:
    return np.ascontiguousarray(torch.as_tensor(t).cpu().numpy().astype(np.int64)).tobytes()


def _tensor(b: bytes) -> torch.Tensor:
    return torch.from_numpy(np.frombuffer(b, dtype=np.int64).copy())


class _Instance:
    def __init__(self, engine: LMCacheEngine, conn, caches):
        self.engine, self.conn, self.caches = engine, conn, caches
        self.device = conn.layout.device
        self.lock = threading.Lock()


class MPCacheServer:
    def __init__(self, config: LMCacheEngineConfig, host: str = "127.0.0.1", port: int = 0):
        self.config = config
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.host = host
        self.port = self.sock.bind_to_random_port(f"tcp://{host}") if port == 0 else port
        if port:
            self.sock.bind(f"tcp://{host}:{port}")
        self.storage: Optional[StorageManager] = None
        self.instances: Dict[str, _Instance] = {}
        self._stop = threading.Event()
        self._t: Optional[threading.Thread] = None

    @property
    def url(self) -> str:
        return f"tcp://{self.host}:{self.port}"

    # ------------------------------------------------------------- ops
    def _register(self, inst: str, p: dict) -> int:
        caches = unwrap_kv_caches(p["kv"])
        first = caches[0][0] if isinstance(caches[0], tuple) else caches[0]
        md = LMCacheEngineMetadata(p.get("model", "model"), int(p.get("world_size", 1)),
                                   int(p.get("worker_id", 0)), "vllm", first.dtype)
        conn = VLLMPagedMemGPUConnector(self.config, kvcaches=caches)
        if self.storage is None:
            self.storage = StorageManager(self.config, md)
        eng = LMCacheEngine(self.config, md, conn, storage_manager=self.storage)
        self.instances[inst] = _Instance(eng, conn, caches)
        logger.info("registered %s: %d layers on %s", inst, len(caches), conn.layout.device)
        return len(caches)

    def _get(self, inst: str) -> _Instance:
        i = self.instances.get(inst)
        if i is None:
            raise KeyError(f"instance {inst} has not registered its KV caches")
        return i

    def _run(self, i: _Instance, fn):
        with i.lock:
            if i.device.type == "cuda":
                with torch.cuda.device(i.device):
                    return fn()
            return fn()

    def _handle(self, op: str, inst: str, p):
        if op == "ping":
            return True
        if op == "register":
            return self._register(inst, p)
        if op == "unregister":
            self.instances.pop(inst, None)  # the shared storage stays
            return True
        i = self._get(inst)
        tokens = _tensor(p["tokens"])
        if op == "lookup":
            return int(self._run(i, lambda: i.engine.lookup(tokens)))
        slots = _tensor(p["slots"])
        if i.device.type == "cuda":
            slots = slots.to(i.device)
        if op == "store":
            self._run(i, lambda: i.engine.store(tokens, slot_mapping=slots))
            return int(tokens.numel())
        if op == "retrieve":
            ret = self._run(i, lambda: i.engine.retrieve(tokens, slot_mapping=slots))
            return int(ret.sum())
        raise ValueError(f"unknown op {op}")

    # ------------------------------------------------------------ serve
    def serve_forever(self) -> None:
        poller = zmq.Poller()
        poller.register(self.sock, zmq.POLLIN)
        while not self._stop.is_set():
            if not poller.poll(100):
                continue
            ident, _, body = self.sock.recv_multipart()
            try:
                op, inst, payload = msgpack.unpackb(body, raw=False)
                res = ["ok", self._handle(op, inst, payload)]
            except Exception as e:  # report to the caller, keep serving
                logger.warning("cache server: %s failed: %s", locals().get("op"), e)
                res = ["err", f"{type(e).__name__}: {e}"]
            self.sock.send_multipart([ident, b"", msgpack.packb(res, use_bin_type=True)])
        self.sock.close()

    def start(self) -> "MPCacheServer":
        self._t = threading.Thread(target=self.serve_forever, daemon=True, name="lmc-mp-server")
        self._t.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)
        if self.storage is not None:
            self.storage.close()


class MPCacheClient:
    """Worker side: register caches, then store / lookup / retrieve."""

    def __init__(self, url: str, instance_id: str, timeout_ms: int = 30000):
        self.instance_id = instance_id
        self.sock = zmq.Context.instance().socket(zmq.REQ)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.sock.setsockopt(zmq.RCVTIMEO, timeout_ms)
        self.sock.setsockopt(zmq.SNDTIMEO, timeout_ms)
        self.sock.connect(url)
        self._device = None

    def _rpc(self, op: str, payload=None):
        self.sock.send(msgpack.packb([op, self.instance_id, payload], use_bin_type=True))
        try:
            st, res = msgpack.unpackb(self.sock.recv(), raw=False)
        except zmq.Again:
            raise TimeoutError(f"cache server did not answer {op}")
        if st != "ok":
            raise RuntimeError(f"cache server: {res}")
        return res

    def register_kv_caches(self, kv_caches, model_name: str = "model", world_size: int = 1,
                           worker_id: int = 0) -> int:
        caches = list(kv_caches.values()) if isinstance(kv_caches, dict) else list(kv_caches)
        first = caches[0][0] if isinstance(caches[0], (tuple, list)) else caches[0]
        self._device = first.device
        return self._rpc("register", {"kv": wrap_kv_caches(caches), "model": model_name,
                                      "world_size": world_size, "worker_id": worker_id})

    def _sync(self) -> None:
        # the server reads / writes these caches from another process
        if self._device is not None and self._device.type == "cuda":
            torch.cuda.synchronize(self._device)

    def store(self, tokens: Sequence[int], slot_mapping) -> int:
        self._sync()
        return self._rpc("store", {"tokens": _ints(tokens), "slots": _ints(slot_mapping)})

    def retrieve(self, tokens: Sequence[int], slot_mapping) -> int:
        self._sync()
        return self._rpc("retrieve", {"tokens": _ints(tokens), "slots": _ints(slot_mapping)})

    def lookup(self, tokens: Sequence[int]) -> int:
        return self._rpc("lookup", {"tokens": _ints(tokens)})

    def close(self, unregister: bool = True) -> None:
        if unregister:
            try:
                self._rpc("unregister")
            except (TimeoutError, RuntimeError):
                pass
        self.sock.close()


def run_cache_server(host: str, port: int, chunk_size: int = 256,
                     cpu_buffer_size: float = 5.0, **kw) -> None:
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=chunk_size, local_cpu=True,
                                            max_local_cpu_size=cpu_buffer_size, **kw)
    srv = MPCacheServer(cfg, host, port)
    print(f"lmcache cache server on {srv.url}", flush=True)
    try:
        srv.serve_forever()
    finally:
        if srv.storage is not None:
            srv.storage.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=5555)
    ap.add_argument("--chunk-size", type=int, default=256)
    ap.add_argument("--cpu-buffer-size", type=float, default=5.0, help="GB of CPU cache")
    a = ap.parse_args()
    run_cache_server(a.host, a.port, a.chunk_size, a.cpu_buffer_size)


if __name__ == "__main__":
    main()
