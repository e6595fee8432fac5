"""Standalone KV chunk server for the remote tier (``remote_url: lm://host:port``).

``python -m lmcache_ascend_b200.server --host 0.0.0.0 --port 65432 [--max-gb N]``

The reference's remote backend talks to upstream LMCache's ``lmcache_server``
(docs/cachegen/Cachegen.md: "The remote backend is LMCache server which
stores cache in CPU").  This server keeps serialized chunks (naive or
CacheGen bytes) in host memory with LRU eviction by size, behind a ZMQ
ROUTER socket; requests are msgpack ``[op, key, payload]`` with op in
put / get / exists / remove / list / ping.
"""

from __future__ import annotations

import argparse
import threading
from collections import OrderedDict
from typing import Optional

import msgpack
import zmq


class LMCacheServer:
    def __init__(self, host: str = "127.0.0.1", port: int = 0, max_bytes: int = 8 << 30):
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        if port == 0:
            self.port = self.sock.bind_to_random_port(f"tcp://{host}")
        else:
            self.sock.bind(f"tcp://{host}:{port}")
            self.port = port
        self.host = host
        self.max_bytes = max_bytes
        self.store: "OrderedDict[str, bytes]" = OrderedDict()
        self.used = 0
        self._stop = threading.Event()
        self._thr: Optional[threading.Thread] = None

    @property
    def url(self) -> str:
        h = "127.0.0.1" if self.host in ("0.0.0.0", "*") else self.host
        return f"lm://{h}:{self.port}"

    def _handle(self, op: str, key: str, payload):
        if op == "put":
            old = self.store.pop(key, None)
            if old is not None:
                self.used -= len(old)
            self.store[key] = payload
            self.used += len(payload)
            while self.used > self.max_bytes and len(self.store) > 1:
                _, v = self.store.popitem(last=False)
                self.used -= len(v)
            return True
        if op == "get":
            v = self.store.get(key)
            if v is not None:
                self.store.move_to_end(key)
            return v
        if op == "exists":
            return key in self.store
        if op == "remove":
            v = self.store.pop(key, None)
            if v is not None:
                self.used -= len(v)
            return v is not None
        if op == "list":
            return list(self.store.keys())
        if op == "ping":
            return "pong"
        raise ValueError(f"unknown op {op}")

    def serve_forever(self) -> None:
        poller = zmq.Poller()
        poller.register(self.sock, zmq.POLLIN)
        while not self._stop.is_set():
            if not poller.poll(100):
                continue
            ident, _, body = self.sock.recv_multipart()
            try:
                op, key, payload = msgpack.unpackb(body, raw=False)
                res = ["ok", self._handle(op, key, payload)]
            except Exception as e:
                res = ["err", str(e)]
            self.sock.send_multipart([ident, b"", msgpack.packb(res, use_bin_type=True)])
        self.sock.close()

    def start(self) -> "LMCacheServer":
        self._thr = threading.Thread(target=self.serve_forever, daemon=True,
                                     name="lmc-server")
        self._thr.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thr is not None:
            self._thr.join(timeout=2)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=65432)
    ap.add_argument("--max-gb", type=float, default=8.0)
    a = ap.parse_args()
    srv = LMCacheServer(a.host, a.port, int(a.max_gb * (1 << 30)))
    print(f"lmcache_ascend_b200 server on {srv.url}", flush=True)
    srv.serve_forever()


if __name__ == "__main__":
    main()
