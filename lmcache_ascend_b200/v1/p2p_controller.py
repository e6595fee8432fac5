"""Key-location controller for cross-instance (P2P) KV sharing.

Instances report the chunk keys they hold (admit) and drop (evict); a lookup
returns the instances holding a key together with their peer endpoints.
Counterpart of the controller the reference's P2P backend queries
(lmcache_ascend/v1/storage_backend/p2p_backend.py:838-960; upstream LMCache
cache_controller).  ZMQ ROUTER server, msgpack ``[op, instance, payload]``.

``python -m lmcache_ascend_b200.v1.p2p_controller --port 9000``
"""

from __future__ import annotations

import argparse
import threading
from collections import defaultdict
from typing import Dict, Optional, Set

import msgpack
import zmq


class P2PController:
    def __init__(self, host: str = "127.0.0.1", port: int = 0):
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.port = self.sock.bind_to_random_port(f"tcp://{host}") if port == 0 else port
        if port:
            self.sock.bind(f"tcp://{host}:{port}")
        self.host = host
        self.urls: Dict[str, str] = {}                 # instance -> peer url
        self.where: Dict[str, Set[str]] = defaultdict(set)  # key -> instances
        self._stop = threading.Event()
        self._t: Optional[threading.Thread] = None

    @property
    def url(self) -> str:
        return f"tcp://{self.host}:{self.port}"

    def _handle(self, op: str, inst: str, payload):
        if op == "register":
            self.urls[inst] = payload
            return True
        if op == "deregister":
            self.urls.pop(inst, None)
            for s in self.where.values():
                s.discard(inst)
            return True
        if op == "admit":
            for k in payload:
                self.where[k].add(inst)
            return True
        if op == "evict":
            for k in payload:
                s = self.where.get(k)
                if s:
                    s.discard(inst)
                    if not s:
                        del self.where[k]
            return True
        if op == "lookup":
            return [[i, self.urls[i]] for i in sorted(self.where.get(payload, ()))
                    if i != inst and i in self.urls]
        raise ValueError(f"unknown op {op}")

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
            except Exception as e:
                res = ["err", str(e)]
            self.sock.send_multipart([ident, b"", msgpack.packb(res, use_bin_type=True)])
        self.sock.close()

    def start(self) -> "P2PController":
        self._t = threading.Thread(target=self.serve_forever, daemon=True, name="lmc-p2p-ctl")
        self._t.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=2)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=9000)
    a = ap.parse_args()
    c = P2PController(a.host, a.port)
    print(f"p2p controller on {c.url}", flush=True)
    c.serve_forever()


if __name__ == "__main__":
    main()
