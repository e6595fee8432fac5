"""Scheduler <-> worker lookup channel (ZMQ IPC).

vLLM's scheduler process decides how many prompt tokens to load from the
cache before the worker holding the engine ever sees the request, so it asks
the worker-side engine over a short-path ZMQ IPC socket (reference: upstream
LMCacheLookupClient/Server, short IPC paths patched in
lmcache_ascend/v1/rpc_utils.py:15-40, token normalisation in
lmcache_ascend/v1/lookup_client/lmcache_lookup_client.py:12-31).
Requests are msgpack ``[lookup_id, token_ids]``; replies the hit length.
"""

from __future__ import annotations

import hashlib
import os
import tempfile
import threading
from typing import Iterable, List, Optional

import msgpack
import zmq

from ...utils.logging import init_logger

logger = init_logger(__name__)


def lookup_ipc_path(instance_id: str, dp_rank: int = 0) -> str:
    """Short IPC path: unix socket paths are limited to ~107 bytes, so the
    instance id is hashed instead of embedded."""
    h = hashlib.sha1(f"{instance_id}:{dp_rank}".encode()).hexdigest()[:12]
    return f"ipc://{tempfile.gettempdir()}/lmc_lkp_{h}.ipc"


def normalize_tokens(tokens) -> List[int]:
    """Accept lists, tuples, numpy arrays and tensors; return a list of ints."""
    if hasattr(tokens, "tolist"):
        tokens = tokens.tolist()
    return [int(t) for t in tokens]


class LookupServer:
    def __init__(self, engine, url: str):
        self.engine = engine
        self.url = url
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.REP)
        self.sock.setsockopt(zmq.LINGER, 0)
        if url.startswith("ipc://"):
            path = url[len("ipc://"):]
            if os.path.exists(path):
                os.unlink(path)
        self.sock.bind(url)
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._loop, daemon=True, name="lmc-lookup")
        self._t.start()

    def _loop(self):
        poller = zmq.Poller()
        poller.register(self.sock, zmq.POLLIN)
        while not self._stop.is_set():
            if not poller.poll(100):
                continue
            try:
                lookup_id, tokens, op = msgpack.unpackb(self.sock.recv(), raw=False)
                if op == "unpin":
                    self.engine.lookup_unpin(lookup_id)
                    res = 0
                else:
                    import torch

                    res = self.engine.lookup(torch.tensor(tokens, dtype=torch.long),
                                             lookup_id=lookup_id, pin=True)
            except Exception:
                logger.exception("lookup failed")
                res = 0
            self.sock.send(msgpack.packb(int(res)))
        self.sock.close()

    def close(self):
        self._stop.set()
        self._t.join(timeout=2)


class LookupClient:
    def __init__(self, url: str, timeout_ms: int = 5000, engine=None):
        self.url = url
        self.engine = engine  # same-process shortcut
        self.timeout_ms = timeout_ms
        self._sock = None
        self._lock = threading.Lock()

    def _socket(self):
        if self._sock is None:
            s = zmq.Context.instance().socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
            s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
            s.connect(self.url)
            self._sock = s
        return self._sock

    def _call(self, lookup_id: str, tokens: List[int], op: str) -> int:
        with self._lock:
            s = self._socket()
            try:
                s.send(msgpack.packb([lookup_id, tokens, op]))
                return int(msgpack.unpackb(s.recv()))
            except zmq.Again:
                s.close()
                self._sock = None
                logger.warning("lookup server %s timed out; treating as a miss", self.url)
                return 0

    def lookup(self, tokens, lookup_id: str) -> int:
        toks = normalize_tokens(tokens)
        if self.engine is not None:
            import torch

            return self.engine.lookup(torch.tensor(toks, dtype=torch.long),
                                      lookup_id=lookup_id, pin=True)
        return self._call(lookup_id, toks, "lookup")

    def unpin(self, lookup_id: str) -> None:
        if self.engine is not None:
            self.engine.lookup_unpin(lookup_id)
        else:
            self._call(lookup_id, [], "unpin")

    def close(self):
        if self._sock is not None:
            self._sock.close()
