"""TCP (ZMQ) channel: host buffers moved as messages.

Used by the CPU test tier and as the cross-box fallback when peers do not
share an NVLink domain.  Every channel runs a small data server (ZMQ REP)
that applies page writes to its registered buffers and serves page reads;
``batched_write`` / ``batched_read`` are one request per batch.
"""

from __future__ import annotations

import threading
from typing import Dict, List, Optional, Sequence, Tuple

import msgpack
import torch
import zmq

from ...utils.logging import init_logger
from .base import BaseTransferChannel, BufferConfig, CompletedEvent, RemoteAddr, RemoteBuffer

logger = init_logger(__name__)


class TCPChannel(BaseTransferChannel):
    def __init__(self, peer_id: str, endpoint: str = "tcp://127.0.0.1:*", buffers=None,
                 timeout_ms: int = 10000):
        super().__init__(peer_id, buffers)
        self.ctx = zmq.Context.instance()
        self.timeout_ms = timeout_ms
        self._srv = self.ctx.socket(zmq.REP)
        self._srv.setsockopt(zmq.LINGER, 0)
        if endpoint.endswith(":*"):
            port = self._srv.bind_to_random_port(endpoint[:-2])
            self.endpoint = f"{endpoint[:-2]}:{port}"
        else:
            self._srv.bind(endpoint)
            self.endpoint = endpoint
        self._peer_eps: Dict[str, str] = {}
        self._socks: Dict[str, zmq.Socket] = {}
        self._stop = threading.Event()
        self._thr = threading.Thread(target=self._serve, name="lmc-tcp-chan", daemon=True)
        self._thr.start()

    def _export(self, buf: BufferConfig) -> dict:
        if buf.tensor.is_cuda:
            raise ValueError("TCP channel serves host buffers only")
        return {"uuid": buf.uuid, "kind": "host", "nbytes": buf.nbytes,
                "page_bytes": buf.page_bytes, "endpoint": self.endpoint}

    def lazy_init_peer_connection(self, peer_id: str, refs: List[dict],
                                  endpoint: Optional[str] = None) -> None:
        mapped = {r["uuid"]: RemoteBuffer(r["uuid"], "host", r["nbytes"], r["page_bytes"])
                  for r in refs}
        ep = endpoint or (refs[0]["endpoint"] if refs else None)
        with self._lock:
            self.remote[peer_id] = mapped
            if ep:
                self._peer_eps[peer_id] = ep

    def _sock(self, peer_id: str) -> zmq.Socket:
        s = self._socks.get(peer_id)
        if s is None:
            s = self.ctx.socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
            s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
            s.connect(self._peer_eps[peer_id])
            self._socks[peer_id] = s
        return s

    def _rpc(self, peer_id: str, msg) -> list:
        s = self._sock(peer_id)
        try:
            s.send(msgpack.packb(msg, use_bin_type=True))
            return msgpack.unpackb(s.recv(), raw=False)
        except zmq.Again:
            # a REQ socket that timed out is unusable: drop it
            s.close()
            self._socks.pop(peer_id, None)
            raise TimeoutError(f"TCP channel: peer {peer_id} did not answer")

    def _serve(self) -> None:
        poller = zmq.Poller()
        poller.register(self._srv, zmq.POLLIN)
        while not self._stop.is_set():
            if not poller.poll(100):
                continue
            req = msgpack.unpackb(self._srv.recv(), raw=False)
            try:
                op, items = req
                out = []
                for it in items:
                    buf = self.local[it[0]]
                    off = it[1] * buf.page_bytes
                    if op == "w":
                        data = it[2]
                        buf.tensor[off:off + len(data)].copy_(
                            torch.frombuffer(bytearray(data), dtype=torch.uint8))
                    else:
                        out.append(bytes(buf.tensor[off:off + it[2]].numpy().tobytes()))
                self._srv.send(msgpack.packb(["ok", out], use_bin_type=True))
            except Exception as e:  # report, keep serving
                self._srv.send(msgpack.packb(["err", str(e)], use_bin_type=True))

    @staticmethod
    def _host_bytes(ptr: int, n: int) -> bytes:
        import ctypes

        return ctypes.string_at(ptr, n)

    def batched_write(self, srcs: Sequence[Tuple[int, int]], peer_id: str,
                      remote: Sequence[RemoteAddr], sync: bool = True):
        items = [[a[0], a[1], self._host_bytes(p, n)] for (p, n), a in zip(srcs, remote)]
        st, payload = self._rpc(peer_id, ["w", items])
        if st != "ok":
            raise RuntimeError(f"remote write failed: {payload}")
        return CompletedEvent()

    def batched_read(self, dsts: Sequence[Tuple[int, int]], peer_id: str,
                     remote: Sequence[RemoteAddr], sync: bool = True):
        import ctypes

        st, payload = self._rpc(peer_id, ["r", [[a[0], a[1], n] for (_, n), a in
                                                zip(dsts, remote)]])
        if st != "ok":
            raise RuntimeError(f"remote read failed: {payload}")
        for (p, n), data in zip(dsts, payload):
            ctypes.memmove(p, data, n)
        return CompletedEvent()

    def close(self) -> None:
        self._stop.set()
        self._thr.join(timeout=2)
        for s in self._socks.values():
            s.close()
        self._srv.close()
