"""Decoder side of RemoteFill: the session service.

Verbs (one msgpack request ``[op, session, op_id, payload]`` -> ``["ok"|"err",
payload]``):
  NEGOTIATE                 version and limits (max window tokens)
  OPEN                      new session for a request: {req_id, num_tokens}
  RESERVE_WINDOW            {window, start, end} -> destination slots of the window
  ARM_WINDOW                {window}: arm completion tracking before the producer writes
  REPORT_TRANSFER_COMPLETE  {window}: verify the window landed (bounded device wait)
  FINISH                    all windows verified: the request's KV is ready
  ABORT                     either side gives up: release everything
  STATUS                    session state
Requests are idempotent by ``op_id``: a producer that lost a reply resends the
same ``op_id`` and gets the recorded reply without the verb running twice.
A session that makes no progress for ``deadline_s`` is aborted by a sweep
thread, which releases its reservations (a producer that died mid-session
cannot pin decoder blocks).  Destination slots come from ``slot_provider``
(the decoder's scheduler: the request's block table).
"""

from __future__ import annotations

import threading
import time
import uuid
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Callable, Dict, Optional, Tuple

import msgpack
import numpy as np
import torch
import zmq

from ...utils.logging import init_logger
from .metrics import DecoderMetrics

logger = init_logger(__name__)

PROTOCOL_VERSION = 1
OPENED, RESERVED, ARMED, VERIFIED, FINISHED, ABORTED = (
    "OPENED", "RESERVED", "ARMED", "VERIFIED", "FINISHED", "ABORTED")


class CopyVerifier:
    """Completion check of a synchronous data plane: nothing to wait for."""

    def arm(self, num_tokens: int):
        return None

    def verify(self, token) -> bool:
        return True


class PushVerifier:
    """Completion of an NVLink push: the per-layer flags reach the counts the
    window adds (bounded device wait), and the receiver's status stays clean."""

    def __init__(self, receiver, tile_tokens: int = 128, timeout_s: float = 5.0):
        self.receiver, self.tile, self.timeout_s = receiver, tile_tokens, timeout_s

    def arm(self, num_tokens: int):
        return self.receiver.expect(num_tokens, tile_tokens=self.tile)

    def verify(self, targets) -> bool:
        self.receiver.wait(targets, timeout_s=self.timeout_s)
        torch.cuda.synchronize(self.receiver.device)
        code = int(self.receiver.status.tensor[0].item())
        if code != 0:
            self.receiver.status.tensor.zero_()
            return False
        return True


@dataclass
class _Session:
    req_id: str
    num_tokens: int
    slots: torch.Tensor
    state: str = OPENED
    windows: Dict[int, Tuple[int, int]] = field(default_factory=dict)
    armed: Dict[int, object] = field(default_factory=dict)
    verified: set = field(default_factory=set)
    last: float = field(default_factory=time.monotonic)
    replies: Dict[str, list] = field(default_factory=dict)


class RemoteFillService:
    def __init__(self, slot_provider: Callable[[str, int], Optional[torch.Tensor]],
                 verifier=None, host: str = "127.0.0.1", port: int = 0,
                 deadline_s: float = 10.0, max_window_tokens: int = 4096,
                 on_ready: Optional[Callable[[str, int], None]] = None,
                 on_abort: Optional[Callable[[str, str], None]] = None,
                 data_plane_desc: Optional[dict] = None, max_sessions: int = 64):
        self.slot_provider = slot_provider
        self.verifier = verifier or CopyVerifier()
        self.deadline_s = deadline_s
        self.max_window_tokens = max_window_tokens
        self.on_ready, self.on_abort = on_ready, on_abort
        self.data_plane_desc = data_plane_desc
        self.sessions: Dict[str, _Session] = {}
        self.ready: Dict[str, int] = {}
        self.aborted: Dict[str, str] = {}
        self._lock = threading.RLock()
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.host = host
        self.port = self.sock.bind_to_random_port(f"tcp://{host}") if port == 0 else port
        if port:
            self.sock.bind(f"tcp://{host}:{port}")
        self._stop = threading.Event()
        self._threads = []
        self._open_replies: "OrderedDict[str, list]" = OrderedDict()  # session-less verbs
        self.metrics = DecoderMetrics()
        self.max_sessions = max_sessions

    @property
    def url(self) -> str:
        return f"tcp://{self.host}:{self.port}"

    token_bytes = 0  # bytes of one token's KV (set by the caller; 0 counts tokens only)

    def metrics_snapshot(self, publish: bool = False) -> dict:
        snap = self.metrics.snapshot()
        if publish:
            self.metrics.publish()
        return snap

    # ------------------------------------------------------------ verbs
    def _active(self, s: "_Session") -> int:
        return sum(b - a for a, b in s.windows.values())

    def _retire(self, s: "_Session", published: bool) -> None:
        m = self.metrics
        m.add("active_sessions", -1)
        m.add("active_windows", -len(s.windows))
        nbytes = self._active(s) * self.token_bytes
        m.add("active_bytes", -nbytes)
        m.add("published_bytes_total" if published else "discarded_bytes_total", nbytes)

    def _abort(self, sid: str, why: str) -> None:
        s = self.sessions.get(sid)
        if s is None or s.state in (FINISHED, ABORTED):
            return
        s.state = ABORTED
        self._retire(s, published=False)
        self.metrics.add("aborted_sessions_total")
        if why == "deadline expired":
            self.metrics.add("expired_sessions_total")
        s.armed.clear()
        self.aborted[s.req_id] = why
        logger.warning("remote fill session %s (%s) aborted: %s", sid, s.req_id, why)
        if self.on_abort:
            self.on_abort(s.req_id, why)

    def _handle(self, op: str, sid: str, p: dict):
        if op == "NEGOTIATE":
            return {"version": PROTOCOL_VERSION, "max_window_tokens": self.max_window_tokens,
                    "data_plane": self.data_plane_desc}
        if op == "OPEN":
            active = sum(1 for x in self.sessions.values() if x.state not in (FINISHED, ABORTED))
            if active >= self.max_sessions:
                self.metrics.add("capacity_rejections_total")
                raise RuntimeError("decoder at its session capacity")
            slots = self.slot_provider(p["req_id"], int(p["num_tokens"]))
            if slots is None or slots.numel() < int(p["num_tokens"]):
                self.metrics.add("capacity_rejections_total")
                raise RuntimeError("no destination blocks for the request")
            sid = uuid.uuid4().hex
            self.sessions[sid] = _Session(p["req_id"], int(p["num_tokens"]), slots)
            self.metrics.add("active_sessions")
            return {"session": sid}
        s = self.sessions.get(sid)
        if s is None:
            raise KeyError(f"unknown session {sid}")
        if op == "STATUS":
            return {"state": s.state, "verified": sorted(s.verified), "req_id": s.req_id}
        if op == "ABORT":
            self._abort(sid, p.get("reason", "producer abort"))
            return {"state": s.state}
        if s.state in (FINISHED, ABORTED):
            raise RuntimeError(f"session is {s.state}")
        s.last = time.monotonic()
        w = int(p.get("window", -1))
        if op == "RESERVE_WINDOW":
            a, b = int(p["start"]), int(p["end"])
            if not (0 <= a < b <= s.num_tokens) or b - a > self.max_window_tokens:
                raise ValueError("window outside the request or too large")
            if w not in s.windows:
                self.metrics.add("active_windows")
                self.metrics.add("active_bytes", (b - a) * self.token_bytes)
                self.metrics.add("reserved_bytes_total", (b - a) * self.token_bytes)
            s.windows[w] = (a, b)
            s.state = RESERVED
            return {"dst_slots": s.slots[a:b].cpu().numpy().astype(np.int64).tobytes()}
        if op == "ARM_WINDOW":
            a, b = s.windows[w]
            s.armed[w] = self.verifier.arm(b - a)
            s.state = ARMED
            return {"armed": w}
        if op == "REPORT_TRANSFER_COMPLETE":
            if w not in s.armed:
                raise RuntimeError("window was not armed")
            if not self.verifier.verify(s.armed.pop(w)):
                self.metrics.add("verify_failures_total")
                self._abort(sid, f"window {w} failed verification")
                raise RuntimeError(f"window {w} failed verification")
            s.verified.add(w)
            s.state = VERIFIED
            return {"verified": w}
        if op == "FINISH":
            if set(s.windows) != s.verified:
                raise RuntimeError("FINISH before every window was verified")
            covered = sum(b - a for a, b in s.windows.values())
            s.state = FINISHED
            self._retire(s, published=True)
            self.metrics.add("finished_sessions_total")
            self.ready[s.req_id] = covered
            if self.on_ready:
                self.on_ready(s.req_id, covered)
            return {"ready_tokens": covered}
        raise ValueError(f"unknown verb {op}")

    def _dispatch(self, body: bytes) -> list:
        op, sid, op_id, payload = msgpack.unpackb(body, raw=False)
        with self._lock:
            s = self.sessions.get(sid)
            cache = s.replies if s is not None else self._open_replies
            if op_id in cache:  # a lost reply: replay it, do not run the verb again
                return cache[op_id]
            try:
                res = ["ok", self._handle(op, sid, payload or {})]
            except Exception as e:
                res = ["err", f"{type(e).__name__}: {e}"]
            if op != "STATUS":
                cache[op_id] = res
                if cache is self._open_replies and len(cache) > 4096:
                    cache.popitem(last=False)
            return res

    # ------------------------------------------------------------ threads
    def _serve(self) -> None:
        poller = zmq.Poller()
        poller.register(self.sock, zmq.POLLIN)
        while not self._stop.is_set():
            if not poller.poll(50):
                continue
            ident, _, body = self.sock.recv_multipart()
            self.sock.send_multipart([ident, b"", msgpack.packb(self._dispatch(body),
                                                                use_bin_type=True)])
        self.sock.close()

    def _sweep(self) -> None:
        while not self._stop.wait(min(0.5, self.deadline_s / 4)):
            now = time.monotonic()
            with self._lock:
                for sid, s in list(self.sessions.items()):
                    if s.state not in (FINISHED, ABORTED) and now - s.last > self.deadline_s:
                        self._abort(sid, "deadline expired")

    def start(self) -> "RemoteFillService":
        for fn, name in ((self._serve, "lmc-rfill-srv"), (self._sweep, "lmc-rfill-sweep")):
            t = threading.Thread(target=fn, name=name, daemon=True)
            t.start()
            self._threads.append(t)
        return self

    def stop(self) -> None:
        self._stop.set()
        for t in self._threads:
            t.join(timeout=2)
