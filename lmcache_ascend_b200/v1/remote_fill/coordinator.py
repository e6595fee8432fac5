"""Admission and per-peer circuit breaking for RemoteFill producers
(reference lmcache_ascend/v1/remote_fill_coordinator.py:77-1528): at most
``max_sessions`` sessions and ``max_bytes`` in flight (a single request larger
than the byte limit is admitted into an otherwise idle producer); a peer whose
fills failed ``threshold`` times in a row is skipped for ``ttl_s`` seconds."""

from __future__ import annotations

import threading
import time
from typing import Dict


class Admission:
    def __init__(self, max_sessions: int = 8, max_bytes: int = 8 << 30):
        self.max_sessions, self.max_bytes = max_sessions, max_bytes
        self.sessions = 0
        self.bytes = 0
        self.admitted = self.waited = self.rejected = 0
        self._cv = threading.Condition()

    def acquire(self, nbytes: int, timeout_s: float) -> bool:
        deadline = time.monotonic() + timeout_s
        with self._cv:
            waited = False
            while self.sessions >= self.max_sessions or (
                    self.sessions > 0 and self.bytes + nbytes > self.max_bytes):
                left = deadline - time.monotonic()
                if left <= 0:
                    self.rejected += 1
                    return False
                waited = True
                self._cv.wait(left)
            self.sessions += 1
            self.bytes += nbytes
            self.admitted += 1
            self.waited += int(waited)
            return True

    def report(self) -> dict:
        """Admission state for operators (bounded fields only)."""
        with self._cv:
            return {"sessions": self.sessions, "bytes": self.bytes,
                    "max_sessions": self.max_sessions, "max_bytes": self.max_bytes,
                    "admitted_total": self.admitted, "waited_total": self.waited,
                    "rejected_total": self.rejected}

    def release(self, nbytes: int) -> None:
        with self._cv:
            self.sessions = max(0, self.sessions - 1)
            self.bytes = max(0, self.bytes - nbytes)
            self._cv.notify_all()


class CircuitBreaker:
    def __init__(self, threshold: int = 3, ttl_s: float = 30.0, clock=time.monotonic):
        self.threshold, self.ttl_s, self.clock = threshold, ttl_s, clock
        self._fails: Dict[str, int] = {}
        self._open_until: Dict[str, float] = {}
        self._lock = threading.Lock()

    def allow(self, peer: str) -> bool:
        with self._lock:
            until = self._open_until.get(peer)
            if until is None:
                return True
            if self.clock() >= until:  # half-open: one more try
                del self._open_until[peer]
                self._fails[peer] = self.threshold - 1
                return True
            return False

    def success(self, peer: str) -> None:
        with self._lock:
            self._fails.pop(peer, None)
            self._open_until.pop(peer, None)

    def open_peers(self) -> int:
        with self._lock:
            now = self.clock()
            return sum(1 for t in self._open_until.values() if t > now)

    def failure(self, peer: str) -> None:
        with self._lock:
            n = self._fails.get(peer, 0) + 1
            self._fails[peer] = n
            if n >= self.threshold:
                self._open_until[peer] = self.clock() + self.ttl_s
