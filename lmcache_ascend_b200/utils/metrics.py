"""Counters, phase timers and Prometheus export.

The reference logs throughput lines and exports Prometheus gauges for its
RemoteFill path (reference lmcache_ascend/v1/remote_fill.py:218-269) and
relies on upstream ``stats_monitor`` phase timers
(reference lmcache_ascend/v1/cache_engine.py:3540-3643).  Here one
process-wide ``Stats`` object holds counters and phase timers; when
``prometheus_client`` is importable the same values are exported.
"""

from __future__ import annotations

import threading
import time
from collections import defaultdict
from contextlib import contextmanager
from typing import Dict

try:
    import prometheus_client as _prom
except Exception:  # pragma: no cover
    _prom = None


class Stats:
    def __init__(self):
        self._lock = threading.Lock()
        self.counters: Dict[str, float] = defaultdict(float)
        self.timers: Dict[str, float] = defaultdict(float)
        self.timer_counts: Dict[str, int] = defaultdict(int)
        self._prom_counters = {}

    def inc(self, name: str, v: float = 1.0) -> None:
        with self._lock:
            self.counters[name] += v
        if _prom is not None:
            c = self._prom_counters.get(name)
            if c is None:
                try:
                    c = _prom.Counter("lmcache_b200_" + name, name)
                except ValueError:  # already registered in this process
                    c = None
                self._prom_counters[name] = c
            if c is not None:
                c.inc(v)

    @contextmanager
    def phase(self, name: str):
        t0 = time.perf_counter()
        try:
            yield
        finally:
            dt = time.perf_counter() - t0
            with self._lock:
                self.timers[name] += dt
                self.timer_counts[name] += 1

    def snapshot(self) -> dict:
        with self._lock:
            return {"counters": dict(self.counters), "timers_s": dict(self.timers),
                    "timer_counts": dict(self.timer_counts)}

    def reset(self) -> None:
        with self._lock:
            self.counters.clear()
            self.timers.clear()
            self.timer_counts.clear()


_STATS = Stats()


def get_stats() -> Stats:
    return _STATS
