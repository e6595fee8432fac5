"""Fixed-cardinality RemoteFill metrics, admission reports and Prometheus
gauges (the reference keeps the same kind of bounded aggregates:
lmcache_ascend/v1/remote_fill.py:218-269 decoder gauges,
remote_fill_producer.py:253 producer counters).

Only names from fixed sets enter an aggregate -- never request ids, session
ids, keys or addresses -- so a long-running server exports a bounded number of
series.  An unknown reason or outcome is counted as "other".
"""

from __future__ import annotations

import threading
from typing import Dict, Mapping, Optional

DECODER_GAUGES = ("active_sessions", "active_windows", "active_bytes")
DECODER_COUNTERS = ("reserved_bytes_total", "published_bytes_total",
                    "discarded_bytes_total", "capacity_rejections_total",
                    "expired_sessions_total", "aborted_sessions_total",
                    "finished_sessions_total", "verify_failures_total")

PRODUCER_OUTCOMES = ("LOCAL_FULL", "PERSISTENT_ONLY", "PERSISTENCE_FAILED", "ABORTED")
PRODUCER_REASONS = ("none", "circuit_open", "admission_timeout", "open_rejected",
                    "reservation_rejected", "arm_rejected", "transfer_failed",
                    "verify_failed", "control_timeout", "finish_rejected", "other")
PRODUCER_GAUGES = ("active_sessions", "inflight_bytes", "circuit_open_peers")

_PROM_LOCK = threading.Lock()
_PROM: Dict[str, object] = {}


def _gauge(name: str, doc: str):
    """A process-wide Prometheus gauge (created once; None without the
    client library or on a registration conflict)."""
    with _PROM_LOCK:
        if name in _PROM:
            return _PROM[name]
        g = None
        try:
            from prometheus_client import Gauge

            g = Gauge(name, doc)
        except Exception:
            g = None
        _PROM[name] = g
        return g


def publish(prefix: str, snapshot: Mapping[str, float]) -> None:
    for k, v in snapshot.items():
        g = _gauge(f"lmcache_b200_remote_fill_{prefix}_{k}", f"remote fill {prefix} {k}")
        if g is not None:
            g.set(float(v))


class DecoderMetrics:
    def __init__(self):
        self._lock = threading.Lock()
        self.values: Dict[str, float] = {k: 0 for k in DECODER_GAUGES + DECODER_COUNTERS}

    def add(self, name: str, v: float = 1) -> None:
        if name not in self.values:
            raise KeyError(f"not a decoder metric: {name}")
        with self._lock:
            self.values[name] += v

    def snapshot(self) -> Dict[str, float]:
        with self._lock:
            return dict(self.values)

    def publish(self) -> None:
        publish("decoder", self.snapshot())


class ProducerMetrics:
    def __init__(self):
        self._lock = threading.Lock()
        self.outcomes: Dict[str, int] = {o: 0 for o in PRODUCER_OUTCOMES}
        self.reasons: Dict[str, int] = {r: 0 for r in PRODUCER_REASONS}
        self.gauges: Dict[str, float] = {g: 0 for g in PRODUCER_GAUGES}
        self.bytes: Dict[str, int] = {"submitted": 0, "published": 0, "discarded": 0}

    def outcome(self, outcome: str, reason: str = "none", nbytes: int = 0) -> None:
        o = outcome if outcome in self.outcomes else "ABORTED"
        r = reason if reason in self.reasons else "other"
        with self._lock:
            self.outcomes[o] += 1
            self.reasons[r] += 1
            self.bytes["published" if o == "LOCAL_FULL" else "discarded"] += nbytes

    def submitted(self, nbytes: int) -> None:
        with self._lock:
            self.bytes["submitted"] += nbytes

    def set_gauge(self, name: str, v: float) -> None:
        if name not in self.gauges:
            raise KeyError(f"not a producer gauge: {name}")
        with self._lock:
            self.gauges[name] = v

    def snapshot(self) -> Dict[str, float]:
        with self._lock:
            out = {f"outcome_{k}": v for k, v in self.outcomes.items()}
            out.update({f"reason_{k}": v for k, v in self.reasons.items()})
            out.update({f"{k}_bytes": v for k, v in self.bytes.items()})
            out.update(self.gauges)
            return out

    def publish(self) -> None:
        publish("producer", self.snapshot())


def classify(reason: str) -> str:
    """Bounded reason label of a failure message."""
    r = reason.lower()
    for needle, label in (("circuit", "circuit_open"), ("admission", "admission_timeout"),
                          ("open", "open_rejected"), ("reserve", "reservation_rejected"),
                          ("arm", "arm_rejected"), ("verification", "verify_failed"),
                          ("did not answer", "control_timeout"),
                          ("finish", "finish_rejected"), ("transfer", "transfer_failed")):
        if needle in r:
            return label
    return "other"
