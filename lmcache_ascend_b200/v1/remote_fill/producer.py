"""Producer (prefiller) side of RemoteFill.

``fill`` runs one request's session against a decoder: NEGOTIATE (once per
decoder), OPEN, then per planned window RESERVE_WINDOW -> ARM_WINDOW -> data
plane transfer -> REPORT_TRANSFER_COMPLETE, then FINISH.  Every verb has a
deadline; a lost reply is retried with the same ``op_id`` (the decoder
replays its recorded answer).  Any failure sends ABORT (best effort), counts
against the decoder in the circuit breaker and runs ``fallback`` (the
persistent path: store to the shared tier so the decoder loads or
recomputes).  Admission bounds sessions and bytes in flight.
"""

from __future__ import annotations

import time
import uuid
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional

import msgpack
import numpy as np
import torch
import zmq

from ...utils.logging import init_logger
from .coordinator import Admission, CircuitBreaker
from .metrics import ProducerMetrics, classify
from .planning import plan_windows

logger = init_logger(__name__)


class CopyDataPlane:
    """Same-process data plane (host tests, single-process serving): moves
    rows from the source layout to the destination layout directly."""

    def __init__(self, src_layout, dst_layout):
        self.src, self.dst = src_layout, dst_layout

    def transfer(self, src_slots: torch.Tensor, dst_slots: torch.Tensor) -> None:
        n = src_slots.numel()
        buf = torch.empty(self.src.chunk_shape(n), dtype=self.src.dtype,
                          device=self.src.device)
        self.src.gather_ref(buf, src_slots)
        self.dst.scatter_ref(buf.to(self.dst.device), dst_slots.to(self.dst.device))


class PushDataPlane:
    """NVLink push kernel into the decoder's paged blocks (asynchronous: the
    decoder verifies arrival through its per-layer flags)."""

    def __init__(self, sender, tile_tokens: int = 128):
        self.sender, self.tile = sender, tile_tokens

    def transfer(self, src_slots: torch.Tensor, dst_slots: torch.Tensor) -> None:
        dev = self.sender.device
        self.sender.push(src_slots.to(dev), dst_slots.to(dev), tile_tokens=self.tile)


@dataclass
class FillResult:
    req_id: str
    ok: bool
    windows: int = 0
    ready_tokens: int = 0
    fell_back: bool = False
    reason: str = ""


class RemoteFillProducer:
    def __init__(self, decoder_url: str, data_plane, window_tokens: int = 2048,
                 block_size: int = 16, op_timeout_s: float = 5.0, retries: int = 2,
                 admission: Optional[Admission] = None,
                 breaker: Optional[CircuitBreaker] = None,
                 fallback: Optional[Callable[[str], None]] = None):
        self.url = decoder_url
        self.plane = data_plane
        self.window_tokens, self.block_size = window_tokens, block_size
        self.timeout_ms = int(op_timeout_s * 1000)
        self.retries = retries
        self.admission = admission or Admission()
        self.breaker = breaker or CircuitBreaker()
        self.fallback = fallback
        self.ctx = zmq.Context.instance()
        self._sock = None
        self._negotiated: Optional[Dict] = None
        self.results: List[FillResult] = []
        self.metrics = ProducerMetrics()

    # ------------------------------------------------------------- rpc
    def _socket(self):
        if self._sock is None:
            s = self.ctx.socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
            s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
            s.connect(self.url)
            self._sock = s
        return self._sock

    def _reset(self) -> None:
        if self._sock is not None:
            self._sock.close()
            self._sock = None

    def _rpc(self, op: str, session: str, payload=None, op_id: Optional[str] = None):
        op_id = op_id or uuid.uuid4().hex
        msg = msgpack.packb([op, session, op_id, payload], use_bin_type=True)
        for attempt in range(self.retries + 1):
            try:
                s = self._socket()
                s.send(msg)
                st, res = msgpack.unpackb(s.recv(), raw=False)
            except zmq.Again:
                self._reset()  # a REQ socket that lost its reply cannot send again
                logger.warning("remote fill %s timed out (attempt %d)", op, attempt + 1)
                continue
            if st != "ok":
                raise RuntimeError(f"{op}: {res}")
            return res
        raise TimeoutError(f"decoder did not answer {op}")

    # ------------------------------------------------------------ fill
    def fill(self, req_id: str, src_slots: torch.Tensor, num_tokens: Optional[int] = None,
             nbytes: int = 0, admit_timeout_s: float = 5.0) -> FillResult:
        n = int(src_slots.numel() if num_tokens is None else num_tokens)
        self.metrics.submitted(nbytes)
        if not self.breaker.allow(self.url):
            return self._fail(req_id, "circuit open for the decoder", sent_open=None)
        if not self.admission.acquire(nbytes, admit_timeout_s):
            return self._fail(req_id, "admission timed out", sent_open=None, count=False)
        session = None
        try:
            if self._negotiated is None:
                self._negotiated = self._rpc("NEGOTIATE", "", {"version": 1})
            wmax = int(self._negotiated.get("max_window_tokens", self.window_tokens))
            session = self._rpc("OPEN", "", {"req_id": req_id, "num_tokens": n})["session"]
            windows = plan_windows(n, self.block_size, min(self.window_tokens, wmax))
            for w, (a, b) in enumerate(windows):
                r = self._rpc("RESERVE_WINDOW", session, {"window": w, "start": a, "end": b})
                dst = torch.from_numpy(np.frombuffer(r["dst_slots"], dtype=np.int64).copy())
                self._rpc("ARM_WINDOW", session, {"window": w})
                self.plane.transfer(src_slots[a:b], dst)
                self._rpc("REPORT_TRANSFER_COMPLETE", session, {"window": w})
            done = self._rpc("FINISH", session)
            self.breaker.success(self.url)
            res = FillResult(req_id, True, len(windows), int(done["ready_tokens"]))
            self.results.append(res)
            self.metrics.outcome("LOCAL_FULL", "none", nbytes)
            return res
        except (RuntimeError, TimeoutError, KeyError, ValueError) as e:
            return self._fail(req_id, str(e), sent_open=session)
        finally:
            self.admission.release(nbytes)

    def _fail(self, req_id: str, reason: str, sent_open: Optional[str],
              count: bool = True) -> FillResult:
        if sent_open:
            try:
                self._rpc("ABORT", sent_open, {"reason": reason})
            except (RuntimeError, TimeoutError):
                pass
        if count:
            self.breaker.failure(self.url)
        fell_back = False
        if self.fallback is not None:
            self.fallback(req_id)
            fell_back = True
        logger.warning("remote fill of %s failed (%s)%s", req_id, reason,
                       "; persistent fallback" if fell_back else "")
        res = FillResult(req_id, False, fell_back=fell_back, reason=reason)
        self.results.append(res)
        self.metrics.outcome("PERSISTENT_ONLY" if fell_back else "ABORTED", classify(reason))
        return res

    def admission_report(self, publish: bool = False) -> dict:
        """Admission and breaker state plus the bounded outcome counters."""
        self.metrics.set_gauge("active_sessions", self.admission.sessions)
        self.metrics.set_gauge("inflight_bytes", self.admission.bytes)
        self.metrics.set_gauge("circuit_open_peers", self.breaker.open_peers())
        rep = {"admission": self.admission.report(), "metrics": self.metrics.snapshot()}
        if publish:
            self.metrics.publish()
        return rep

    def status(self, session: str) -> dict:
        return self._rpc("STATUS", session)

    def close(self) -> None:
        self._reset()
