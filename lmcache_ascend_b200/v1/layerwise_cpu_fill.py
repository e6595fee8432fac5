"""Layerwise CPU fill: page leases and a bounded queue of asynchronous puts.

Behaviour of the reference (lmcache_ascend/v1/layerwise_cpu_fill.py:16-174):

* :class:`CPUFillLease` keeps CPU chunk pages alive (one reference each, the
  same page counted once) while a reader outside the allocator's view, such
  as a remote fill or a DMA engine, still reads them.  It proves ownership
  only; the caller waits for the producer's copies separately.  Released once.
* :class:`LayerwisePutQueue` bounds the puts that layerwise stores submit to
  slower tiers, so the model thread is not fenced every forward: admission
  waits only at a batch boundary when the byte or batch limit is reached (one
  oversized batch is admitted into an empty queue), completed puts are reaped
  out of order, failures are sticky (a later local hit does not prove the put
  persisted), and fences can target the puts of given requests, including
  puts of chunks a request reused from an earlier request.
"""

from __future__ import annotations

import threading
import time
from collections import deque
from concurrent.futures import Future, wait
from typing import Any, Deque, Dict, Iterable, List, Optional, Sequence, Set, Tuple


class CPUFillLease:
    def __init__(self, pages: Sequence[Any]):
        self._lock = threading.Lock()
        self._pages: List[Any] = []
        seen: Set[int] = set()
        try:
            for p in pages:
                if id(p) in seen:
                    continue
                seen.add(id(p))
                raw = getattr(p, "raw_data", None)
                if not p.is_valid or raw is None or raw.device.type != "cpu":
                    raise ValueError("a CPU fill lease needs valid CPU pages")
                p.ref_count_up()
                self._pages.append(p)
        except BaseException:
            self.release()
            raise

    @property
    def num_pages(self) -> int:
        return len(self._pages)

    def release(self) -> None:
        with self._lock:
            pages, self._pages = self._pages, []
        for p in pages:
            p.ref_count_down()

    def __enter__(self) -> "CPUFillLease":
        return self

    def __exit__(self, *exc) -> None:
        self.release()


class LayerwisePutQueue:
    def __init__(self, max_bytes: int, max_batches: int, timeout: float):
        if max_bytes <= 0 or max_batches <= 0 or timeout < 0:
            raise ValueError("put queue limits must be positive and the timeout >= 0")
        self.max_bytes = int(max_bytes)
        self.max_batches = int(max_batches)
        self.timeout = float(timeout)
        self.pending: Deque[Tuple[int, Tuple[Future, ...]]] = deque()
        self.pending_bytes = 0
        self.error: Optional[BaseException] = None
        self._by_req: Dict[str, Set[Future]] = {}
        self._by_key: Dict[Any, Set[Future]] = {}

    def fail(self, error: BaseException) -> None:
        """Latch a failure seen outside the futures (a synchronous submit)."""
        if self.error is None:
            self.error = error

    def _raise(self) -> None:
        if self.error is not None:
            raise self.error

    def poll(self) -> None:
        """Reap finished batches (in any order) without waiting."""
        self._raise()
        finished: Set[Future] = set()
        keep: Deque[Tuple[int, Tuple[Future, ...]]] = deque()
        keep_bytes = 0
        try:
            for size, futs in self.pending:
                all_done = True
                for f in futs:
                    if f.done():
                        f.result()  # raises the put's error
                        finished.add(f)
                    else:
                        all_done = False
                if not all_done:
                    keep.append((size, futs))
                    keep_bytes += size
        except BaseException as e:
            self.error = e
            raise
        self.pending, self.pending_bytes = keep, keep_bytes
        if finished:
            for table in (self._by_req, self._by_key):
                for k in list(table):
                    table[k] -= finished
                    if not table[k]:
                        del table[k]

    def _wait_oldest(self, deadline: float) -> None:
        _, left = wait(self.pending[0][1], timeout=max(0.0, deadline - time.monotonic()))
        if left:
            self.error = TimeoutError("layerwise puts did not complete in time")
            raise self.error
        self.poll()

    def reserve(self, size: int) -> None:
        """Wait until a batch of ``size`` bytes may be submitted."""
        self.poll()
        deadline = time.monotonic() + self.timeout
        while self.pending and (len(self.pending) >= self.max_batches or
                                self.pending_bytes + size > self.max_bytes):
            self._wait_oldest(deadline)

    def add(self, size: int, futures: Sequence[Future], *, req_id: str = "",
            keys: Iterable[Any] = ()) -> None:
        """Track a submitted batch (after :meth:`reserve`)."""
        futs = tuple(f for f in futures if f is not None)
        if not futs:
            return
        self.pending.append((int(size), futs))
        self.pending_bytes += int(size)
        if req_id:
            self._by_req.setdefault(req_id, set()).update(futs)
        for k in keys:
            self._by_key.setdefault(k, set()).update(futs)

    def track_keys(self, req_id: str, keys: Iterable[Any]) -> None:
        """A request reuses chunks whose puts may still run: fence them with it."""
        if not req_id or not self._by_key:
            return
        for k in keys:
            futs = self._by_key.get(k)
            if futs:
                self._by_req.setdefault(req_id, set()).update(futs)

    def drain_requests(self, req_ids: Iterable[str]) -> None:
        """Wait for the puts of these requests only."""
        self.poll()
        futs: Set[Future] = set()
        for r in req_ids:
            futs |= self._by_req.get(r, set())
        if futs:
            _, left = wait(futs, timeout=self.timeout)
            if left:
                self.error = TimeoutError("layerwise puts did not complete in time")
                raise self.error
        self.poll()

    def drain(self) -> None:
        """Wait for every pending put (before the allocator is torn down)."""
        self.poll()
        deadline = time.monotonic() + self.timeout
        while self.pending:
            self._wait_oldest(deadline)
        self.poll()
