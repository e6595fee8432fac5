"""Layerwise CPU fill: held CPU pages and a window of asynchronous puts.

Contract (the reference's lmcache_ascend/v1/layerwise_cpu_fill.py:16-174
defines the same two duties; the design below is this repo's own):

* :class:`PageHold` -- while something the allocator cannot see (a DMA
  engine, a remote fill) still reads CPU chunk pages, those pages must not
  be reused.  A hold takes one reference on every distinct page it is given
  and gives all of them back exactly once.
* :class:`PutWindow` -- layerwise stores hand each layer's chunks to the
  slower tiers as asynchronous puts.  The window bounds what is in flight
  (bytes and batches), so the model thread only waits when a bound is hit;
  it learns of completions through future callbacks (no polling), keeps the
  first failure (a put that failed leaves a later lookup hit unproven, so the
  error stays raised), and fences by request, including requests that reuse
  chunks whose puts are still running.
"""

from __future__ import annotations

import threading
import time
from concurrent.futures import Future
from typing import Any, Dict, Iterable, List, Optional, Sequence, Set


class PageHold:
    """One reference on each distinct CPU page in ``pages`` until
    :meth:`release` (idempotent; also the context-manager exit)."""

    def __init__(self, pages: Sequence[Any]):
        distinct: Dict[int, Any] = {}
        for p in pages:
            distinct.setdefault(id(p), p)
        for p in distinct.values():  # check everything before touching counts
            raw = getattr(p, "raw_data", None)
            if not getattr(p, "is_valid", False) or raw is None or raw.device.type != "cpu":
                raise ValueError("a page hold needs valid CPU pages")
        self._held = tuple(distinct.values())
        for p in self._held:
            p.ref_count_up()
        self._gone = threading.Event()

    @property
    def num_pages(self) -> int:
        return 0 if self._gone.is_set() else len(self._held)

    def release(self) -> None:
        if self._gone.is_set():
            return
        self._gone.set()
        held, self._held = self._held, ()
        for p in held:
            p.ref_count_down()

    def __enter__(self) -> "PageHold":
        return self

    def __exit__(self, *exc) -> None:
        self.release()


class _Batch:
    __slots__ = ("size", "left", "reqs", "keys")

    def __init__(self, size: int, n: int):
        self.size, self.left = size, n
        self.reqs: Set[str] = set()
        self.keys: List[Any] = []


class PutWindow:
    """Bounded set of in-flight put batches.

    ``admit(size)`` blocks until a batch of ``size`` bytes fits (an empty
    window always takes one batch, however large); ``submit`` registers the
    batch's futures; ``fence(req_ids)`` / ``fence_all()`` wait for puts.  Every
    wait is bounded by ``timeout`` seconds; running out is a failure too.
    """

    def __init__(self, max_bytes: int, max_batches: int, timeout: float):
        if max_bytes <= 0 or max_batches <= 0 or timeout < 0:
            raise ValueError("put window limits must be positive and the timeout >= 0")
        self.max_bytes, self.max_batches = int(max_bytes), int(max_batches)
        self.timeout = float(timeout)
        self._cv = threading.Condition()
        self._live: Set[_Batch] = set()
        self._bytes = 0
        self._by_req: Dict[str, Set[_Batch]] = {}
        self._by_key: Dict[Any, Set[_Batch]] = {}
        self._error: Optional[BaseException] = None

    # ---------------------------------------------------------- state
    @property
    def inflight_batches(self) -> int:
        with self._cv:
            return len(self._live)

    @property
    def inflight_bytes(self) -> int:
        with self._cv:
            return self._bytes

    @property
    def error(self) -> Optional[BaseException]:
        return self._error

    def record_failure(self, err: BaseException) -> None:
        """Latch a failure seen outside the futures (a submit that raised)."""
        with self._cv:
            if self._error is None:
                self._error = err
            self._cv.notify_all()

    def check(self) -> None:
        if self._error is not None:
            raise self._error

    # ------------------------------------------------------ completion
    def _retire(self, b: _Batch) -> None:  # under the lock
        self._live.discard(b)
        self._bytes -= b.size
        for table, names in ((self._by_req, b.reqs), (self._by_key, b.keys)):
            for n in names:
                s = table.get(n)
                if s is not None:
                    s.discard(b)
                    if not s:
                        del table[n]

    def _on_done(self, b: _Batch, fut: Future) -> None:
        err = fut.exception() if not fut.cancelled() else RuntimeError("put cancelled")
        with self._cv:
            if err is not None and self._error is None:
                self._error = err
            b.left -= 1
            if b.left == 0:
                self._retire(b)
            self._cv.notify_all()

    # -------------------------------------------------------- waiting
    def _wait(self, ready, what: str) -> None:
        """Wait (bounded) until ``ready()`` holds; raises the latched error."""
        deadline = time.monotonic() + self.timeout
        with self._cv:
            while True:
                if self._error is not None:
                    raise self._error
                if ready():
                    return
                left = deadline - time.monotonic()
                if left <= 0:
                    self._error = TimeoutError(f"layerwise puts: {what} timed out")
                    raise self._error
                self._cv.wait(left)

    def admit(self, size: int) -> None:
        self._wait(lambda: not self._live or (len(self._live) < self.max_batches and
                                              self._bytes + size <= self.max_bytes),
                   "admission")

    def submit(self, size: int, futures: Sequence[Optional[Future]], *, req_id: str = "",
               keys: Iterable[Any] = ()) -> None:
        """Register a batch the caller just submitted (after :meth:`admit`)."""
        futs = [f for f in futures if f is not None]
        if not futs:
            return
        b = _Batch(int(size), len(futs))
        with self._cv:
            self._live.add(b)
            self._bytes += b.size
            if req_id:
                b.reqs.add(req_id)
                self._by_req.setdefault(req_id, set()).add(b)
            for k in keys:
                b.keys.append(k)
                self._by_key.setdefault(k, set()).add(b)
        for f in futs:  # may run the callback at once (already finished)
            f.add_done_callback(lambda fut, b=b: self._on_done(b, fut))

    def inherit(self, req_id: str, keys: Iterable[Any]) -> None:
        """``req_id`` reuses chunks whose puts may still run: its fence
        covers them too."""
        if not req_id:
            return
        with self._cv:
            for k in keys:
                for b in self._by_key.get(k, ()):
                    b.reqs.add(req_id)
                    self._by_req.setdefault(req_id, set()).add(b)

    def fence(self, req_ids: Iterable[str]) -> None:
        ids = list(req_ids)
        self._wait(lambda: not any(self._by_req.get(r) for r in ids), "request fence")

    def fence_all(self) -> None:
        self._wait(lambda: not self._live, "drain")
