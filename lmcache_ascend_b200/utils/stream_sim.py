"""CPU model of CUDA streams and events for stream-ordering tests.

Work enqueued on a ``SimStream`` does not run when it is enqueued: the
simulator executes it later, one operation at a time, in any order that
respects (a) the order of each stream and (b) event waits, choosing among the
runnable streams with a seeded random generator.  So an ordering the code did
not establish (a missing ``wait_event``, an event recorded before the work it
should cover) shows up as a different interleaving on some seed.

Memory effects are modelled on host tensors:
* a write has a start and a completion.  At its start the destination rows
  are poisoned (NaN for floating dtypes, all ones for integers) and marked as
  having a pending writer; at its completion the payload is written and the
  mark cleared.  A write is split into start and completion steps that the
  simulator may separate by other operations;
* a read fails (records a violation) if a source row has a pending writer or
  holds poison.
Checking the final contents against an independent expectation catches a
corrupted payload.  ``SimCuda`` patches ``torch.cuda.Stream/Event/stream/
current_stream`` so code written against torch's stream API runs unchanged.
"""

from __future__ import annotations

import contextlib
import random
from collections import deque
from typing import Callable, Deque, Dict, List, Optional, Sequence, Tuple

import torch


class Violation(AssertionError):
    pass


class SimEvent:
    def __init__(self, sim: "Sim"):
        self.sim = sim
        self.token: Optional[int] = None  # completion token to wait for; None: never recorded

    # torch.cuda.Event API
    def record(self, stream: Optional["SimStream"] = None) -> None:
        s = stream or self.sim.current
        self.token = s.mark()

    def query(self) -> bool:
        return self.token is None or self.token in self.sim.done

    def synchronize(self) -> None:
        if self.token is not None:
            self.sim.run_until(lambda: self.token in self.sim.done)


class SimStream:
    def __init__(self, sim: "Sim", name: str):
        self.sim, self.name = sim, name
        self.q: Deque[Tuple[str, object, int]] = deque()  # (kind, payload, token)

    def _push(self, kind: str, payload) -> int:
        tok = self.sim.next_token()
        self.q.append((kind, payload, tok))
        return tok

    def mark(self) -> int:
        return self._push("mark", None)

    def enqueue(self, fn: Callable[[], None], name: str = "op") -> int:
        return self._push("op", (fn, name))

    def enqueue_write(self, dst: torch.Tensor, rows: torch.Tensor, payload,
                      name: str = "write") -> None:
        """dst[rows] = payload (a tensor, or a callable giving it at completion),
        as a start step and a completion step."""
        self._push("wstart", (dst, rows, name))
        self._push("wend", (dst, rows, payload, name))

    def enqueue_cond_wait(self, pred: Callable[[], bool]) -> None:
        """Later work on this stream waits until ``pred()`` holds (a device-side
        spin on a flag another agent sets)."""
        self._push("cond", pred)

    def enqueue_read(self, src: torch.Tensor, rows: torch.Tensor,
                     sink: Callable[[torch.Tensor], None], name: str = "read") -> None:
        self._push("read", (src, rows, sink, name))

    # torch.cuda.Stream API
    def wait_event(self, ev: SimEvent) -> None:
        if ev.token is not None:
            self._push("wait", ev.token)

    def wait_stream(self, other: "SimStream") -> None:
        self._push("wait", other.mark())

    def synchronize(self) -> None:
        tok = self.mark()
        self.sim.run_until(lambda: tok in self.sim.done)

    def record_event(self, ev: Optional[SimEvent] = None) -> SimEvent:
        ev = ev or SimEvent(self.sim)
        ev.record(self)
        return ev


class Sim:
    def __init__(self, seed: int = 0):
        self.rng = random.Random(seed)
        self.streams: List[SimStream] = []
        self.done: set = set()
        self._tok = 0
        self.pending: Dict[int, List[Tuple[int, torch.Tensor]]] = {}  # id(t) -> writes
        self.violations: List[str] = []
        self.default = self.new_stream("default")
        self.current = self.default

    def next_token(self) -> int:
        self._tok += 1
        return self._tok

    def new_stream(self, name: str = "") -> SimStream:
        s = SimStream(self, name or f"s{len(self.streams)}")
        self.streams.append(s)
        return s

    # ------------------------------------------------------------ memory
    @staticmethod
    def _poison(t: torch.Tensor, rows: torch.Tensor) -> None:
        if t.dtype.is_floating_point:
            t[rows] = float("nan")
        else:
            t[rows] = -1

    def _pending_rows(self, t: torch.Tensor) -> List[torch.Tensor]:
        return [r for _, r in self.pending.get(id(t), [])]

    def _check_read(self, src: torch.Tensor, rows: torch.Tensor, name: str) -> None:
        for pr in self._pending_rows(src):
            if bool(torch.isin(rows, pr).any()):
                self.violations.append(f"{name}: read a row whose write has not completed")
                return
        vals = src[rows]
        bad = torch.isnan(vals).any() if vals.dtype.is_floating_point else (vals == -1).all(
            dim=-1).any() if vals.dim() > 1 else False
        if bool(bad):
            self.violations.append(f"{name}: read poisoned (never completed) data")

    # --------------------------------------------------------- execution
    def _runnable(self, s: SimStream) -> bool:
        if not s.q:
            return False
        kind, payload, _ = s.q[0]
        if kind == "wait":
            return payload in self.done
        if kind == "cond":
            return bool(payload())
        return True

    def step(self) -> bool:
        ready = [s for s in self.streams if self._runnable(s)]
        if not ready:
            return False
        s = self.rng.choice(ready)
        kind, payload, tok = s.q.popleft()
        if kind == "op":
            payload[0]()
        elif kind == "wstart":
            dst, rows, name = payload
            self._poison(dst, rows)
            self.pending.setdefault(id(dst), []).append((tok, rows))
        elif kind == "wend":
            dst, rows, data, name = payload
            dst[rows] = data() if callable(data) else data
            lst = self.pending.get(id(dst), [])
            for i, (_, r) in enumerate(lst):
                if r is rows:
                    del lst[i]
                    break
        elif kind == "read":
            src, rows, sink, name = payload
            self._check_read(src, rows, name)
            sink(src[rows].clone())
        self.done.add(tok)
        return True

    def run_until(self, cond: Callable[[], bool]) -> None:
        while not cond():
            if not self.step():
                raise Violation("deadlock: nothing runnable but the condition does not hold")

    def drain(self) -> None:
        while self.step():
            pass
        stuck = [s.name for s in self.streams if s.q]
        if stuck:
            raise Violation(f"streams never drained (a wait on an event that never "
                            f"completes): {stuck}")

    def check(self) -> None:
        if self.violations:
            raise Violation("; ".join(self.violations))


class SimCuda(contextlib.AbstractContextManager):
    """Patch torch.cuda's stream/event API onto a ``Sim`` for the duration."""

    def __init__(self, sim: Sim):
        self.sim = sim
        self._saved = {}

    def __enter__(self):
        sim = self.sim
        c = torch.cuda
        self._saved = {k: getattr(c, k) for k in ("Stream", "Event", "stream",
                                                  "current_stream", "synchronize")}

        @contextlib.contextmanager
        def stream(s):
            prev, sim.current = sim.current, s
            try:
                yield s
            finally:
                sim.current = prev

        c.Stream = lambda *a, **k: sim.new_stream()
        c.Event = lambda *a, **k: SimEvent(sim)
        c.stream = stream
        c.current_stream = lambda *a, **k: sim.current
        c.synchronize = lambda *a, **k: sim.drain()
        return sim

    def __exit__(self, *exc):
        for k, v in self._saved.items():
            setattr(torch.cuda, k, v)
        return False
