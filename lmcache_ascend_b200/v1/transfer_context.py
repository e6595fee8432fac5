"""Transfer contexts: the shared lifecycle of a batch of deferred-fetch chunks.

Behaviour of the reference (lmcache_ascend/v1/transfer_context.py:35-310):
a context belongs to one retrieve that reads ``num_proxies`` chunks from a
peer.  It hands out bounce buffers ("ping-pong" banks) from a registered
allocator, no more at a time than the pipeline depth allows; it counts the
proxies still to be consumed; and it sends the peer a Done signal exactly
once, when the last proxy is consumed or when the retrieve gives up early
(:meth:`send_done_now`), so the peer can unpin the chunks it holds for us.
Subclasses deliver the signal: :class:`P2PTransferContext` for cross-instance
pulls and :class:`PDTransferContext` for disaggregated-prefill pulls.
"""

from __future__ import annotations

import threading
from typing import Callable, List, Optional

import torch

from ..utils.logging import init_logger
from .memory_management import BaseAllocator, MemoryFormat, MemoryObj

logger = init_logger(__name__)

DEFAULT_PIPELINE_DEPTH = 4


class BaseTransferContext:
    def __init__(self, num_proxies: int, allocator: Optional[BaseAllocator] = None,
                 shape: Optional[torch.Size] = None, dtype: Optional[torch.dtype] = None,
                 fmt: MemoryFormat = MemoryFormat.KV_2LTD,
                 pipeline_depth: int = DEFAULT_PIPELINE_DEPTH):
        if num_proxies < 0:
            raise ValueError("num_proxies must be >= 0")
        self.num_proxies = num_proxies
        self.allocator = allocator
        self.shape, self.dtype, self.fmt = shape, dtype, fmt
        self._depth = max(1, int(pipeline_depth))
        self._remaining = num_proxies
        self._done_sent = False
        self._lock = threading.Lock()
        self._outstanding: List[MemoryObj] = []

    @property
    def max_pipeline_depth(self) -> int:
        """Bounce buffers in flight: the configured depth, capped by the number
        of proxies and by the free pages of a paged allocator."""
        d = min(self._depth, max(1, self.num_proxies))
        free = getattr(self.allocator, "num_free", None)
        if free is not None:
            d = min(d, max(1, int(free)))
        return d

    def allocate_buffers(self, count: int) -> List[MemoryObj]:
        """``count`` bounce buffers of the context's shape; all or none."""
        if self.allocator is None or self.shape is None:
            raise RuntimeError("transfer context has no allocator / buffer shape")
        got: List[MemoryObj] = []
        for _ in range(count):
            obj = self.allocator.allocate(self.shape, self.dtype, self.fmt)
            if obj is None:
                for o in got:
                    o.ref_count_down()
                raise MemoryError(f"could not allocate {count} transfer buffers")
            got.append(obj)
        with self._lock:
            self._outstanding.extend(got)
        return got

    def release_buffers(self, buffers: List[MemoryObj]) -> None:
        with self._lock:
            for b in buffers:
                if b in self._outstanding:
                    self._outstanding.remove(b)
        for b in buffers:
            b.ref_count_down()

    @property
    def done_sent(self) -> bool:
        return self._done_sent

    @property
    def remaining(self) -> int:
        return self._remaining

    def decref(self) -> None:
        """One proxy consumed; the last one sends Done."""
        with self._lock:
            if self._remaining > 0:
                self._remaining -= 1
            last = self._remaining == 0
        if last:
            self.send_done_now()

    def send_done_now(self) -> None:
        with self._lock:
            if self._done_sent:
                return
            self._done_sent = True
        try:
            self._send_done()
        except Exception as e:  # the peer's TTL sweep releases the pins anyway
            logger.warning("transfer Done signal failed: %s", e)

    def close(self) -> None:
        """Release leftover buffers and make sure Done went out."""
        with self._lock:
            left, self._outstanding = self._outstanding, []
        for b in left:
            b.ref_count_down()
        self.send_done_now()

    def _send_done(self) -> None:
        raise NotImplementedError


class P2PTransferContext(BaseTransferContext):
    """Cross-instance pull: Done tells the holder to unpin the looked-up chunks."""

    def __init__(self, num_proxies: int, lookup_id: str, target_peer_url: str,
                 send_done: Callable[[str, str], None], **kw):
        super().__init__(num_proxies, **kw)
        self._lookup_id = lookup_id
        self._peer = target_peer_url
        self._send = send_done

    @property
    def lookup_id(self) -> str:
        return self._lookup_id

    @property
    def target_peer_url(self) -> str:
        return self._peer

    def _send_done(self) -> None:
        self._send(self._peer, self._lookup_id)


class PDTransferContext(BaseTransferContext):
    """Disaggregated-prefill pull: Done acknowledges the sender's pull request."""

    def __init__(self, num_proxies: int, req_id: str, on_done: Callable[[str], None], **kw):
        super().__init__(num_proxies, **kw)
        self.req_id = req_id
        self._on_done = on_done

    def _send_done(self) -> None:
        self._on_done(self.req_id)
