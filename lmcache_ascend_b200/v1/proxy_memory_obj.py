"""ProxyMemoryObj: a chunk that still lives on a peer.

Behaviour of the reference (lmcache_ascend/v1/proxy_memory_obj.py:36-467):
instead of fetching every hit chunk from a peer during lookup-and-prefetch,
the engine carries proxies that name the peer's buffer page; the GPU
connector resolves them in batches into bounce buffers taken from the
transfer context and scatters each batch into the paged cache while the next
batch is being read, then releases the buffers and marks the proxies
consumed (the last one sends the Done signal through the context).

Reads go through a transfer channel's ``batched_read`` /
``submit_batched_read`` (:mod:`lmcache_ascend_b200.v1.transfer_channel`):
remote memory is named ``(buffer uuid, page index)``, never by pointer.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch

from .memory_management import MemoryFormat, MemoryObj, MemoryObjMetadata
from .transfer_context import BaseTransferContext


class ProxyMemoryObj(MemoryObj):
    def __init__(self, shape: torch.Size, dtype: torch.dtype, fmt: MemoryFormat, channel,
                 peer_id: str, remote_addr: Tuple[str, int], context: BaseTransferContext,
                 nbytes: Optional[int] = None):
        n = nbytes if nbytes is not None else \
            int(torch.Size(shape).numel()) * torch.empty((), dtype=dtype).element_size()
        super().__init__(None, MemoryObjMetadata(torch.Size(shape), dtype, 0, n, fmt), None)
        self._channel = channel
        self._peer = peer_id
        self._addr = (remote_addr[0], int(remote_addr[1]))
        self._ctx = context
        self._backing: Optional[MemoryObj] = None
        self._resolved = False
        self._consumed = False

    # ------------------------------------------------------------ state
    @property
    def is_proxy(self) -> bool:
        return True

    @property
    def resolved(self) -> bool:
        return self._resolved

    @property
    def consumed(self) -> bool:
        return self._consumed

    @property
    def transfer_context(self) -> BaseTransferContext:
        return self._ctx

    @property
    def backing_obj(self) -> Optional[MemoryObj]:
        return self._backing

    @property
    def remote_addr(self) -> Tuple[str, int]:
        return self._addr

    def set_backing_obj(self, obj: MemoryObj) -> None:
        """Assign a bounce buffer; the data must be (re)fetched into it."""
        if obj.get_size() < self.get_size():
            raise ValueError("backing buffer smaller than the proxied chunk")
        self._backing = obj
        self._resolved = False

    def clear_backing_obj(self) -> None:
        self._backing = None

    def mark_consumed(self) -> None:
        """The data reached its destination; counts once toward Done."""
        if self._consumed:
            return
        self._consumed = True
        self._ctx.decref()

    # ------------------------------------------------------------ views
    @property
    def tensor(self) -> Optional[torch.Tensor]:
        if self._backing is None or not self._resolved:
            return None
        t = self._backing.tensor
        return t.reshape(-1)[: self.get_shape().numel()].view(self.get_shape()) \
            if t is not None else None

    @property
    def raw_data(self):  # noqa: D401 - mirrors MemoryObj.raw_data
        return self._backing.raw_data if self._backing is not None else None

    @raw_data.setter
    def raw_data(self, value) -> None:
        if value is not None:
            raise AttributeError("a proxy's data lives in its backing buffer")

    def data_ptr(self) -> int:
        return self._backing.data_ptr() if self._backing is not None else 0

    def free(self) -> None:
        self._valid = False  # nothing owned; the context owns the bounce buffers

    # ------------------------------------------------------------ fetch
    def resolve(self) -> None:
        ProxyMemoryObj.resolve_batch([self])

    @staticmethod
    def _read_args(unresolved: Sequence["ProxyMemoryObj"]):
        peer = unresolved[0]._peer
        dsts, addrs = [], []
        for p in unresolved:
            if p._backing is None:
                raise RuntimeError("cannot resolve a proxy without a backing buffer")
            if p._peer != peer or p._channel is not unresolved[0]._channel:
                raise ValueError("a batch must share one channel and one peer")
            dsts.append((p._backing.data_ptr(), p.get_size()))
            addrs.append(p._addr)
        return peer, dsts, addrs

    @staticmethod
    def resolve_batch(proxies: Sequence["ProxyMemoryObj"]) -> None:
        """Blocking read of every unresolved proxy in one channel call."""
        todo = [p for p in proxies if not p._resolved]
        if not todo:
            return
        peer, dsts, addrs = ProxyMemoryObj._read_args(todo)
        todo[0]._channel.batched_read(dsts, peer, addrs, sync=True)
        for p in todo:
            p._resolved = True

    @staticmethod
    def submit_resolve_batch(proxies: Sequence["ProxyMemoryObj"]):
        """Start the read and return its event (``synchronize()``/``query()``),
        or None when nothing was left to read."""
        todo = [p for p in proxies if not p._resolved]
        if not todo:
            return None
        peer, dsts, addrs = ProxyMemoryObj._read_args(todo)
        ch = todo[0]._channel
        if hasattr(ch, "submit_batched_read"):
            ev = ch.submit_batched_read(dsts, peer, addrs)
        else:
            ch.batched_read(dsts, peer, addrs, sync=True)
            ev = None
        for p in todo:
            p._resolved = True
        return ev

    def __repr__(self) -> str:
        return (f"ProxyMemoryObj(shape={tuple(self.get_shape())}, peer={self._peer}, "
                f"addr={self._addr}, resolved={self._resolved}, consumed={self._consumed})")


def is_proxy(obj) -> bool:
    return getattr(obj, "is_proxy", False) is True


def load_proxies_pipelined(proxies: Sequence[ProxyMemoryObj], starts: Sequence[int],
                           ends: Sequence[int],
                           scatter: Callable[[List[MemoryObj], List[int], List[int]], object]
                           ) -> None:
    """Resolve ``proxies`` in two banks of bounce buffers and scatter each bank
    while the other one is being read.  ``scatter(objs, starts, ends)`` moves
    resolved chunks to their destination and returns an object with
    ``synchronize()`` (a CUDA event) or None when it finished synchronously;
    a bank is refilled only after its scatter completed."""
    if not proxies:
        return
    ctx = proxies[0].transfer_context
    depth = ctx.max_pipeline_depth
    bank = max(1, depth // 2)
    nbanks = 2 if depth >= 2 and len(proxies) > bank else 1
    bufs = ctx.allocate_buffers(bank * nbanks)
    banks = [bufs[i * bank:(i + 1) * bank] for i in range(nbanks)]
    pending = [None] * nbanks  # scatter completion per bank
    try:
        batches = [list(range(i, min(i + bank, len(proxies))))
                   for i in range(0, len(proxies), bank)]

        def submit(k: int):
            b = k % nbanks
            if pending[b] is not None:
                pending[b].synchronize()
                pending[b] = None
            for j, i in enumerate(batches[k]):
                proxies[i].set_backing_obj(banks[b][j])
            return ProxyMemoryObj.submit_resolve_batch([proxies[i] for i in batches[k]])

        read_ev = submit(0)
        for k, idx in enumerate(batches):
            nxt = submit(k + 1) if k + 1 < len(batches) and nbanks > 1 else None
            if read_ev is not None:
                read_ev.synchronize()
            objs = [proxies[i] for i in idx]
            done = scatter(objs, [starts[i] for i in idx], [ends[i] for i in idx])
            pending[k % nbanks] = done
            for p in objs:
                p.mark_consumed()
            if nbanks == 1 and k + 1 < len(batches):
                if done is not None:
                    done.synchronize()
                    pending[0] = None
                nxt = submit(k + 1)
            read_ev = nxt
        for ev in pending:
            if ev is not None:
                ev.synchronize()
    finally:
        for p in proxies:
            p.clear_backing_obj()
        ctx.release_buffers(bufs)
