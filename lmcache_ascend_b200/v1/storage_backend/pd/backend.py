"""Disaggregated-prefill (PD) storage backend.

One class, two roles (reference lmcache_ascend/v1/storage_backend/pd/
backend.py:42-337 with sender_mixin.py / receiver_mixin.py):

* sender (prefiller): chunk objects are allocated from this backend's page
  pool (device pages: the gather kernel writes them in one launch), then
  pushed to pages the receiver allocated (AllocRequest/AllocResponse over
  ZMQ, data over the transfer channel), or -- pull mode -- advertised for the
  receiver to read.  A per-peer circuit breaker skips pushes for
  ``pd_alloc_fail_backoff_ttl`` seconds after the receiver refused an
  allocation; pull pins are released after ``pd_pull_pending_ttl`` if the
  receiver never reports completion.
* receiver (decoder): owns the page pool the prefiller writes into, serves
  allocation and handshake requests, keeps received chunks until the
  decoder retrieves them, refuses allocations that would dip into the
  ``pd_backpressure_reserve`` fraction of its pool.
* direct paged push (B200 fast path): the receiver shares a descriptor of
  its paged KV cache in the handshake; the sender's ``direct_push`` launches
  the fused NVLink kernel from its paged blocks into the decoder's paged
  blocks, and the decoder waits per layer on device flags
  (``wait_direct``).  No page pool, no chunk objects, no NCCL.
"""

from __future__ import annotations

import os
import threading
import time
import uuid as _uuid
from typing import Any, Dict, List, Optional, Sequence

import torch
import zmq

from ....config import LMCacheEngineConfig, LMCacheEngineMetadata
from ....utils.keys import CacheEngineKey
from ....utils.logging import init_logger
from ....utils.metrics import get_stats
from ...memory_management import (
    DeviceBuffer,
    HostBuffer,
    MemoryFormat,
    MemoryObj,
    PagedTensorAllocator,
)
from ...transfer_channel import BufferConfig, CreateTransferChannel
from ..abstract_backend import StorageBackendInterface
from . import messages as M
from .receiver import ReceiverMixin
from .sender import SenderMixin

logger = init_logger(__name__)

_DTYPES = {str(d).removeprefix("torch."): d for d in
           (torch.float32, torch.float16, torch.bfloat16, torch.uint8, torch.int8,
            torch.float8_e4m3fn)}


def dtype_from_str(s: str) -> torch.dtype:
    return _DTYPES[s]


class PDBackend(SenderMixin, ReceiverMixin, StorageBackendInterface):
    name = "PDBackend"

    def __init__(self, config: LMCacheEngineConfig,
                 metadata: Optional[LMCacheEngineMetadata] = None, channel=None,
                 page_bytes: Optional[int] = None, **kw):
        self.config = config
        self.metadata = metadata
        self.role = config.pd_role
        self.tp_rank = metadata.worker_id if metadata is not None else 0
        self.peer_id = f"{self.role}-{config.lmcache_instance_id}-{self.tp_rank}-" \
                       f"{os.getpid()}-{_uuid.uuid4().hex[:6]}"
        self.stats = get_stats()
        self.ctx = zmq.Context.instance()
        self.timeout_ms = int(config.blocking_timeout_secs * 1000)
        self._lock = threading.RLock()
        self._req_lock = threading.Lock()
        self._closed = threading.Event()
        self._threads: List[threading.Thread] = []
        self.device = torch.device(config.pd_buffer_device if config.pd_buffer_device != "cuda"
                                   else f"cuda:{torch.cuda.current_device()}") \
            if torch.cuda.is_available() or config.pd_buffer_device == "cpu" else \
            torch.device("cpu")
        self.channel = channel
        self.allocator: Optional[PagedTensorAllocator] = None
        self.buffer_cfg: Optional[BufferConfig] = None
        self._page_bytes = page_bytes
        self._gpu_connector = None
        self.push_receiver = None  # parallel.pd_push.PushReceiver (receiver role)
        self.push_sender = None    # parallel.pd_push.PushSender (sender role)
        self._init_role(**kw)

    # --------------------------------------------------------- set-up
    def _make_pool(self, page_bytes: int) -> None:
        self._page_bytes = page_bytes
        nbytes = max(page_bytes, (self.config.pd_buffer_size // page_bytes) * page_bytes)
        if self.device.type == "cuda":
            buf = DeviceBuffer(nbytes, self.device)
            self.buffer_cfg = BufferConfig(buf.tensor, page_bytes)
        else:
            shm = None
            if self.config.transfer_channel == "nvlink":
                shm = f"/lmc_pd_{os.getpid()}_{_uuid.uuid4().hex[:8]}"
            hb = HostBuffer(nbytes, shm_name=shm)
            self._host_buffer = hb
            self.buffer_cfg = BufferConfig(hb.tensor, page_bytes, shm_name=shm)
        self.allocator = PagedTensorAllocator(self.buffer_cfg.tensor, page_bytes)
        if self.channel is None:
            dev = self.device if self.device.type == "cuda" else None
            self.channel = CreateTransferChannel(self.config.transfer_channel, self.peer_id,
                                                 device=dev)
        self.channel.register_buffer(self.buffer_cfg)

    def _init_role(self, **kw) -> None:
        if self._page_bytes:
            self._make_pool(self._page_bytes)
        if self.role == "receiver":
            self._init_receiver(**kw)
        else:
            self._init_sender(**kw)

    def post_init(self, gpu_connector=None, engine=None, **kw) -> None:
        """Size the page pool from the chunk shape and register the paged
        cache for the direct push once KV caches are known."""
        self._gpu_connector = gpu_connector
        if gpu_connector is None or getattr(gpu_connector, "layout", None) is None:
            return
        if self.allocator is None:
            self._make_pool(gpu_connector.chunk_bytes(self.config.chunk_size))
        if gpu_connector.layout.device.type == "cuda":
            from ....parallel.pd_push import PushReceiver, PushSender

            if self.role == "receiver" and self.push_receiver is None:
                self.push_receiver = PushReceiver(gpu_connector.layout)
            if self.role == "sender" and self.push_sender is None:
                self.push_sender = PushSender(gpu_connector.layout)

    # ------------------------------------------------------- allocation
    def get_allocator_backend(self):
        return self if self.role == "sender" and self._page_bytes else None

    def allocate(self, shape, dtype, fmt: MemoryFormat = MemoryFormat.KV_2LTD,
                 eviction: bool = True) -> Optional[MemoryObj]:
        if self.allocator is None:
            raise RuntimeError("PD page pool not initialised (post_init not called)")
        deadline = time.monotonic() + (self.config.blocking_timeout_secs if eviction else 0)
        while True:
            obj = self.allocator.allocate(shape, dtype, fmt)
            if obj is not None or time.monotonic() >= deadline:
                return obj
            time.sleep(0.001)  # pages return as in-flight pushes complete

    def batched_allocate(self, shape, dtype, batch_size, fmt=MemoryFormat.KV_2LTD,
                         eviction=True):
        out = []
        for _ in range(batch_size):
            o = self.allocate(shape, dtype, fmt, eviction)
            if o is None:
                for p in out:
                    p.ref_count_down()
                return None
            out.append(o)
        return out

    # ------------------------------------------------------------- zmq
    def _rep_server(self, url: str, handler, name: str) -> str:
        sock = self.ctx.socket(zmq.REP)
        sock.setsockopt(zmq.LINGER, 0)
        if url.endswith(":0"):
            port = sock.bind_to_random_port(url[:-2])
            url = f"{url[:-2]}:{port}"
        else:
            sock.bind(url)

        def loop():
            poller = zmq.Poller()
            poller.register(sock, zmq.POLLIN)
            while not self._closed.is_set():
                if not poller.poll(100):
                    continue
                try:
                    msg = M.decode(sock.recv())
                    reply = handler(msg)
                except Exception as e:  # never leave the REQ side hanging
                    logger.exception("%s handler failed", name)
                    reply = M.Ack(False, str(e))
                sock.send(M.encode(reply))
            sock.close()

        t = threading.Thread(target=loop, name=name, daemon=True)
        t.start()
        self._threads.append(t)
        return url

    def _req(self, url: str, msg, timeout_ms: Optional[int] = None):
        """One request/reply with the peer at ``url`` over a REQ socket kept
        per URL (a new TCP connection per request costs more than the round
        trip); a timeout discards the socket so the next request starts clean."""
        to = timeout_ms or self.timeout_ms
        with self._req_lock:
            socks = self.__dict__.setdefault("_req_socks", {})
            s = socks.get((url, to))
            if s is None:
                s = self.ctx.socket(zmq.REQ)
                s.setsockopt(zmq.LINGER, 0)
                s.setsockopt(zmq.RCVTIMEO, to)
                s.setsockopt(zmq.SNDTIMEO, to)
                s.connect(url)
                socks[(url, to)] = s
            try:
                s.send(M.encode(msg))
                return M.decode(s.recv())
            except zmq.Again:
                socks.pop((url, to), None)
                s.close()
                raise TimeoutError(f"PD peer at {url} did not answer within {to} ms")

    def close(self) -> None:
        self._closed.set()
        for t in self._threads:
            t.join(timeout=2)
        with self._req_lock:
            for sock in self.__dict__.get("_req_socks", {}).values():
                sock.close()
            self.__dict__.get("_req_socks", {}).clear()
        self._close_role()
        if self.push_sender is not None:
            self.push_sender.close()
        if self.channel is not None:
            self.channel.close()

    # ------------------------------------------------- storage interface
    def contains(self, key: CacheEngineKey, pin: bool = False) -> bool:
        return self.role == "receiver" and self._contains_receiver(key, pin)

    def get_blocking(self, key: CacheEngineKey) -> Optional[MemoryObj]:
        return self._get_receiver(key) if self.role == "receiver" else None

    def remove(self, key: CacheEngineKey, force: bool = True) -> bool:
        if self.role != "receiver":
            return False
        obj = self._get_receiver(key)
        if obj is None:
            return False
        obj.ref_count_down()
        return True

    def keys(self) -> List[CacheEngineKey]:
        if self.role != "receiver":
            return []
        return [CacheEngineKey.from_string(k) for k in self.ready_keys()]

    def _close_role(self) -> None:
        if self.role == "receiver":
            self._close_receiver()
        else:
            self._close_sender()
