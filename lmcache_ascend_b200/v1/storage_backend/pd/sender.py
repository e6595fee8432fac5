"""Sender (prefiller) side of the PD backend (reference
lmcache_ascend/v1/storage_backend/pd/sender_mixin.py:39-578: TTL sweep :138-189,
backpressure :191, peer connection :254, remote allocation :269, circuit
breaker :301-327, push :339-423, pull :425-578)."""

from __future__ import annotations

import threading
import time
import uuid as _uuid
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch
import zmq

from ....utils.keys import CacheEngineKey
from ....utils.logging import init_logger
from ...memory_management import MemoryObj
from . import messages as M

logger = init_logger(__name__)


class SenderMixin:
    # ------------------------------------------------------------ set-up
    def _init_sender(self, peer_init_url: Optional[str] = None,
                     peer_alloc_url: Optional[str] = None, **kw) -> None:
        cfg = self.config
        host = cfg.pd_peer_host or "127.0.0.1"
        pi = cfg.pd_peer_init_port or [7300]
        pa = cfg.pd_peer_alloc_port or [7400]
        self.peer_init_url = peer_init_url or f"tcp://{host}:{pi[self.tp_rank % len(pi)]}"
        self.peer_alloc_url = peer_alloc_url or f"tcp://{host}:{pa[self.tp_rank % len(pa)]}"
        self.remote_peer_id: Optional[str] = None
        self._receiver_epoch: Optional[str] = None  # decoder registration we mapped
        self._alloc_fail_until = 0.0
        self.pull_pending: Dict[str, Tuple[List[MemoryObj], float]] = {}
        self._proxy_sock = None
        if cfg.pd_proxy_host and cfg.pd_proxy_port:
            self._proxy_sock = self.ctx.socket(zmq.PUSH)
            self._proxy_sock.setsockopt(zmq.LINGER, 1000)
            self._proxy_sock.connect(f"tcp://{cfg.pd_proxy_host}:{cfg.pd_proxy_port}")
        self.done_url = None
        if cfg.pd_pull_mode:
            self._done_sock = self.ctx.socket(zmq.PULL)
            self._done_sock.setsockopt(zmq.LINGER, 0)
            port = self._done_sock.bind_to_random_port("tcp://0.0.0.0")
            self.done_url = f"tcp://{kw.get('advertise_host', '127.0.0.1')}:{port}"
            t = threading.Thread(target=self._done_loop, name="lmc-pd-done", daemon=True)
            t.start()
            self._threads.append(t)
        t = threading.Thread(target=self._sweep_loop, name="lmc-pd-ttl", daemon=True)
        t.start()
        self._threads.append(t)

    # -------------------------------------------------------- connection
    def _ensure_peer_connection(self) -> None:
        if self.remote_peer_id is not None:
            return
        refs = self.channel.get_local_buffer_refs() if self.channel is not None else []
        resp = self._req(self.peer_init_url, M.HandshakeRequest(self.peer_id, refs, None))
        if not isinstance(resp, M.HandshakeResponse) or not resp.ok:
            raise RuntimeError(f"PD handshake failed: {resp}")
        if resp.buffer_refs and self.channel is not None:
            self.channel.lazy_init_peer_connection(resp.peer_id, resp.buffer_refs)
        if resp.receiver_desc is not None and self.push_sender is not None:
            from ....parallel.pd_push import ReceiverDesc

            rd = ReceiverDesc.from_dict(resp.receiver_desc)
            self.push_sender.connect([rd])
            self._receiver_epoch = rd.epoch
        self.remote_peer_id = resp.peer_id

    def breaker_open(self) -> bool:
        return time.monotonic() < self._alloc_fail_until

    def _trip_breaker(self) -> None:
        self._alloc_fail_until = time.monotonic() + self.config.pd_alloc_fail_backoff_ttl
        self.stats.inc("pd_breaker_trips")

    # -------------------------------------------------------------- puts
    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey],
                                objs: Sequence[MemoryObj], transfer_spec: Any = None):
        if self.role != "sender":
            return None
        if self.breaker_open():
            self.stats.inc("pd_breaker_skips", len(keys))
            return None
        try:
            self._ensure_peer_connection()
            if self.config.pd_pull_mode:
                self._put_pull(keys, objs)
            else:
                self._put_push(keys, objs)
        except (TimeoutError, RuntimeError, zmq.ZMQError) as e:
            logger.warning("PD put of %d chunks failed: %s", len(keys), e)
            self.remote_peer_id = None  # force a new handshake next time
            self._trip_breaker()
            return None
        spec = transfer_spec or {}
        if self._proxy_sock is not None and spec.get("req_id") and spec.get("is_last", True):
            self._proxy_sock.send(M.encode(M.ProxyNotif(str(spec["req_id"]))))
        return None

    def _req_fields(self, objs: Sequence[MemoryObj]):
        o0 = objs[0]
        return (o0.get_memory_format().value, list(o0.get_shape()),
                str(o0.get_dtype()).removeprefix("torch."), objs[-1].get_num_tokens())

    def _put_push(self, keys, objs) -> None:
        fmt, shape, dtype, last = self._req_fields(objs)
        skeys = [k.to_string() for k in keys]
        resp = self._req(self.peer_alloc_url,
                         M.AllocRequest(skeys, fmt, shape, dtype, last, self.peer_id))
        if not isinstance(resp, M.AllocResponse):
            raise RuntimeError(f"bad alloc response {resp}")
        if resp.alloc_failed:
            logger.warning("PD receiver refused allocation for %d chunks", len(keys))
            self._trip_breaker()
            return
        sent = set(resp.already_sent_indexes)
        todo = [i for i in range(len(keys)) if i not in sent]
        srcs = [(objs[i].data_ptr(), objs[i].get_size()) for i in todo]
        addrs = list(zip(resp.remote_buffer_uuids, resp.remote_indexes))
        if srcs:
            self.channel.batched_write(srcs, self.remote_peer_id, addrs, sync=True)
        self._req(self.peer_alloc_url, M.WriteDone([skeys[i] for i in todo]))
        self.stats.inc("pd_pushed_chunks", len(todo))
        self.stats.inc("pd_pushed_bytes", sum(n for _, n in srcs))

    def _put_pull(self, keys, objs) -> None:
        fmt, shape, dtype, last = self._req_fields(objs)
        for o in objs:
            o.ref_count_up()  # pinned until the receiver reports the pull done
        pull_id = _uuid.uuid4().hex
        idx = [self.allocator.page_index(o) for o in objs]
        notif = M.PullReadyNotif(pull_id, [k.to_string() for k in keys],
                                 [self.buffer_cfg.uuid] * len(objs), idx, self.peer_id,
                                 self.done_url, fmt, shape, dtype, last)
        with self._lock:
            self.pull_pending[pull_id] = (list(objs),
                                          time.monotonic() + self.config.pd_pull_pending_ttl)
        ack = self._req(self.peer_alloc_url, notif)
        if not isinstance(ack, M.PullReadyDoneAck) or ack.alloc_failed:
            self._release_pull(pull_id)
            self._trip_breaker()
            return
        if len(ack.already_sent_indexes) == len(objs):
            self._release_pull(pull_id)

    def _release_pull(self, pull_id: str) -> None:
        with self._lock:
            ent = self.pull_pending.pop(pull_id, None)
        if ent is not None:
            for o in ent[0]:
                o.ref_count_down()

    def _done_loop(self) -> None:
        poller = zmq.Poller()
        poller.register(self._done_sock, zmq.POLLIN)
        while not self._closed.is_set():
            if not poller.poll(100):
                continue
            msg = M.decode(self._done_sock.recv())
            if isinstance(msg, M.PullDoneSignal):
                self._release_pull(msg.pull_id)
        self._done_sock.close()

    def _sweep_loop(self) -> None:
        """Release pull pins whose receiver never reported completion."""
        while not self._closed.wait(0.05):
            now = time.monotonic()
            with self._lock:
                expired = [p for p, (_, dl) in self.pull_pending.items() if dl < now]
            for p in expired:
                logger.warning("PD pull %s expired after %.1fs; releasing pinned pages", p,
                               self.config.pd_pull_pending_ttl)
                self.stats.inc("pd_pull_expired")
                self._release_pull(p)

    # ------------------------------------------------------- direct push
    def _drop_peer_mapping(self) -> None:
        """Forget the decoder's mapping (after its epoch changed): wait for
        the pushes already enqueued through it, then unmap."""
        if self.push_sender is not None:
            self.push_sender.close()
        self.remote_peer_id = None
        self._receiver_epoch = None

    def reserve_direct_push(self, req_id: str, num_tokens: int, dst_slots_host,
                            layer_begin: int = 0, num_layers: Optional[int] = None,
                            tile_tokens: int = 512, token_begin: int = 0,
                            prompt_end: int = -1) -> Tuple[List[int], int]:
        """Ask the decoder to grant a direct push of ``req_id`` before anything
        is launched.  ``dst_slots_host`` (host tensor or sequence) are the
        destination slots the sender was given; ``None`` asks the decoder for
        the slots it reserved, from reserved token ``token_begin`` on, at most
        ``num_tokens`` (-1: all) and not past prompt position ``prompt_end``.
        Returns (the destination slots: the decoder's list when it chose them,
        else ``dst_slots_host`` as given; prompt position of the
        reservation's first token).
        Raises -- and trips the per-peer circuit breaker -- when the decoder
        does not answer, answers with a stale registration epoch twice, or
        refuses (no reservation in time, slots that differ from its
        reservation, slots out of range).  No kernel that stores into the
        decoder's memory runs unless this returned."""
        if self.push_sender is None:
            raise RuntimeError("direct push needs a registered paged cache on the prefiller")
        want = dst_slots_host is None
        digest, max_slot = ("", -1) if want else M.slot_digest(dst_slots_host)
        deadline = time.monotonic() + self.config.pd_reserve_timeout_s
        reconnects = 0
        try:
            while True:
                self._ensure_peer_connection()
                if self.push_sender.replicas == 0 or not getattr(self, "_receiver_epoch", None):
                    raise RuntimeError("the decoder shared no paged-cache descriptor")
                L = self.push_sender.layout.num_layers
                nl = L - layer_begin if num_layers is None else num_layers
                resp = self._req(self.peer_alloc_url, M.DirectPushReserve(
                    str(req_id), self._receiver_epoch, int(num_tokens), int(layer_begin),
                    int(nl), int(tile_tokens), digest, max_slot, self.peer_id,
                    int(token_begin), want, int(prompt_end)))
                if isinstance(resp, M.DirectPushGrant) and resp.ok:
                    self.stats.inc("pd_direct_grants")
                    if want:
                        return list(resp.slots), int(resp.first_token)
                    return dst_slots_host, int(resp.first_token)  # as given
                if isinstance(resp, M.DirectPushGrant) and resp.epoch and \
                        resp.epoch != self._receiver_epoch and reconnects < 1:
                    reconnects += 1  # the decoder re-registered: map it again
                    self._drop_peer_mapping()
                    continue
                if isinstance(resp, M.DirectPushGrant) and resp.retry and \
                        time.monotonic() < deadline:
                    time.sleep(0.001)
                    continue
                raise RuntimeError(f"decoder refused direct push of {req_id}: "
                                   f"{getattr(resp, 'error', resp)}")
        except (TimeoutError, RuntimeError, zmq.ZMQError):
            self.stats.inc("pd_direct_refusals")
            self.remote_peer_id = None  # handshake again next time
            self._trip_breaker()
            raise

    def direct_push(self, src_slots: torch.Tensor, dst_slots: torch.Tensor, req_id: str,
                    layer_begin: int = 0, num_layers: Optional[int] = None,
                    tile_tokens: int = 512, dst_slots_host=None) -> None:
        """Reserve (``reserve_direct_push``), then push the prefiller's paged
        KV rows ``src_slots`` straight into the decoder's paged blocks
        ``dst_slots`` with the fused kernel on the current stream.
        ``dst_slots_host`` is the host copy of ``dst_slots`` the grant is
        checked against (taken from ``dst_slots`` when omitted)."""
        if self.breaker_open():
            self.stats.inc("pd_breaker_skips")
            raise RuntimeError("PD circuit breaker open: decoder recently refused or failed")
        host = dst_slots_host if dst_slots_host is not None else dst_slots.cpu()
        self.reserve_direct_push(req_id, int(src_slots.numel()), host, layer_begin,
                                 num_layers, tile_tokens)
        L = self.push_sender.layout.num_layers
        nl = L - layer_begin if num_layers is None else num_layers
        self.push_sender.push(src_slots, dst_slots, layer_begin, nl, tile_tokens)
        self.stats.inc("pd_direct_push_bytes",
                       src_slots.numel() * nl * sum(self.push_sender.layout.row_bytes))

    def push_granted_layers(self, src_slots: torch.Tensor, dst_slots: torch.Tensor,
                            layer_begin: int, num_layers: int, tile_tokens: int = 512) -> None:
        """Launch layers of a push that ``reserve_direct_push`` granted (for
        the layer-by-layer push during prefill: one grant per request, then
        one launch per layer with no round trip)."""
        self.push_sender.push(src_slots, dst_slots, layer_begin, num_layers, tile_tokens)
        self.stats.inc("pd_direct_push_bytes",
                       src_slots.numel() * num_layers * sum(self.push_sender.layout.row_bytes))

    def _close_sender(self) -> None:
        with self._lock:
            ids = list(self.pull_pending)
        for p in ids:
            self._release_pull(p)
        if self._proxy_sock is not None:
            self._proxy_sock.close()
