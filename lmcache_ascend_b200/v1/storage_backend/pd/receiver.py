"""Receiver (decoder) side of the PD backend (reference
lmcache_ascend/v1/storage_backend/pd/receiver_mixin.py:43-463: allocation
loop :61-134 and :389, eager / delayed pull :136-348, done signal :350)."""

from __future__ import annotations

import threading
import time
from typing import Dict, List, Optional, Tuple

import torch
import zmq

from ....utils.keys import CacheEngineKey
from ....utils.logging import init_logger
from ...memory_management import MemoryFormat, MemoryObj
from . import messages as M

logger = init_logger(__name__)


class ReceiverMixin:
    # ------------------------------------------------------------ set-up
    def _init_receiver(self, bind_host: str = "0.0.0.0", init_port: Optional[int] = None,
                       alloc_port: Optional[int] = None, **kw) -> None:
        cfg = self.config
        ports_i = cfg.pd_peer_init_port or [0]
        ports_a = cfg.pd_peer_alloc_port or [0]
        ip = init_port if init_port is not None else ports_i[self.tp_rank % len(ports_i)]
        ap = alloc_port if alloc_port is not None else ports_a[self.tp_rank % len(ports_a)]
        self.data: Dict[str, MemoryObj] = {}
        self.pending: Dict[str, MemoryObj] = {}
        self.delayed: Dict[str, Tuple[str, Tuple[str, int], MemoryObj]] = {}
        # granted direct pushes: req_id -> [device targets, layer_begin,
        # num_layers, next layer to wait for]
        self.direct: Dict[str, list] = {}
        # destination slots the decoder reserved per request, and how many of
        # its tokens were granted so far
        self.reservations: Dict[str, dict] = {}
        self._grant_cv = threading.Condition(self._lock)  # signalled on every grant
        self._done_socks: Dict[str, zmq.Socket] = {}
        self.init_url = self._rep_server(f"tcp://{bind_host}:{ip}", self._handle_init,
                                         "lmc-pd-init")
        self.alloc_url = self._rep_server(f"tcp://{bind_host}:{ap}", self._handle_alloc,
                                          "lmc-pd-alloc")

    def endpoints(self) -> Tuple[str, str]:
        """(init url, alloc url) with the bound ports (for tests/launchers)."""
        return self.init_url.replace("0.0.0.0", "127.0.0.1"), \
            self.alloc_url.replace("0.0.0.0", "127.0.0.1")

    # ---------------------------------------------------------- handlers
    def _handle_init(self, msg):
        if not isinstance(msg, M.HandshakeRequest):
            return M.HandshakeResponse(self.peer_id, [], None, False, "expected handshake")
        if msg.buffer_refs and self.channel is not None:
            self.channel.lazy_init_peer_connection(msg.peer_id, msg.buffer_refs)
        refs = self.channel.get_local_buffer_refs() if self.channel is not None else []
        desc = self.push_receiver.desc.to_dict() if self.push_receiver is not None else None
        return M.HandshakeResponse(self.peer_id, refs, desc)

    def _handle_alloc(self, msg):
        if isinstance(msg, M.AllocRequest):
            return self._allocate_and_put(msg)
        if isinstance(msg, M.WriteDone):
            with self._lock:
                for k in msg.keys:
                    obj = self.pending.pop(k, None)
                    if obj is not None:
                        self.data[k] = obj
            self.stats.inc("pd_recv_chunks", len(msg.keys))
            return M.Ack()
        if isinstance(msg, M.PullReadyNotif):
            return self._handle_pull_ready(msg)
        if isinstance(msg, M.DirectPushReserve):
            return self._handle_direct_reserve(msg)
        return M.Ack(False, f"unexpected message {type(msg).__name__}")

    # ------------------------------------------------- direct paged push
    def reserve_direct(self, req_id: str, dst_slots, first_token: int = 0) -> None:
        """Decoder: ``dst_slots`` (host tensor or sequence, one per token) are
        the paged-cache slots this decoder allocated for ``req_id``.  A
        prefiller's direct push of that request is granted only into these
        slots, in token order, possibly over several pushes (chunked prefill);
        the request is complete for ``wait_direct*`` once every reserved token
        was granted.  ``first_token``: prompt position of the first reserved
        token (tokens before it are already in this decoder's cache)."""
        import numpy as np

        arr = (dst_slots.detach().to("cpu", torch.int64).numpy()
               if isinstance(dst_slots, torch.Tensor) else np.asarray(list(dst_slots), np.int64))
        with self._lock:
            self.reservations[str(req_id)] = {"slots": arr, "granted": 0, "targets": None,
                                              "first": int(first_token)}
            self.direct.pop(str(req_id), None)

    def cancel_direct(self, req_id: str) -> None:
        with self._lock:
            self.reservations.pop(str(req_id), None)
            self.direct.pop(str(req_id), None)

    def _handle_direct_reserve(self, msg: "M.DirectPushReserve") -> "M.DirectPushGrant":
        pr = self.push_receiver
        if pr is None:
            return M.DirectPushGrant(False, error="receiver has no registered paged cache")
        epoch = pr.desc.epoch
        if msg.epoch != epoch:
            self.stats.inc("pd_direct_refused_epoch")
            return M.DirectPushGrant(False, epoch, "stale epoch: the paged cache was "
                                                   "registered again since the sender mapped it")
        nl_total = pr.layout.num_layers
        if msg.layer_begin < 0 or msg.num_layers < 1 or \
                msg.layer_begin + msg.num_layers > nl_total:
            return M.DirectPushGrant(False, epoch, "layer range out of the paged cache")
        with self._lock:
            res = self.reservations.get(msg.req_id)
            slots_out: List[int] = []
            if res is None:
                if self.config.pd_direct_require_reservation or msg.want_slots:
                    return M.DirectPushGrant(False, epoch, "no reservation for this request",
                                             retry=True)
                n = msg.num_tokens
                if msg.dst_max_slot >= pr.layout.num_slots:
                    self.stats.inc("pd_direct_refused_range")
                    return M.DirectPushGrant(False, epoch,
                                             "destination slot out of the paged cache")
                tg = pr.expect_host(n, msg.layer_begin, msg.num_layers, msg.tile_tokens)
                self.direct[msg.req_id] = [tg, msg.layer_begin, msg.num_layers, msg.layer_begin]
                self._grant_cv.notify_all()
                self.stats.inc("pd_direct_granted")
                return M.DirectPushGrant(True, epoch)
            arr = res["slots"]
            tb = msg.token_begin
            if tb != res["granted"]:
                return M.DirectPushGrant(False, epoch, f"push starts at token {tb}, the "
                                                       f"reservation continues at "
                                                       f"{res['granted']}")
            n = len(arr) - tb if msg.num_tokens < 0 else msg.num_tokens
            n = min(n, len(arr) - tb)
            if msg.want_slots and msg.prompt_end >= 0:
                n = min(n, msg.prompt_end - (res["first"] + tb))
            if n <= 0:
                return M.DirectPushGrant(False, epoch, "nothing left of the reservation")
            part = arr[tb:tb + n]
            if msg.want_slots:
                slots_out = part.tolist()
            else:
                digest, _ = M.slot_digest(part)
                if n != msg.num_tokens or digest != msg.dst_digest:
                    self.stats.inc("pd_direct_refused_slots")
                    return M.DirectPushGrant(False, epoch, "destination slots differ from "
                                                           "the decoder's reservation")
            if int(part.max()) >= pr.layout.num_slots:
                return M.DirectPushGrant(False, epoch, "reserved slot out of the paged cache")
            res["targets"] = pr.expect_host(n, msg.layer_begin, msg.num_layers,
                                            msg.tile_tokens)
            res["granted"] = tb + n
            res["layers"] = (msg.layer_begin, msg.num_layers)
            if res["granted"] >= len(arr):  # every reserved token is on its way
                self.reservations.pop(msg.req_id, None)
                lb, nl = res["layers"]
                self.direct[msg.req_id] = [res["targets"], lb, nl, lb]
                self._grant_cv.notify_all()
        self.stats.inc("pd_direct_granted")
        return M.DirectPushGrant(True, epoch, slots=slots_out, first_token=res["first"])

    def direct_granted(self, req_id: str) -> bool:
        """Every reserved token of ``req_id`` was granted to a prefiller."""
        with self._lock:
            return str(req_id) in self.direct

    def _shapes(self, shape: List[int], n: int, last_toks: int, fmt: int):
        shp = list(shape)
        tdim = MemoryFormat(fmt).token_dim()
        out = [torch.Size(shp)] * n
        if n and last_toks and tdim >= 0:
            last = list(shp)
            last[tdim] = last_toks
            out[-1] = torch.Size(last)
        return out

    def _alloc_pages(self, keys: List[str], shapes, dtype, fmt) -> Optional[List[MemoryObj]]:
        if self.allocator is None:
            return None
        need = len(keys)
        reserve = int(self.config.pd_backpressure_reserve * self.allocator.num_pages)
        if self.allocator.num_free - need < reserve:
            self.stats.inc("pd_backpressure_refusals")
            return None
        objs = []
        for shp in shapes:
            o = self.allocator.allocate(shp, dtype, MemoryFormat(fmt))
            if o is None:
                for p in objs:
                    p.ref_count_down()
                return None
            objs.append(o)
        return objs

    def _allocate_and_put(self, req: "M.AllocRequest"):
        from .backend import dtype_from_str

        with self._lock:
            already = [i for i, k in enumerate(req.keys) if k in self.data or k in self.pending]
            todo = [i for i in range(len(req.keys)) if i not in set(already)]
            shapes = self._shapes(req.shape, len(req.keys), req.last_chunk_toks, req.fmt)
            objs = self._alloc_pages([req.keys[i] for i in todo], [shapes[i] for i in todo],
                                     dtype_from_str(req.dtype), req.fmt)
            if objs is None:
                self.stats.inc("pd_alloc_failed")
                return M.AllocResponse(already, [], [], alloc_failed=True)
            idxs = []
            for i, o in zip(todo, objs):
                self.pending[req.keys[i]] = o
                idxs.append(self.allocator.page_index(o))
        return M.AllocResponse(already, idxs, [self.buffer_cfg.uuid] * len(idxs))

    # --------------------------------------------------------- pull mode
    def _handle_pull_ready(self, msg: "M.PullReadyNotif"):
        from .backend import dtype_from_str

        with self._lock:
            already = [i for i, k in enumerate(msg.keys) if k in self.data]
            todo = [i for i in range(len(msg.keys)) if i not in set(already)]
            shapes = self._shapes(msg.shape, len(msg.keys), msg.last_chunk_toks, msg.fmt)
            objs = self._alloc_pages([msg.keys[i] for i in todo], [shapes[i] for i in todo],
                                     dtype_from_str(msg.dtype), msg.fmt)
            if objs is None:
                return M.PullReadyDoneAck(already, alloc_failed=True)
        remote = [(msg.sender_buffer_uuids[i], msg.sender_mem_indexes[i]) for i in todo]
        if self.config.pd_delay_pull:
            with self._lock:
                for i, o, r in zip(todo, objs, remote):
                    self.delayed[msg.keys[i]] = (msg.sender_id, r, o)
                self._delayed_pull_ids = getattr(self, "_delayed_pull_ids", {})
                self._delayed_pull_ids[msg.pull_id] = (msg.sender_done_url,
                                                       [msg.keys[i] for i in todo])
            return M.PullReadyDoneAck(already)

        def eager():
            try:
                self.channel.batched_read([(o.data_ptr(), o.get_size()) for o in objs],
                                          msg.sender_id, remote, sync=True)
                with self._lock:
                    for i, o in zip(todo, objs):
                        self.data[msg.keys[i]] = o
            except Exception:
                logger.exception("eager pull failed")
                for o in objs:
                    o.ref_count_down()
            self._send_done(msg.sender_done_url, msg.pull_id)

        threading.Thread(target=eager, daemon=True, name="lmc-pd-pull").start()
        return M.PullReadyDoneAck(already)

    def _send_done(self, url: str, pull_id: str) -> None:
        s = self._done_socks.get(url)
        if s is None:
            s = self.ctx.socket(zmq.PUSH)
            s.setsockopt(zmq.LINGER, 1000)
            s.connect(url)
            self._done_socks[url] = s
        s.send(M.encode(M.PullDoneSignal(pull_id)))

    def _resolve_delayed(self, key: str) -> Optional[MemoryObj]:
        with self._lock:
            ent = self.delayed.pop(key, None)
        if ent is None:
            return None
        sender_id, remote, obj = ent
        self.channel.batched_read([(obj.data_ptr(), obj.get_size())], sender_id, [remote],
                                  sync=True)
        # a pull batch is done once none of its keys is still delayed
        for pid, (url, keys) in list(getattr(self, "_delayed_pull_ids", {}).items()):
            if key in keys and not any(k in self.delayed for k in keys):
                self._delayed_pull_ids.pop(pid, None)
                self._send_done(url, pid)
        return obj

    # ----------------------------------------------------- storage API
    def ready_keys(self) -> List[str]:
        with self._lock:
            return list(self.data.keys()) + list(self.delayed.keys())

    def _contains_receiver(self, key: CacheEngineKey, pin: bool = False) -> bool:
        s = key.to_string()
        with self._lock:
            return s in self.data or s in self.delayed

    def _get_receiver(self, key: CacheEngineKey) -> Optional[MemoryObj]:
        s = key.to_string()
        with self._lock:
            obj = self.data.pop(s, None)
        if obj is None:
            obj = self._resolve_delayed(s)
        if obj is not None:
            self.stats.inc("pd_retrieved_chunks")
        return obj  # the caller owns the backend's reference

    def _granted(self, req_id: str, timeout_s: float):
        """The granted entry of ``req_id``, waiting (bounded) for the grant."""
        deadline = time.monotonic() + timeout_s
        with self._grant_cv:
            while True:
                ent = self.direct.get(req_id)
                left = deadline - time.monotonic()
                if ent is not None or left <= 0:
                    return ent
                self._grant_cv.wait(left)

    def wait_direct(self, req_id: str, timeout_s: Optional[float] = None,
                    sync: bool = False) -> bool:
        """Enqueue the bounded flag wait for every layer of a granted direct
        push (not yet waited for) on the current stream.  With ``sync`` also
        waits on the host and checks the status word.  Returns False if the
        push was never granted within ``timeout_s``."""
        to = timeout_s or self.config.pd_flag_timeout_s
        ent = self._granted(req_id, to)
        if ent is None:
            return False
        tg, lb, nl, nxt = ent
        with self._lock:
            self.direct.pop(req_id, None)
        if nxt < lb + nl:
            self.push_receiver.wait(list(tg[nxt - lb:]), nxt, to)
        if sync:
            torch.cuda.current_stream().synchronize()
            self.push_receiver.check()
        return True

    def wait_direct_layer(self, req_id: str, layer: int,
                          timeout_s: Optional[float] = None) -> bool:
        """Enqueue the bounded flag wait of layers up to ``layer`` (inclusive)
        of a granted direct push on the current stream, so the kernels queued
        after it (attention of that layer) see the pushed rows.  No host
        wait.  Returns False if the push was never granted."""
        to = timeout_s or self.config.pd_flag_timeout_s
        ent = self._granted(req_id, to)
        if ent is None:
            return False
        tg, lb, nl, nxt = ent
        last = min(layer, lb + nl - 1)
        if last >= nxt:
            self.push_receiver.wait(list(tg[nxt - lb:last - lb + 1]), nxt, to)
            ent[3] = last + 1
        if ent[3] >= lb + nl:
            with self._lock:
                self.direct.pop(req_id, None)
        return True

    def _close_receiver(self) -> None:
        with self._lock:
            objs = list(self.data.values()) + list(self.pending.values()) + \
                [e[2] for e in self.delayed.values()]
            self.data.clear()
            self.pending.clear()
            self.delayed.clear()
        for o in objs:
            o.ref_count_down()
        for s in self._done_socks.values():
            s.close()
