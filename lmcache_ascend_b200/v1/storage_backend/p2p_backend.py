"""P2P backend: share cached chunks between serving instances.

Behaviour of the reference's ``P2PBackend`` (lmcache_ascend/v1/storage_backend/
p2p_backend.py:106-985): chunks stored locally are announced to the
controller (and withdrawn when no local tier holds them any more); a lookup
miss in the local tiers asks the controller which instance holds the key; a
get pulls the chunk from that instance, retrying other holders (up to
``p2p_max_retries``) when a peer fails or times out.

Data plane:
* chunk in the holder's HBM tier (one box): the holder pins the object under
  a lease and answers with its offset in its HBM slab, which every instance
  exported over CUDA IPC when it registered; the reader maps the slab once
  and copies the chunk over NVLink into its own tier (one device-to-device
  peer copy), then returns the lease.  Leases a reader never returns expire
  after ``p2p_pull_pending_ttl`` seconds (reference delayed pull with proxy
  objects, p2p_backend.py:838-960);
* chunk in the holder's CPU tier: naive-serde bytes over ZMQ.
"""

from __future__ import annotations

import threading
import time
import uuid as _uuid
from typing import Any, Dict, List, Optional, Sequence, Tuple

import msgpack
import torch
import zmq

from ...config import LMCacheEngineConfig
from ...utils.keys import CacheEngineKey
from ...utils.logging import init_logger
from ...utils.metrics import get_stats
from ..memory_management import MemoryObj
from .abstract_backend import StorageBackendInterface
from .serde import NaiveSerde

logger = init_logger(__name__)


class P2PBackend(StorageBackendInterface):
    name = "P2PBackend"

    def __init__(self, config: LMCacheEngineConfig, metadata, local_cpu, hbm=None, **kw):
        self.config = config
        self.local = local_cpu
        self.hbm = hbm                      # LocalGPUBackend or None
        self._leases: Dict[str, Tuple[MemoryObj, float]] = {}
        self._lease_lock = threading.Lock()
        self._peer_maps = None              # PeerMappings of the holders' HBM slabs
        self._slab_desc = None
        if hbm is not None:
            from ...parallel.ipc import export_local

            slab = hbm.allocator.dev.tensor
            self._slab_base = slab.data_ptr()
            self._slab_desc = export_local(self._slab_base, hbm.device.index or 0).to_dict()
        self.instance = f"{config.lmcache_instance_id}-{metadata.worker_id if metadata else 0}" \
                        f"-{_uuid.uuid4().hex[:6]}"
        self.timeout_ms = int(config.blocking_timeout_secs * 1000)
        self.ctx = zmq.Context.instance()
        self.serde = NaiveSerde()
        self.stats = get_stats()
        self._stop = threading.Event()
        self._ctl_lock = threading.Lock()
        self._ctl = None
        self._loc_cache: Dict[str, Tuple[float, List]] = {}
        host = config.p2p_host or "127.0.0.1"
        ports = config.p2p_init_ports or [0]
        port = ports[(metadata.worker_id if metadata else 0) % len(ports)]
        self._srv = self.ctx.socket(zmq.REP)
        self._srv.setsockopt(zmq.LINGER, 0)
        if port == 0:
            port = self._srv.bind_to_random_port(f"tcp://{host}")
        else:
            self._srv.bind(f"tcp://{host}:{port}")
        self.peer_url = f"tcp://{host}:{port}"
        self._t = threading.Thread(target=self._serve, daemon=True, name="lmc-p2p-peer")
        self._t.start()
        if not config.controller_url:
            raise ValueError("enable_p2p needs controller_url")
        self._ctl_rpc("register", {"url": self.peer_url, "hbm": self._slab_desc})
        local_cpu.evict_listeners.append(self._on_evict)
        if hbm is not None:
            hbm.evict_listeners.append(self._on_evict)

    # ----------------------------------------------------------- controller
    def _ctl_rpc(self, op: str, payload):
        with self._ctl_lock:
            if self._ctl is None:
                s = self.ctx.socket(zmq.REQ)
                s.setsockopt(zmq.LINGER, 0)
                s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
                s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
                s.connect(self.config.controller_url)
                self._ctl = s
            try:
                self._ctl.send(msgpack.packb([op, self.instance, payload], use_bin_type=True))
                st, res = msgpack.unpackb(self._ctl.recv(), raw=False)
            except zmq.Again:
                self._ctl.close()
                self._ctl = None
                raise TimeoutError("P2P controller did not answer")
        if st != "ok":
            raise RuntimeError(f"controller error: {res}")
        return res

    def _on_evict(self, key: CacheEngineKey) -> None:
        for tier in (self.hbm, self.local):
            if tier is not None and tier.contains(key):
                return  # still held here (an HBM eviction writes back to the CPU tier)
        try:
            self._ctl_rpc("evict", [key.to_string()])
        except (TimeoutError, RuntimeError):
            logger.warning("P2P: could not withdraw %s", key)

    # ----------------------------------------------------------- peer server
    def _serve(self) -> None:
        poller = zmq.Poller()
        poller.register(self._srv, zmq.POLLIN)
        while not self._stop.is_set():
            if not poller.poll(100):
                continue
            try:
                op, key = msgpack.unpackb(self._srv.recv(), raw=False)
                self._expire_leases()
                if op == "release":
                    self._release_lease(key)
                    self._srv.send(msgpack.packb(["ok", None], use_bin_type=True))
                    continue
                reply = ["ok", None]
                if op == "get":
                    ck = CacheEngineKey.from_string(key)
                    obj = self.hbm.get_blocking(ck) if self.hbm is not None else None
                    if obj is not None:  # stays pinned by the lease until released
                        lease = _uuid.uuid4().hex
                        with self._lease_lock:
                            self._leases[lease] = (obj, time.monotonic() +
                                                   self.config.p2p_pull_pending_ttl)
                        reply = ["dev", {"off": obj.data_ptr() - self._slab_base,
                                         "n": obj.get_size(), "shape": list(obj.get_shape()),
                                         "dtype": str(obj.get_dtype()).removeprefix("torch."),
                                         "fmt": obj.get_memory_format().name,
                                         "lease": lease}]
                    else:
                        obj = self.local.get_blocking(ck)
                        if obj is not None:
                            try:
                                reply = ["ok", self.serde.serialize(obj)]
                            finally:
                                obj.ref_count_down()
                self._srv.send(msgpack.packb(reply, use_bin_type=True))
            except Exception as e:
                self._srv.send(msgpack.packb(["err", str(e)], use_bin_type=True))
        self._srv.close()

    def _release_lease(self, lease: str) -> None:
        with self._lease_lock:
            ent = self._leases.pop(lease, None)
        if ent is not None:
            ent[0].ref_count_down()

    def _expire_leases(self) -> None:
        now = time.monotonic()
        with self._lease_lock:
            dead = [k for k, (_, dl) in self._leases.items() if dl < now]
        for k in dead:
            logger.warning("P2P lease %s expired (reader never returned it)", k)
            self.stats.inc("p2p_lease_expired")
            self._release_lease(k)

    # ------------------------------------------------- NVLink peer reads
    def _read_peer_hbm(self, inst: str, desc: dict, meta: dict) -> Optional[MemoryObj]:
        """Copy a chunk out of a holder's HBM slab (peer mapping, one
        device-to-device copy over NVLink) into this instance's tier."""
        from ... import ops
        from ...parallel.ipc import IpcDesc, PeerMappings
        from .pd.backend import dtype_from_str
        from ..memory_management import MemoryFormat

        dest_tier = self.hbm if self.hbm is not None else self.local
        if self._peer_maps is None:
            dev = torch.cuda.current_device()
            self._peer_maps = (PeerMappings(dev), {})
        maps, bases = self._peer_maps
        base = bases.get(inst)
        if base is None:
            base = bases[inst] = maps.resolve(IpcDesc.from_dict(desc))
        obj = dest_tier.allocate(torch.Size(meta["shape"]), dtype_from_str(meta["dtype"]),
                                 MemoryFormat[meta["fmt"]])
        if obj is None:
            return None
        n = int(meta["n"])
        t = torch.tensor
        ops.native().layerwise_prefill_dma_copy(t([obj.data_ptr()]), t([base + meta["off"]]),
                                                t([n]))
        torch.cuda.current_stream().synchronize()
        self.stats.inc("p2p_nvlink_bytes", n)
        return obj

    # ------------------------------------------------------- storage API
    def batched_submit_put_task(self, keys: Sequence[CacheEngineKey], objs: Sequence[MemoryObj],
                                transfer_spec: Any = None):
        # the CPU tier keeps the data; announce where it can be found
        if keys:
            try:
                self._ctl_rpc("admit", [k.to_string() for k in keys])
            except (TimeoutError, RuntimeError) as e:
                logger.warning("P2P admit failed: %s", e)
        return None

    def _holders(self, key: str) -> List:
        now = time.monotonic()
        ent = self._loc_cache.get(key)
        if ent is not None and now - ent[0] < 1.0:
            return ent[1]
        try:
            res = self._ctl_rpc("lookup", key)
        except (TimeoutError, RuntimeError):
            res = []
        self._loc_cache[key] = (now, res)
        return res

    def contains(self, key: CacheEngineKey, pin: bool = False) -> bool:
        return bool(self._holders(key.to_string()))

    def get_blocking(self, key: CacheEngineKey) -> Optional[MemoryObj]:
        k = key.to_string()
        holders = self._holders(k)[: max(1, self.config.p2p_max_retries)]
        for inst, ent in holders:
            url = ent["url"] if isinstance(ent, dict) else ent
            desc = ent.get("hbm") if isinstance(ent, dict) else None
            s = self.ctx.socket(zmq.REQ)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.RCVTIMEO, self.timeout_ms)
            s.setsockopt(zmq.SNDTIMEO, self.timeout_ms)
            s.connect(url)
            try:
                s.send(msgpack.packb(["get", k], use_bin_type=True))
                st, data = msgpack.unpackb(s.recv(), raw=False)
                if st == "dev":
                    obj = None
                    try:
                        if desc is not None and torch.cuda.is_available():
                            obj = self._read_peer_hbm(inst, desc, data)
                    finally:  # return the lease whether or not the copy happened
                        s.send(msgpack.packb(["release", data["lease"]], use_bin_type=True))
                        s.recv()
                    if obj is not None:
                        return obj
                    self.stats.inc("p2p_retries")
                    continue
            except zmq.Again:
                logger.warning("P2P peer %s timed out for %s; trying the next holder", inst, k)
                self.stats.inc("p2p_retries")
                continue
            finally:
                s.close()
            if st == "ok" and data is not None:
                self.stats.inc("p2p_get_bytes", len(data))
                return self.serde.deserialize(data, self.local)
            self.stats.inc("p2p_retries")
        self._loc_cache.pop(k, None)
        return None

    def close(self) -> None:
        try:
            self._ctl_rpc("deregister", None)
        except (TimeoutError, RuntimeError):
            pass
        self._stop.set()
        self._t.join(timeout=2)
        if self._ctl is not None:
            self._ctl.close()
