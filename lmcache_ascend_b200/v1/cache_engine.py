"""The LMCache engine: store / retrieve / lookup over token-hash chunks.

Public surface follows the reference's ``AscendLMCacheEngine`` and the
upstream ``LMCacheEngine`` it extends (reference
lmcache_ascend/v1/cache_engine.py: ``store`` :8951, ``store_layer`` :6030,
``lookup`` :3801, ``lookup_unpin`` :3823, ``get_finished_stores`` :3651,
``wait_for_pending_stores`` :3679, ``get_kv_events`` :3796, ``close`` :10153,
async store worker :3451-3649, health gate :8979; upstream ``retrieve``,
``retrieve_layer``, ``prefetch``).
"""

from __future__ import annotations

import queue
import threading
import time
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Generator, List, Optional, Sequence, Tuple

import torch

from ..config import LMCacheEngineConfig, LMCacheEngineMetadata
from ..utils.keys import CacheEngineKey
from ..utils.logging import init_logger
from ..utils.metrics import get_stats
from ..utils.nvtx import nvtx_range
from .gpu_connector import GPUConnectorInterface
from .memory_management import MemoryFormat, MemoryObj
from .storage_backend.storage_manager import StorageManager
from .token_database import ChunkedTokenDatabase, SegmentTokenDatabase, TokenDatabase

logger = init_logger(__name__)


@dataclass
class CacheStoreEvent:
    """KV cache event (reference cache_engine.py:3588-3616)."""

    block_hashes: List[int]
    parent_block_hash: Optional[int]
    token_ids: List[int]
    block_size: int
    lora_id: Optional[int] = None
    medium: str = "cpu"


class ThreadSafeEventList:
    """Append/drain list of KV events (reference cache_engine.py:221-254)."""

    def __init__(self):
        self._lock = threading.Lock()
        self._events: List[CacheStoreEvent] = []

    def append(self, e: CacheStoreEvent) -> None:
        with self._lock:
            self._events.append(e)

    def drain(self) -> List[CacheStoreEvent]:
        with self._lock:
            out, self._events = self._events, []
            return out

    def __len__(self) -> int:
        return len(self._events)


@dataclass
class _StoreRequest:
    req_id: Any
    tokens: torch.Tensor
    mask: Optional[torch.Tensor]
    kwargs: Dict[str, Any]
    done: threading.Event = field(default_factory=threading.Event)
    error: Optional[BaseException] = None


class _LazyLayers:
    """Per-layer chunk objects of a layerwise retrieve, fetched from the tiers
    when the connector first asks for a layer, so the CPU-tier lookups of
    later layers overlap the transfers of earlier ones.  A chunk missing in a
    later layer (evicted despite the lookup pin) borrows the same chunk's
    object of the previous layer (same shape) and ends the usable prefix
    there: the caller recomputes, and overwrites, those tokens."""

    def __init__(self, storage_manager, chunk_layer_keys, num_layers: int):
        self.sm = storage_manager
        self.keys = chunk_layer_keys  # [chunk][layer]
        self.L = num_layers
        self.rows: Dict[int, List[MemoryObj]] = {}
        self.owned: List[MemoryObj] = []
        self.complete = len(chunk_layer_keys)

    def prefix_of_layer0(self) -> int:
        got = self.sm.batched_get([ks[0] for ks in self.keys])
        n = 0
        while n < len(got) and got[n] is not None:
            n += 1
        for o in got[n:]:
            if o is not None:
                o.ref_count_down()
        self.keys = self.keys[:n]
        self.complete = n
        self.rows[0] = list(got[:n])
        self.owned.extend(got[:n])
        return n

    def __len__(self) -> int:
        return self.L

    def __getitem__(self, layer: int) -> List[MemoryObj]:
        row = self.rows.get(layer)
        if row is None:
            got = self.sm.batched_get([ks[layer] for ks in self.keys])
            if None not in got:
                self.owned.extend(got)
                self.rows[layer] = got
                return got
            prev = self[layer - 1]
            row = []
            for c, o in enumerate(got):
                if o is None:
                    self.complete = min(self.complete, c)
                    row.append(prev[c])
                else:
                    self.owned.append(o)
                    row.append(o)
            self.rows[layer] = row
        return row

    def __iter__(self):
        return (self[l] for l in range(self.L))

    def release(self) -> None:
        for o in self.owned:
            o.ref_count_down()
        self.owned = []


@dataclass
class SparseLayerRequest:
    """One layer of a sparse load: paged slot ``slot_mapping[i]`` receives
    token ``selected_token_idx[i]`` of the request (device tensors, same
    integer dtype and length)."""

    selected_token_idx: torch.Tensor
    slot_mapping: torch.Tensor


@dataclass
class SparseRetrieveState:
    """Warm metadata of one long-context request for sparse (top-k) loads,
    kept by the caller between decode steps: the request's cached chunks,
    one held object per chunk, and the device table of their addresses.
    Later steps reuse it without touching the storage tiers; a longer
    context extends it (``extend``), and a failed extension leaves it as it
    was (reference rollback guard: lmcache_ascend/v1/cache_engine.py:257-300)."""

    keys: List[CacheEngineKey] = field(default_factory=list)
    ends: List[int] = field(default_factory=list)
    objs: List[MemoryObj] = field(default_factory=list)
    ptrs: Optional[torch.Tensor] = None
    chunk_tokens: int = 0

    @property
    def total_tokens(self) -> int:
        return self.ends[-1] if self.ends else 0

    def release(self) -> None:
        objs, self.objs = self.objs, []
        for o in objs:
            o.ref_count_down()
        self.keys, self.ends, self.ptrs = [], [], None


class _SparseAppend:
    """Transaction over a SparseRetrieveState: an extension may replace the
    state's partial last chunk and append chunks.  ``commit`` releases the
    replaced chunk; ``rollback`` (unless committed) releases what was
    appended and puts the state back exactly as it was."""

    def __init__(self, st: SparseRetrieveState):
        self.st = st
        self.snap = (list(st.keys), list(st.ends), list(st.objs), st.ptrs)
        self.dropped: List[MemoryObj] = []
        self.done = False

    def drop_last(self) -> None:
        st = self.st
        st.keys.pop()
        st.ends.pop()
        self.dropped.append(st.objs.pop())

    def commit(self) -> None:
        self.done = True
        for o in self.dropped:
            o.ref_count_down()
        self.dropped = []

    def rollback(self) -> None:
        if self.done:
            return
        st = self.st
        keep = {id(o) for o in self.snap[2]}
        for o in st.objs:
            if id(o) not in keep:
                o.ref_count_down()
        st.keys[:], st.ends[:], st.objs[:] = self.snap[0], self.snap[1], self.snap[2]
        st.ptrs = self.snap[3]


class LMCacheEngine:
    def __init__(self, config: LMCacheEngineConfig, metadata: LMCacheEngineMetadata,
                 gpu_connector: GPUConnectorInterface,
                 token_database: Optional[TokenDatabase] = None,
                 storage_manager: Optional[StorageManager] = None,
                 broadcast_fn: Optional[Callable] = None,
                 broadcast_object_fn: Optional[Callable] = None,
                 collective_all_true_fn: Optional[Callable] = None, **kw):
        self.config = config
        self.metadata = metadata
        self.gpu_connector = gpu_connector
        if token_database is None:
            token_database = (SegmentTokenDatabase(config, metadata)
                              if config.enable_blending else
                              ChunkedTokenDatabase(config, metadata))
        self.token_database = token_database
        self.storage_manager = storage_manager or StorageManager(config, metadata, **kw)
        self.broadcast_fn = broadcast_fn
        self.broadcast_object_fn = broadcast_object_fn
        self.collective_all_true_fn = collective_all_true_fn
        self.stats = get_stats()
        self.kv_events = ThreadSafeEventList()
        self._engine_state_lock = threading.RLock()
        self._lookup_pins: Dict[Any, List[CacheEngineKey]] = {}
        # chunk key -> its per-layer keys, shared by the stores and retrieves
        # of the same prefix so the tiers' dict lookups hit on identity
        self._layer_keys: "OrderedDict[CacheEngineKey, list]" = OrderedDict()
        self._layer_keys_lock = threading.Lock()
        self._healthy = True
        self._closed = False
        # async store worker (reference cache_engine.py:412-421, 3451)
        self._store_queue: "queue.Queue[Optional[_StoreRequest]]" = queue.Queue(
            maxsize=max(1, config.store_async_max_queue_size))
        self._finished_stores: List[Any] = []
        self._finished_lock = threading.Lock()
        self._pending = 0
        self._pending_cv = threading.Condition()
        self._worker: Optional[threading.Thread] = None
        if config.store_async:
            self._worker = threading.Thread(target=self._store_worker_loop,
                                            name="lmc-store", daemon=True)
            self._worker.start()

    # ----------------------------------------------------------- set-up
    def post_init(self, kvcaches=None, **kw) -> None:
        if kvcaches is not None and hasattr(self.gpu_connector, "register_kv_caches"):
            self.gpu_connector.register_kv_caches(kvcaches)
        for b in self.storage_manager.backends.values():
            hook = getattr(b, "post_init", None)
            if hook is not None:
                hook(gpu_connector=self.gpu_connector, engine=self, **kw)

    def is_healthy(self) -> bool:
        return self._healthy and not self._closed

    def mark_unhealthy(self, why: str) -> None:
        logger.error("engine marked unhealthy: %s", why)
        self._healthy = False

    def _passive(self) -> bool:
        """MLA latent is replicated across TP ranks: only rank 0 stores."""
        return self.config.save_only_first_rank and self.metadata.worker_id != 0

    def _key(self, key: CacheEngineKey) -> CacheEngineKey:
        if self.config.save_only_first_rank and key.worker_id != 0:
            return key.with_worker(0)
        return key

    # ------------------------------------------------------------ store
    def _chunks(self, tokens, mask=None, request_configs=None,
                hashes=None, offsets=None) -> List[Tuple[int, int, CacheEngineKey]]:
        return [(s, e, self._key(k)) for s, e, k in self.token_database.process_tokens(
            tokens=tokens, hashes=hashes, offsets=offsets, mask=mask,
            request_configs=request_configs)]

    @nvtx_range("lmc.store")
    def store(self, tokens: Optional[torch.Tensor] = None,
              mask: Optional[torch.Tensor] = None, **kwargs) -> None:
        """Store the KV of ``tokens`` (chunks not yet cached) from the paged cache.

        kwargs: ``slot_mapping`` (device tensor, one slot per token),
        ``kvcaches`` (optional re-registration), ``req_id``,
        ``request_configs``, ``hashes``/``offsets`` (precomputed chunk hashes).
        """
        if not self.is_healthy():
            logger.warning("store skipped: engine unhealthy")
            return
        if self._passive():
            return
        if self.config.store_async and self._worker is not None:
            req = _StoreRequest(kwargs.get("req_id"), tokens, mask, kwargs)
            with self._pending_cv:
                self._pending += 1
            self._store_queue.put(req)
            return
        self._run_store(tokens, mask, **kwargs)

    def _run_store(self, tokens, mask=None, **kwargs) -> int:
        with self.stats.phase("store.process_tokens"):
            chunks = self._chunks(tokens, mask, kwargs.get("request_configs"),
                                  kwargs.get("hashes"), kwargs.get("offsets"))
        todo = [(s, e, k) for s, e, k in chunks
                if self.storage_manager.contains(k) is None]
        if not todo:
            return 0
        if "kvcaches" in kwargs and kwargs["kvcaches"] is not None and \
                not getattr(self.gpu_connector, "kvcaches_registered", True):
            self.gpu_connector.register_kv_caches(kwargs["kvcaches"])
        objs, starts, ends, keys = [], [], [], []
        fmt = getattr(self.gpu_connector, "memory_format", MemoryFormat.KV_2LTD)
        dtype = self.gpu_connector.layout.dtype
        for s, e, k in todo:
            obj = self.storage_manager.allocate(self.gpu_connector.get_shape(e - s), dtype, fmt)
            if obj is None:
                logger.warning("store: out of CPU cache memory after %d chunks", len(objs))
                break
            objs.append(obj)
            starts.append(s)
            ends.append(e)
            keys.append(k)
        if not objs:
            return 0
        with self.stats.phase("store.from_gpu"):
            self.gpu_connector.batched_from_gpu(objs, starts, ends,
                                                slot_mapping=kwargs["slot_mapping"])
        with self.stats.phase("store.put"):
            self.storage_manager.batched_put(keys, objs,
                                             transfer_spec=kwargs.get("transfer_spec"))
        for o in objs:
            o.ref_count_down()
        if self.config.enable_kv_events:
            self._emit_events(tokens, starts, ends, keys)
        n = sum(e - s for s, e in zip(starts, ends))
        self.stats.inc("stored_tokens", n)
        return n

    # ---------------------------------------------- direct prefill push
    def _pd_backend(self):
        pd = self.storage_manager.backends.get("PDBackend")
        if pd is None:
            raise RuntimeError("direct prefill push needs enable_pd")
        return pd

    @staticmethod
    def _host_and_device(slots: torch.Tensor, dev, dtype=None):
        """(host copy, device copy) of a slot mapping; host tensors travel to
        the device without blocking when pinned."""
        host = slots if slots.device.type == "cpu" else slots.cpu()
        d = slots.to(dev, non_blocking=True) if dev is not None else slots
        if dtype is not None and d.dtype != dtype:
            d = d.to(dtype)
        return host, d

    @nvtx_range("lmc.store_direct_prefill")
    def store_direct_prefill(self, tokens: Optional[torch.Tensor] = None, *,
                             slot_mapping: torch.Tensor, dst_slot_mapping: torch.Tensor,
                             req_id: str, layer_begin: int = 0,
                             num_layers: Optional[int] = None) -> int:
        """Prefiller: push this request's KV rows from the local paged cache
        straight into the decoder's paged blocks (``dst_slot_mapping``, the
        decoder's block allocation) with the fused kernel, on the current
        stream.  The decoder must grant the push first (its registration is
        current and the slots are the ones it reserved for ``req_id``); a
        refusal or a dead decoder raises before anything is launched.
        Returns the number of tokens pushed (reference cache_engine.py:2634
        ``store_direct_prefill``)."""
        if not self.is_healthy() or self._passive():
            return 0
        pd = self._pd_backend()
        n = int(slot_mapping.numel())
        dev = pd.push_sender.device if pd.push_sender is not None else None
        _, src = self._host_and_device(slot_mapping, dev)
        host_dst, dst = self._host_and_device(dst_slot_mapping, dev, src.dtype)
        pd.direct_push(src, dst, req_id, layer_begin, num_layers, dst_slots_host=host_dst)
        self.stats.inc("stored_tokens", n)
        return n

    def begin_direct_prefill(self, req_id: str, *, slot_mapping: torch.Tensor,
                             dst_slot_mapping: Optional[torch.Tensor] = None,
                             num_layers: Optional[int] = None, token_begin: int = 0,
                             tile_tokens: int = 512) -> "DirectPrefillPush":
        """Prefiller, layer-by-layer push during the prefill forward: get the
        decoder's grant for every layer of ``req_id`` now (raises, with
        nothing launched, on refusal), then call ``push_layer`` on the
        returned handle as each layer's KV is written.

        ``slot_mapping``: this prefiller's slots of the tokens to push.
        ``dst_slot_mapping``: the decoder's slots for them, when the caller
        knows them; ``None`` takes them from the decoder's reservation of
        ``req_id`` (from reserved token ``token_begin`` on): ``slot_mapping``
        then covers prompt positions 0 .. len-1 and the push covers the
        reserved positions among them (``handle.num_tokens``)."""
        pd = self._pd_backend()
        if pd.push_sender is None:
            raise RuntimeError("direct push needs a registered paged cache on the prefiller")
        dev = pd.push_sender.device
        L = pd.push_sender.layout.num_layers
        nl = L if num_layers is None else num_layers
        if dst_slot_mapping is None:
            # slot_mapping covers prompt positions [0, len); the decoder's
            # reservation starts at its own first_token
            granted, first = pd.reserve_direct_push(req_id, -1, None, 0, nl, tile_tokens,
                                                    token_begin, int(slot_mapping.numel()))
            n = len(granted)
            start = first + token_begin
            _, src = self._host_and_device(slot_mapping[start:start + n], dev)
            host = torch.tensor(granted, dtype=torch.int64).pin_memory() \
                if torch.cuda.is_available() else torch.tensor(granted, dtype=torch.int64)
            _, dst = self._host_and_device(host, dev, src.dtype)
        else:
            _, src = self._host_and_device(slot_mapping, dev)
            host_dst, dst = self._host_and_device(dst_slot_mapping, dev, src.dtype)
            pd.reserve_direct_push(req_id, int(src.numel()), host_dst, 0, nl, tile_tokens,
                                   token_begin)
        self.stats.inc("stored_tokens", int(src.numel()))
        return DirectPrefillPush(pd, req_id, src, dst, nl, tile_tokens)

    def wait_direct_prefill(self, req_id: str, timeout_s: Optional[float] = None,
                            sync: bool = False) -> bool:
        """Decoder: enqueue the bounded per-layer wait for a direct push on the
        current stream (``sync`` also checks the device status on the host)."""
        return self._pd_backend().wait_direct(req_id, timeout_s, sync)

    def reserve_direct_prefill(self, req_id: str, dst_slot_mapping,
                               first_token: int = 0) -> None:
        """Decoder: these paged-cache slots (for prompt positions
        ``first_token`` ..) are allocated for ``req_id``; only a push into
        exactly them is granted."""
        self._pd_backend().reserve_direct(req_id, dst_slot_mapping, first_token)

    def direct_prefill_granted(self, req_id: str) -> bool:
        """Decoder: every reserved token of ``req_id`` was granted to the
        prefiller (its flags can now be waited for)."""
        return self._pd_backend().direct_granted(req_id)

    def cancel_direct_prefill(self, req_id: str) -> None:
        self._pd_backend().cancel_direct(req_id)

    def wait_direct_prefill_layer(self, req_id: str, layer: int,
                                  timeout_s: Optional[float] = None) -> bool:
        """Decoder: enqueue the bounded wait for layers up to ``layer`` of a
        granted direct push on the current stream (no host wait)."""
        return self._pd_backend().wait_direct_layer(req_id, layer, timeout_s)

    def _emit_events(self, tokens, starts, ends, keys) -> None:
        toks = tokens.tolist() if isinstance(tokens, torch.Tensor) else list(tokens)
        parent = None
        for s, e, k in zip(starts, ends, keys):
            self.kv_events.append(CacheStoreEvent([k.chunk_hash], parent, toks[s:e], e - s))
            parent = k.chunk_hash

    def _store_worker_loop(self) -> None:
        while True:
            req = self._store_queue.get()
            if req is None:
                return
            try:
                self._run_store(req.tokens, req.mask, **req.kwargs)
            except BaseException as e:  # keep the worker alive
                req.error = e
                logger.exception("async store failed")
            finally:
                with self._finished_lock:
                    if req.req_id is not None:
                        self._finished_stores.append(req.req_id)
                with self._pending_cv:
                    self._pending -= 1
                    self._pending_cv.notify_all()
                req.done.set()

    def get_finished_stores(self) -> List[Any]:
        with self._finished_lock:
            out, self._finished_stores = self._finished_stores, []
            return out

    def wait_for_pending_stores(self, timeout: Optional[float] = None) -> bool:
        with self._pending_cv:
            return self._pending_cv.wait_for(lambda: self._pending == 0, timeout=timeout)

    # --------------------------------------------------------- retrieve
    @nvtx_range("lmc.retrieve")
    def retrieve(self, tokens: torch.Tensor, mask: Optional[torch.Tensor] = None,
                 **kwargs) -> torch.Tensor:
        """Load the longest cached prefix of ``tokens`` into the paged cache.

        Returns a bool mask over ``tokens``: True where KV was loaded.
        """
        n = len(tokens)
        ret = torch.zeros(n, dtype=torch.bool)
        if not self.is_healthy():
            return ret
        chunks = self._chunks(tokens, mask, kwargs.get("request_configs"),
                              kwargs.get("hashes"), kwargs.get("offsets"))
        if not chunks:
            return ret
        with self.stats.phase("retrieve.get"):
            objs = self.storage_manager.batched_get([k for _, _, k in chunks])
        good, starts, ends = [], [], []
        for (s, e, _), o in zip(chunks, objs):
            if o is None:
                break  # prefix semantics: stop at the first miss
            good.append(o)
            starts.append(s)
            ends.append(e)
        for o in objs[len(good):]:
            if o is not None:
                o.ref_count_down()
        if good:
            with self.stats.phase("retrieve.to_gpu"):
                self.gpu_connector.batched_to_gpu(good, starts, ends,
                                                  slot_mapping=kwargs["slot_mapping"])
            for o in good:
                o.ref_count_down()
            for s, e in zip(starts, ends):
                ret[s:e] = True
        self.stats.inc("retrieved_tokens", int(ret.sum()))
        return ret

    # ----------------------------------------------------------- lookup
    def lookup(self, tokens: Optional[torch.Tensor] = None,
               search_range: Optional[List[str]] = None, lookup_id: Any = None,
               pin: bool = False, request_configs: Optional[dict] = None,
               hashes: Optional[List[int]] = None, offsets: Optional[List[int]] = None
               ) -> int:
        """Number of prefix tokens whose chunks are cached (pinned if asked)."""
        with self._engine_state_lock:
            end = 0
            pinned = []
            for s, e, k in self._chunks(tokens, None, request_configs, hashes, offsets):
                k = self._lookup_key(k)
                if self.storage_manager.contains(k, search_range, pin=pin) is None:
                    break
                if pin:
                    pinned.append(k)
                end = e
            if pin and lookup_id is not None:
                self._lookup_pins.setdefault(lookup_id, []).extend(pinned)
            self.stats.inc("lookup_hit_tokens", end)
            return end

    _LAYER_KEY_MEMO = 2048  # chunks (a 512k-token working set at 256 tokens a chunk)

    def _split(self, key: CacheEngineKey, num_layers: int) -> list:
        """The per-layer keys of ``key``, memoised (LRU over chunk keys)."""
        memo = self._layer_keys
        with self._layer_keys_lock:
            got = memo.get(key)
            if got is not None and len(got) == num_layers:
                memo.move_to_end(key)
                return got
        got = key.split_layers(num_layers)
        with self._layer_keys_lock:
            memo[key] = got
            while len(memo) > self._LAYER_KEY_MEMO:
                memo.popitem(last=False)
        return got

    def _lookup_key(self, key: CacheEngineKey) -> CacheEngineKey:
        """Layerwise stores keep one object per layer: probe the last layer,
        which is written together with the others once the store finished."""
        if self.config.use_layerwise and getattr(self.gpu_connector, "layout", None) is not None:
            L = self.gpu_connector.layout.num_layers
            return self._split(key, L)[L - 1]
        return key

    def agree_restorable(self, tokens: torch.Tensor) -> bool:
        """Every TP rank holds all chunks of ``tokens`` (restore agreement,
        reference cache_engine.py:9685-9742).  Each rank checks its own tiers;
        with ``collective_all_true_fn`` (a TP-group all-reduce every rank runs
        in the same step) the answer is the same on every rank."""
        local = self.lookup(tokens) >= len(tokens)
        fn = self.collective_all_true_fn
        return bool(fn(local)) if fn is not None else local

    def lookup_unpin(self, lookup_id: Any) -> None:
        with self._engine_state_lock:
            for k in self._lookup_pins.pop(lookup_id, []):
                self.storage_manager.unpin(k)

    # -------------------------------------------------------- layerwise
    def store_layer(self, tokens: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    **kwargs) -> Generator[None, None, None]:
        """Generator: yields num_layers + 1 times; resume after each layer's KV
        is written so that layer is gathered while the next one computes."""
        conn = self.gpu_connector
        if not self.is_healthy() or self._passive():
            for _ in range(conn.layout.num_layers + 1):
                yield
            return
        chunks = [(s, e, k) for s, e, k in self._chunks(tokens, mask)
                  if self.storage_manager.contains(k) is None]
        L = conn.layout.num_layers
        dtype = conn.layout.dtype
        fmt = getattr(conn, "memory_format", MemoryFormat.KV_2LTD)
        per_layer: List[List[MemoryObj]] = []
        for layer in range(L):
            row = []
            for s, e, k in chunks:
                o = self.storage_manager.allocate(conn.get_shape(e - s), dtype, fmt)
                if o is None:
                    raise RuntimeError("store_layer: out of CPU cache memory")
                # positions the keys were rotated for (CacheBlend re-positions them)
                o.meta.cached_positions = torch.arange(s, e)
                row.append(o)
            per_layer.append(row)
        starts = [s for s, _, _ in chunks]
        ends = [e for _, e, _ in chunks]
        gen = conn.batched_from_gpu(per_layer, starts, ends,
                                    slot_mapping=kwargs["slot_mapping"])
        next(gen)
        for layer in range(L):
            yield
            next(gen, None)
        next(gen, None)  # finish the generator: every layer's bytes are in the objects
        q = self.layerwise_put_queue
        req_id = kwargs.get("req_id", "")
        split = [self._split(k, L) for _, _, k in chunks]
        for layer in range(L):
            lkeys = [ks[layer] for ks in split]
            size = sum(o.get_size() for o in per_layer[layer])
            q.admit(size)
            try:
                futs = self.storage_manager.batched_put(lkeys, per_layer[layer])
            except BaseException as e:
                q.record_failure(e)
                raise
            q.submit(size, futs, req_id=req_id, keys=lkeys)
            for o in per_layer[layer]:
                o.ref_count_down()
        yield

    @property
    def layerwise_put_queue(self):
        """Bound on layerwise puts in flight to asynchronous tiers."""
        if getattr(self, "_put_queue", None) is None:
            from .layerwise_cpu_fill import PutWindow

            c = self.config
            self._put_queue = PutWindow(c.layerwise_put_max_bytes,
                                        c.layerwise_put_max_batches,
                                        c.layerwise_put_timeout_secs)
        return self._put_queue

    def wait_layerwise_puts(self, req_ids: Optional[List[str]] = None) -> None:
        """Fence the layerwise puts of ``req_ids`` (all puts when None)."""
        q = self.layerwise_put_queue
        if req_ids is None:
            q.fence_all()
        else:
            q.fence(req_ids)

    # -------------------------------------------------- sparse retrieve
    def _extend_sparse_state(self, st: SparseRetrieveState, txn: "_SparseAppend", tokens,
                             mask, kwargs) -> None:
        """Fetch the chunks of ``tokens`` past ``st.total_tokens`` (prefix
        semantics: stop at the first miss) and rebuild the pointer table.  A
        partial last chunk of a shorter context is fetched again whole."""
        chunks = self._chunks(tokens, mask, kwargs.get("request_configs"),
                              kwargs.get("hashes"), kwargs.get("offsets"))
        if st.ends and chunks and chunks[-1][1] > st.total_tokens and \
                st.total_tokens % self.config.chunk_size:
            txn.drop_last()
        new = [(s_, e, k) for s_, e, k in chunks if e > st.total_tokens]
        if not new:
            return
        if new[0][0] != st.total_tokens:
            raise ValueError("sparse state and token chunks disagree on chunk boundaries")
        objs = self.storage_manager.batched_get([k for _, _, k in new])
        got = 0
        while got < len(objs) and objs[got] is not None:
            got += 1
        for o in objs[got:]:
            if o is not None:
                o.ref_count_down()
        for (_, e, k), o in zip(new[:got], objs[:got]):
            st.keys.append(k)
            st.ends.append(e)
            st.objs.append(o)
        if st.objs:
            st.chunk_tokens = st.chunk_tokens or self.config.chunk_size
            dev = self.gpu_connector.layout.device
            table = torch.tensor([o.data_ptr() for o in st.objs], dtype=torch.int64)
            st.ptrs = table.to(dev) if dev.type == "cuda" else table

    def _quarantine_sparse(self, st: SparseRetrieveState, why: str) -> None:
        """A sparse copy's completion is unknown: keep its source chunks
        referenced until the process restarts (they may still be read) and
        stop serving."""
        self.__dict__.setdefault("_quarantined", []).append(tuple(st.objs))
        for o in st.objs:
            o.ref_count_up()
        self.mark_unhealthy(f"sparse load failed ({why}); its source chunks are retained")

    def retrieve_layer_head_token_wise(self, tokens: torch.Tensor,
                                       mask: Optional[torch.Tensor] = None, *,
                                       sparse_state: SparseRetrieveState, **kwargs
                                       ) -> Generator[Optional[torch.Tensor], Any, None]:
        """Sparse (top-k) layerwise retrieve for long contexts whose KV stays
        in the CPU tier (reference lmcache_ascend/v1/cache_engine.py:7457):

            g = engine.retrieve_layer_head_token_wise(tokens, sparse_state=st)
            cached = next(g)            # bool mask of tokens the state covers
            for layer in range(L):
                g.send(SparseLayerRequest(selected_idx, dst_slots))
            done = next(g)              # bool mask of tokens loaded

        The first step (or a longer context) fetches the missing chunks once
        into ``st``; later steps only launch copies: each layer's selected
        rows move straight from the pinned chunks into the paged slots (one
        launch per layer, rows read through the device pointer table).  A
        copy that fails quarantines the chunks and marks the engine
        unhealthy, since the transfer may still be reading them."""
        n = len(tokens)
        ret = torch.zeros(n, dtype=torch.bool)
        if not self.is_healthy():
            yield ret
            return
        st = sparse_state
        txn = _SparseAppend(st)
        try:
            self._extend_sparse_state(st, txn, tokens, mask, kwargs)
            txn.commit()
        finally:
            txn.rollback()
        ret[:st.total_tokens] = True
        layout = self.gpu_connector.layout
        loaded = torch.zeros(n, dtype=torch.bool)
        req = yield ret
        from ..ops import api

        status = kwargs.get("status")
        for layer in range(layout.num_layers):
            if req is None:
                break
            if st.objs:
                try:
                    idx = req.selected_token_idx
                    sm = req.slot_mapping
                    if layout.device.type == "cuda":
                        idx = idx.to(layout.device, sm.dtype)
                        api._xfer(layout, None, sm.to(layout.device), False,
                                  chunk_ptrs=st.ptrs, chunk_tokens=st.chunk_tokens,
                                  chunk_on_device=st.objs[0].tensor.is_cuda,
                                  layer_begin=layer, num_layers=1, chunk_layer_begin=layer,
                                  chunk_idx=idx, chunk_idx_limit=st.total_tokens,
                                  mode=api.MODE_SIMT if not st.objs[0].tensor.is_cuda
                                  else api.MODE_AUTO, status=status)
                    else:
                        self._sparse_layer_ref(layout, st, layer, idx, sm)
                    sel = req.selected_token_idx.long().cpu()
                    loaded[sel[(sel >= 0) & (sel < st.total_tokens)]] = True
                except BaseException as e:
                    self._quarantine_sparse(st, repr(e))
                    raise
            req = yield None
        self.stats.inc("sparse_retrieved_rows", int(loaded.sum()))
        yield loaded

    @staticmethod
    def _sparse_layer_ref(layout, st: SparseRetrieveState, layer: int, idx, slots) -> None:
        """CPU oracle of one sparse layer copy (host-resident caches)."""
        full = torch.cat([o.tensor for o in st.objs], dim=2)
        keep = (idx >= 0) & (idx < st.total_tokens)
        rows = full.index_select(2, idx[keep].long())
        layout.scatter_ref(rows, slots[keep], layer_begin=layer, num_layers=1,
                           chunk_layer_begin=layer)

    def retrieve_layer(self, tokens: torch.Tensor, mask: Optional[torch.Tensor] = None,
                       **kwargs) -> Generator[Optional[torch.Tensor], None, None]:
        """Generator: yields num_layers + 2 times.  The first yield returns
        after lookup; each following resume loads one layer; the last yield
        returns the retrieved-token mask."""
        conn = self.gpu_connector
        L = conn.layout.num_layers
        n = len(tokens)
        ret = torch.zeros(n, dtype=torch.bool)
        chunks = self._chunks(tokens, mask)
        sm = self.storage_manager
        # the hit: chunks whose last layer is stored (store_layer puts layers
        # in order, so the last layer present means every layer is)
        hit = 0
        split = []
        for _, _, k in chunks:
            ks = self._split(k, L)
            if sm.contains(ks[L - 1]) is None:
                break
            split.append(ks)
            hit += 1
        chunks = chunks[:hit]
        layers = _LazyLayers(sm, split, L)
        if hit:
            hit = layers.prefix_of_layer0()  # layer 0 now; later layers on demand
            chunks = chunks[:hit]
        starts = [s for s, _, _ in chunks]
        ends = [e for _, e, _ in chunks]
        yield None
        if hit:
            gen = conn.batched_to_gpu(None, starts, ends, slot_mapping=kwargs["slot_mapping"])
            next(gen)
            gen.send(layers)
            for layer in range(1, L):
                yield None
                next(gen)
            yield None
            next(gen, None)
            layers.release()
            for s, e in zip(starts[:layers.complete], ends[:layers.complete]):
                ret[s:e] = True
        else:
            for _ in range(L):
                yield None
        yield ret

    # ------------------------------------------------------------- misc
    def prefetch(self, tokens: torch.Tensor, mask: Optional[torch.Tensor] = None) -> None:
        """Promote cached chunks from lower tiers into the CPU tier."""
        for _, _, k in self._chunks(tokens, mask):
            obj = self.storage_manager.get(k)
            if obj is None:
                break
            obj.ref_count_down()

    def remove(self, tokens: torch.Tensor, locations: Optional[List[str]] = None) -> int:
        n = 0
        for _, _, k in self._chunks(tokens):
            n += self.storage_manager.remove(k, locations)
        return n

    def clear(self, locations: Optional[List[str]] = None) -> int:
        n = 0
        for name, b in self.storage_manager.backends.items():
            if locations is not None and name not in locations:
                continue
            for k in b.keys():
                n += int(b.remove(k))
        return n

    def get_kv_events(self) -> List[CacheStoreEvent]:
        return self.kv_events.drain()

    def close(self) -> None:
        if self._closed:
            return
        if self._worker is not None:
            self.wait_for_pending_stores(timeout=self.config.blocking_timeout_secs)
            self._store_queue.put(None)
            self._worker.join(timeout=5)
        if getattr(self, "_put_queue", None) is not None:
            try:
                self._put_queue.fence_all()  # fence puts before the allocator goes away
            except BaseException as e:
                logger.warning("layerwise puts failed before close: %s", e)
        self._closed = True
        self.storage_manager.close()
        close = getattr(self.gpu_connector, "close", None)
        if close:
            close()


class LMCacheEngineBuilder:
    """Process-wide registry of engines by instance id (upstream builder)."""

    _engines: Dict[str, LMCacheEngine] = {}
    _lock = threading.Lock()

    @classmethod
    def get_or_create(cls, instance_id: str, config: LMCacheEngineConfig,
                      metadata: LMCacheEngineMetadata,
                      gpu_connector: GPUConnectorInterface, **kw) -> LMCacheEngine:
        with cls._lock:
            eng = cls._engines.get(instance_id)
            if eng is None or eng._closed:  # a closed engine is never handed out again
                eng = LMCacheEngine(config, metadata, gpu_connector, **kw)
                cls._engines[instance_id] = eng
            return eng

    @classmethod
    def register(cls, instance_id: str, engine: "LMCacheEngine") -> None:
        with cls._lock:
            cls._engines[instance_id] = engine

    @classmethod
    def get(cls, instance_id: str) -> Optional[LMCacheEngine]:
        return cls._engines.get(instance_id)

    @classmethod
    def destroy(cls, instance_id: str) -> None:
        with cls._lock:
            eng = cls._engines.pop(instance_id, None)
        if eng is not None:
            eng.close()


class DirectPrefillPush:
    """A granted layer-by-layer direct push of one request (prefiller side).

    ``push_layer(l, ready)`` makes a side stream wait for ``ready`` (the event
    after layer ``l``'s KV write; default: the current stream's position) and
    launches layer ``l``'s push there, so the push overlaps the next layers'
    forward.  ``finish()`` records completion; ``done()`` polls it; the
    source blocks must stay allocated until it is True."""

    def __init__(self, pd, req_id: str, src: torch.Tensor, dst: torch.Tensor,
                 num_layers: int, tile_tokens: int):
        self.pd, self.req_id = pd, req_id
        self.src, self.dst = src, dst
        self.num_tokens = int(src.numel())
        self.num_layers, self.tile_tokens = num_layers, tile_tokens
        self.pushed = 0
        self._done_event: Optional[torch.cuda.Event] = None
        self._finished = False
        self.stream = None
        if src.is_cuda:
            self.stream = torch.cuda.Stream(device=src.device)
            # the slot tables were copied on the caller's stream
            staged = torch.cuda.Event()
            staged.record()
            self.stream.wait_event(staged)
            src.record_stream(self.stream)
            dst.record_stream(self.stream)

    def push_layer(self, layer: int, ready: Optional[torch.cuda.Event] = None) -> None:
        if self.stream is None:  # host-resident caches (CPU tier tests)
            self.pd.push_granted_layers(self.src, self.dst, layer, 1, self.tile_tokens)
            self.pushed += 1
            return
        if ready is None:
            ready = torch.cuda.Event()
            ready.record()
        self.stream.wait_event(ready)
        with torch.cuda.stream(self.stream):
            self.pd.push_granted_layers(self.src, self.dst, layer, 1, self.tile_tokens)
        self.pushed += 1

    def finish(self) -> Optional[torch.cuda.Event]:
        self._finished = True
        if self.stream is None:
            return None
        ev = torch.cuda.Event()
        ev.record(self.stream)
        self._done_event = ev
        return ev

    def done(self) -> bool:
        if not self._finished:
            return False
        return self._done_event is None or self._done_event.query()
