"""vLLM v1 KV-connector logic (scheduler and worker roles).

Behaviour of the reference's ``LMCacheAscendConnectorV1Impl``
(lmcache_ascend/integration/vllm/vllm_v1_adapter.py:211-1950) and upstream
LMCache's vLLM v1 adapter, re-implemented against the v1 connector API:

scheduler role
  ``get_num_new_matched_tokens`` asks the engine (over the lookup channel)
  how many prompt tokens are cached, never the whole prompt (vLLM must
  compute at least one token); ``update_state_after_alloc`` records the
  blocks vLLM gave the request; ``build_connector_meta`` turns each
  scheduled request into a ``ReqMeta`` (token ids, slot mapping from the
  block table, what to load, what to save).
worker role
  ``register_kv_caches`` hands vLLM's per-layer KV tensors to the engine;
  ``start_load_kv`` / ``wait_for_layer_load`` retrieve (whole or layer by
  layer); ``save_kv_layer`` / ``wait_for_save`` store (layer by layer or at
  the end of the step).

disaggregated prefill, direct paged push (``enable_pd`` with the NVLink
channel; the reference drives the same from ``save_kv_layer`` with
per-layer source-ready events, vllm_v1_adapter.py:668-752, and submits after
a preflight, :803-818)
  The router gives the prefill and the decode instance the same
  ``kv_transfer_params = {"lmcache_direct_push": True, "pd_req_id": ID}``.
  Decoder (``kv_consumer``): the scheduler reports the prompt (minus the
  token vLLM computes itself) as an asynchronous external hit, vLLM
  allocates blocks, and the worker reserves exactly those slots for ID.
  Prefiller (``kv_producer``): at the first ``save_kv_layer`` of a step the
  worker asks the decoder for the grant (its slots come back in it; a dead
  decoder, a stale registration or a refusal raises before anything is
  launched), then launches layer l's push on a side stream behind layer
  l's KV write, so it overlaps layers l+1.. of the forward.  vLLM keeps the
  prefiller's blocks until ``get_finished`` reports the push done; the
  decoder's ``get_finished`` reports the request received once every
  layer's flag arrived (bounded device wait).

This module only uses attribute access on vLLM's objects, so the logic can be
exercised with light stand-ins in tests; ``connector.py`` binds it to
``KVConnectorBase_V1``.
"""

from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from ...config import LMCacheEngineConfig, LMCacheEngineMetadata
from ...utils.logging import init_logger
from .lookup import LookupClient, LookupServer, lookup_ipc_path

logger = init_logger(__name__)


@dataclass
class LoadSpec:
    vllm_cached_tokens: int
    lmcache_cached_tokens: int
    can_load: bool = False


@dataclass
class SaveSpec:
    skip_leading_tokens: int
    can_save: bool


@dataclass
class RequestTracker:
    req_id: str
    prompt_len: int
    token_ids: List[int]
    allocated_block_ids: List[int]
    num_saved_tokens: int = 0
    disagg_spec: Optional[dict] = None
    num_pushed_tokens: int = 0  # prompt tokens handed to the direct push so far
    group_block_ids: List[List[int]] = field(default_factory=list)  # groups 1..

    def update(self, new_token_ids: Sequence[int], new_block_ids: Optional[Sequence[int]],
               new_group_blocks: Optional[Sequence[Sequence[int]]] = None):
        self.token_ids.extend(new_token_ids)
        if new_block_ids:
            self.allocated_block_ids.extend(new_block_ids)
        for g, blocks in enumerate(new_group_blocks or ()):
            while len(self.group_block_ids) <= g:
                self.group_block_ids.append([])
            if blocks:
                self.group_block_ids[g].extend(blocks)


@dataclass
class ReqMeta:
    req_id: str
    token_ids: torch.Tensor
    slot_mapping: torch.Tensor
    save_spec: Optional[SaveSpec] = None
    load_spec: Optional[LoadSpec] = None
    is_last_prefill: bool = False
    disagg_spec: Optional[dict] = None
    # direct paged push: {"mode": "send"|"recv", "pd_req_id": ID, ...}
    direct: Optional[dict] = None
    # KV cache groups after the first (e.g. the DSA indexer cache): slots of
    # the same tokens in each group's own block table
    group_slot_mappings: List[torch.Tensor] = field(default_factory=list)

    def slots_of_group(self, g: int) -> torch.Tensor:
        return self.slot_mapping if g == 0 else self.group_slot_mappings[g - 1]

    @staticmethod
    def build(tracker: RequestTracker, block_size: int, chunk_size: int,
              load_spec: Optional[LoadSpec], tokens_done: int, save_unfull_chunk: bool,
              skip_save: bool) -> Optional["ReqMeta"]:
        """``tokens_done``: prompt tokens whose KV exists once this step ran."""
        tokens_done = min(tokens_done, tracker.prompt_len)
        is_last_prefill = tokens_done >= tracker.prompt_len
        save = None
        n_save = 0
        if not skip_save:
            n_save = tokens_done if (is_last_prefill and save_unfull_chunk) else \
                (tokens_done // chunk_size) * chunk_size
            if n_save > tracker.num_saved_tokens:
                save = SaveSpec((tracker.num_saved_tokens // chunk_size) * chunk_size, True)
                tracker.num_saved_tokens = n_save
            else:
                n_save = 0
        loading = load_spec is not None and load_spec.can_load
        if save is None and not loading:
            return None
        ntoks = max(n_save, load_spec.lmcache_cached_tokens if loading else 0)
        blocks = torch.tensor(tracker.allocated_block_ids, dtype=torch.long)
        t = torch.arange(ntoks)
        slot = blocks[t // block_size] * block_size + t % block_size
        r = ReqMeta(tracker.req_id, torch.tensor(tracker.token_ids[:ntoks], dtype=torch.long),
                    slot, save, load_spec if loading else None, is_last_prefill,
                    tracker.disagg_spec)
        for gb in tracker.group_block_ids:
            b = torch.tensor(gb, dtype=torch.long)
            r.group_slot_mappings.append(b[t // block_size] * block_size + t % block_size)
        return r


@dataclass
class LMCacheConnectorMetadata:
    requests: List[ReqMeta] = field(default_factory=list)
    # preemption checkpoints: KV of a preempted request to copy out before
    # vLLM reuses its blocks ({"req_id", "generation", "token_ids",
    # "slot_mapping"}), and generations to forget
    preemption_captures: List[dict] = field(default_factory=list)
    preemption_cancels: List[Tuple[str, int]] = field(default_factory=list)

    def add_request(self, r: ReqMeta) -> None:
        self.requests.append(r)


def direct_push_id(request) -> Optional[str]:
    """The disaggregated request id shared by prefiller and decoder, when the
    router asked for a direct paged push of this request."""
    params = getattr(request, "kv_transfer_params", None) or {}
    if params.get("lmcache_direct_push") and params.get("pd_req_id"):
        return str(params["pd_req_id"])
    return None


def block_ids_of(blocks) -> List[int]:
    """Block ids of vLLM's ``KVCacheBlocks`` (first group) or a plain list."""
    if blocks is None:
        return []
    get = getattr(blocks, "get_block_ids", None)
    if callable(get):
        ids = get()
        return list(ids[0]) if ids and isinstance(ids[0], (list, tuple)) else list(ids)
    return list(blocks)


def slots_of(block_ids: Sequence[int], block_size: int, begin: int, end: int) -> torch.Tensor:
    blocks = torch.tensor(list(block_ids), dtype=torch.long)
    t = torch.arange(begin, end)
    return blocks[t // block_size] * block_size + t % block_size


def config_from_extra(extra: Optional[Dict[str, Any]]) -> LMCacheEngineConfig:
    """Engine config from LMCACHE_CONFIG_FILE / LMCACHE_* env, overridden by
    ``kv_connector_extra_config`` keys prefixed with ``lmcache.``
    (reference lmcache_ascend_connector_v1.py:46-49)."""
    cfg = LMCacheEngineConfig.from_env()
    over = {k: v for k, v in (extra or {}).items() if str(k).startswith("lmcache.")}
    if over:
        cfg.update(over)
    return cfg


class _GroupedLookup:
    """Lookup over every KV cache group's engine: a prefix counts as cached
    only as far as every group holds it."""

    def __init__(self, engines):
        self.engines = engines

    def lookup(self, tokens, lookup_id=None, pin: bool = False, **kw) -> int:
        hit = None
        for e in self.engines:
            n = e.lookup(tokens, lookup_id=lookup_id, pin=pin, **kw)
            hit = n if hit is None else min(hit, n)
        return hit or 0

    def lookup_unpin(self, lookup_id) -> None:
        for e in self.engines:
            e.lookup_unpin(lookup_id)


class _DoneEvent:
    @staticmethod
    def query() -> bool:
        return True


class LMCacheConnectorV1Impl:
    """Role-split connector logic.  ``role`` is "scheduler" or "worker".

    ``model_name``, ``world_size``/``rank``, ``block_size`` and ``use_mla``
    describe the model shard (taken from vLLM's config by ``connector.py``).
    A scheduler and a worker in one process can share one engine (``engine``
    argument); otherwise the scheduler reaches the worker's engine through
    the lookup channel.
    """

    def __init__(self, role: str, config: LMCacheEngineConfig, model_name: str,
                 block_size: int, world_size: int = 1, rank: int = 0, use_mla: bool = False,
                 dp_rank: int = 0, engine=None, kv_dtype=None, kv_role: str = "kv_both"):
        if kv_role not in ("kv_both", "kv_producer", "kv_consumer"):
            raise ValueError(f"unknown kv_role {kv_role!r}")
        self.role = role
        # vLLM's KVTransferConfig.kv_role: a consumer (disaggregated decoder)
        # only loads; producers and kv_both instances also save
        self.kv_role = kv_role
        self.config = config
        self.block_size = block_size
        self.chunk_size = config.chunk_size
        self.use_mla = use_mla
        self.rank = rank
        self.engine = engine
        self.metadata = LMCacheEngineMetadata(model_name, world_size, rank, "vllm", kv_dtype,
                                              use_mla=use_mla, role=role, dp_rank=dp_rank)
        self.lookup_url = lookup_ipc_path(config.lmcache_instance_id, dp_rank)
        # scheduler state
        self._trackers: Dict[str, RequestTracker] = {}
        self._load_specs: Dict[str, LoadSpec] = {}
        self._lookup = None
        if role == "scheduler":
            self._lookup = LookupClient(self.lookup_url, engine=engine)
        # worker state
        self._lookup_server = None
        self._meta: Optional[LMCacheConnectorMetadata] = None
        self._layer_names: List[str] = []
        self._layer_load_gens: List = []
        self._layer_store_gens: List = []
        self._layer_idx = 0
        # preemption checkpoints (scheduler side): live request objects,
        # computed-token count and preemption generation per request
        self._requests: Dict[str, Any] = {}
        self._computed: Dict[str, int] = {}
        self._generation: Dict[str, int] = {}
        self._checkpointer = None                   # worker: PreemptionCheckpointer
        # direct paged push state
        self._direct_recv: Dict[str, dict] = {}     # scheduler: decoder requests awaiting blocks
        self._direct_senders: set = set()           # scheduler: prefiller requests that push
        self._push_handles: Dict[str, Any] = {}     # worker: vLLM req id -> DirectPrefillPush
        self._step_handles: List[Tuple[str, Any]] = []
        self._sending: Dict[str, Any] = {}          # worker: pushes whose blocks vLLM holds
        self._receiving: Dict[str, dict] = {}       # worker: reserved decoder requests
        self._recv_stream = None
        self.load_error_block_ids: set = set()
        self._pushed: Dict[str, int] = {}   # worker: reserved tokens pushed per request
        self._push_failed: set = set()
        self._finished_pushers: set = set()  # finished in vLLM, blocks held for the push
        self._layer_index: Dict[str, int] = {}
        self._engines: List[Any] = []       # one engine per KV cache group
        self._group_names: List[List[str]] = []
        self._layer_group: Dict[str, int] = {}

    # ============================================================ scheduler
    @staticmethod
    def _all_tokens(request) -> List[int]:
        """Prompt plus generated tokens (a resumed request's prefix)."""
        allt = getattr(request, "all_token_ids", None)
        return list(allt) if allt is not None else list(request.prompt_token_ids or [])

    def on_new_request(self, request) -> None:
        self._requests[request.request_id] = request

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> Tuple[int, bool]:
        self._requests.setdefault(request.request_id, request)
        tokens = self._all_tokens(request)
        if not tokens:
            return 0, False
        pid = direct_push_id(request)
        if pid is not None and self.kv_role == "kv_consumer":
            # the prefiller pushes the prompt's KV: an asynchronous external hit
            # of every prompt token vLLM does not compute itself
            need = len(tokens) - 1 - num_computed_tokens
            if need <= 0:
                return 0, False
            self._direct_recv[request.request_id] = {"pd_req_id": pid,
                                                     "first": num_computed_tokens, "n": need}
            return need, True
        hit = self._lookup.lookup(tokens, lookup_id=request.request_id)
        # vLLM must compute at least the last prompt token itself, so report
        # one token less; the load still covers every cached chunk (a chunk
        # cut short would hash differently) and vLLM overwrites that token.
        need = min(hit, len(tokens) - 1) - num_computed_tokens
        if need <= 0:
            self._lookup.unpin(request.request_id)
            return 0, False
        self._load_specs[request.request_id] = LoadSpec(num_computed_tokens, hit, False)
        return need, False

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        rec = self._direct_recv.get(request.request_id)
        if rec is not None:
            if num_external_tokens == 0:
                self._direct_recv.pop(request.request_id, None)
            else:
                rec["n"] = num_external_tokens
                rec["blocks"] = block_ids_of(blocks)
            return
        spec = self._load_specs.get(request.request_id)
        if spec is None:
            return
        if num_external_tokens == 0:
            spec.can_load = False
            return
        spec.can_load = True

    def _direct_send_meta(self, tr: RequestTracker, done: int) -> Optional[ReqMeta]:
        """Prefiller: the tokens computed by this step go to the decoder."""
        done = min(done, tr.prompt_len)
        if done <= tr.num_pushed_tokens:
            return None
        slots = slots_of(tr.allocated_block_ids, self.block_size, 0, done)
        r = ReqMeta(tr.req_id, torch.tensor(tr.token_ids[:done], dtype=torch.long), slots,
                    is_last_prefill=done >= tr.prompt_len)
        r.direct = {"mode": "send", "pd_req_id": tr.disagg_spec["pd_req_id"],
                    "token_begin": tr.num_pushed_tokens}
        tr.num_pushed_tokens = done
        return r

    def _capture_specs(self, scheduler_output, meta: LMCacheConnectorMetadata) -> None:
        """Preempted requests: their blocks still hold the KV computed so far
        (vLLM reuses them in this step's forward); the worker copies it out in
        ``handle_preemptions`` and publishes it under the request's token
        chain, so the resumed request finds it as a prefix hit."""
        for req_id in getattr(scheduler_output, "preempted_req_ids", None) or ():
            tr = self._trackers.get(req_id)
            n = self._computed.get(req_id, 0)
            req = self._requests.get(req_id)
            if tr is None or n <= 0:
                continue
            tokens = self._all_tokens(req) if req is not None else tr.token_ids
            n = min(n, len(tokens), len(tr.allocated_block_ids) * self.block_size)
            gen = self._generation.get(req_id, 0) + 1
            self._generation[req_id] = gen
            meta.preemption_captures.append({
                "req_id": req_id, "generation": gen,
                "token_ids": torch.tensor(tokens[:n], dtype=torch.long),
                "slot_mapping": slots_of(tr.allocated_block_ids, self.block_size, 0, n)})

    def build_connector_meta(self, scheduler_output) -> LMCacheConnectorMetadata:
        meta = LMCacheConnectorMetadata()
        self._capture_specs(scheduler_output, meta)
        for req_id in getattr(scheduler_output, "finished_req_ids", ()) or ():
            self._trackers.pop(req_id, None)
            self._load_specs.pop(req_id, None)
            self._direct_recv.pop(req_id, None)
            self._requests.pop(req_id, None)
            self._computed.pop(req_id, None)
            gen = self._generation.pop(req_id, None)
            if gen is not None:
                meta.preemption_cancels.append((req_id, gen))
        # decoder: requests whose blocks were just allocated for the push
        for req_id, rec in list(self._direct_recv.items()):
            if "blocks" not in rec:
                continue
            self._direct_recv.pop(req_id)
            slots = slots_of(rec["blocks"], self.block_size, rec["first"],
                             rec["first"] + rec["n"])
            r = ReqMeta(req_id, torch.empty(0, dtype=torch.long), slots)
            r.direct = {"mode": "recv", "pd_req_id": rec["pd_req_id"], "first": rec["first"]}
            meta.add_request(r)
        for new in scheduler_output.scheduled_new_reqs:
            tokens = list(new.prompt_token_ids or [])
            blocks = list(new.block_ids[0]) if new.block_ids else []
            tr = RequestTracker(new.req_id, len(tokens), tokens, blocks)
            if new.block_ids and len(new.block_ids) > 1:
                tr.group_block_ids = [list(b) for b in new.block_ids[1:]]
            self._trackers[new.req_id] = tr
            pid = direct_push_id(new) if self.kv_role == "kv_producer" else None
            if pid is not None and self.engine_supports_direct():
                tr.disagg_spec = {"pd_req_id": pid}
                self._direct_senders.add(new.req_id)
                done = new.num_computed_tokens + scheduler_output.num_scheduled_tokens[new.req_id]
                r = self._direct_send_meta(tr, done)
                if r is not None:
                    meta.add_request(r)
                continue
            spec = self._load_specs.pop(new.req_id, None)
            done = new.num_computed_tokens + scheduler_output.num_scheduled_tokens[new.req_id]
            self._computed[new.req_id] = done
            if spec is not None and spec.can_load:
                tr.num_saved_tokens = (spec.lmcache_cached_tokens // self.chunk_size) * \
                    self.chunk_size  # already cached: do not store again
            r = ReqMeta.build(tr, self.block_size, self.chunk_size, spec, done,
                              self.config.save_unfull_chunk, skip_save=False)
            if r is not None:
                meta.add_request(r)
        cached = scheduler_output.scheduled_cached_reqs
        resumed = set(getattr(cached, "resumed_req_ids", None) or ())
        for i, req_id in enumerate(getattr(cached, "req_ids", []) or []):
            tr = self._trackers.get(req_id)
            if tr is None:
                continue
            new_blocks = cached.new_block_ids[i]
            done = cached.num_computed_tokens[i] + scheduler_output.num_scheduled_tokens[req_id]
            self._computed[req_id] = done
            if req_id in resumed:
                # back from preemption: a fresh block table; load what the
                # checkpoint (or any earlier store) holds of its prefix
                req = self._requests.get(req_id)
                tokens = self._all_tokens(req) if req is not None else tr.token_ids
                tr.token_ids = list(tokens)
                tr.allocated_block_ids = list(new_blocks[0]) if new_blocks else []
                tr.group_block_ids = [list(b) for b in new_blocks[1:]] if new_blocks else []
                spec = self._load_specs.pop(req_id, None)
                if spec is not None and spec.can_load:
                    tr.num_saved_tokens = max(tr.num_saved_tokens,
                                              (spec.lmcache_cached_tokens // self.chunk_size)
                                              * self.chunk_size)
                    r = ReqMeta.build(tr, self.block_size, self.chunk_size, spec, done,
                                      self.config.save_unfull_chunk, skip_save=True)
                    if r is not None:
                        meta.add_request(r)
                continue
            tr.update(cached.new_token_ids[i] if cached.new_token_ids else [],
                      list(new_blocks[0]) if new_blocks else None,
                      [list(b) for b in new_blocks[1:]] if new_blocks and len(new_blocks) > 1
                      else None)
            if tr.disagg_spec is not None:  # chunked prefill of a direct push
                r = self._direct_send_meta(tr, done)
                if r is not None:
                    meta.add_request(r)
                continue
            if tr.num_saved_tokens >= tr.prompt_len:
                continue  # decode phase: nothing to store
            r = ReqMeta.build(tr, self.block_size, self.chunk_size, None, done,
                              self.config.save_unfull_chunk, skip_save=False)
            if r is not None:
                meta.add_request(r)
        return meta

    def engine_supports_direct(self) -> bool:
        return bool(self.config.enable_pd and self.config.pd_role == "sender")

    def request_finished(self, request, block_ids) -> Tuple[bool, Optional[dict]]:
        self._trackers.pop(request.request_id, None)
        self._requests.pop(request.request_id, None)
        self._direct_recv.pop(request.request_id, None)
        if self._lookup is not None:
            self._lookup.unpin(request.request_id)
        if request.request_id in self._direct_senders:
            # keep the blocks until the worker reports the push done
            self._direct_senders.discard(request.request_id)
            return True, None
        return False, None

    # =============================================================== worker
    def _ensure_engine(self):
        if self.engine is None:
            from ...v1.cache_engine import LMCacheEngineBuilder
            from ...v1.gpu_connector import CreateGPUConnector

            from ...v1.cache_engine import LMCacheEngine

            conn = CreateGPUConnector(self.config, self.metadata)
            self.engine = LMCacheEngine(self.config, self.metadata, conn)
            LMCacheEngineBuilder.register(f"{self.config.lmcache_instance_id}-{self.rank}",
                                          self.engine)
        return self.engine

    def register_kv_caches(self, kv_caches: Dict[str, torch.Tensor]) -> None:
        """vLLM passes {layer_name: tensor}; layer order is the model's."""
        def layer_index(name: str) -> int:
            for part in name.split("."):
                if part.isdigit():
                    return int(part)
            return 0

        self._layer_names = sorted(kv_caches, key=layer_index)
        from ...v1.kv_layer_groups import KVLayerGroupsManager

        self.layer_groups = KVLayerGroupsManager()
        self.layer_groups.build_kv_layer_groups({n: kv_caches[n] for n in self._layer_names})
        ng = self.layer_groups.num_groups
        # group g's layers, in layer order; index of a layer inside its group
        self._group_names = [list(grp.layer_names) for grp in self.layer_groups.kv_layer_groups]
        self._layer_group = {n: g for g, names in enumerate(self._group_names) for n in names}
        self._layer_index = {n: i for names in self._group_names for i, n in enumerate(names)}
        eng = self._ensure_engine()
        caches0 = [kv_caches[n] for n in self._group_names[0]]
        first = caches0[0] if isinstance(caches0[0], torch.Tensor) else caches0[0][0]
        if self.metadata.kv_dtype is None:
            self.metadata.kv_dtype = first.dtype
        eng.post_init(kvcaches=caches0)
        self._caches0 = caches0
        self._engines = [eng]
        for g in range(1, ng):
            self._engines.append(self._group_engine(g, [kv_caches[n]
                                                        for n in self._group_names[g]]))
        if self.rank == 0 and self._lookup_server is None:
            self._lookup_server = LookupServer(_GroupedLookup(self._engines), self.lookup_url)

    def _group_engine(self, g: int, caches):
        """Engine of KV cache group ``g`` > 0 (e.g. the DSA indexer): its own
        paged layout, chunk keys under its own instance id, a CPU tier sized
        by its share of the bytes per token."""
        import copy

        from ...v1.cache_engine import LMCacheEngine
        from ...v1.gpu_connector import CreateGPUConnector

        grp = self.layer_groups.kv_layer_groups
        per_tok = [x.num_layers * x.hidden_dim_size * (2 if len(x.shape) == 5 else 1)
                   for x in grp]
        cfg = copy.deepcopy(self.config)
        cfg.lmcache_instance_id = f"{self.config.lmcache_instance_id}-g{g}"
        cfg.max_local_cpu_size = max(0.01, self.config.max_local_cpu_size * per_tok[g] /
                                     max(1, sum(per_tok)))
        cfg.enable_pd = False  # the direct push moves the first group
        md = copy.deepcopy(self.metadata)
        md.model_name = f"{self.metadata.model_name}#g{g}"
        first = caches[0] if isinstance(caches[0], torch.Tensor) else caches[0][0]
        md.kv_dtype = first.dtype
        eng = LMCacheEngine(cfg, md, CreateGPUConnector(cfg, md))
        eng.post_init(kvcaches=caches)
        return eng

    def bind_connector_metadata(self, meta: LMCacheConnectorMetadata) -> None:
        self._meta = meta

    @property
    def checkpointer(self):
        if self._checkpointer is None:
            from ...v1.preemption_checkpoint import PreemptionCheckpointer

            self._checkpointer = PreemptionCheckpointer(self._ensure_engine())
        return self._checkpointer

    def handle_preemptions(self, meta: Optional[LMCacheConnectorMetadata] = None) -> None:
        """Before vLLM reuses a preempted request's blocks: copy its computed
        KV out (every TP rank its own shard) and publish it under the
        request's token chain; forget generations of finished requests
        (reference vllm_v1_adapter.py:1546-1614).  Stores still in flight for
        those requests are drained first, since they read the same blocks."""
        meta = meta if meta is not None else self._meta
        if meta is None or self.kv_role == "kv_consumer":
            return
        ck = self.checkpointer
        for req_id, gen in meta.preemption_cancels:
            ck.cancel(req_id, gen)
        if not meta.preemption_captures:
            return
        eng = self._ensure_engine()
        if self.config.store_async:
            eng.wait_for_pending_stores(timeout=self.config.blocking_timeout_secs)
        for cap in meta.preemption_captures:
            try:
                n = ck.capture(cap["req_id"], cap["generation"], cap["token_ids"].tolist(),
                               cap["slot_mapping"])
                if n:
                    ck.seal(cap["req_id"], cap["generation"], cap["token_ids"].tolist())
            except Exception as e:  # the request recomputes instead
                logger.warning("preemption checkpoint of %s failed: %s", cap["req_id"], e)
                ck.cancel(cap["req_id"], cap["generation"])

    def clear_connector_metadata(self) -> None:
        self._meta = None

    def _mask(self, n: int, skip: int) -> Optional[torch.Tensor]:
        if skip <= 0:
            return None
        m = torch.ones(n, dtype=torch.bool)
        m[:skip] = False
        return m

    def start_load_kv(self, forward_context=None, **kwargs) -> None:
        if self._meta is None:
            return
        eng = self._ensure_engine()
        self._layer_load_gens = []
        self._layer_idx = 0
        for r in self._meta.requests:
            if r.direct is not None and r.direct["mode"] == "recv":
                # decoder: these freshly allocated blocks take the prefiller's push
                eng.reserve_direct_prefill(r.direct["pd_req_id"], r.slot_mapping,
                                           first_token=r.direct["first"])
                self._receiving[r.req_id] = {
                    "pd_req_id": r.direct["pd_req_id"], "event": None,
                    "slots": r.slot_mapping, "deadline": time.monotonic()
                    + self.config.pd_reserve_timeout_s + self.config.pd_flag_timeout_s}
                continue
            spec = r.load_spec
            if spec is None or not spec.can_load:
                continue
            n = spec.lmcache_cached_tokens
            skip = (spec.vllm_cached_tokens // self.chunk_size) * self.chunk_size
            toks = r.token_ids[:n]
            mask = self._mask(n, skip)
            if not eng.agree_restorable(toks):
                # some TP rank cannot load this prefix: no rank loads it, and
                # vLLM recomputes the tokens of these blocks
                logger.warning("req %s: TP ranks disagree on a %d-token hit; recomputing",
                               r.req_id, n)
                self.load_error_block_ids.update(
                    (r.slot_mapping[skip:n] // self.block_size).unique().tolist())
                continue
            if self.config.enable_blending:
                # CacheBlend: retrieve the cached segments and recompute the
                # deviating tokens with the served model's weights, writing
                # the blended KV into this request's blocks (the serving
                # process registers its model under the instance id)
                from ...v1.blend.vllm_model import get_or_create_blender

                b = get_or_create_blender(self.config.lmcache_instance_id, eng,
                                          eng.gpu_connector, self.config, self._caches0)
                ret = b.blend(toks, mask, slot_mapping=r.slots_of_group(0)[:n])
                got = int(ret.sum())
                if got < n - skip:
                    logger.warning("req %s: blended %d of %d expected tokens", r.req_id,
                                   got, n - skip)
                continue
            for gi, geng in enumerate(self._engines):
                slots = r.slots_of_group(gi)[:n]
                if self.config.use_layerwise:
                    g = geng.retrieve_layer(toks, mask, slot_mapping=slots)
                    next(g)
                    self._layer_load_gens.append((gi, g))
                else:
                    ret = geng.retrieve(toks, mask, slot_mapping=slots)
                    got = int(ret.sum())
                    if got < n - skip:
                        logger.warning("req %s group %d: loaded %d of %d expected tokens",
                                       r.req_id, gi, got, n - skip)

    def wait_for_layer_load(self, layer_name: str) -> None:
        gi = self._layer_group.get(layer_name, 0)
        for g_, gen in self._layer_load_gens:
            if g_ == gi:
                next(gen, None)

    def _begin_direct_pushes(self, eng) -> None:
        """Prefiller, first layer of a step: one grant per pushing request
        (nothing is launched for a request whose grant failed)."""
        self._step_handles = []
        for r in self._meta.requests:
            if r.direct is None or r.direct["mode"] != "send":
                continue
            try:
                h = eng.begin_direct_prefill(r.direct["pd_req_id"], slot_mapping=r.slot_mapping,
                                             token_begin=self._pushed_of(r))
            except Exception as e:  # refused / dead decoder: no launch, request not pushed
                logger.warning("direct push of %s not granted: %s", r.req_id, e)
                self._push_failed.add(r.req_id)
                continue
            self._pushed[r.req_id] = self._pushed_of(r) + h.num_tokens
            self._step_handles.append((r.req_id, h))

    def _pushed_of(self, r: ReqMeta) -> int:
        return self._pushed.get(r.req_id, 0)

    def save_kv_layer(self, layer_name: str, kv_layer=None, attn_metadata=None, **kw) -> None:
        if self._meta is None or self.kv_role == "kv_consumer":
            return
        if any(r.direct is not None for r in self._meta.requests):
            eng = self._ensure_engine()
            idx = self._layer_index.get(layer_name, 0)
            if idx == 0:
                self._begin_direct_pushes(eng)
            # this layer's KV write is enqueued on the current stream: the push
            # of layer idx waits for it on the handle's side stream
            for _, h in self._step_handles:
                h.push_layer(idx)
        if not self.config.use_layerwise:
            return
        self._ensure_engine()
        gi = self._layer_group.get(layer_name, 0)
        if self._layer_index.get(layer_name, 0) == 0:  # first layer of its group
            if gi == 0:
                self._layer_store_gens = []
            geng = self._engines[gi]
            for r in self._meta.requests:
                if r.save_spec is None:
                    continue
                n = r.token_ids.numel()
                g = geng.store_layer(r.token_ids,
                                     self._mask(n, r.save_spec.skip_leading_tokens),
                                     slot_mapping=r.slots_of_group(gi))
                next(g)  # before the first layer
                self._layer_store_gens.append((gi, g))
        for g_, gen in self._layer_store_gens:
            if g_ == gi:
                next(gen, None)

    def wait_for_save(self) -> None:
        if self._meta is None or self.kv_role == "kv_consumer":
            return
        for req_id, h in self._step_handles:
            h.finish()  # the blocks stay with vLLM until get_finished reports it
            self._sending.setdefault(req_id, []).append(h)
        self._step_handles = []
        self._ensure_engine()
        if self.config.use_layerwise:
            for _, g in self._layer_store_gens:
                for _ in g:
                    pass
            self._layer_store_gens = []
            return
        for r in self._meta.requests:
            if r.save_spec is None or not r.save_spec.can_save:
                continue
            n = r.token_ids.numel()
            for gi, geng in enumerate(self._engines):
                geng.store(r.token_ids, self._mask(n, r.save_spec.skip_leading_tokens),
                           slot_mapping=r.slots_of_group(gi), req_id=r.req_id)

    def _poll_receiving(self) -> set:
        """Decoder: requests whose pushed KV has fully arrived.  Once every
        reserved token is granted, a bounded flag wait is enqueued on a side
        stream; its event completing means every layer landed.  A request
        never granted before its deadline is cancelled, and its blocks are
        reported as load errors."""
        done = set()
        eng = self.engine
        for req_id, st in list(self._receiving.items()):
            pid = st["pd_req_id"]
            if st["event"] is None:
                if eng.direct_prefill_granted(pid):
                    if not st["slots"].is_cuda and not torch.cuda.is_available():
                        eng.wait_direct_prefill(pid)  # host-resident caches: no device wait
                        st["event"] = _DoneEvent()
                    else:
                        if self._recv_stream is None:
                            self._recv_stream = torch.cuda.Stream()
                        with torch.cuda.stream(self._recv_stream):
                            eng.wait_direct_prefill(pid)
                            ev = torch.cuda.Event()
                            ev.record()
                        st["event"] = ev
                elif time.monotonic() > st["deadline"]:
                    logger.error("direct push of %s (%s) never granted; failing its load",
                                 req_id, pid)
                    eng.cancel_direct_prefill(pid)
                    self.load_error_block_ids.update(
                        (st["slots"] // self.block_size).unique().tolist())
                    self._receiving.pop(req_id)
                    done.add(req_id)
                    continue
            if st["event"] is not None and st["event"].query():
                pd = eng.storage_manager.backends.get("PDBackend")
                try:
                    pd.push_receiver.check()
                except RuntimeError as e:
                    logger.error("direct push of %s failed on the device: %s", req_id, e)
                    self.load_error_block_ids.update(
                        (st["slots"] // self.block_size).unique().tolist())
                self._receiving.pop(req_id)
                done.add(req_id)
        return done

    def _poll_sending(self) -> set:
        """Prefiller: finished requests whose pushes have all run (vLLM may
        free their blocks now)."""
        done = set()
        for req_id in list(self._finished_pushers):
            hs = self._sending.get(req_id, [])
            if all(h.done() for h in hs):
                self._sending.pop(req_id, None)
                self._pushed.pop(req_id, None)
                self._push_failed.discard(req_id)
                self._finished_pushers.discard(req_id)
                done.add(req_id)
        return done

    def get_finished(self, finished_req_ids) -> Tuple[Optional[set], Optional[set]]:
        sending = set()
        if self.engine is not None and self.config.store_async:
            sending |= set(self.engine.get_finished_stores())
        for req_id in finished_req_ids or ():
            if req_id in self._sending or req_id in self._push_failed or req_id in self._pushed:
                self._finished_pushers.add(req_id)
        sending |= self._poll_sending()
        recving = self._poll_receiving() if self._receiving else set()
        return (sending or None), (recving or None)

    def join_pushes_on_current_stream(self) -> None:
        """Make the current stream wait for every direct push this worker has
        finished enqueuing (for timing a step end to end)."""
        for hs in self._sending.values():
            for h in hs:
                if h._done_event is not None:
                    torch.cuda.current_stream().wait_event(h._done_event)

    def get_block_ids_with_load_errors(self) -> set:
        out, self.load_error_block_ids = self.load_error_block_ids, set()
        return out

    @property
    def lookup_engine(self):
        """What the scheduler's lookups should ask: the engine, or every
        group's engine when the model has several KV cache groups."""
        return _GroupedLookup(self._engines) if len(self._engines) > 1 else self.engine

    def shutdown(self) -> None:
        if self._lookup_server is not None:
            self._lookup_server.close()
        if self._lookup is not None:
            self._lookup.close()
        for e in self._engines[1:]:
            e.close()
        self._engines = self._engines[:1]
