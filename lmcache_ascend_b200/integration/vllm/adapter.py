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

This module only uses attribute access on vLLM's objects, so the logic can be
exercised with light stand-ins in tests; ``connector.py`` binds it to
``KVConnectorBase_V1``.
"""

from __future__ import annotations

import os
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

    def update(self, new_token_ids: Sequence[int], new_block_ids: Optional[Sequence[int]]):
        self.token_ids.extend(new_token_ids)
        if new_block_ids:
            self.allocated_block_ids.extend(new_block_ids)


@dataclass
class ReqMeta:
    req_id: str
    token_ids: torch.Tensor
    slot_mapping: torch.Tensor
    save_spec: Optional[SaveSpec] = None
    load_spec: Optional[LoadSpec] = None
    is_last_prefill: bool = False
    disagg_spec: Optional[dict] = None

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
        return ReqMeta(tracker.req_id, torch.tensor(tracker.token_ids[:ntoks], dtype=torch.long),
                       slot, save, load_spec if loading else None, is_last_prefill,
                       tracker.disagg_spec)


@dataclass
class LMCacheConnectorMetadata:
    requests: List[ReqMeta] = field(default_factory=list)

    def add_request(self, r: ReqMeta) -> None:
        self.requests.append(r)


def config_from_extra(extra: Optional[Dict[str, Any]]) -> LMCacheEngineConfig:
    """Engine config from LMCACHE_CONFIG_FILE / LMCACHE_* env, overridden by
    ``kv_connector_extra_config`` keys prefixed with ``lmcache.``
    (reference lmcache_ascend_connector_v1.py:46-49)."""
    cfg = LMCacheEngineConfig.from_env()
    over = {k: v for k, v in (extra or {}).items() if str(k).startswith("lmcache.")}
    if over:
        cfg.update(over)
    return cfg


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

    # ============================================================ scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> Tuple[int, bool]:
        tokens = list(request.prompt_token_ids or [])
        if not tokens:
            return 0, False
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
        spec = self._load_specs.get(request.request_id)
        if spec is None:
            return
        if num_external_tokens == 0:
            spec.can_load = False
            return
        spec.can_load = True

    def build_connector_meta(self, scheduler_output) -> LMCacheConnectorMetadata:
        meta = LMCacheConnectorMetadata()
        for req_id in getattr(scheduler_output, "finished_req_ids", ()) or ():
            self._trackers.pop(req_id, None)
            self._load_specs.pop(req_id, None)
        for new in scheduler_output.scheduled_new_reqs:
            tokens = list(new.prompt_token_ids or [])
            blocks = list(new.block_ids[0]) if new.block_ids else []
            tr = RequestTracker(new.req_id, len(tokens), tokens, blocks)
            self._trackers[new.req_id] = tr
            spec = self._load_specs.pop(new.req_id, None)
            done = new.num_computed_tokens + scheduler_output.num_scheduled_tokens[new.req_id]
            if spec is not None and spec.can_load:
                tr.num_saved_tokens = (spec.lmcache_cached_tokens // self.chunk_size) * \
                    self.chunk_size  # already cached: do not store again
            r = ReqMeta.build(tr, self.block_size, self.chunk_size, spec, done,
                              self.config.save_unfull_chunk, skip_save=False)
            if r is not None:
                meta.add_request(r)
        cached = scheduler_output.scheduled_cached_reqs
        for i, req_id in enumerate(getattr(cached, "req_ids", []) or []):
            tr = self._trackers.get(req_id)
            if tr is None:
                continue
            new_blocks = cached.new_block_ids[i]
            tr.update(cached.new_token_ids[i] if cached.new_token_ids else [],
                      list(new_blocks[0]) if new_blocks else None)
            done = cached.num_computed_tokens[i] + scheduler_output.num_scheduled_tokens[req_id]
            if tr.num_saved_tokens >= tr.prompt_len:
                continue  # decode phase: nothing to store
            r = ReqMeta.build(tr, self.block_size, self.chunk_size, None, done,
                              self.config.save_unfull_chunk, skip_save=False)
            if r is not None:
                meta.add_request(r)
        return meta

    def request_finished(self, request, block_ids) -> Tuple[bool, Optional[dict]]:
        self._trackers.pop(request.request_id, None)
        if self._lookup is not None:
            self._lookup.unpin(request.request_id)
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
        caches = [kv_caches[n] for n in self._layer_names]
        from ...v1.kv_layer_groups import KVLayerGroupsManager

        self.layer_groups = KVLayerGroupsManager()
        self.layer_groups.build_kv_layer_groups({n: kv_caches[n] for n in self._layer_names})
        if self.layer_groups.num_groups > 1:
            raise ValueError("layers with different KV cache shapes/dtypes "
                             f"({self.layer_groups.num_groups} groups) need one engine per group")
        eng = self._ensure_engine()
        first = caches[0]
        if self.metadata.kv_dtype is None:
            self.metadata.kv_dtype = first.dtype
        eng.post_init(kvcaches=caches)
        if self.rank == 0 and self._lookup_server is None:
            self._lookup_server = LookupServer(eng, self.lookup_url)

    def bind_connector_metadata(self, meta: LMCacheConnectorMetadata) -> None:
        self._meta = meta

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
            spec = r.load_spec
            if spec is None or not spec.can_load:
                continue
            n = spec.lmcache_cached_tokens
            skip = (spec.vllm_cached_tokens // self.chunk_size) * self.chunk_size
            toks, slots = r.token_ids[:n], r.slot_mapping[:n]
            mask = self._mask(n, skip)
            if self.config.use_layerwise:
                g = eng.retrieve_layer(toks, mask, slot_mapping=slots)
                next(g)
                self._layer_load_gens.append(g)
            else:
                ret = eng.retrieve(toks, mask, slot_mapping=slots)
                got = int(ret.sum())
                if got < n - skip:
                    logger.warning("req %s: loaded %d of %d expected tokens", r.req_id, got,
                                   n - skip)

    def wait_for_layer_load(self, layer_name: str) -> None:
        for g in self._layer_load_gens:
            next(g, None)

    def save_kv_layer(self, layer_name: str, kv_layer=None, attn_metadata=None, **kw) -> None:
        if self._meta is None or not self.config.use_layerwise or self.kv_role == "kv_consumer":
            return
        eng = self._ensure_engine()
        if layer_name == self._layer_names[0]:
            self._layer_store_gens = []
            for r in self._meta.requests:
                if r.save_spec is None:
                    continue
                n = r.token_ids.numel()
                g = eng.store_layer(r.token_ids, self._mask(n, r.save_spec.skip_leading_tokens),
                                    slot_mapping=r.slot_mapping)
                next(g)  # before the first layer
                self._layer_store_gens.append(g)
        for g in self._layer_store_gens:
            next(g, None)

    def wait_for_save(self) -> None:
        if self._meta is None or self.kv_role == "kv_consumer":
            return
        eng = self._ensure_engine()
        if self.config.use_layerwise:
            for g in self._layer_store_gens:
                for _ in g:
                    pass
            self._layer_store_gens = []
            return
        for r in self._meta.requests:
            if r.save_spec is None or not r.save_spec.can_save:
                continue
            n = r.token_ids.numel()
            eng.store(r.token_ids, self._mask(n, r.save_spec.skip_leading_tokens),
                      slot_mapping=r.slot_mapping, req_id=r.req_id)

    def get_finished(self, finished_req_ids) -> Tuple[Optional[set], Optional[set]]:
        if self.engine is not None and self.config.store_async:
            done = set(self.engine.get_finished_stores())
            return (done or None), None
        return None, None

    def shutdown(self) -> None:
        if self._lookup_server is not None:
            self._lookup_server.close()
        if self._lookup is not None:
            self._lookup.close()
