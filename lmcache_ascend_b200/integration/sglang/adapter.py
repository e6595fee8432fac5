"""SGLang integration: the LMCache connector SGLang's scheduler calls.

Behaviour of the reference's SGLang patches
(lmcache_ascend/integration/sglang/sglang_adapter.py:16-137):
* the connector is built from SGLang's per-layer K and V token pools
  (``k_pool[layer]``: [pool_size, heads, head_dim], page size 1, or paged
  [num_pages, page_size, heads, head_dim]);
* ``start_load_kv`` looks up the request's tokens, agrees on the minimum hit
  across TP ranks (``global_min_tokens``: every rank must load the same
  prefix), skips what SGLang's radix cache already holds (``offset``) and
  loads the rest, whole or layer by layer; it returns the number of newly
  loaded tokens;
* ``store_kv`` saves the tokens after ``offset``.
"""

from __future__ import annotations

import uuid
from dataclasses import dataclass
from typing import List, Optional

import torch

from ...config import LMCacheEngineConfig, LMCacheEngineMetadata
from ...utils.logging import init_logger
from ...v1.cache_engine import LMCacheEngine
from ...v1.gpu_connector import SGLangGPUConnector, SGLangLayerwiseGPUConnector

logger = init_logger(__name__)


@dataclass
class LoadMetadata:
    token_ids: List[int]
    slot_mapping: torch.Tensor
    offset: int = 0


@dataclass
class StoreMetadata:
    token_ids: List[int]
    slot_mapping: torch.Tensor
    offset: int = 0


class LMCacheSGLangConnector:
    def __init__(self, model_name: str, tp_size: int, rank: int, k_pool: List[torch.Tensor],
                 v_pool: List[torch.Tensor], config: Optional[LMCacheEngineConfig] = None,
                 tp_group=None, layerwise: bool = False):
        if k_pool is None or len(k_pool) == 0:
            raise ValueError("k_pool cannot be empty during initialization")
        self.config = config or LMCacheEngineConfig.from_env()
        self.tp_size, self.rank, self.tp_group = tp_size, rank, tp_group
        self.layerwise = layerwise
        self.num_layers = len(k_pool)
        kv_dtype = k_pool[0].dtype
        md = LMCacheEngineMetadata(model_name, tp_size, rank, "sglang", kv_dtype)
        self.kvcaches = [(self._paged(k), self._paged(v)) for k, v in zip(k_pool, v_pool)]
        if layerwise and not self.config.use_layerwise:
            self.config.use_layerwise = True
        conn = (SGLangLayerwiseGPUConnector(self.config) if layerwise
                else SGLangGPUConnector(self.config))
        conn.register_kv_caches(self.kvcaches)
        self.engine = LMCacheEngine(self.config, md, conn)
        self.engine.post_init()
        self._retrievers = []
        self._lookup_ids: List[str] = []

    @staticmethod
    def _paged(t: torch.Tensor) -> torch.Tensor:
        """Token pool [size, H, D] -> [size, 1, H, D] (page size 1)."""
        return t.unsqueeze(1) if t.dim() == 3 else t

    # ----------------------------------------------------------------- TP
    @torch.no_grad()
    def global_min_tokens(self, local_tokens: int) -> int:
        if self.tp_size == 1 or self.tp_group is None:
            return local_tokens
        import torch.distributed as dist

        t = torch.tensor([local_tokens], dtype=torch.int64)
        backend = dist.get_backend(self.tp_group)
        if backend == "nccl":
            t = t.cuda()
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.tp_group)
        return int(t.item())

    # --------------------------------------------------------------- load
    def start_load_kv(self, meta: LoadMetadata) -> int:
        tokens = torch.tensor(meta.token_ids, dtype=torch.long)
        slots = meta.slot_mapping
        lookup_id = str(uuid.uuid4())
        hit = self.engine.lookup(tokens, lookup_id=lookup_id, pin=True)
        hit = self.global_min_tokens(hit)
        if hit <= meta.offset:
            self.engine.lookup_unpin(lookup_id)
            return 0
        mask = torch.ones(hit, dtype=torch.bool)
        cs = self.config.chunk_size
        mask[:(meta.offset // cs) * cs] = False
        if self.layerwise:
            g = self.engine.retrieve_layer(tokens[:hit], mask, slot_mapping=slots[:hit])
            next(g)
            next(g)  # first layer
            self._retrievers.append(g)
            self._lookup_ids.append(lookup_id)
        else:
            self.engine.retrieve(tokens[:hit], mask, slot_mapping=slots[:hit])
            self.engine.lookup_unpin(lookup_id)
        return hit - meta.offset

    def load_kv_layerwise(self, layer_id: int) -> None:
        """Called before layer ``layer_id + 1`` runs: load the next layer."""
        if layer_id >= self.num_layers - 1:
            for g in self._retrievers:
                for _ in g:
                    pass
            self._retrievers = []
            for lid in self._lookup_ids:
                self.engine.lookup_unpin(lid)
            self._lookup_ids = []
            return
        for g in self._retrievers:
            next(g, None)

    # -------------------------------------------------------------- store
    def store_kv(self, meta: StoreMetadata) -> None:
        tokens = torch.tensor(meta.token_ids, dtype=torch.long)
        cs = self.config.chunk_size
        mask = None
        skip = (meta.offset // cs) * cs
        if skip:
            mask = torch.ones(len(tokens), dtype=torch.bool)
            mask[:skip] = False
        if self.layerwise:
            for _ in self.engine.store_layer(tokens, mask, slot_mapping=meta.slot_mapping):
                pass
        else:
            self.engine.store(tokens, mask, slot_mapping=meta.slot_mapping)

    def close(self) -> None:
        self.engine.close()
