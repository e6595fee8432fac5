"""CacheBlend: reuse the KV of independently cached document segments and
recompute only the tokens whose keys deviate most.

Semantics of the reference's ``LMCBlender`` (lmcache_ascend/v1/blend/
blender.py:17-183): layers are computed layer by layer while the retriever
loads the cached KV of the same layer; on ``blend_check_layers`` the fresh
keys are compared with the cached (re-positioned) keys and the
``blend_recompute_ratios`` fraction with the largest squared difference is
kept as the query set for the remaining layers; their fresh K/V are merged
into the cached K/V, which the other tokens keep.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Union

import torch

from ...config import LMCacheEngineConfig
from ...utils.logging import init_logger

logger = init_logger(__name__)


@dataclass
class LMCBlendCommonMetadata:
    check_layers: List[int]
    recomp_ratios: List[float]
    thresholds: Optional[List[float]] = None


@dataclass
class LMCBlendMetadata:
    imp_indices: Optional[torch.Tensor] = None
    attn_mask: Optional[torch.Tensor] = None
    positions: Optional[torch.Tensor] = None

    def clean(self) -> None:
        self.imp_indices = None
        self.attn_mask = None
        self.positions = None


class LMCBlender:
    def __init__(self, cache_engine, gpu_connector, model, config: LMCacheEngineConfig,
                 kv_caches=None):
        self.cache_engine = cache_engine
        self.gpu_connector = gpu_connector
        self.layerwise_model = model
        self.num_layers = model.config.num_layers
        self.kv_caches = kv_caches
        self.common_metadata = LMCBlendCommonMetadata(
            check_layers=list(config.blend_check_layers),
            recomp_ratios=list(config.blend_recompute_ratios),
            thresholds=config.extra_config.get("blend_thresholds"))
        self.metadata = LMCBlendMetadata()
        if getattr(gpu_connector, "fused_rope", "absent") is None:
            from .positional_encoding import get_fused_rope

            c = model.config
            gpu_connector.fused_rope = get_fused_rope(
                c.head_dim, c.head_dim, c.max_position, c.rope_theta, True,
                device=str(model.device))

    def process_qkv(self, q, k, v, residual, layer_id: int, model,
                    mask: Optional[torch.Tensor] = None, **kwargs):
        """q [T', H, D], k/v [T', KH, D] fresh (pre-RoPE) for the current
        query set.  Returns (q, k_all, v_all, residual, attn_output)."""
        old_k, old_v = self.gpu_connector.get_kv(layer_id)
        kh, d = k.shape[1], k.shape[2]
        old_k = old_k.view(-1, kh, d)
        old_v = old_v.view(-1, kh, d)
        num_falses = 0 if mask is None else int(mask.numel() - mask.long().sum().item())
        if self.metadata.positions is None:
            self.metadata.positions = torch.arange(q.shape[0], device=q.device,
                                                   dtype=torch.int64)
        q, k = model.rotary_emb(self.metadata.positions, q, k)
        ratios = self.common_metadata.recomp_ratios
        if layer_id in self.common_metadata.check_layers and ratios and ratios[0] > 0:
            if k[num_falses:].shape[0] != old_k.shape[0]:
                raise ValueError("token count of fresh K (after the masked prefix) and cached K "
                                 "differ")
            diff = torch.sum((k[num_falses:].float() - old_k.float()) ** 2, dim=[1, 2])
            total = diff.shape[0]
            topk = max(1, int(total * ratios[0]))
            top = torch.sort(torch.topk(diff, k=topk).indices).values
            q, k, v, residual = q[top], k[top], v[top], residual[top]
            self.metadata.imp_indices = top
            self.metadata.positions = self.metadata.positions[top]
            logger.debug("blend layer %d: recomputing %d of %d tokens", layer_id, topk, total)
        if self.metadata.imp_indices is not None:
            old_k = old_k.clone()
            old_v = old_v.clone()
            old_k[self.metadata.imp_indices] = k.to(old_k.dtype)
            old_v[self.metadata.imp_indices] = v.to(old_v.dtype)
            return q, old_k, old_v, residual, None
        return q, k, v, residual, None

    def blend_layer(self, tokens: torch.Tensor, mask: Optional[torch.Tensor] = None,
                    slot_mapping: Optional[torch.Tensor] = None, **kwargs):
        """Layerwise retrieve + blend; yields num_layers + 2 times."""
        executor = self.layerwise_model.compute_layer(tokens, self, self.kv_caches,
                                                      slot_mapping)
        retriever = self.cache_engine.retrieve_layer(tokens, mask, slot_mapping=slot_mapping,
                                                     **kwargs)
        next(retriever)
        yield
        for _ in range(self.num_layers):
            next(retriever)
            next(executor)
            yield
        self.retrieved = next(retriever)
        self.metadata.clean()
        yield

    def blend(self, tokens: Union[torch.Tensor, List[int]], mask: Optional[torch.Tensor] = None,
              **kwargs):
        if isinstance(tokens, list):
            tokens = torch.tensor(tokens)
        gen = self.blend_layer(tokens, mask, **kwargs)
        for _ in range(self.num_layers + 2):
            next(gen)
        return self.retrieved
