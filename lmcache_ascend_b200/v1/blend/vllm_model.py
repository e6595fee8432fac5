"""CacheBlend over a serving engine's own model.

The blender drives a model layer by layer: fresh Q/K/V of the request,
the top-k deviation check against the retrieved KV on the check layers,
attention of the recomputed tokens over the merged KV, and the merged KV
written back into the paged cache.  ``LMCVLLMModel`` runs that loop on the
modules of a vLLM decoder model (``LlamaForCausalLM``, ``Qwen3ForCausalLM``
and subclasses): its embeddings, fused RMSNorms, ``qkv_proj``, the
attention's ``rotary_emb``, Qwen3's per-head ``q_norm`` / ``k_norm``,
``o_proj`` and MLP, so the blended prefill uses the served weights
(reference lmcache_ascend/v1/blend/models/llama.py:13-98, qwen3.py,
models/utils.py:15-64 ``infer_model_from_vllm`` / ``VLLMModelTracker``).

Attention of the recomputed query rows over all key rows is causal by
position (a query at position p sees keys at positions <= p), computed with
``scaled_dot_product_attention`` and grouped-query heads (reference
blend/attention/attention.py:30-70, 150-190).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F
from torch import nn

from ...utils.logging import init_logger

logger = init_logger(__name__)


class VLLMModelTracker:
    """Serving-engine models by instance id, registered by the code that
    loads the model and looked up by the blender of that instance."""

    _models: Dict[str, nn.Module] = {}

    @classmethod
    def register_model(cls, instance_id: str, vllm_model: nn.Module) -> None:
        if instance_id in cls._models:
            logger.warning("a model is already registered for %s; keeping it", instance_id)
            return
        cls._models[instance_id] = vllm_model

    @classmethod
    def get_model(cls, instance_id: str) -> nn.Module:
        if instance_id not in cls._models:
            raise ValueError(f"no model registered for instance {instance_id!r}")
        return cls._models[instance_id]

    @classmethod
    def unregister(cls, instance_id: str) -> None:
        cls._models.pop(instance_id, None)


@dataclass
class _BlendModelConfig:
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    max_position: int
    rope_theta: float


def _first(x):
    return x[0] if isinstance(x, tuple) else x


class LMCVLLMModel:
    """Layerwise blending forward over a vLLM decoder model's modules."""

    def __init__(self, vllm_model: nn.Module, qk_norm: bool = False):
        self.vllm_model = vllm_model
        inner = vllm_model.model
        start = getattr(inner, "start_layer", 0)
        end = getattr(inner, "end_layer", len(inner.layers))
        self.layers = list(inner.layers[start:end])
        attn = self.layers[0].self_attn
        hf = getattr(vllm_model, "config", None)
        self.config = _BlendModelConfig(
            num_layers=len(self.layers), num_heads=attn.num_heads,
            num_kv_heads=attn.num_kv_heads, head_dim=attn.head_dim,
            max_position=int(getattr(hf, "max_position_embeddings", 8192)),
            rope_theta=float(getattr(hf, "rope_theta", 10000.0)))
        self.qk_norm = qk_norm
        p = next(vllm_model.parameters())
        self.device, self.dtype = p.device, p.dtype

    # ------------------------------------------------------------ helpers
    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        m = self.vllm_model
        if hasattr(m, "get_input_embeddings"):
            return m.get_input_embeddings(tokens)
        return m.model.embed_tokens(tokens)

    def rotary_emb(self, positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor):
        """RoPE of q [T, H, D] and k [T, KH, D] by the model's own rotary
        module (it takes and returns flattened rows)."""
        T = q.shape[0]
        rq, rk = self.layers[0].self_attn.rotary_emb(positions, q.reshape(T, -1),
                                                      k.reshape(T, -1))
        return rq.view(q.shape), rk.view(k.shape)

    def _split_qkv(self, layer, h: torch.Tensor):
        a = layer.self_attn
        qkv = _first(a.qkv_proj(h))
        q, k, v = qkv.split([a.q_size, a.kv_size, a.kv_size], dim=-1)
        c = self.config
        q = q.reshape(-1, c.num_heads, c.head_dim)
        k = k.reshape(-1, c.num_kv_heads, c.head_dim)
        v = v.reshape(-1, c.num_kv_heads, c.head_dim)
        if self.qk_norm:
            q = a.q_norm(q.contiguous())
            k = a.k_norm(k.contiguous())
        return q, k, v

    def attend(self, q, k, v, q_pos, k_pos) -> torch.Tensor:
        """q [Tq, H, D] at q_pos over k, v [Tk, KH, D] at k_pos, causal by
        position; returns [Tq, H * D]."""
        c = self.config
        rep = c.num_heads // c.num_kv_heads
        mask = q_pos[:, None] >= k_pos[None, :]
        o = F.scaled_dot_product_attention(
            q.transpose(0, 1), k.repeat_interleave(rep, 1).transpose(0, 1),
            v.repeat_interleave(rep, 1).transpose(0, 1), attn_mask=mask[None],
            scale=getattr(self.layers[0].self_attn, "scaling", None))
        return o.transpose(0, 1).reshape(q.shape[0], -1)

    @staticmethod
    def write_kv(kv_layer, slot_mapping, k, v) -> None:
        kc, vc = kv_layer
        kc.view(-1, kc.shape[-2] * kc.shape[-1])[slot_mapping.long()] = \
            k.reshape(k.shape[0], -1).to(kc.dtype)
        vc.view(-1, vc.shape[-2] * vc.shape[-1])[slot_mapping.long()] = \
            v.reshape(v.shape[0], -1).to(vc.dtype)

    # ----------------------------------------------------------- forward
    @torch.no_grad()
    def compute_layer(self, tokens: torch.Tensor, blender, kv_caches: Optional[List],
                      slot_mapping: Optional[torch.Tensor]):
        """Generator over the layers (one yield per layer); returns the final
        normed hidden states of the rows still computed."""
        tokens = tokens.to(self.device)
        n = tokens.numel()
        all_pos = torch.arange(n, device=self.device)
        h = self.embed(tokens)
        residual = None
        for idx, layer in enumerate(self.layers):
            if residual is None:
                residual = h
                h = layer.input_layernorm(h)
            else:
                h, residual = layer.input_layernorm(h, residual)
            q, k, v = self._split_qkv(layer, h)
            q, k, v, residual, _ = blender.process_qkv(q, k, v, residual, idx, self)
            if kv_caches is not None and slot_mapping is not None:
                self.write_kv(kv_caches[idx], slot_mapping.to(self.device), k, v)
            o = self.attend(q, k, v, blender.metadata.positions, all_pos)
            h = _first(layer.self_attn.o_proj(o))
            h, residual = layer.post_attention_layernorm(h, residual)
            h = layer.mlp(h)
            yield
        norm = self.vllm_model.model.norm
        out = norm(h, residual)
        return _first(out)


def infer_model_from_vllm(vllm_model: nn.Module) -> LMCVLLMModel:
    """The blending wrapper for a served vLLM model, chosen by class name."""
    name = type(vllm_model).__name__
    if name == "LlamaForCausalLM":
        return LMCVLLMModel(vllm_model, qk_norm=False)
    if "Qwen3ForCausalLM" in name:
        return LMCVLLMModel(vllm_model, qk_norm=True)
    raise NotImplementedError(f"CacheBlend does not support model type {name}")


_blenders: Dict[str, object] = {}


def _kv_pairs(kv_caches):
    """Per layer (K, V) paged views of vLLM's caches ([2, NB, BS, KH, D]
    tensors, or (K, V) pairs already)."""
    out = []
    for t in kv_caches:
        if isinstance(t, torch.Tensor):
            out.append((t[0], t[1]) if t.shape[0] == 2 else (t[:, 0], t[:, 1]))
        else:
            out.append((t[0], t[1]))
    return out


def get_or_create_blender(instance_id: str, cache_engine, gpu_connector, config, kv_caches):
    """The blender of a serving instance over its registered model
    (reference lmcache_ascend/v1/blend/utils.py:21-45)."""
    b = _blenders.get(instance_id)
    if b is None:
        from .blender import LMCBlender

        model = infer_model_from_vllm(VLLMModelTracker.get_model(instance_id))
        b = _blenders[instance_id] = LMCBlender(cache_engine, gpu_connector, model, config,
                                                kv_caches=_kv_pairs(kv_caches))
    return b


def drop_blender(instance_id: str) -> None:
    _blenders.pop(instance_id, None)
