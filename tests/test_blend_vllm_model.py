"""CacheBlend driven through a serving engine's model (``LMCVLLMModel``).

The served model here is built from vLLM's module conventions (fused
residual RMSNorm, ``qkv_proj`` / ``o_proj`` returning ``(out, bias)``, a
rotary module over flattened rows, optional Qwen3 per-head q/k norms) and
shares its weights with this repo's reference model.  With every token
recomputed, blending a prompt through the wrapper must leave the same KV in
the paged cache as a plain prefill of that prompt.  CPU only.
"""

import pytest
import torch
import torch.nn.functional as F
from torch import nn

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.models.llama import LlamaConfig, LlamaForBlend
from lmcache_ascend_b200.v1.blend.blender import LMCBlender
from lmcache_ascend_b200.v1.blend.vllm_model import (LMCVLLMModel, VLLMModelTracker,
                                                     infer_model_from_vllm)
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMBufferLayerwiseGPUConnector
from lmcache_ascend_b200.v1.token_database import SegmentTokenDatabase

SEP = [999, 998]
NB, BS = 32, 16


class _FusedNorm(nn.Module):
    def __init__(self, norm):
        super().__init__()
        self.norm = norm

    def forward(self, x, residual=None):
        if residual is None:
            return self.norm(x)
        x = x + residual
        return self.norm(x), x


class _QKV(nn.Module):
    def __init__(self, q, k, v):
        super().__init__()
        self.q, self.k, self.v = q, k, v

    def forward(self, h):
        return torch.cat([self.q(h), self.k(h), self.v(h)], dim=-1), None


class _Out(nn.Module):
    def __init__(self, lin):
        super().__init__()
        self.lin = lin

    def forward(self, x):
        return self.lin(x), None


class _Rotary(nn.Module):
    def __init__(self, ref, D):
        super().__init__()
        self.ref, self.D = ref, D

    def forward(self, positions, q, k):
        T = q.shape[0]
        return (self.ref.rope(positions, q.view(T, -1, self.D)).reshape(T, -1),
                self.ref.rope(positions, k.view(T, -1, self.D)).reshape(T, -1))


class _Attn(nn.Module):
    def __init__(self, layer, ref, c):
        super().__init__()
        self.num_heads, self.num_kv_heads, self.head_dim = c.num_heads, c.num_kv_heads, \
            c.head_dim
        self.q_size, self.kv_size = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
        self.qkv_proj = _QKV(layer.q_proj, layer.k_proj, layer.v_proj)
        self.o_proj = _Out(layer.o_proj)
        self.rotary_emb = _Rotary(ref, c.head_dim)
        if layer.q_norm is not None:
            self.q_norm, self.k_norm = layer.q_norm, layer.k_norm


class _MLP(nn.Module):
    def __init__(self, layer):
        super().__init__()
        self.l = layer

    def forward(self, x):
        return self.l.down_proj(F.silu(self.l.gate_proj(x)) * self.l.up_proj(x))


class _Layer(nn.Module):
    def __init__(self, layer, ref, c):
        super().__init__()
        self.input_layernorm = _FusedNorm(layer.input_layernorm)
        self.self_attn = _Attn(layer, ref, c)
        self.post_attention_layernorm = _FusedNorm(layer.post_attention_layernorm)
        self.mlp = _MLP(layer)


class _Inner(nn.Module):
    def __init__(self, ref, c):
        super().__init__()
        self.embed_tokens = ref.embed_tokens
        self.layers = nn.ModuleList([_Layer(l, ref, c) for l in ref.layers])
        self.norm = _FusedNorm(ref.norm)
        self.start_layer, self.end_layer = 0, len(self.layers)


def _served(ref, c, qwen3):
    cls = type("Qwen3ForCausalLM" if qwen3 else "LlamaForCausalLM", (nn.Module,), {})
    m = cls()
    m.model = _Inner(ref, c)
    m.config = type("HF", (), {"max_position_embeddings": c.max_position,
                               "rope_theta": c.rope_theta})()
    return m


def _setup(qwen3):
    cfg = LlamaConfig.tiny(vocab_size=1000, hidden_size=128, num_layers=4, num_heads=4,
                           num_kv_heads=2, head_dim=32, intermediate_size=256,
                           max_position=4096, qk_norm=qwen3)
    ref = LlamaForBlend(cfg, device="cpu")
    served = _served(ref, cfg, qwen3)
    kv = [(torch.zeros(NB, BS, 2, 32), torch.zeros(NB, BS, 2, 32)) for _ in range(4)]
    ec = LMCacheEngineConfig.from_defaults(chunk_size=256, enable_blending=True,
                                           use_layerwise=True, max_local_cpu_size=0.05,
                                           blend_recompute_ratios=[1.0],
                                           blend_check_layers=[0])
    md = LMCacheEngineMetadata("tiny", 1, 0, "vllm", torch.float32)
    conn = VLLMBufferLayerwiseGPUConnector(ec, kvcaches=kv)
    eng = LMCacheEngine(ec, md, conn, token_database=SegmentTokenDatabase(ec, md, SEP))
    VLLMModelTracker.unregister("blend-test")
    VLLMModelTracker.register_model("blend-test", served)
    wrapped = infer_model_from_vllm(VLLMModelTracker.get_model("blend-test"))
    assert isinstance(wrapped, LMCVLLMModel) and wrapped.qk_norm == qwen3
    blender = LMCBlender(eng, conn, wrapped, ec, kv_caches=kv)
    return ref, eng, blender, kv


@pytest.mark.parametrize("qwen3", [False, True])
def test_blend_through_served_model_equals_prefill(qwen3):
    ref, eng, blender, kv = _setup(qwen3)
    g = torch.Generator().manual_seed(0)
    d1 = torch.randint(0, 900, (40,), generator=g)
    d2 = torch.randint(0, 900, (50,), generator=g)
    for doc, seed in ((d1, 1), (d2, 2)):
        slots = torch.randperm(NB * BS, generator=torch.Generator().manual_seed(seed))[:len(doc)]
        ref.prefill(doc, kv, slots)
        for _ in eng.store_layer(doc, slot_mapping=slots):
            pass
    prompt = torch.cat([d1, torch.tensor(SEP), d2])
    slots = torch.randperm(NB * BS, generator=torch.Generator().manual_seed(7))[:len(prompt)]
    got = blender.blend(prompt, slot_mapping=slots)
    assert int(got.sum()) == len(d1) + len(d2)
    blended = [(kv[l][0].view(NB * BS, -1)[slots].clone(), kv[l][1].view(NB * BS, -1)[slots]
                .clone()) for l in range(4)]
    ref.prefill(prompt, kv, slots)
    for l in range(4):
        for which in range(2):
            want = kv[l][which].view(NB * BS, -1)[slots]
            assert torch.allclose(blended[l][which], want, atol=1e-4, rtol=1e-4), (l, which)


def test_unsupported_model_type_is_refused():
    with pytest.raises(NotImplementedError):
        infer_model_from_vllm(nn.Linear(2, 2))
