"""CacheBlend on the CPU tier: documents cached standalone, reused inside a
new prompt at new positions (fused RoPE re-rotation), top-k recompute."""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.models.llama import LlamaConfig, LlamaForBlend
from lmcache_ascend_b200.v1.blend.blender import LMCBlender
from lmcache_ascend_b200.v1.blend.positional_encoding import get_fused_rope
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMBufferLayerwiseGPUConnector
from lmcache_ascend_b200.v1.token_database import SegmentTokenDatabase

SEP = [999, 998]
NB, BS = 32, 16


def _setup(ratio, check_layers, dev="cpu"):
    cfg = LlamaConfig.tiny(vocab_size=1000, hidden_size=128, num_layers=4, num_heads=4,
                           num_kv_heads=2, head_dim=32, intermediate_size=256,
                           max_position=4096)
    model = LlamaForBlend(cfg, device=dev)
    kv = [(torch.zeros(NB, BS, 2, 32, device=dev), torch.zeros(NB, BS, 2, 32, device=dev))
          for _ in range(cfg.num_layers)]
    ec = LMCacheEngineConfig.from_defaults(chunk_size=256, enable_blending=True,
                                           use_layerwise=True, max_local_cpu_size=0.05,
                                           blend_recompute_ratios=[ratio],
                                           blend_check_layers=check_layers)
    md = LMCacheEngineMetadata("tiny", 1, 0, "vllm", torch.float32)
    conn = VLLMBufferLayerwiseGPUConnector(ec, kvcaches=kv)
    eng = LMCacheEngine(ec, md, conn, token_database=SegmentTokenDatabase(ec, md, SEP))
    blender = LMCBlender(eng, conn, model, ec, kv_caches=kv)
    return model, eng, conn, blender, kv


def _precompute(model, eng, kv, doc, seed):
    g = torch.Generator().manual_seed(seed)
    slots = torch.randperm(NB * BS, generator=g)[:len(doc)]
    model.prefill(doc, kv, slots)
    for _ in eng.store_layer(doc, slot_mapping=slots):
        pass


def _rows(kv, slots, layer, which):
    return kv[layer][which].view(NB * BS, -1)[slots.long()]


def test_fused_rope_self_check():
    assert get_fused_rope(32, 32, 4096, 10000.0, True, device="cpu") is not None
    assert get_fused_rope(32, 16, 4096, 10000.0, True, device="cpu") is None


@pytest.mark.parametrize("ratio,check", [(1.0, [0])])
def test_blend_full_recompute_equals_prefill(ratio, check):
    model, eng, conn, blender, kv = _setup(ratio, check)
    g = torch.Generator().manual_seed(0)
    d1 = torch.randint(0, 900, (40,), generator=g)
    d2 = torch.randint(0, 900, (50,), generator=g)
    _precompute(model, eng, kv, d1, 1)
    _precompute(model, eng, kv, d2, 2)
    prompt = torch.cat([d1, torch.tensor(SEP), d2])
    T = prompt.numel()
    slots = torch.randperm(NB * BS, generator=g)[:T]
    ret = blender.blend(prompt, slot_mapping=slots)
    assert bool(ret[:40].all()) and bool(ret[42:].all()) and not bool(ret[40:42].any())
    # re-positioned cached K of d2 (layer 0) == K computed at its new positions
    ref_kv = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in kv]
    ref_slots = torch.arange(T)
    model.prefill(prompt, ref_kv, ref_slots)
    k0 = conn.get_kv(0)[0]
    assert torch.allclose(k0[42:], ref_kv[0][0].view(NB * BS, -1)[42:T], atol=1e-4)
    # full recompute from layer 0 reproduces the plain prefill for all layers
    for layer in range(model.config.num_layers):
        for which in (0, 1):
            got = _rows(kv, slots, layer, which)
            want = ref_kv[layer][which].view(NB * BS, -1)[:T]
            assert torch.allclose(got, want, atol=1e-4), (layer, which)
    eng.close()


def test_blend_partial_recompute_selects_topk():
    model, eng, conn, blender, kv = _setup(0.25, [1])
    g = torch.Generator().manual_seed(5)
    d1 = torch.randint(0, 900, (60,), generator=g)
    d2 = torch.randint(0, 900, (60,), generator=g)
    _precompute(model, eng, kv, d1, 3)
    _precompute(model, eng, kv, d2, 4)
    prompt = torch.cat([d1, torch.tensor(SEP), d2])
    T = prompt.numel()
    slots = torch.randperm(NB * BS, generator=g)[:T]
    picked = []
    orig = blender.process_qkv

    def spy(*a, **kw):
        out = orig(*a, **kw)
        picked.append(out[0].shape[0])
        return out

    blender.process_qkv = spy
    blender.blend(prompt, slot_mapping=slots)
    # layers 0-1 before selection see all tokens; after the check layer 25 % remain
    assert picked[0] == T and picked[1] == int(T * 0.25) and picked[-1] == int(T * 0.25)
    eng.close()
