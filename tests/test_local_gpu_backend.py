"""HBM tier: stores land in device pages, hits are device-to-device, and an
evicted chunk is written back to the CPU tier and still hits from there."""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import (VLLMPagedMemGPUConnector,
                                                  VLLMPagedMemLayerwiseGPUConnector)

from .utils import make_separate_kv, random_slots

pytestmark = pytest.mark.gpu
L, NB, BS, H, D = 4, 64, 16, 2, 64


def _rows(kv, slots):
    return [t.view(NB * BS, -1)[slots.long()] for layer in kv for t in layer]


@pytest.mark.parametrize("layerwise", [False, True])
def test_hbm_tier_hits_and_writes_back(layerwise):
    chunk_bytes = 2 * L * 64 * H * D * 2
    cfg = LMCacheEngineConfig.from_defaults(
        chunk_size=64, local_gpu=True, max_local_gpu_size=(6.5 * chunk_bytes) / (1 << 30),
        max_local_cpu_size=0.05, use_layerwise=layerwise)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.bfloat16)
    kv = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=1)
    conn = (VLLMPagedMemLayerwiseGPUConnector if layerwise else VLLMPagedMemGPUConnector)(
        cfg, kvcaches=kv)
    eng = LMCacheEngine(cfg, md, conn)
    sm = eng.storage_manager
    gpu = sm.backends["LocalGPUBackend"]
    cpu = sm.backends["LocalCPUBackend"]

    def store(tokens, slots):
        if layerwise:
            for _ in eng.store_layer(tokens, slot_mapping=slots):
                pass
        else:
            eng.store(tokens, slot_mapping=slots)

    def load(tokens, slots):
        if layerwise:
            g = eng.retrieve_layer(tokens, slot_mapping=slots)
            out = None
            for out in g:
                pass
            return out
        return eng.retrieve(tokens, slot_mapping=slots)

    a_tok = torch.arange(256)
    a_slots = random_slots(256, NB * BS, seed=2, device="cuda")
    want = _rows(kv, a_slots)
    store(a_tok, a_slots)
    assert len(gpu) > 0 and all(o.raw_data.is_cuda for o in gpu.hot_cache.values())
    assert len(cpu) == 0  # the CPU tier holds nothing until a write-back
    b_slots = random_slots(256, NB * BS, seed=3, device="cuda")
    ret = load(a_tok, b_slots)
    torch.cuda.synchronize()
    assert bool(ret.all())
    for x, y in zip(want, _rows(kv, b_slots)):
        assert torch.equal(x, y)
    # more stores than the HBM tier holds: the oldest chunks move to the CPU tier
    for i in range(1, 4):
        store(torch.arange(256) + 1000 * i, random_slots(256, NB * BS, seed=10 + i,
                                                         device="cuda"))
    assert gpu.writebacks > 0 and len(cpu) > 0
    c_slots = random_slots(256, NB * BS, seed=20, device="cuda")
    ret = load(a_tok, c_slots)
    torch.cuda.synchronize()
    assert bool(ret.all())
    for x, y in zip(want, _rows(kv, c_slots)):
        assert torch.equal(x, y)
    eng.close()
