"""Decoder preemption checkpoints: capture at HBM reuse, seal with accepted
tokens, restore as a prefix hit (CPU tier)."""

import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector
from lmcache_ascend_b200.v1.preemption_checkpoint import PreemptionCheckpointer

from .utils import make_separate_kv, random_slots

L, NB, BS, H, D, CS = 2, 64, 16, 2, 32, 64


def _setup():
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=1)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=CS, max_local_cpu_size=0.05,
                                            save_unfull_chunk=False)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    conn = VLLMPagedMemGPUConnector(cfg, kvcaches=kv)
    eng = LMCacheEngine(cfg, md, conn)
    return eng, conn, kv


def _rows(kv, slots):
    return [t.reshape(NB * BS, -1)[slots.long()].clone() for layer in kv for t in layer]


def test_capture_seal_restore_round_trip():
    eng, conn, kv = _setup()
    ck = PreemptionCheckpointer(eng)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 1000, (130,), generator=g)
    generated = torch.randint(0, 1000, (70,), generator=g)
    tokens = torch.cat([prompt, generated])          # 200 tokens decoded so far
    slots = random_slots(200, NB * BS, seed=2)
    eng.store(prompt, slot_mapping=slots[:130])      # prompt chunks stored at prefill
    want = _rows(kv, slots[:192])
    # preemption: capture the generated span, then the blocks are reused
    assert ck.capture("r1", 0, tokens, slots, start=130) == 200 - 128
    for layer in kv:
        for t in layer:
            t.zero_()
    # speculative tail rejected: 195 tokens accepted
    res = ck.seal("r1", 0, tokens[:195].tolist())
    assert res.stored_chunks == 1 and res.published_tokens == 192  # chunk [128, 192)
    assert ck.available(tokens[:195]) == 192 and ck.pending() == 0
    new_slots = random_slots(195, NB * BS, seed=3)
    assert ck.restore(tokens[:195], new_slots) == 192
    for a, b in zip(want, _rows(kv, new_slots[:192])):
        assert torch.equal(a, b)
    eng.close()


def test_rejected_tokens_and_stale_generations():
    eng, conn, kv = _setup()
    ck = PreemptionCheckpointer(eng)
    tokens = torch.arange(256)
    slots = random_slots(256, NB * BS, seed=4)
    ck.capture("r", 1, tokens, slots)
    assert ck.capture("r", 0, tokens, slots) == 0          # older generation ignored
    other = tokens.clone()
    other[100] = 9999                                      # accepted tokens diverge at 100
    res = ck.seal("r", 1, other.tolist())
    assert res.published_tokens == 64 and res.dropped_tokens == 256 - 64
    assert ck.seal("r", 1, tokens.tolist()) is None        # already sealed
    ck.capture("q", 0, tokens, slots)
    ck.cancel("q")
    assert ck.pending() == 0
    cpu = eng.storage_manager.backends["LocalCPUBackend"]
    assert cpu.allocator.num_active == len(cpu.keys())     # cancelled pages returned
    eng.close()
