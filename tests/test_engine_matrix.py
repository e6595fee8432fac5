"""Engine store/retrieve matrix (the upstream cache-engine test grid the
reference re-runs): tier (CPU, local disk, remote) x chunk size (128, 256) x
save_unfull_chunk, for prefix hits, masked offsets, reads through the slower
tier after the CPU tier dropped its copy, and allocator leaks."""

import time

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

from .utils import make_separate_kv, random_slots

L, NB, BS, H, D = 2, 128, 16, 2, 32


def _rows(kv, slots):
    return [t.reshape(NB * BS, -1)[slots.long()].clone() for layer in kv for t in layer]


def _flush(eng):
    for b in eng.storage_manager.backends.values():
        for f in ("wait_for_puts", "wait_for_writes"):
            if hasattr(b, f):
                getattr(b, f)()


@pytest.mark.parametrize("tier", ["cpu", "disk", "remote"])
@pytest.mark.parametrize("chunk", [128, 256])
@pytest.mark.parametrize("unfull", [True, False])
def test_engine_matrix(tier, chunk, unfull, tmp_path):
    extra = {}
    if tier == "disk":
        extra = dict(local_disk=str(tmp_path), max_local_disk_size=0.1)
    elif tier == "remote":
        extra = dict(remote_url=f"mem://matrix-{time.time()}-{chunk}-{unfull}",
                     remote_serde="naive")
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=chunk)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=chunk, max_local_cpu_size=0.05,
                                            save_unfull_chunk=unfull, **extra)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    conn = VLLMPagedMemGPUConnector(cfg, kvcaches=kv)
    eng = LMCacheEngine(cfg, md, conn)
    try:
        g = torch.Generator().manual_seed(chunk + unfull)
        T = 700
        prompt = torch.randint(0, 30000, (T + 100,), generator=g)
        s1 = random_slots(T, NB * BS, seed=1)
        want = _rows(kv, s1)
        eng.store(prompt[:T], slot_mapping=s1)
        _flush(eng)
        full = (T // chunk) * chunk
        stored = T if unfull else full
        cpu = eng.storage_manager.backends["LocalCPUBackend"]
        if tier != "cpu":  # read through the slower tier
            for k in cpu.keys():
                cpu.remove(k)
        # a longer request hits the full chunks (a partial chunk is keyed by its
        # own tokens); the same request hits everything stored
        assert eng.lookup(prompt) == full
        assert eng.lookup(prompt[:T]) == stored
        for layer in kv:
            for t in layer:
                t.zero_()
        s2 = random_slots(T + 100, NB * BS, seed=2)
        ret = eng.retrieve(prompt[:T], slot_mapping=s2[:T])
        assert int(ret.sum()) == stored and bool(ret[:stored].all())
        got = _rows(kv, s2[:stored])
        for a, b in zip(want, got):
            assert torch.equal(a[:stored], b)
        ret = eng.retrieve(prompt, slot_mapping=s2)
        assert int(ret.sum()) == full
        # masked offset: the first chunk is already on the GPU
        mask = torch.ones(T + 100, dtype=torch.bool)
        mask[:chunk] = False
        ret = eng.retrieve(prompt, mask=mask, slot_mapping=s2)
        assert not bool(ret[:chunk].any()) and int(ret.sum()) == full - chunk
        # no leaked CPU pages: every active allocation is a resident chunk
        alloc = cpu.allocator
        assert alloc.num_active == len(cpu.keys()) and alloc.memcheck()
    finally:
        eng.close()
