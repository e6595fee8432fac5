"""Sparse (top-k) layerwise retrieve through the engine.

A long context is stored in the CPU tier; decode steps then load only
selected tokens per layer into given paged slots.  Checks: rows land exactly
(PyTorch oracle), the warm state is reused without touching the tiers, a
longer context extends it, a failed extension rolls it back, and a failed
copy quarantines the source chunks and marks the engine unhealthy.  CPU
tier + host caches here; the GPU variant uses the kernel on pinned chunks.
"""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import (LMCacheEngine, SparseLayerRequest,
                                                 SparseRetrieveState)
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

from .utils import make_separate_kv, random_slots, zeros_like_kv

L, NB, BS, H, D = 3, 96, 16, 2, 32


def _engine(dev="cpu"):
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=128, max_local_cpu_size=0.05)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, dev, seed=3)
    eng = LMCacheEngine(cfg, md, VLLMPagedMemGPUConnector(cfg, kvcaches=kv))
    return eng, kv


def _rows(kv, layer, slots):
    return [t.view(NB * BS, -1)[slots.long()] for t in kv[layer]]


def _run(eng, tokens, st, picks):
    g = eng.retrieve_layer_head_token_wise(tokens, sparse_state=st)
    cached = next(g)
    for req in picks:
        g.send(req)
    done = next(g)
    return cached, done


def test_sparse_steps_warm_state_and_extension():
    eng, kv = _engine()
    T = 900
    tokens = torch.arange(T) + 7
    src_slots = random_slots(T, NB * BS, seed=1)
    eng.store(tokens, slot_mapping=src_slots)
    src_rows = [_rows(kv, l, src_slots) for l in range(L)]
    dst_kv = zeros_like_kv(kv)
    eng.gpu_connector.register_kv_caches(dst_kv)  # decode into a fresh cache
    st = SparseRetrieveState()
    g = torch.Generator().manual_seed(2)
    for step in range(2):
        picks, want = [], []
        for l in range(L):
            sel = torch.randperm(T, generator=g)[:64]
            dst = torch.randperm(NB * BS, generator=g)[:64]
            picks.append(SparseLayerRequest(sel, dst))
            want.append((sel, dst))
        gets = eng.stats.get("sparse_fetches") if hasattr(eng.stats, "get") else None
        calls = {"n": 0}
        real = eng.storage_manager.batched_get

        def counting(keys, *a, **k):
            calls["n"] += 1
            return real(keys, *a, **k)

        eng.storage_manager.batched_get = counting
        cached, done = _run(eng, tokens, st, picks)
        eng.storage_manager.batched_get = real
        assert bool(cached.all())
        assert calls["n"] == (1 if step == 0 else 0)  # warm steps never touch the tiers
        for l, (sel, dst) in enumerate(want):
            got = _rows(dst_kv, l, dst)
            for p in range(2):
                assert torch.equal(got[p], src_rows[l][p][sel])
        assert int(done.sum()) == len(torch.cat([w[0] for w in want]).unique())
    # a longer context extends the state by the new chunks only
    T2 = 1200
    tokens2 = torch.cat([tokens, torch.arange(T2 - T) + 5000])
    slots2 = torch.cat([src_slots, random_slots(T2, NB * BS, seed=9)[:T2 - T]])
    eng.gpu_connector.register_kv_caches(kv)
    eng.store(tokens2, slot_mapping=slots2)
    n_before = len(st.objs)
    eng.gpu_connector.register_kv_caches(dst_kv)
    cached, _ = _run(eng, tokens2, st, [])
    assert st.total_tokens == T2 and len(st.objs) > n_before and bool(cached.all())
    st.release()
    eng.close()


def test_failed_extension_rolls_back():
    eng, kv = _engine()
    tokens = torch.arange(600)
    eng.store(tokens, slot_mapping=random_slots(600, NB * BS, seed=4))
    st = SparseRetrieveState()
    _run(eng, tokens[:256], st, [])
    keys, objs = list(st.keys), list(st.objs)

    def broken(*a, **k):
        raise RuntimeError("tier failed")

    eng.storage_manager.batched_get = broken
    with pytest.raises(RuntimeError):
        next(eng.retrieve_layer_head_token_wise(tokens, sparse_state=st))
    assert st.keys == keys and st.objs == objs  # unchanged
    st.release()
    eng.close()


def test_failed_copy_quarantines_and_marks_unhealthy():
    eng, kv = _engine()
    tokens = torch.arange(300)
    eng.store(tokens, slot_mapping=random_slots(300, NB * BS, seed=5))
    st = SparseRetrieveState()

    def broken(*a, **k):
        raise RuntimeError("copy failed")

    eng._sparse_layer_ref = broken
    g = eng.retrieve_layer_head_token_wise(tokens, sparse_state=st)
    next(g)
    with pytest.raises(RuntimeError):
        g.send(SparseLayerRequest(torch.tensor([1, 2]), torch.tensor([3, 4])))
    assert not eng.is_healthy()
    held = eng._quarantined[0]
    refs = [o.get_ref_count() for o in held]
    st.release()  # the caller lets go; the quarantine still holds them
    assert all(o.get_ref_count() == r - 1 >= 1 for o, r in zip(held, refs))
    eng.close()


@pytest.mark.gpu
def test_sparse_steps_gpu_pinned_chunks():
    eng, kv = _engine("cuda")
    T = 1000
    tokens = torch.arange(T)
    src_slots = random_slots(T, NB * BS, seed=11, device="cuda")
    eng.store(tokens, slot_mapping=src_slots)
    src_rows = [_rows(kv, l, src_slots) for l in range(L)]
    dst_kv = zeros_like_kv(kv)
    eng.gpu_connector.register_kv_caches(dst_kv)
    st = SparseRetrieveState()
    g = torch.Generator().manual_seed(3)
    picks = []
    for l in range(L):
        sel = torch.randperm(T, generator=g)[:200].cuda()
        dst = torch.randperm(NB * BS, generator=g)[:200].cuda()
        picks.append(SparseLayerRequest(sel, dst))
    _run(eng, tokens, st, picks)
    torch.cuda.synchronize()
    for l, pk in enumerate(picks):
        got = _rows(dst_kv, l, pk.slot_mapping)
        for p in range(2):
            assert torch.equal(got[p], src_rows[l][p][pk.selected_token_idx])
    st.release()
    eng.close()
