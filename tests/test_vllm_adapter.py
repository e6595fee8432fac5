"""vLLM v1 connector logic driven with light stand-ins for vLLM's scheduler
objects (CPU tier): request A is prefilled and saved; request B with the same
prompt is matched by the scheduler, and its KV is loaded into B's blocks by
the worker; chunked prefill saves chunk by chunk; the lookup channel works
across a ZMQ IPC socket."""

from types import SimpleNamespace

import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig
from lmcache_ascend_b200.integration.vllm.adapter import LMCacheConnectorV1Impl
from lmcache_ascend_b200.integration.vllm.lookup import LookupClient, LookupServer

L, NB, BS, H, D = 2, 128, 16, 2, 32


def _kv():
    torch.manual_seed(0)
    return {f"model.layers.{i}.self_attn.attn": torch.zeros(2, NB, BS, H, D) for i in range(L)}


def _sched_out(new=(), cached=None, scheduled=None, finished=()):
    cached = cached or SimpleNamespace(req_ids=[], new_token_ids=[], new_block_ids=[],
                                       num_computed_tokens=[], resumed_req_ids=set())
    return SimpleNamespace(scheduled_new_reqs=list(new), scheduled_cached_reqs=cached,
                           num_scheduled_tokens=scheduled or {}, finished_req_ids=set(finished))


def _pair(cfg):
    worker = LMCacheConnectorV1Impl("worker", cfg, "m", BS)
    kv = _kv()
    worker.register_kv_caches(kv)
    sched = LMCacheConnectorV1Impl("scheduler", cfg, "m", BS, engine=worker.engine)
    return sched, worker, kv


def _slots(blocks, n):
    b = torch.tensor(blocks)
    t = torch.arange(n)
    return b[t // BS] * BS + t % BS


def _fill(kv, slots, seed):
    g = torch.Generator().manual_seed(seed)
    for t in kv.values():
        t.view(2, NB * BS, -1)[:, slots] = torch.randn(2, len(slots), H * D, generator=g)


def _read(kv, slots):
    return [t.view(2, NB * BS, -1)[:, slots].clone() for t in kv.values()]


def _step(worker, meta):
    worker.bind_connector_metadata(meta)
    worker.start_load_kv(None)
    for name in worker._layer_names:
        worker.wait_for_layer_load(name)
        worker.save_kv_layer(name, None, None)
    worker.wait_for_save()
    worker.clear_connector_metadata()


def test_save_then_prefix_hit_loads_into_new_blocks():
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=256, max_local_cpu_size=0.05)
    sched, worker, kv = _pair(cfg)
    prompt = list(range(1000, 1600))  # 600 tokens
    blocks_a = list(range(0, 38))
    req_a = SimpleNamespace(request_id="A", prompt_token_ids=prompt)
    assert sched.get_num_new_matched_tokens(req_a, 0) == (0, False)
    sched.update_state_after_alloc(req_a, None, 0)
    new_a = SimpleNamespace(req_id="A", prompt_token_ids=prompt, block_ids=(blocks_a,),
                            num_computed_tokens=0)
    meta = sched.build_connector_meta(_sched_out([new_a], scheduled={"A": 600}))
    assert len(meta.requests) == 1 and meta.requests[0].save_spec is not None
    sa = _slots(blocks_a, 600)
    _fill(kv, sa, seed=1)  # the model's forward wrote A's KV
    want = _read(kv, sa)
    _step(worker, meta)

    req_b = SimpleNamespace(request_id="B", prompt_token_ids=prompt)
    need, is_async = sched.get_num_new_matched_tokens(req_b, 0)
    assert need == 599 and not is_async
    sched.update_state_after_alloc(req_b, None, need)
    blocks_b = list(range(40, 78))
    new_b = SimpleNamespace(req_id="B", prompt_token_ids=prompt, block_ids=(blocks_b,),
                            num_computed_tokens=0)
    meta = sched.build_connector_meta(_sched_out([new_b], scheduled={"B": 1}))
    r = meta.requests[0]
    assert r.load_spec is not None and r.load_spec.lmcache_cached_tokens == 600
    _step(worker, meta)
    got = _read(kv, _slots(blocks_b, 600))
    for a, b in zip(want, got):
        assert torch.equal(a, b)
    sched.request_finished(req_b, blocks_b)
    worker.shutdown()
    worker.engine.close()


def test_chunked_prefill_saves_per_chunk_and_layerwise():
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=128, max_local_cpu_size=0.05,
                                            use_layerwise=True)
    sched, worker, kv = _pair(cfg)
    prompt = list(range(300))
    blocks = list(range(0, 19))
    req = SimpleNamespace(request_id="C", prompt_token_ids=prompt)
    sched.get_num_new_matched_tokens(req, 0)
    new = SimpleNamespace(req_id="C", prompt_token_ids=prompt, block_ids=(blocks,),
                          num_computed_tokens=0)
    s = _slots(blocks, 300)
    _fill(kv, s, seed=2)
    meta = sched.build_connector_meta(_sched_out([new], scheduled={"C": 200}))
    assert meta.requests[0].token_ids.numel() == 128  # one full chunk so far
    _step(worker, meta)
    cached = SimpleNamespace(req_ids=["C"], new_token_ids=[[]], new_block_ids=[None],
                             num_computed_tokens=[200], resumed_req_ids=set())
    meta = sched.build_connector_meta(_sched_out(cached=cached, scheduled={"C": 100}))
    assert meta.requests[0].save_spec.skip_leading_tokens == 128
    assert meta.requests[0].token_ids.numel() == 300  # last prefill saves the tail
    _step(worker, meta)
    assert worker.engine.lookup(torch.tensor(prompt)) == 300  # found through the layer keys
    worker.shutdown()
    worker.engine.close()


def test_lookup_over_ipc():
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.01,
                                            lmcache_instance_id="ipc-test")
    worker = LMCacheConnectorV1Impl("worker", cfg, "m", BS)
    kv = _kv()
    worker.register_kv_caches(kv)
    toks = torch.arange(128)
    worker.engine.store(toks, slot_mapping=_slots(list(range(8)), 128))
    client = LookupClient(worker.lookup_url)
    assert client.lookup(toks.tolist(), "r1") == 128
    client.unpin("r1")
    assert client.lookup(list(range(500, 564)), "r2") == 0
    client.close()
    worker.shutdown()
    worker.engine.close()


def test_kv_consumer_loads_but_never_saves():
    import pytest

    cfg = LMCacheEngineConfig.from_defaults(chunk_size=256, max_local_cpu_size=0.05)
    worker = LMCacheConnectorV1Impl("worker", cfg, "m", BS, kv_role="kv_consumer")
    kv = _kv()
    worker.register_kv_caches(kv)
    sched = LMCacheConnectorV1Impl("scheduler", cfg, "m", BS, engine=worker.engine,
                                   kv_role="kv_consumer")
    prompt = list(range(3000, 3600))
    req = SimpleNamespace(request_id="C", prompt_token_ids=prompt)
    sched.get_num_new_matched_tokens(req, 0)
    sched.update_state_after_alloc(req, None, 0)
    new = SimpleNamespace(req_id="C", prompt_token_ids=prompt, block_ids=(list(range(38)),),
                          num_computed_tokens=0)
    meta = sched.build_connector_meta(_sched_out([new], scheduled={"C": 600}))
    _fill(kv, _slots(list(range(38)), 600), seed=3)
    _step(worker, meta)
    assert worker.engine.lookup(torch.tensor(prompt)) == 0  # nothing was stored
    with pytest.raises(ValueError):
        LMCacheConnectorV1Impl("worker", cfg, "m", BS, kv_role="kv_sideways")
    worker.shutdown()
    worker.engine.close()


def test_two_group_model_latent_and_indexer():
    """A DSA-shaped model registers two KV cache groups (MLA latent layers
    and indexer layers, different shapes and dtypes); each group gets its own
    block table from vLLM, is stored by its own engine, and a prefix hit
    loads both groups into the new request's blocks.  The scheduler's lookup
    counts a prefix only as far as every group holds it."""
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.05)
    worker = LMCacheConnectorV1Impl("worker", cfg, "dsa", BS, use_mla=True)
    kv = {}
    for i in range(2):
        kv[f"model.layers.{i}.self_attn.attn"] = torch.zeros(NB, BS, 96)           # latent
        kv[f"model.layers.{i}.self_attn.indexer.k_cache"] = torch.zeros(NB, BS, 32,
                                                                        dtype=torch.bfloat16)
    worker.register_kv_caches(kv)
    assert len(worker._engines) == 2
    sched = LMCacheConnectorV1Impl("scheduler", cfg, "dsa", BS, use_mla=True,
                                   engine=worker.lookup_engine)
    prompt = list(range(200))
    lat_a, idx_a = list(range(0, 13)), list(range(60, 73))
    g = torch.Generator().manual_seed(5)
    t = torch.arange(200)
    s_lat = torch.tensor(lat_a)[t // BS] * BS + t % BS
    s_idx = torch.tensor(idx_a)[t // BS] * BS + t % BS
    for name, x in kv.items():
        s = s_idx if "indexer" in name else s_lat
        x.view(NB * BS, -1)[s] = torch.randn(200, x.shape[-1], generator=g).to(x.dtype)
    want = {n: x.view(NB * BS, -1)[s_idx if "indexer" in n else s_lat].clone()
            for n, x in kv.items()}
    req = SimpleNamespace(request_id="A", prompt_token_ids=prompt)
    sched.get_num_new_matched_tokens(req, 0)
    new = SimpleNamespace(req_id="A", prompt_token_ids=prompt, block_ids=(lat_a, idx_a),
                          num_computed_tokens=0)
    meta = sched.build_connector_meta(_sched_out([new], scheduled={"A": 200}))
    assert len(meta.requests[0].group_slot_mappings) == 1
    _step(worker, meta)
    # request B: same prompt, new blocks in both groups
    req_b = SimpleNamespace(request_id="B", prompt_token_ids=prompt)
    need, _ = sched.get_num_new_matched_tokens(req_b, 0)
    assert need == 199
    sched.update_state_after_alloc(req_b, None, need)
    lat_b, idx_b = list(range(20, 33)), list(range(80, 93))
    new_b = SimpleNamespace(req_id="B", prompt_token_ids=prompt, block_ids=(lat_b, idx_b),
                            num_computed_tokens=0)
    meta = sched.build_connector_meta(_sched_out([new_b], scheduled={"B": 1}))
    _step(worker, meta)
    s_lat_b = torch.tensor(lat_b)[t // BS] * BS + t % BS
    s_idx_b = torch.tensor(idx_b)[t // BS] * BS + t % BS
    for n, x in kv.items():
        got = x.view(NB * BS, -1)[s_idx_b if "indexer" in n else s_lat_b]
        assert torch.equal(got, want[n]), n
    # drop the indexer group's chunks: the grouped lookup no longer reports a hit
    worker._engines[1].clear()
    req_c = SimpleNamespace(request_id="C", prompt_token_ids=prompt)
    assert sched.get_num_new_matched_tokens(req_c, 0) == (0, False)
    worker.shutdown()
    worker.engine.close()


def test_blending_on_load_through_the_served_model():
    """enable_blending: the worker's load of a hit runs CacheBlend on the
    model the serving process registered (here a vLLM-shaped wrapper around
    this repo's reference model); with every token recomputed the request's
    blocks end up with exactly the KV a prefill of the prompt writes, although
    the cached KV it started from was different."""
    from lmcache_ascend_b200.models.llama import LlamaConfig, LlamaForBlend
    from lmcache_ascend_b200.v1.blend.vllm_model import VLLMModelTracker, drop_blender

    from .test_blend_vllm_model import _served

    cfg = LMCacheEngineConfig.from_defaults(
        chunk_size=256, max_local_cpu_size=0.05, enable_blending=True, use_layerwise=True,
        blend_recompute_ratios=[1.0], blend_check_layers=[0],
        lmcache_instance_id="adapter-blend-test")
    mc = LlamaConfig.tiny(vocab_size=2000, hidden_size=128, num_layers=L, num_heads=4,
                          num_kv_heads=H, head_dim=D, intermediate_size=256, max_position=4096)
    ref = LlamaForBlend(mc, device="cpu")
    VLLMModelTracker.unregister(cfg.lmcache_instance_id)
    drop_blender(cfg.lmcache_instance_id)
    VLLMModelTracker.register_model(cfg.lmcache_instance_id, _served(ref, mc, False))
    sched, worker, kv = _pair(cfg)
    try:
        prompt = list(range(1000, 1300))  # 300 tokens
        blocks_a = list(range(0, 19))
        req_a = SimpleNamespace(request_id="A", prompt_token_ids=prompt)
        sched.get_num_new_matched_tokens(req_a, 0)
        sched.update_state_after_alloc(req_a, None, 0)
        new_a = SimpleNamespace(req_id="A", prompt_token_ids=prompt, block_ids=(blocks_a,),
                                num_computed_tokens=0)
        meta = sched.build_connector_meta(_sched_out([new_a], scheduled={"A": 300}))
        sa = _slots(blocks_a, 300)
        # the cached KV of A is NOT what the model computes for this prompt, so
        # only a recompute (the blend) can produce the model's KV for B
        _fill(kv, sa, seed=1)
        _step(worker, meta)

        req_b = SimpleNamespace(request_id="B", prompt_token_ids=prompt)
        need, _ = sched.get_num_new_matched_tokens(req_b, 0)
        assert need > 0
        sched.update_state_after_alloc(req_b, None, need)
        blocks_b = list(range(40, 59))
        new_b = SimpleNamespace(req_id="B", prompt_token_ids=prompt, block_ids=(blocks_b,),
                                num_computed_tokens=0)
        meta = sched.build_connector_meta(_sched_out([new_b], scheduled={"B": 1}))
        _step(worker, meta)
        n = meta.requests[0].load_spec.lmcache_cached_tokens
        sb = _slots(blocks_b, 300)[:n]
        got = _read(kv, sb)
        fresh = {k: torch.zeros_like(t) for k, t in kv.items()}
        ref.prefill(torch.tensor(prompt[:n]), [(t[0], t[1]) for t in fresh.values()], sb)
        for a, b in zip(got, _read(fresh, sb)):
            assert torch.allclose(a, b, atol=1e-4, rtol=1e-4)
        from lmcache_ascend_b200.v1.blend.vllm_model import _blenders

        assert cfg.lmcache_instance_id in _blenders
        sched.request_finished(req_b, blocks_b)
    finally:
        worker.shutdown()
        worker.engine.close()
        drop_blender(cfg.lmcache_instance_id)
        VLLMModelTracker.unregister(cfg.lmcache_instance_id)
