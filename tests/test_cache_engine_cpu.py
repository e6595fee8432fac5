"""CPU tier: engine store/retrieve round trip and the
engine's lookup / pin / eviction / layerwise semantics."""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import (
    VLLMPagedMemGPUConnector,
    VLLMPagedMemLayerwiseGPUConnector,
)
from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

from .utils import make_merged_kv, make_mla_kv, make_separate_kv, random_slots, zeros_like_kv


def _engine(kv, chunk=256, layerwise=False, **cfg):
    config = LMCacheEngineConfig.from_defaults(chunk_size=chunk, max_local_cpu_size=0.05,
                                               use_layerwise=layerwise, **cfg)
    md = LMCacheEngineMetadata("test-model", 1, 0, "vllm", torch.float32)
    cls = VLLMPagedMemLayerwiseGPUConnector if layerwise else VLLMPagedMemGPUConnector
    conn = cls(config, kvcaches=kv)
    return LMCacheEngine(config, md, conn), conn


def _rows(layout: PagedKVLayout, slots):
    """[L, T, sum(E)] copy of the rows at `slots` (planes concatenated)."""
    s = slots.long()
    blk, off = s // layout.block_size, s % layout.block_size
    return torch.stack([torch.cat([p.rows(l, blk, off) for p in layout.planes], dim=-1)
                        for l in range(layout.num_layers)])


def test_config1_round_trip_bit_exact():
    # 2 layers, 4 KV heads, head_dim 64, block 16, 64 blocks,
    # fp32 N(0,1) seed 0; 4 x 512-token prompts sharing a 256-token prefix.
    torch.manual_seed(0)
    L, H, D, BS, NB = 2, 4, 64, 16, 64
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=0)
    eng, conn = _engine(kv)
    g = torch.Generator().manual_seed(0)
    prefix = torch.randint(0, 32000, (256,), generator=g)
    prompts = [torch.cat([prefix, torch.randint(0, 32000, (256,), generator=g)])
               for _ in range(4)]
    expected = []
    for i, p in enumerate(prompts):
        slots = random_slots(512, NB * BS, seed=100 + i)
        # fresh KV for this request's slots
        for layer in kv:
            for t in layer:
                t.view(NB * BS, -1)[slots] = torch.randn(512, H * D, generator=g)
        exp = _rows(conn.layout, slots)
        if i > 0:  # the shared prefix chunk was stored by prompt 0
            exp[:, :256] = expected[0][:, :256]
        expected.append(exp)
        eng.store(p, slot_mapping=slots)
    assert len(eng.storage_manager.backends["LocalCPUBackend"]) == 1 + 4  # 1 shared + 4 tails
    for i, p in enumerate(prompts):
        fresh = zeros_like_kv(kv)
        conn.register_kv_caches(fresh)
        slots = random_slots(512, NB * BS, seed=200 + i)
        assert eng.lookup(p) == 512
        ret = eng.retrieve(p, slot_mapping=slots)
        assert bool(ret.all())
        got = _rows(conn.layout, slots)
        assert torch.equal(got, expected[i])
    eng.close()


@pytest.mark.parametrize("fmt", ["merged", "flashinfer", "mla", "mla_flat", "dsa"])
def test_formats_round_trip(fmt):
    L, BS, NB = 3, 16, 32
    if fmt == "merged":
        kv = make_merged_kv(L, NB, BS, 2, 32, torch.float16, "cpu")
        mla = False
    elif fmt == "flashinfer":
        kv = make_merged_kv(L, NB, BS, 2, 32, torch.float16, "cpu", flashinfer=True)
        mla = False
    elif fmt == "mla":
        kv = make_mla_kv(L, NB, BS, 64, 16, torch.bfloat16, "cpu")
        mla = True
    elif fmt == "mla_flat":
        kv = make_mla_kv(L, NB, BS, 64, 16, torch.bfloat16, "cpu", flat=True)
        mla = True
    else:
        kv = make_mla_kv(L, NB, BS, 64, 16, torch.bfloat16, "cpu", indexer_dim=32)
        mla = True
    config = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", kv[0][0].dtype if isinstance(kv[0], tuple)
                               else kv[0].dtype, use_mla=mla)
    conn = VLLMPagedMemGPUConnector(config, use_mla=mla, kvcaches=kv)
    eng = LMCacheEngine(config, md, conn)
    tokens = torch.arange(200)
    slots = random_slots(200, NB * BS, seed=1)
    exp = _rows(conn.layout, slots)
    eng.store(tokens, slot_mapping=slots)
    conn.register_kv_caches(zeros_like_kv(kv))
    slots2 = random_slots(200, NB * BS, seed=2)
    ret = eng.retrieve(tokens, slot_mapping=slots2)
    assert bool(ret.all())
    assert torch.equal(_rows(conn.layout, slots2), exp)
    eng.close()


def test_prefix_semantics_and_mask():
    kv = make_separate_kv(1, 32, 16, 2, 16, torch.float32, "cpu")
    eng, conn = _engine(kv, chunk=64)
    tokens = torch.arange(256)
    slots = random_slots(256, 512, seed=3)
    eng.store(tokens, slot_mapping=slots)
    assert eng.lookup(tokens) == 256
    # diverging third chunk: only two chunks hit
    other = tokens.clone()
    other[130] = 99999
    assert eng.lookup(other) == 128
    ret = eng.retrieve(other, slot_mapping=slots)
    assert int(ret.sum()) == 128 and bool(ret[:128].all())
    # mask: skip the first chunk
    mask = torch.ones(256, dtype=torch.bool)
    mask[:64] = False
    ret = eng.retrieve(tokens, mask=mask, slot_mapping=slots)
    assert not bool(ret[:64].any()) and bool(ret[64:].all())
    eng.close()


def test_lookup_pin_and_eviction():
    kv = make_separate_kv(1, 64, 16, 2, 64, torch.float32, "cpu")
    # 64 tokens x 2 x 1 x 128 x 4 B = 64 KiB per chunk; 200 KiB cache = 3 chunks
    config = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=200 / (1 << 20))
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    conn = VLLMPagedMemGPUConnector(config, kvcaches=kv)
    eng = LMCacheEngine(config, md, conn)
    a = torch.arange(128)
    b = torch.arange(1000, 1128)
    eng.store(a, slot_mapping=random_slots(128, 1024, seed=4))
    assert eng.lookup(a, lookup_id="r1", pin=True) == 128
    eng.store(b, slot_mapping=random_slots(128, 1024, seed=5))
    # a's chunks are pinned and survive; b could keep at most one chunk
    assert eng.lookup(a) == 128
    assert eng.lookup(b) <= 64
    eng.lookup_unpin("r1")
    c = torch.arange(2000, 2128)
    eng.store(c, slot_mapping=random_slots(128, 1024, seed=6))
    assert eng.lookup(c) >= 64
    eng.close()


def test_async_store_and_finished():
    kv = make_separate_kv(1, 32, 16, 2, 16, torch.float32, "cpu")
    eng, conn = _engine(kv, chunk=64, store_async=True)
    for i in range(5):
        eng.store(torch.arange(i * 1000, i * 1000 + 128),
                  slot_mapping=random_slots(128, 512, seed=i), req_id=f"r{i}")
    assert eng.wait_for_pending_stores(timeout=10)
    assert sorted(eng.get_finished_stores()) == [f"r{i}" for i in range(5)]
    assert eng.lookup(torch.arange(4000, 4128)) == 128
    eng.close()


def test_layerwise_store_and_retrieve():
    L = 4
    kv = make_separate_kv(L, 32, 16, 2, 16, torch.float32, "cpu")
    eng, conn = _engine(kv, chunk=64, layerwise=True)
    tokens = torch.arange(160)
    slots = random_slots(160, 512, seed=7)
    exp = _rows(conn.layout, slots)
    gen = eng.store_layer(tokens, slot_mapping=slots)
    n = sum(1 for _ in gen)
    assert n == L + 1
    conn.register_kv_caches(zeros_like_kv(kv))
    slots2 = random_slots(160, 512, seed=8)
    gen = eng.retrieve_layer(tokens, slot_mapping=slots2)
    outs = list(gen)
    assert len(outs) == L + 2
    ret = outs[-1]
    assert bool(ret.all())
    assert torch.equal(_rows(conn.layout, slots2), exp)
    eng.close()


def test_kv_events_and_unhealthy():
    kv = make_separate_kv(1, 32, 16, 2, 16, torch.float32, "cpu")
    eng, conn = _engine(kv, chunk=64, enable_kv_events=True)
    eng.store(torch.arange(128), slot_mapping=random_slots(128, 512))
    ev = eng.get_kv_events()
    assert len(ev) == 2 and ev[1].parent_block_hash == ev[0].block_hashes[0]
    eng.mark_unhealthy("test")
    eng.store(torch.arange(500, 628), slot_mapping=random_slots(128, 512))
    assert eng.lookup(torch.arange(500, 628)) == 0
    eng.close()


def test_head_major_cache_round_trip():
    """vLLM can store heads apart behind a token-major shape (HND)."""
    g = torch.Generator().manual_seed(3)
    kv = [torch.randn(16, 2, 2, 16, 32, generator=g).permute(0, 1, 3, 2, 4) for _ in range(2)]
    eng, conn = _engine(kv, chunk=64)
    assert conn.layout.planes[0].segmented
    tokens = torch.arange(100)
    slots = random_slots(100, 256, seed=1)
    exp = _rows(conn.layout, slots)
    eng.store(tokens, slot_mapping=slots)
    fresh = [torch.zeros(16, 2, 2, 16, 32).permute(0, 1, 3, 2, 4) for _ in range(2)]
    conn.register_kv_caches(fresh)
    slots2 = random_slots(100, 256, seed=2)
    assert bool(eng.retrieve(tokens, slot_mapping=slots2).all())
    assert torch.equal(_rows(conn.layout, slots2), exp)
    eng.close()


def test_key_hash_cache_is_not_pickled():
    import pickle
    import subprocess
    import sys

    from lmcache_ascend_b200.utils.keys import CacheEngineKey

    k = CacheEngineKey("vllm", "model-x", 2, 1, 0xABCDEF, "bfloat16", 0, (("tag", "v"),))
    hash(k)  # fills the cache in this process
    blob = pickle.dumps(k)
    assert "_h" not in pickle.loads(blob).__dict__
    # another process (another str-hash salt) finds the key by equality
    code = ("import pickle,sys; from lmcache_ascend_b200.utils.keys import CacheEngineKey as K;"
            "k=pickle.loads(sys.stdin.buffer.read());"
            "d={K('vllm','model-x',2,1,0xABCDEF,'bfloat16',0,(('tag','v'),)):1};"
            "print(d.get(k))")
    out = subprocess.run([sys.executable, "-c", code], input=blob, capture_output=True,
                         env={**__import__("os").environ, "PYTHONHASHSEED": "123"})
    assert out.stdout.strip() == b"1", out.stderr


def test_layerwise_retrieve_survives_a_chunk_evicted_between_layers():
    L = 4
    kv = make_separate_kv(L, 32, 16, 2, 16, torch.float32, "cpu")
    eng, conn = _engine(kv, chunk=64, layerwise=True)
    tokens = torch.arange(192)
    slots = random_slots(192, 512, seed=9)
    exp = _rows(conn.layout, slots)
    for _ in eng.store_layer(tokens, slot_mapping=slots):
        pass
    cpu = eng.storage_manager.backends["LocalCPUBackend"]
    conn.register_kv_caches(zeros_like_kv(kv))
    slots2 = random_slots(192, 512, seed=10)
    gen = eng.retrieve_layer(tokens, slot_mapping=slots2)
    next(gen)  # lookup done: all 3 chunks hit
    keys = [k for _, _, k in eng._chunks(tokens)]
    cpu.remove(keys[1].layer_key(2))  # chunk 1 of layer 2 goes away mid-retrieve
    ret = list(gen)[-1]
    assert int(ret.sum()) == 64 and bool(ret[:64].all())  # usable prefix: chunk 0
    got = _rows(conn.layout, slots2)  # [L, T, E]
    assert torch.equal(got[:, :64], exp[:, :64])
    assert cpu.allocator.num_active == len(cpu.keys())  # no leaked references
    eng.close()
