"""Remote tier (mem:// and lm:// server), naive and CacheGen serde, and the
local-disk tier, through the engine; CacheGen quantisation error bounds and
CPU/GPU bitstream identity."""

import time

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.server import LMCacheServer
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.cachegen import CacheGenConfig, decode_kv, encode_kv, CacheGenEncoded
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

from .utils import make_separate_kv, random_slots, zeros_like_kv

L, NB, BS, H, D = 3, 32, 16, 2, 64


def _engine(**cfg):
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=1)
    c = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02, **cfg)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    conn = VLLMPagedMemGPUConnector(c, kvcaches=kv)
    return LMCacheEngine(c, md, conn), conn, kv


def _rows(kv, slots):
    return [t.view(NB * BS, -1)[slots.long()] for layer in kv for t in layer]


def _flush(eng):
    for b in eng.storage_manager.backends.values():
        for f in ("wait_for_puts", "wait_for_writes"):
            if hasattr(b, f):
                getattr(b, f)()


@pytest.mark.parametrize("url_kind", ["mem", "lm"])
def test_remote_naive_round_trip(url_kind):
    srv = None
    if url_kind == "lm":
        srv = LMCacheServer().start()
        url = srv.url
    else:
        url = f"mem://naive-{time.time()}"
    try:
        eng, conn, kv = _engine(remote_url=url, remote_serde="naive")
        tokens = torch.arange(150)
        s1 = random_slots(150, NB * BS, seed=2)
        want = _rows(kv, s1)
        eng.store(tokens, slot_mapping=s1)
        _flush(eng)
        eng.storage_manager.backends["LocalCPUBackend"].close()  # force remote hits
        eng.storage_manager.backends["LocalCPUBackend"].__init__(eng.config)
        assert eng.lookup(tokens) == 150
        conn.register_kv_caches(zeros_like_kv(kv))
        s2 = random_slots(150, NB * BS, seed=3)
        assert bool(eng.retrieve(tokens, slot_mapping=s2).all())
        got = [t.view(NB * BS, -1)[s2.long()] for p in [conn.layout.planes]
               for l in range(L) for t in (p[0].views[l], p[1].views[l])]
        for a, b in zip(want, got):
            assert torch.equal(a.view(-1), b.reshape(-1))
        eng.close()
    finally:
        if srv:
            srv.stop()


def test_local_disk_round_trip(tmp_path):
    eng, conn, kv = _engine(local_disk=str(tmp_path), max_local_disk_size=0.1)
    tokens = torch.arange(130)
    s1 = random_slots(130, NB * BS, seed=4)
    want = _rows(kv, s1)
    eng.store(tokens, slot_mapping=s1)
    _flush(eng)
    cpu = eng.storage_manager.backends["LocalCPUBackend"]
    for k in cpu.keys():
        cpu.remove(k)
    assert eng.lookup(tokens) == 130
    conn.register_kv_caches(zeros_like_kv(kv))
    s2 = random_slots(130, NB * BS, seed=5)
    assert bool(eng.retrieve(tokens, slot_mapping=s2).all())
    got = [t.view(NB * BS, -1)[s2.long()] for l in range(L)
           for t in (conn.layout.planes[0].views[l], conn.layout.planes[1].views[l])]
    for a, b in zip(want, got):
        assert torch.equal(a.view(-1), b.reshape(-1))
    eng.close()


def _kv_chunk(L, T, C, dev="cpu", seed=0):
    g = torch.Generator().manual_seed(seed)
    scale = torch.rand(C, generator=g) * 1.5 + 0.5  # per-channel U(0.5, 2)
    return (torch.randn(2, L, T, C, generator=g) * scale).to(torch.bfloat16).to(dev)


@pytest.mark.parametrize("dev", ["cpu", pytest.param("cuda", marks=pytest.mark.gpu)])
def test_cachegen_round_trip_error(dev):
    L, T, C = 4, 256, 128
    kv = _kv_chunk(L, T, C, dev)
    cfg = CacheGenConfig.from_ranges(L, [(0, 2, 32), (2, 4, 16)], [(0, 1, 256), (1, 4, 16)])
    enc = encode_kv(kv, cfg)
    raw = kv.numel() * 2
    data = enc.to_bytes()
    assert len(data) < raw * 0.45  # well below the bf16 size (includes the entropy model)
    dec = decode_kv(CacheGenEncoded.from_bytes(data), dev)
    # error <= half a quantisation step per element
    for i, bins in ((0, cfg.bins("k")), (1, cfg.bins("v"))):
        half = (bins // 2 - 1).float().view(-1, 1, 1)
        step = kv[i].float().abs().amax(-1, keepdim=True).cpu() / half
        err = (dec[i].float().cpu() - kv[i].float().cpu()).abs()
        # half a step, plus the bf16 rounding of the dequantised value
        tol = step * 0.51 + kv[i].float().abs().cpu() * 2 ** -7 + 1e-3
        assert bool((err <= tol).all())


@pytest.mark.gpu
def test_cachegen_gpu_matches_cpu_bytes():
    L, T, C = 3, 128, 256
    kv = _kv_chunk(L, T, C, "cpu", seed=3)
    cfg = CacheGenConfig.default(L)
    a = encode_kv(kv, cfg).to_bytes()
    b = encode_kv(kv.cuda(), cfg).to_bytes()
    assert a == b


def test_remote_cachegen_serde_engine():
    eng, conn, kv = _engine(remote_url=f"mem://cg-{time.time()}", remote_serde="cachegen",
                            cachegen_k_bins=[[0, 100, 256]], cachegen_v_bins=[[0, 100, 256]])
    # cachegen quantises: compare within a step
    tokens = torch.arange(64)
    s1 = random_slots(64, NB * BS, seed=6)
    want = _rows(kv, s1)
    eng.store(tokens, slot_mapping=s1)
    _flush(eng)
    cpu = eng.storage_manager.backends["LocalCPUBackend"]
    for k in cpu.keys():
        cpu.remove(k)
    conn.register_kv_caches(zeros_like_kv(kv))
    s2 = random_slots(64, NB * BS, seed=7)
    assert bool(eng.retrieve(tokens, slot_mapping=s2).all())
    got = [t.view(NB * BS, -1)[s2.long()] for l in range(L)
           for t in (conn.layout.planes[0].views[l], conn.layout.planes[1].views[l])]
    for a, b in zip(want, got):
        step = a.abs().amax(-1, keepdim=True) / 127
        assert bool(((a - b.reshape(a.shape)).abs() <= step * 0.51 + 1e-6).all())
    eng.close()
