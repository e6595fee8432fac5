"""P2P cross-instance sharing through the controller, peer failure handling,
and the audit wrapper (CPU tier, loopback ZMQ)."""

import time

import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector
from lmcache_ascend_b200.v1.p2p_controller import P2PController

from .utils import make_separate_kv, random_slots, zeros_like_kv

L, NB, BS, H, D = 2, 32, 16, 2, 32


def _engine(ctl_url, seed, **kw):
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=seed)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02,
                                            enable_p2p=True, controller_url=ctl_url,
                                            p2p_init_ports=[0], blocking_timeout_secs=1.0, **kw)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    conn = VLLMPagedMemGPUConnector(cfg, kvcaches=kv)
    return LMCacheEngine(cfg, md, conn), conn, kv


def _rows(kv, slots):
    return [t.view(NB * BS, -1)[slots.long()] for layer in kv for t in layer]


def test_p2p_share_between_instances():
    ctl = P2PController().start()
    a, ca, kva = _engine(ctl.url, 1, lmcache_instance_id="A")
    b, cb, kvb = _engine(ctl.url, 2, lmcache_instance_id="B")
    try:
        tokens = torch.arange(192)
        s1 = random_slots(192, NB * BS, seed=3)
        want = _rows(kva, s1)
        a.store(tokens, slot_mapping=s1)
        assert b.lookup(tokens) == 192  # found on A through the controller
        cb.register_kv_caches(zeros_like_kv(kvb))
        s2 = random_slots(192, NB * BS, seed=4)
        assert bool(b.retrieve(tokens, slot_mapping=s2).all())
        got = [t.view(NB * BS, -1)[s2.long()] for l in range(L)
               for t in (cb.layout.planes[0].views[l], cb.layout.planes[1].views[l])]
        for x, y in zip(want, got):
            assert torch.equal(x.view(-1), y.reshape(-1))
        # evicting on A withdraws the keys
        cpu = a.storage_manager.backends["LocalCPUBackend"]
        for k in cpu.keys():
            cpu.remove(k)
        bcpu = b.storage_manager.backends["LocalCPUBackend"]
        for k in bcpu.keys():
            bcpu.remove(k)
        time.sleep(1.1)  # location cache TTL
        assert b.lookup(tokens) == 0
    finally:
        a.close()
        b.close()
        ctl.stop()


def test_p2p_dead_peer_is_a_miss():
    ctl = P2PController().start()
    a, ca, kva = _engine(ctl.url, 1, lmcache_instance_id="A2")
    b, cb, kvb = _engine(ctl.url, 2, lmcache_instance_id="B2")
    try:
        tokens = torch.arange(64)
        a.store(tokens, slot_mapping=random_slots(64, NB * BS, seed=5))
        # A's peer server stops answering (host-side fault), its keys stay registered
        p2p_a = a.storage_manager.backends["P2PBackend"]
        p2p_a._stop.set()
        p2p_a._t.join(timeout=2)
        t0 = time.time()
        ret = b.retrieve(tokens, slot_mapping=random_slots(64, NB * BS, seed=6))
        assert not bool(ret.any()) and time.time() - t0 < 5
    finally:
        b.close()
        ctl.stop()


def test_audit_backend_checks_and_keeps_data():
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=7)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02,
                                            enable_audit=True, remote_url=f"mem://audit-{time.time()}")
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    conn = VLLMPagedMemGPUConnector(cfg, kvcaches=kv)
    eng = LMCacheEngine(cfg, md, conn)
    tokens = torch.arange(128)
    eng.store(tokens, slot_mapping=random_slots(128, NB * BS, seed=8))
    rb = eng.storage_manager.backends["RemoteBackend"]
    rb.wait_for_puts()
    cpu = eng.storage_manager.backends["LocalCPUBackend"]
    for k in cpu.keys():
        cpu.remove(k)
    assert bool(eng.retrieve(tokens, slot_mapping=random_slots(128, NB * BS, seed=9)).all())
    assert rb.mismatches == 0
    assert eng.remove(tokens, locations=["RemoteBackend"]) == 0  # audit does not remove
    eng.close()


import pytest


@pytest.mark.gpu
def test_p2p_reads_peer_hbm_tier():
    """Both instances keep an HBM tier: B's miss is served by A leasing the
    chunk in its HBM slab and B copying it over the peer mapping (same GPU
    here: the same kernels and leases, local addresses); the lease is
    returned and B then holds the chunk in its own HBM tier."""
    ctl = P2PController().start()

    def eng(seed, name):
        kv = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=seed)
        cfg = LMCacheEngineConfig.from_defaults(
            chunk_size=64, max_local_cpu_size=0.02, local_gpu=True, max_local_gpu_size=0.02,
            enable_p2p=True, controller_url=ctl.url, p2p_init_ports=[0],
            blocking_timeout_secs=2.0, lmcache_instance_id=name)
        md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.bfloat16)
        conn = VLLMPagedMemGPUConnector(cfg, kvcaches=kv)
        return LMCacheEngine(cfg, md, conn), conn, kv

    a, ca, kva = eng(1, "A")
    b, cb, kvb = eng(2, "B")
    try:
        tokens = torch.arange(192)
        s1 = random_slots(192, NB * BS, seed=3, device="cuda")
        want = _rows(kva, s1)
        a.store(tokens, slot_mapping=s1)
        pa = a.storage_manager.backends["P2PBackend"]
        assert b.lookup(tokens) == 192
        s2 = random_slots(192, NB * BS, seed=4, device="cuda")
        assert bool(b.retrieve(tokens, slot_mapping=s2).all())
        torch.cuda.synchronize()
        for x, y in zip(want, _rows(kvb, s2)):
            assert torch.equal(x, y)
        pb = b.storage_manager.backends["P2PBackend"]
        assert pb.stats.counters.get("p2p_nvlink_bytes", 0) > 0
        assert not pa._leases  # every lease came back
        bh = b.storage_manager.backends["LocalGPUBackend"]
        assert len(bh) == 3  # the three chunks now live in B's HBM tier
    finally:
        a.close()
        b.close()
        ctl.stop()
