"""PD backend protocol on the host (CPU tier): sender and receiver engines
in one process, ZMQ control plane on loopback, TCP data channel, host page
pools.  Covers push, eager and delayed pull, back-pressure refusal, the
per-peer circuit breaker, the pull-pin TTL release and a dead receiver.
Faults are injected on the host only (refused allocations, a receiver that
never answers)."""

import time

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector
from lmcache_ascend_b200.utils.metrics import get_stats

from .utils import make_separate_kv, random_slots, zeros_like_kv

L, NB, BS, H, D = 2, 32, 16, 2, 32
CHUNK = 64


def _pair(pull=False, delay=False, recv_pages=64, ttl=5.0, backoff=5.0, timeout=5.0):
    base = dict(chunk_size=CHUNK, enable_pd=True, transfer_channel="tcp",
                pd_buffer_device="cpu", max_local_cpu_size=0.01, local_cpu=False,
                pd_pull_mode=pull, pd_delay_pull=delay, pd_pull_pending_ttl=ttl,
                pd_alloc_fail_backoff_ttl=backoff, blocking_timeout_secs=timeout,
                pd_backpressure_reserve=0.0, pd_peer_init_port=[0], pd_peer_alloc_port=[0])
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    kv_r = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=1)
    page = 2 * L * CHUNK * H * D * 4
    rcfg = LMCacheEngineConfig.from_defaults(pd_role="receiver",
                                             pd_buffer_size=recv_pages * page, **base)
    rconn = VLLMPagedMemGPUConnector(rcfg, kvcaches=zeros_like_kv(kv_r))
    recv = LMCacheEngine(rcfg, md, rconn)
    recv.post_init()
    pd_r = recv.storage_manager.backends["PDBackend"]
    init_url, alloc_url = pd_r.endpoints()
    kv_s = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=2)
    scfg = LMCacheEngineConfig.from_defaults(pd_role="sender", pd_buffer_size=64 * page, **base)
    sconn = VLLMPagedMemGPUConnector(scfg, kvcaches=kv_s)
    send = LMCacheEngine(scfg, md, sconn, peer_init_url=init_url, peer_alloc_url=alloc_url)
    send.post_init()
    return send, recv, kv_s


def _rows(kv, slots):
    return [t.view(NB * BS, -1)[slots.long()] for layer in kv for t in layer]


@pytest.mark.parametrize("pull,delay", [(False, False), (True, False), (True, True)])
def test_pd_round_trip(pull, delay):
    send, recv, kv_s = _pair(pull=pull, delay=delay)
    try:
        tokens = torch.arange(200)
        s_slots = random_slots(200, NB * BS, seed=3)
        want = _rows(kv_s, s_slots)
        send.store(tokens, slot_mapping=s_slots)
        deadline = time.time() + 10
        while recv.lookup(tokens) < 200 and time.time() < deadline:
            time.sleep(0.01)
        assert recv.lookup(tokens) == 200
        r_slots = random_slots(200, NB * BS, seed=4)
        ret = recv.retrieve(tokens, slot_mapping=r_slots)
        assert bool(ret.all())
        got = _rows(recv.gpu_connector.layout_kv if hasattr(recv.gpu_connector, "layout_kv")
                    else [tuple(p.views[l] for p in recv.gpu_connector.layout.planes)
                          for l in range(L)], r_slots)
        for a, b in zip(want, got):
            assert torch.equal(a, b)
        if pull:  # pins released once the receiver reported completion
            deadline = time.time() + 5
            pd_s = send.storage_manager.backends["PDBackend"]
            while pd_s.pull_pending and time.time() < deadline:
                time.sleep(0.01)
            assert not pd_s.pull_pending
    finally:
        send.close()
        recv.close()


def test_pd_backpressure_trips_breaker():
    # receiver pool of 2 pages, request of 4 chunks -> refused, breaker opens
    send, recv, _ = _pair(recv_pages=2, backoff=0.3)
    try:
        st = get_stats()
        before = st.snapshot()["counters"].get("pd_breaker_trips", 0)
        send.store(torch.arange(256), slot_mapping=random_slots(256, NB * BS, seed=5))
        assert recv.lookup(torch.arange(256)) == 0
        assert send.storage_manager.backends["PDBackend"].breaker_open()
        assert st.snapshot()["counters"]["pd_breaker_trips"] == before + 1
        skips = st.snapshot()["counters"].get("pd_breaker_skips", 0)
        send.store(torch.arange(1000, 1064), slot_mapping=random_slots(64, NB * BS, seed=6))
        assert st.snapshot()["counters"]["pd_breaker_skips"] == skips + 1
        time.sleep(0.35)  # after the back-off a small request goes through
        send.store(torch.arange(2000, 2064), slot_mapping=random_slots(64, NB * BS, seed=7))
        assert recv.lookup(torch.arange(2000, 2064)) == 64
    finally:
        send.close()
        recv.close()


def test_pd_pull_pins_released_after_ttl():
    # delayed pull that the decoder never retrieves: the sender's TTL sweep
    # releases the pinned pages
    send, recv, _ = _pair(pull=True, delay=True, ttl=0.3)
    try:
        pd_s = send.storage_manager.backends["PDBackend"]
        free0 = pd_s.allocator.num_free
        send.store(torch.arange(128), slot_mapping=random_slots(128, NB * BS, seed=8))
        assert pd_s.pull_pending
        time.sleep(0.8)
        assert not pd_s.pull_pending
        assert pd_s.allocator.num_free == free0
    finally:
        send.close()
        recv.close()


def test_pd_dead_receiver_times_out():
    send, recv, _ = _pair(timeout=0.5, backoff=10.0)
    recv.close()  # the decoder goes away before the prefiller pushes
    try:
        t0 = time.time()
        send.store(torch.arange(64), slot_mapping=random_slots(64, NB * BS, seed=9))
        assert time.time() - t0 < 5
        assert send.storage_manager.backends["PDBackend"].breaker_open()
    finally:
        send.close()
