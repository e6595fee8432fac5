"""Direct paged push: the decoder's grant comes before any launch.

Host-side protocol test (CPU, ZMQ on loopback).  The prefiller's push
launcher and the decoder's flag receiver are fakes that record what would
have run on a GPU, so the test can assert that NO kernel that stores into the
decoder's memory is launched when the decoder is dead, when the sender holds
a mapping of an earlier registration (stale epoch), or when the decoder
refuses (no reservation, other slots, out of range); and that a granted push
launches exactly once, after the grant.  Faults are made on the host only.
"""

import uuid

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.parallel.pd_push import ReceiverDesc
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

from .utils import make_separate_kv, zeros_like_kv

L, NB, BS, H, D = 2, 16, 16, 2, 32


class FakeLayout:
    def __init__(self, layout):
        self.num_layers, self.num_slots = layout.num_layers, layout.num_slots
        self.row_bytes = layout.row_bytes


class FakeReceiver:
    def __init__(self, layout):
        self.layout = FakeLayout(layout)
        self.new_epoch()
        self.expected = []
        self.waits = []

    def new_epoch(self):
        self.desc = ReceiverDesc(num_layers=self.layout.num_layers, block_size=BS,
                                 num_slots=self.layout.num_slots, block_stride=[0, 0],
                                 slot_stride=[0, 0], row_bytes=self.layout.row_bytes,
                                 planes=[], flags={}, device=0, epoch=uuid.uuid4().hex)

    def expect_host(self, n, lb, nl, tile):
        self.expected.append((n, lb, nl, tile))
        return list(range(nl))

    def wait(self, tg, lb, timeout):
        self.waits.append((list(tg), lb))

    def check(self):
        pass


class FakeSender:
    def __init__(self, layout):
        self.layout = FakeLayout(layout)
        self.device = torch.device("cpu")
        self.replicas = 0
        self.connected = []
        self.launches = []
        self.closes = 0

    def connect(self, descs):
        self.connected.append(descs[0].epoch)
        self.replicas = 1

    def push(self, src, dst, lb, nl, tile=128):
        self.launches.append((src.clone(), dst.clone(), lb, nl))

    def close(self):
        self.closes += 1
        self.replicas = 0


def _pair(require=True, reserve_timeout=0.3, blocking=2.0):
    base = dict(chunk_size=64, enable_pd=True, transfer_channel="tcp", pd_buffer_device="cpu",
                pd_buffer_size=1 << 20, local_cpu=False, max_local_cpu_size=0.01,
                pd_peer_init_port=[0], pd_peer_alloc_port=[0], pd_backpressure_reserve=0.0,
                pd_direct_require_reservation=require, pd_reserve_timeout_s=reserve_timeout,
                blocking_timeout_secs=blocking, pd_alloc_fail_backoff_ttl=30.0)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    kv = make_separate_kv(L, NB, BS, H, D, torch.float32, "cpu", seed=1)
    rcfg = LMCacheEngineConfig.from_defaults(pd_role="receiver", **base)
    recv = LMCacheEngine(rcfg, md, VLLMPagedMemGPUConnector(rcfg, kvcaches=zeros_like_kv(kv)))
    recv.post_init()
    pd_r = recv.storage_manager.backends["PDBackend"]
    pd_r.push_receiver = FakeReceiver(recv.gpu_connector.layout)
    iu, au = pd_r.endpoints()
    scfg = LMCacheEngineConfig.from_defaults(pd_role="sender", **base)
    send = LMCacheEngine(scfg, md, VLLMPagedMemGPUConnector(scfg, kvcaches=kv),
                         peer_init_url=iu, peer_alloc_url=au)
    send.post_init()
    pd_s = send.storage_manager.backends["PDBackend"]
    pd_s.push_sender = FakeSender(send.gpu_connector.layout)
    return send, recv, pd_s, pd_r


def _slots(seed, n=40):
    g = torch.Generator().manual_seed(seed)
    return torch.randperm(NB * BS, generator=g)[:n]


def test_granted_push_launches_once_after_the_grant():
    send, recv, pd_s, pd_r = _pair()
    try:
        src, dst = _slots(1), _slots(2)
        recv.reserve_direct_prefill("r1", dst)
        assert send.store_direct_prefill(slot_mapping=src, dst_slot_mapping=dst,
                                         req_id="r1") == 40
        assert len(pd_s.push_sender.launches) == 1
        s, d, lb, nl = pd_s.push_sender.launches[0]
        assert torch.equal(d, dst) and torch.equal(s, src) and (lb, nl) == (0, L)
        assert pd_r.push_receiver.expected == [(40, 0, L, 512)]
        assert recv.direct_prefill_granted("r1")
        assert recv.wait_direct_prefill("r1", timeout_s=1.0)
    finally:
        send.close()
        recv.close()


def test_dead_decoder_no_launch_and_breaker_opens():
    send, recv, pd_s, pd_r = _pair(blocking=0.3)
    dst = _slots(2)
    recv.reserve_direct_prefill("r1", dst)
    recv.close()  # the decoder goes away before the request
    try:
        with pytest.raises((TimeoutError, RuntimeError)):
            send.store_direct_prefill(slot_mapping=_slots(1), dst_slot_mapping=dst, req_id="r1")
        assert pd_s.push_sender.launches == []
        assert pd_s.breaker_open()
        # while the breaker is open the next request fails without a round trip
        with pytest.raises(RuntimeError, match="breaker"):
            send.store_direct_prefill(slot_mapping=_slots(1), dst_slot_mapping=dst,
                                      req_id="r2")
        assert pd_s.push_sender.launches == []
    finally:
        send.close()


def test_stale_epoch_remaps_before_any_launch():
    send, recv, pd_s, pd_r = _pair()
    try:
        src, dst = _slots(1), _slots(2)
        recv.reserve_direct_prefill("r1", dst)
        send.store_direct_prefill(slot_mapping=src, dst_slot_mapping=dst, req_id="r1")
        old = pd_r.push_receiver.desc.epoch
        assert pd_s.push_sender.connected == [old]
        # the decoder re-registers its cache (restart / re-allocation)
        pd_r.push_receiver.new_epoch()
        recv.reserve_direct_prefill("r2", dst)
        send.store_direct_prefill(slot_mapping=src, dst_slot_mapping=dst, req_id="r2")
        # the old mapping was dropped and the new registration mapped BEFORE
        # the second launch
        assert pd_s.push_sender.closes >= 1
        assert pd_s.push_sender.connected[-1] == pd_r.push_receiver.desc.epoch != old
        assert len(pd_s.push_sender.launches) == 2
    finally:
        send.close()
        recv.close()


def test_no_reservation_is_refused_without_launch():
    send, recv, pd_s, pd_r = _pair(reserve_timeout=0.2)
    try:
        with pytest.raises(RuntimeError, match="no reservation"):
            send.store_direct_prefill(slot_mapping=_slots(1), dst_slot_mapping=_slots(2),
                                      req_id="nobody-reserved-this")
        assert pd_s.push_sender.launches == []
        assert pd_s.breaker_open()
    finally:
        send.close()
        recv.close()


def test_other_slots_than_reserved_are_refused_without_launch():
    send, recv, pd_s, pd_r = _pair()
    try:
        recv.reserve_direct_prefill("r1", _slots(2))
        with pytest.raises(RuntimeError, match="differ"):
            send.store_direct_prefill(slot_mapping=_slots(1), dst_slot_mapping=_slots(3),
                                      req_id="r1")
        assert pd_s.push_sender.launches == []
        assert pd_r.push_receiver.expected == []
    finally:
        send.close()
        recv.close()


def test_out_of_range_slots_refused_without_reservation_policy():
    send, recv, pd_s, pd_r = _pair(require=False)
    try:
        bad = _slots(2)
        bad[5] = NB * BS + 3
        with pytest.raises(RuntimeError, match="out of"):
            send.store_direct_prefill(slot_mapping=_slots(1), dst_slot_mapping=bad, req_id="r1")
        assert pd_s.push_sender.launches == []
        send.storage_manager.backends["PDBackend"]._alloc_fail_until = 0.0
        ok = _slots(4)
        send.store_direct_prefill(slot_mapping=_slots(1), dst_slot_mapping=ok, req_id="r2")
        assert len(pd_s.push_sender.launches) == 1
    finally:
        send.close()
        recv.close()


def test_decoder_slots_come_back_in_the_grant_and_chunks_advance():
    """want-slots mode (the connector's path): the prefiller does not know the
    decoder's blocks; each grant returns the next reserved slots, offset by
    the decoder's local prefix (first_token), and the request completes on
    the decoder once every reserved token was granted."""
    send, recv, pd_s, pd_r = _pair()
    try:
        dst = _slots(2, n=30)
        recv.reserve_direct_prefill("r1", dst, first_token=10)  # prompt positions 10..39
        src_all = _slots(1, n=40)                               # prefiller prompt 0..39
        h1 = send.begin_direct_prefill("r1", slot_mapping=src_all[:25], token_begin=0)
        assert h1.num_tokens == 15 and not recv.direct_prefill_granted("r1")
        h2 = send.begin_direct_prefill("r1", slot_mapping=src_all, token_begin=15)
        assert h2.num_tokens == 15 and recv.direct_prefill_granted("r1")
        assert torch.equal(h1.dst.long(), dst[:15]) and torch.equal(h1.src.long(),
                                                                    src_all[10:25])
        assert torch.equal(h2.dst.long(), dst[15:]) and torch.equal(h2.src.long(),
                                                                    src_all[25:40])
        assert pd_s.push_sender.launches == []  # grants only; layers launch later
    finally:
        send.close()
        recv.close()
