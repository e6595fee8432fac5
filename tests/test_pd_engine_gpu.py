"""PD through the engine API on one GPU: device page pools moved by the
NVLink channel (gather kernel into pool pages, SIMT page copy, scatter on
retrieve), and the direct paged push (store_direct_prefill /
wait_direct_prefill).  Sender and receiver engines live in one process;
the control plane is ZMQ on loopback."""

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

from .utils import block_slots, make_separate_kv, zeros_like_kv

pytestmark = pytest.mark.gpu
L, NB, BS, H, D = 4, 32, 128, 2, 128


def _pair():
    base = dict(chunk_size=256, enable_pd=True, transfer_channel="nvlink",
                pd_buffer_device="cuda", pd_buffer_size=64 << 20, max_local_cpu_size=0.01,
                local_cpu=False, pd_peer_init_port=[0], pd_peer_alloc_port=[0],
                pd_backpressure_reserve=0.0)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.bfloat16)
    kv_r = zeros_like_kv(make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=1))
    rcfg = LMCacheEngineConfig.from_defaults(pd_role="receiver", **base)
    recv = LMCacheEngine(rcfg, md, VLLMPagedMemGPUConnector(rcfg, kvcaches=kv_r))
    recv.post_init()
    iu, au = recv.storage_manager.backends["PDBackend"].endpoints()
    kv_s = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, "cuda", seed=2)
    scfg = LMCacheEngineConfig.from_defaults(pd_role="sender", **base)
    send = LMCacheEngine(scfg, md, VLLMPagedMemGPUConnector(scfg, kvcaches=kv_s),
                         peer_init_url=iu, peer_alloc_url=au)
    send.post_init()
    return send, recv, kv_s, kv_r


def _rows(kv, slots):
    return [t.view(NB * BS, -1)[slots.long()] for layer in kv for t in layer]


def test_pd_pool_push_and_retrieve():
    send, recv, kv_s, kv_r = _pair()
    try:
        T = 700
        tokens = torch.arange(T)
        ss = block_slots(T, BS, NB, seed=3, device="cuda")
        send.store(tokens, slot_mapping=ss)
        assert recv.lookup(tokens) == T
        rs = block_slots(T, BS, NB, seed=4, device="cuda")
        ret = recv.retrieve(tokens, slot_mapping=rs)
        torch.cuda.synchronize()
        assert bool(ret.all())
        for a, b in zip(_rows(kv_s, ss), _rows(kv_r, rs)):
            assert torch.equal(a, b)
        pd_r = recv.storage_manager.backends["PDBackend"]
        assert pd_r.allocator.num_free == pd_r.allocator.num_pages  # pages returned
    finally:
        send.close()
        recv.close()


def test_direct_prefill_push_engine_api():
    send, recv, kv_s, kv_r = _pair()
    try:
        T = 1000
        ss = block_slots(T, BS, NB, seed=5, device="cuda", dtype=torch.int32)
        rs = block_slots(T, BS, NB, seed=6, device="cuda", dtype=torch.int32)
        for layer in range(L):  # layer by layer, as during prefill
            recv.reserve_direct_prefill(f"req-{layer}", rs.cpu())  # the decoder's allocation
            send.store_direct_prefill(slot_mapping=ss, dst_slot_mapping=rs,
                                      req_id=f"req-{layer}", layer_begin=layer, num_layers=1)
            assert recv.wait_direct_prefill(f"req-{layer}", timeout_s=5.0)
        torch.cuda.synchronize()
        recv.storage_manager.backends["PDBackend"].push_receiver.check()
        for a, b in zip(_rows(kv_s, ss), _rows(kv_r, rs)):
            assert torch.equal(a, b)
    finally:
        send.close()
        recv.close()
