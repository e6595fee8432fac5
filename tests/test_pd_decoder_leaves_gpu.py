"""The decoder leaves between two requests (2 GPUs, one process per GPU).

Request 1 is pushed from the prefiller (cuda:0) into the decoder's paged cache
(cuda:1) over NVLink and checked byte for byte.  Then the decoder closes its
engine and its process exits, with none of its kernels in flight.  Request 2
must fail on the control plane (the decoder's grant never comes) with no push
launched, and open the per-peer breaker; request 3 then fails at once on the
breaker.  The failure is made on the host (a process that exits); nothing
faults or hangs a GPU.  NVLink multicast is not used (NVLS off).
"""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

L, NB, BS, H, D = 4, 32, 128, 2, 128
T = 1000


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _base(iport, aport):
    return dict(chunk_size=256, enable_pd=True, transfer_channel="nvlink",
                pd_buffer_device="cuda", pd_buffer_size=16 << 20, max_local_cpu_size=0.01,
                local_cpu=False, pd_peer_init_port=[iport], pd_peer_alloc_port=[aport],
                pd_backpressure_reserve=0.0, blocking_timeout_secs=1.0,
                pd_reserve_timeout_s=1.0, pd_alloc_fail_backoff_ttl=30.0)


def _decoder(iport, aport, q, go):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
        from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
        from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector
        from tests.utils import block_slots, make_separate_kv, zeros_like_kv

        dev = torch.device("cuda", 1)
        torch.cuda.set_device(dev)
        md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.bfloat16)
        kv = zeros_like_kv(make_separate_kv(L, NB, BS, H, D, torch.bfloat16, dev, seed=1))
        cfg = LMCacheEngineConfig.from_defaults(pd_role="receiver", **_base(iport, aport))
        eng = LMCacheEngine(cfg, md, VLLMPagedMemGPUConnector(cfg, kvcaches=kv))
        eng.post_init()
        rs = block_slots(T, BS, NB, seed=6, device=dev, dtype=torch.int32)
        eng.reserve_direct_prefill("r1", rs.cpu())
        q.put(("ready", None))
        assert eng.wait_direct_prefill("r1", timeout_s=20.0, sync=True)
        torch.cuda.synchronize(dev)
        rows = [t.view(NB * BS, -1)[rs.long()].cpu() for layer in kv for t in layer]
        q.put(("rows", rows))
        go.get(timeout=120)  # the prefiller has what it needs: leave between requests
        eng.close()
        torch.cuda.synchronize(dev)
        q.put(("left", None))
    except Exception:
        q.put(("error", traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_decoder_leaves_between_requests_no_launch_and_breaker():
    from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
    from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
    from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

    from .utils import block_slots, make_separate_kv

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q, go = ctx.Queue(), ctx.Queue()
    iport, aport = _port(), _port()
    p = ctx.Process(target=_decoder, args=(iport, aport, q, go))
    p.start()
    send = None
    try:
        tag, msg = q.get(timeout=180)
        assert tag == "ready", msg
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.bfloat16)
        kv = make_separate_kv(L, NB, BS, H, D, torch.bfloat16, dev, seed=2)
        cfg = LMCacheEngineConfig.from_defaults(pd_role="sender", **_base(0, 0))
        send = LMCacheEngine(cfg, md, VLLMPagedMemGPUConnector(cfg, kvcaches=kv),
                             peer_init_url=f"tcp://127.0.0.1:{iport}",
                             peer_alloc_url=f"tcp://127.0.0.1:{aport}")
        send.post_init()
        ss = block_slots(T, BS, NB, seed=5, device=dev, dtype=torch.int32)
        rs = block_slots(T, BS, NB, seed=6, device=dev, dtype=torch.int32)
        assert send.store_direct_prefill(slot_mapping=ss, dst_slot_mapping=rs,
                                         req_id="r1") == T
        torch.cuda.synchronize(dev)
        tag, rows = q.get(timeout=120)
        assert tag == "rows", rows
        want = [t.view(NB * BS, -1)[ss.long()].cpu() for layer in kv for t in layer]
        for a, b in zip(want, rows):
            assert torch.equal(a, b)

        pd = send.storage_manager.backends["PDBackend"]
        launches = []
        real_push = pd.push_sender.push
        pd.push_sender.push = lambda *a, **k: (launches.append(a), real_push(*a, **k))
        go.put("leave")
        tag, msg = q.get(timeout=120)
        assert tag == "left", msg
        p.join(timeout=60)
        assert not p.is_alive()

        with pytest.raises((TimeoutError, RuntimeError)):
            send.store_direct_prefill(slot_mapping=ss, dst_slot_mapping=rs, req_id="r2")
        assert launches == []
        assert pd.breaker_open()
        with pytest.raises(RuntimeError, match="breaker"):
            send.store_direct_prefill(slot_mapping=ss, dst_slot_mapping=rs, req_id="r3")
        assert launches == []
        torch.cuda.synchronize(dev)  # the prefiller's context is intact
    finally:
        if send is not None:
            send.close()
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
