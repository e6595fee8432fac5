"""Layerwise CPU-fill lease and the bounded put queue (host-side, CPU)."""

import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemLayerwiseGPUConnector
from lmcache_ascend_b200.v1.layerwise_cpu_fill import CPUFillLease, LayerwisePutQueue
from lmcache_ascend_b200.v1.memory_management import TensorMemoryAllocator

from .utils import make_separate_kv, random_slots


def test_lease_holds_pages_once_and_releases_once():
    alloc = TensorMemoryAllocator(torch.empty(1 << 16, dtype=torch.uint8))
    a = alloc.allocate([64], torch.float32)
    b = alloc.allocate([64], torch.float32)
    lease = CPUFillLease([a, b, a])
    assert lease.num_pages == 2 and a.get_ref_count() == 2
    a.ref_count_down()
    b.ref_count_down()  # the producers drop theirs; the lease keeps the pages
    assert alloc.num_active == 2
    lease.release()
    lease.release()
    assert alloc.num_active == 0
    c = alloc.allocate([64], torch.float32)
    c.free()
    with pytest.raises(ValueError):
        CPUFillLease([c])


def _done(v=None):
    f = Future()
    f.set_result(v)
    return f


def test_put_queue_admission_reaping_and_sticky_errors():
    q = LayerwisePutQueue(max_bytes=100, max_batches=2, timeout=0.5)
    slow = Future()
    q.reserve(60)
    q.add(60, [slow], req_id="r1", keys=["k1"])
    q.add(10, [_done()], req_id="r2", keys=["k2"])
    q.poll()  # r2 finished out of order: reaped, r1 still charged
    assert len(q.pending) == 1 and q.pending_bytes == 60
    threading.Timer(0.1, slow.set_result, args=(None,)).start()
    t0 = time.monotonic()
    q.reserve(60)  # 60 + 60 > 100: waits for r1
    assert time.monotonic() - t0 >= 0.05 and not q.pending
    q.reserve(500)  # oversized batch admitted into an empty queue
    bad = Future()
    bad.set_exception(RuntimeError("disk full"))
    q.add(5, [bad])
    with pytest.raises(RuntimeError):
        q.poll()
    with pytest.raises(RuntimeError):  # sticky
        q.reserve(1)


def test_put_queue_request_fences_and_timeout():
    q = LayerwisePutQueue(max_bytes=1 << 20, max_batches=8, timeout=0.2)
    slow, other = Future(), Future()
    q.add(1, [slow], req_id="a", keys=["k"])
    q.add(1, [other], req_id="b", keys=["z"])
    q.track_keys("c", ["k"])  # c reuses a's chunk: fenced together
    threading.Timer(0.05, slow.set_result, args=(None,)).start()
    q.drain_requests(["c"])  # does not wait for b
    assert not other.done()
    with pytest.raises(TimeoutError):
        q.drain()


def test_engine_store_layer_puts_go_through_the_queue(tmp_path):
    L, NB, BS = 3, 32, 16
    kv = make_separate_kv(L, NB, BS, 2, 32, torch.float32, "cpu", seed=1)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02,
                                            use_layerwise=True, local_disk=str(tmp_path),
                                            max_local_disk_size=0.05,
                                            layerwise_put_max_batches=1)
    md = LMCacheEngineMetadata("m", 1, 0, "vllm", torch.float32)
    eng = LMCacheEngine(cfg, md, VLLMPagedMemLayerwiseGPUConnector(cfg, kvcaches=kv))
    tokens = torch.arange(128)
    for _ in eng.store_layer(tokens, slot_mapping=random_slots(128, NB * BS, seed=2),
                             req_id="r"):
        pass
    eng.wait_layerwise_puts(["r"])
    assert not eng.layerwise_put_queue.pending
    assert eng.lookup(tokens) == 128
    eng.close()
