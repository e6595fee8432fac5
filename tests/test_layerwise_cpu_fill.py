"""Layerwise CPU fill: page holds and the put window (host-side, CPU)."""

import threading
import time
from concurrent.futures import Future

import pytest
import torch

from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemLayerwiseGPUConnector
from lmcache_ascend_b200.v1.layerwise_cpu_fill import PageHold, PutWindow
from lmcache_ascend_b200.v1.memory_management import TensorMemoryAllocator

from .utils import make_separate_kv, random_slots


def test_page_hold_counts_each_page_once_and_checks_before_counting():
    alloc = TensorMemoryAllocator(torch.empty(1 << 16, dtype=torch.uint8))
    a = alloc.allocate([64], torch.float32)
    b = alloc.allocate([64], torch.float32)
    with PageHold([a, b, a, b, a]) as hold:
        assert hold.num_pages == 2 and a.get_ref_count() == 2 and b.get_ref_count() == 2
        a.ref_count_down()
        b.ref_count_down()  # the producers are done; only the hold keeps them
        assert alloc.num_active == 2
    assert alloc.num_active == 0 and hold.num_pages == 0
    hold.release()  # a second release gives nothing back twice
    assert alloc.num_active == 0
    good = alloc.allocate([64], torch.float32)
    dead = alloc.allocate([64], torch.float32)
    dead.free()
    with pytest.raises(ValueError):
        PageHold([good, dead])
    assert good.get_ref_count() == 1  # nothing was taken before the check failed
    good.ref_count_down()


def _finished(value=None, error=None):
    f = Future()
    if error is not None:
        f.set_exception(error)
    else:
        f.set_result(value)
    return f


def test_window_bounds_bytes_and_batches_with_callbacks():
    w = PutWindow(max_bytes=100, max_batches=2, timeout=2.0)
    slow = Future()
    w.admit(60)
    w.submit(60, [slow], req_id="r1", keys=["k1"])
    w.admit(10)
    w.submit(10, [_finished()], req_id="r2", keys=["k2"])  # done at once: retired
    assert (w.inflight_batches, w.inflight_bytes) == (1, 60)
    threading.Timer(0.1, slow.set_result, args=(None,)).start()
    t0 = time.monotonic()
    w.admit(60)  # 60 + 60 > 100: waits for the callback of r1's future
    assert time.monotonic() - t0 >= 0.05 and w.inflight_batches == 0
    w.admit(10_000)  # an empty window takes any one batch
    w.submit(10_000, [Future(), Future()])
    with pytest.raises(TimeoutError):
        _blocked_admit()


def _blocked_admit():
    w = PutWindow(max_bytes=10, max_batches=1, timeout=0.05)
    w.submit(5, [Future()])
    w.admit(5)


def test_window_errors_are_sticky():
    w = PutWindow(max_bytes=1 << 20, max_batches=8, timeout=1.0)
    w.submit(5, [_finished(error=OSError("disk full"))], req_id="r")
    with pytest.raises(OSError):
        w.check()
    with pytest.raises(OSError):  # every later wait raises it too
        w.admit(1)
    with pytest.raises(OSError):
        w.fence(["anything"])
    w2 = PutWindow(1 << 20, 8, 0.05)
    w2.submit(1, [Future()])
    with pytest.raises(TimeoutError):
        w2.fence_all()
    with pytest.raises(TimeoutError):  # the timeout is latched as well
        w2.check()


def test_request_fences_and_reused_chunks():
    w = PutWindow(max_bytes=1 << 20, max_batches=8, timeout=1.0)
    a_put, b_put = Future(), Future()
    w.submit(1, [a_put], req_id="a", keys=["chunk-a"])
    w.submit(1, [b_put], req_id="b", keys=["chunk-b"])
    w.inherit("c", ["chunk-a"])  # c reuses a's chunk
    threading.Timer(0.05, a_put.set_result, args=(None,)).start()
    w.fence(["c"])  # covers a's put, not b's
    assert a_put.done() and not b_put.done()
    b_put.set_result(None)
    w.fence_all()
    assert w.inflight_batches == 0


def test_engine_store_layer_puts_go_through_the_window(tmp_path):
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
    assert eng.layerwise_put_queue.inflight_batches == 0
    assert eng.lookup(tokens) == 128
    eng.close()
