"""Multiprocess mode: a cache-server process serving two workers' paged KV
caches by IPC handle (shared-memory host caches on CPU, CUDA IPC on GPU);
a prefix stored by one worker is a hit for the other."""

import multiprocessing as mp
import socket
import time

import pytest
import torch

from lmcache_ascend_b200.v1.multiprocess.server import MPCacheClient

from .utils import make_separate_kv, random_slots

L, NB, BS, H, D = 2, 32, 16, 2, 32


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _server(port):
    from lmcache_ascend_b200.v1.multiprocess.server import run_cache_server

    run_cache_server("127.0.0.1", port, chunk_size=64, cpu_buffer_size=0.05)


def _wait(url):
    c = MPCacheClient(url, "probe", timeout_ms=1000)
    for _ in range(120):
        try:
            c._rpc("ping")
            c.close(unregister=False)
            return
        except TimeoutError:
            c.close(unregister=False)
            c = MPCacheClient(url, "probe", timeout_ms=1000)
    raise RuntimeError("cache server did not start")


def _run(device):
    port = _free_port()
    ctx = mp.get_context("spawn")
    proc = ctx.Process(target=_server, args=(port,), daemon=True)
    proc.start()
    url = f"tcp://127.0.0.1:{port}"
    a = b = None
    try:
        _wait(url)
        src = make_separate_kv(L, NB, BS, H, D, torch.float32, device, seed=1)
        dst = [tuple(torch.zeros_like(t) for t in layer) for layer in src]
        if device == "cpu":
            for layer in src + dst:
                for t in layer:
                    t.share_memory_()
        a = MPCacheClient(url, "worker-a")
        b = MPCacheClient(url, "worker-b")
        assert a.register_kv_caches(src) == L and b.register_kv_caches(dst) == L
        tokens = torch.arange(192)
        s_a = random_slots(192, NB * BS, seed=2)
        s_b = random_slots(192, NB * BS, seed=3)
        assert b.lookup(tokens) == 0
        a.store(tokens, s_a)
        assert b.lookup(tokens) == 192  # shared tier
        assert b.retrieve(tokens, s_b) == 192
        if device == "cuda":
            torch.cuda.synchronize()
        for l in range(L):
            for p in range(2):
                want = src[l][p].reshape(NB * BS, -1)[s_a.to(device)]
                got = dst[l][p].reshape(NB * BS, -1)[s_b.to(device)]
                assert torch.equal(want, got)
        with pytest.raises(RuntimeError):
            MPCacheClient(url, "never-registered").lookup(tokens)
    finally:
        for c in (a, b):
            if c is not None:
                c.close()
        proc.terminate()
        proc.join(timeout=10)


def test_cache_server_shares_prefix_between_workers_cpu():
    _run("cpu")


@pytest.mark.gpu
def test_cache_server_shares_prefix_between_workers_cuda():
    _run("cuda")
