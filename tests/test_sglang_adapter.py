"""SGLang connector on the CPU tier: token pools (page size 1), store then
load into other pool slots, radix-cache offset, layerwise loading, and the
TP min-agreement over two gloo ranks."""

import os

import torch
import torch.multiprocessing as mp

from lmcache_ascend_b200.config import LMCacheEngineConfig
from lmcache_ascend_b200.integration.sglang.adapter import (
    LMCacheSGLangConnector,
    LoadMetadata,
    StoreMetadata,
)

L, POOL, H, D = 2, 1024, 2, 16


def _pools(seed):
    g = torch.Generator().manual_seed(seed)
    return ([torch.randn(POOL, H, D, generator=g) for _ in range(L)],
            [torch.randn(POOL, H, D, generator=g) for _ in range(L)])


def _conn(layerwise=False, **kw):
    k, v = _pools(1)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02, **kw)
    return LMCacheSGLangConnector("m", 1, 0, k, v, cfg, layerwise=layerwise), k, v


def test_store_and_load_with_offset():
    for layerwise in (False, True):
        c, k, v = _conn(layerwise)
        toks = list(range(200))
        perm = torch.randperm(POOL)
        src, dst = perm[:200], perm[200:400]
        c.store_kv(StoreMetadata(toks, src))
        for t in k + v:
            t[dst] = 0
        n = c.start_load_kv(LoadMetadata(toks, dst, offset=64))
        if layerwise:
            for layer in range(L):
                c.load_kv_layerwise(layer)
        assert n == 200 - 64
        for a in k + v:
            assert torch.equal(a[dst[64:]], a[src[64:]])  # loaded past the offset
            assert int(a[dst[:64]].abs().sum()) == 0       # radix cache part untouched
        assert c.start_load_kv(LoadMetadata(list(range(5000, 5100)), dst, 0)) == 0
        c.close()


def _tp_worker(rank, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    k, v = _pools(rank)
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=64, max_local_cpu_size=0.02)
    c = LMCacheSGLangConnector("m", 2, rank, k, v, cfg, tp_group=dist.group.WORLD)
    toks = list(range(256))
    n_store = 256 if rank == 0 else 128  # rank 1 cached less of the prompt
    c.store_kv(StoreMetadata(toks[:n_store], torch.arange(n_store)))
    got = c.start_load_kv(LoadMetadata(toks, torch.arange(256, 512), 0))
    q.put((rank, got))
    c.close()
    dist.destroy_process_group()


def test_tp_min_agreement():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    ps = [ctx.Process(target=_tp_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(60)
    assert res == {0: 128, 1: 128}  # both ranks load the common prefix only
