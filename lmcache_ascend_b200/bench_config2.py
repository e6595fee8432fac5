"""Local offload, one engine per data-parallel replica (one per GPU).

Llama-3-8B-shaped paged KV (32 layers, 8 KV heads, head_dim 128, block 16,
bf16, random N(0, 1)); 64 requests of 8192 tokens per replica, the first
half of every prompt shared by all requests (and replicas), the second half
random per request; chunk 256.  Request i is stored from one block table
(only its chunks not cached yet move: all 8192 tokens for the first request,
the 4096-token suffix after that) and then retrieved on a hit into another
block table, through the engine's public API into the pinned CPU tier and
back.  Reported per replica: store and retrieve GB/s (bytes moved / wall
time of the calls, bracketed by device synchronisation), the p50 retrieve
time, and TTFT on a hit (Llama-3-8B, 8192-token prefix, one new token) from
``bench_ttft``; aggregates over replicas and max over ranks for times.
"""

from __future__ import annotations

import statistics
import time

import torch

L, KH, D, BS = 32, 8, 128, 16


def run_config2(dev, rank: int, world: int, gloo=None, requests: int = 64,
                tokens: int = 8192, shared: float = 0.5, chunk: int = 256,
                ttft_requests: int = 5) -> dict:
    import torch.distributed as dist

    from .bench_ttft import run_ttft
    from .config import LMCacheEngineConfig, LMCacheEngineMetadata
    from .models.llama import LlamaConfig
    from .v1.cache_engine import LMCacheEngine
    from .v1.gpu_connector import VLLMPagedMemGPUConnector

    per_req_blocks = tokens // BS
    nb = 2 * per_req_blocks
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    kv = [(torch.randn(nb, BS, KH, D, device=dev, dtype=torch.bfloat16, generator=g),
           torch.randn(nb, BS, KH, D, device=dev, dtype=torch.bfloat16, generator=g))
          for _ in range(L)]
    tok_bytes = L * 2 * KH * D * 2
    cfg = LMCacheEngineConfig.from_defaults(chunk_size=chunk, local_cpu=True,
                                            max_local_cpu_size=3.5, save_unfull_chunk=True)
    md = LMCacheEngineMetadata("Llama-3-8B", 1, 0, "vllm", torch.bfloat16)
    eng = LMCacheEngine(cfg, md, VLLMPagedMemGPUConnector(cfg, kvcaches=kv))
    cpu = torch.Generator().manual_seed(7)
    perm = torch.randperm(nb, generator=cpu)
    t = torch.arange(tokens)
    store_slots = (perm[:per_req_blocks][t // BS] * BS + t % BS).to(dev)
    load_slots = (perm[per_req_blocks:][t // BS] * BS + t % BS).to(dev)
    n_shared = int(tokens * shared)
    prefix = torch.randint(0, 128000, (n_shared,), generator=cpu)  # same on every replica
    own = torch.Generator().manual_seed(1000 + rank)
    st_ms, rt_ms, stored_bytes, ok = [], [], 0, True
    for i in range(requests):
        suffix = torch.randint(0, 128000, (tokens - n_shared,), generator=own)
        toks = torch.cat([prefix, suffix])
        before = eng.lookup(toks)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        eng.store(toks, slot_mapping=store_slots)
        torch.cuda.synchronize(dev)
        st_ms.append((time.perf_counter() - t0) * 1e3)
        stored_bytes += (tokens - before) * tok_bytes
        t0 = time.perf_counter()
        ret = eng.retrieve(toks, slot_mapping=load_slots)
        torch.cuda.synchronize(dev)
        rt_ms.append((time.perf_counter() - t0) * 1e3)
        if i == 0:
            ok = bool(ret.all()) and all(
                torch.equal(a.view(-1, KH * D)[store_slots.long()],
                            a.view(-1, KH * D)[load_slots.long()])
                for layer in kv for a in layer)
        elif not bool(ret.all()):
            ok = False
    eng.close()
    del kv, eng
    torch.cuda.empty_cache()
    store_s, load_s = sum(st_ms) / 1e3, sum(rt_ms) / 1e3
    mine = {"store_gbps": stored_bytes / store_s / 1e9,
            "retrieve_gbps": requests * tokens * tok_bytes / load_s / 1e9,
            "retrieve_p50_ms": statistics.median(rt_ms)}
    ttft = run_ttft(dev, tokens=tokens, requests=ttft_requests, warmup=2,
                    model_config=LlamaConfig.llama3_8b(), block_size=BS)
    mine["ttft_p50_ms"] = ttft["p50_ms"]
    vals = torch.tensor([mine["store_gbps"], mine["retrieve_gbps"], mine["retrieve_p50_ms"],
                         mine["ttft_p50_ms"], float(ok)], device=dev, dtype=torch.float64)
    if world > 1:
        allv = [torch.zeros_like(vals) for _ in range(world)]
        dist.all_gather(allv, vals)
        allv = torch.stack(allv).cpu()
    else:
        allv = vals.cpu().unsqueeze(0)
    return {"replicas": world, "requests_per_replica": requests, "tokens": tokens,
            "shared_prefix_tokens": n_shared, "chunk": chunk,
            "store_gbps_aggregate": round(float(allv[:, 0].sum()), 2),
            "retrieve_gbps_aggregate": round(float(allv[:, 1].sum()), 2),
            "store_gbps_min_replica": round(float(allv[:, 0].min()), 2),
            "retrieve_gbps_min_replica": round(float(allv[:, 1].min()), 2),
            "retrieve_p50_ms_max_over_ranks": round(float(allv[:, 2].max()), 3),
            "ttft_p50_ms_max_over_ranks": round(float(allv[:, 3].max()), 3),
            "kv_check": bool(allv[:, 4].min() > 0),
            "timing": "wall time of each store / retrieve call, device synchronised "
                      "before and after",
            "tier": "pinned CPU tier (copy-engine staging)",
            "model": "Llama-3-8B KV shape (32 layers, 8 KV heads, head_dim 128, block 16), "
                     "random init; TTFT with a random-init Llama-3-8B"}
