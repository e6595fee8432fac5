"""Time to first token on a prefix hit, through the engine's public API.

A request is a prompt whose first ``tokens`` tokens were stored earlier by
another request (in the CPU tier) plus one new token.  TTFT is the wall time
from the request's arrival to the first generated token id on the host:

  LMCacheEngine.lookup (scheduler side)
  -> LMCacheEngine.retrieve_layer: layer l of every hit chunk moves from the
     pinned CPU tier into fresh paged blocks (one kernel launch per layer on
     the load stream) while the model computes layer l - 1
  -> the model's forward of the new token over the cached context, layer by
     layer (each layer waits only for its own load)
  -> lm_head + argmax and the device-to-host read of the token id.

The model is random-init (no checkpoints here) with the real architecture,
built on the GPU directly; KV is random bf16 of the model's shape.

``python -m lmcache_ascend_b200.bench_ttft --tokens 16384 --requests 8``
"""

from __future__ import annotations

import argparse
import json
import time
from typing import Dict, Optional

import torch

from .config import LMCacheEngineConfig, LMCacheEngineMetadata
from .models.llama import LlamaConfig, LlamaForBlend


def _block_slots(T: int, bs: int, blocks: torch.Tensor) -> torch.Tensor:
    t = torch.arange(T)
    return (blocks[t // bs] * bs + t % bs).long()


@torch.no_grad()
def run_ttft(device, tokens: int = 16384, requests: int = 8, warmup: int = 2,
             model_config: Optional[LlamaConfig] = None, chunk_size: int = 256,
             block_size: int = 128, dtype=torch.bfloat16, seed: int = 0,
             transfer_mode: str = "copy_engine", numa_node: int = -2,
             tier: str = "cpu") -> Dict:
    """``tier``: "cpu" keeps the stored prefix in the pinned CPU tier (the
    hit crosses the host link); "hbm" keeps it in the HBM tier (the hit is a
    device-to-device scatter)."""
    from .v1.cache_engine import LMCacheEngine
    from .v1.gpu_connector import VLLMPagedMemLayerwiseGPUConnector

    dev = torch.device(device)
    mc = model_config or LlamaConfig.qwen3_32b()
    t_build = time.perf_counter()
    model = LlamaForBlend(mc, dev, dtype, seed=seed, lm_head=True)
    L, KH, D, BS = mc.num_layers, mc.num_kv_heads, mc.head_dim, block_size
    per_req_blocks = (tokens + 1 + BS - 1) // BS
    nb = 2 * per_req_blocks  # one block table to seed the cache, one per request
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    kv = [(torch.randn(nb, BS, KH, D, device=dev, dtype=dtype, generator=g),
           torch.randn(nb, BS, KH, D, device=dev, dtype=dtype, generator=g)) for _ in range(L)]
    kv_bytes = tokens * L * 2 * KH * D * torch.empty((), dtype=dtype).element_size()
    hbm = tier == "hbm"
    cfg = LMCacheEngineConfig.from_defaults(
        chunk_size=chunk_size, use_layerwise=True, local_cpu=True,
        max_local_cpu_size=(0.05 if hbm else kv_bytes * 1.05 / (1 << 30) + 0.05),
        save_unfull_chunk=True, local_gpu=hbm,
        max_local_gpu_size=(kv_bytes * 1.05 / (1 << 30) + 0.05) if hbm else 0.0,
        cpu_transfer_mode=transfer_mode, numa_node=numa_node if dev.type == "cuda" else -1)
    md = LMCacheEngineMetadata("Qwen3-32B" if mc.num_layers == 64 else "model", 1, 0, "vllm",
                               dtype)
    conn = VLLMPagedMemLayerwiseGPUConnector(cfg, kvcaches=kv)
    eng = LMCacheEngine(cfg, md, conn)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    build_s = time.perf_counter() - t_build

    cpu = torch.Generator().manual_seed(seed + 2)
    perm = torch.randperm(nb, generator=cpu)
    store_slots = _block_slots(tokens, BS, perm[:per_req_blocks]).to(dev)
    load_table = perm[per_req_blocks:]
    load_slots = _block_slots(tokens + 1, BS, load_table).to(dev)
    prompt = torch.randint(0, mc.vocab_size, (tokens + 1,), generator=cpu)
    prefix = prompt[:tokens]
    # an earlier request computed and stored the prefix
    for _ in eng.store_layer(prefix, slot_mapping=store_slots):
        pass
    want0 = kv[0][0].view(-1, KH * D)[store_slots[:chunk_size]].clone()
    wantL = kv[L - 1][1].view(-1, KH * D)[store_slots[-chunk_size:]].clone()

    times, dev_ms, hits, first_ok = [], [], [], None
    phases = {"lookup_ms": [], "fetch_ms": [], "enqueue_ms": [], "drain_ms": []}
    for r in range(warmup + requests):
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True) if dev.type == "cuda" else None
        e1 = torch.cuda.Event(enable_timing=True) if dev.type == "cuda" else None
        t0 = time.perf_counter()
        if e0 is not None:
            e0.record()
        hit = eng.lookup(prefix)                                     # scheduler
        ta = time.perf_counter()
        gen = eng.retrieve_layer(prefix, slot_mapping=load_slots[:tokens])  # worker
        next(gen)
        tb = time.perf_counter()
        tok = model.decode_step(prompt[tokens:], tokens, kv, load_slots[:tokens],
                                load_slots[tokens:tokens + 1],
                                before_layer=lambda l: next(gen))
        ret = next(gen)
        tc = time.perf_counter()
        if e1 is not None:
            e1.record()
        token_id = int(tok.item())                                   # device -> host
        t1 = time.perf_counter()
        if r == 0:
            got0 = kv[0][0].view(-1, KH * D)[load_slots[:chunk_size]]
            gotL = kv[L - 1][1].view(-1, KH * D)[load_slots[tokens - chunk_size:tokens]]
            first_ok = bool(torch.equal(got0, want0) and torch.equal(gotL, wantL)
                            and int(ret.sum()) == tokens)
        if r >= warmup:
            times.append((t1 - t0) * 1e3)
            for k, v in (("lookup_ms", ta - t0), ("fetch_ms", tb - ta), ("enqueue_ms", tc - tb),
                         ("drain_ms", t1 - tc)):
                phases[k].append(v * 1e3)
            hits.append(hit)
            if e0 is not None:
                dev_ms.append(e0.elapsed_time(e1))
        del token_id
    # the same token's forward with the context already resident (no load):
    # the part of TTFT that belongs to the model, not to the cache
    fwd = []
    for r in range(warmup + requests):
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        tok = model.decode_step(prompt[tokens:], tokens, kv, load_slots[:tokens],
                                load_slots[tokens:tokens + 1])
        int(tok.item())
        if r >= warmup:
            fwd.append((time.perf_counter() - t0) * 1e3)
    eng.close()
    times.sort()
    p = lambda q: times[min(len(times) - 1, int(q * (len(times) - 1) + 0.5))]
    res = {"p50_ms": round(p(0.5), 3), "p90_ms": round(p(0.9), 3),
           "min_ms": round(times[0], 3), "requests": requests, "warmup": warmup,
           "prefix_hit_tokens": int(min(hits)) if hits else 0, "new_tokens": 1,
           "kv_bytes": kv_bytes, "kv_load_gbps_at_p50": round(kv_bytes / p(0.5) / 1e6, 2),
           "device_span_p50_ms": round(sorted(dev_ms)[len(dev_ms) // 2], 3) if dev_ms else None,
           "forward_only_p50_ms": round(sorted(fwd)[len(fwd) // 2], 3),
           "kv_check": first_ok, "setup_s": round(build_s, 2), "transfer_mode": transfer_mode,
           "numa_node": numa_node,
           "phases_p50_ms": {k: round(sorted(v)[len(v) // 2], 3) for k, v in phases.items() if v},
           "model": f"{md.model_name} (random init, TP1: {L} layers, {mc.num_heads} heads, "
                    f"{KH} KV heads)",
           "tier": tier,
           "path": ("lookup + layerwise " + ("HBM-tier device->paged" if hbm else "CPU->GPU")
                    + " retrieve overlapped with the new token's forward + lm_head argmax "
                      "+ D2H")}
    del model, kv, conn, eng
    if dev.type == "cuda":
        torch.cuda.empty_cache()
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--requests", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--mode", default="copy_engine", choices=["copy_engine", "zero_copy"])
    ap.add_argument("--numa", type=int, default=-2, help="-2 auto, -1 none, >= 0 node")
    ap.add_argument("--tier", default="cpu", choices=["cpu", "hbm"])
    a = ap.parse_args()
    print(json.dumps(run_ttft("cuda", a.tokens, a.requests, a.warmup, transfer_mode=a.mode,
                              numa_node=a.numa, tier=a.tier)), flush=True)


if __name__ == "__main__":
    main()
