"""Per-kernel microbenchmarks (device-timed with CUDA events).

``python -m lmcache_ascend_b200.bench_kernels [--only NAME] [--small]``
prints one JSON line per case with GB/s and the fraction of the measured HBM
copy bandwidth (``MEASURED_PEAKS.json`` at the repo root when present).

Cases (BASELINE shapes):
* ``gather`` / ``scatter``: K1 paged <-> chunk, Llama-3-8B KV (32 layers,
  8 KV heads, head_dim 128, block 16, bf16), 8192 tokens per launch, TMA and
  SIMT engines, device chunks (multi-chunk pointer table, chunk 256).
* ``offload_store`` / ``offload_load``: the connector's store/retrieve of the
  same request to/from pinned host chunks (copy-engine pipeline and
  zero-copy kernel).
* ``cachegen``: CDF + encode + decode of a Llama-3-8B 256-token chunk.
* ``rope``: K re-rotation, 8192 tokens x 8 heads x 128.
* ``push_loopback``: K9 on one GPU (Qwen3-32B TP4 shard, 16k tokens).
"""

from __future__ import annotations

import argparse
import json
import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peak_hbm() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return 6650.0  # fallback figure of this pool


def _time(fn, iters=10, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _emit(name, ms, moved_bytes, traffic_bytes=None, **extra):
    hbm = _peak_hbm()
    traffic = traffic_bytes if traffic_bytes is not None else 2 * moved_bytes
    d = {"case": name, "ms": round(ms, 4), "payload_GBps": round(moved_bytes / ms / 1e6, 1),
         "hbm_traffic_GBps": round(traffic / ms / 1e6, 1),
         "frac_of_measured_hbm": round(traffic / ms / 1e6 / hbm, 3)}
    d.update(extra)
    print(json.dumps(d), flush=True)


def _llama_cache(T, dev, L=32, H=8, D=128, BS=16):
    nb = 2 * ((T + BS - 1) // BS)
    kv = [(torch.randn(nb, BS, H, D, device=dev, dtype=torch.bfloat16),
           torch.randn(nb, BS, H, D, device=dev, dtype=torch.bfloat16)) for _ in range(L)]
    g = torch.Generator().manual_seed(0)
    blocks = torch.randperm(nb, generator=g)[: (T + BS - 1) // BS]
    t = torch.arange(T)
    slots = (blocks[t // BS] * BS + t % BS).to(dev)
    return kv, slots


def bench_gather_scatter(small: bool):
    from . import ops
    from .v1.kv_format import PagedKVLayout

    dev = torch.device("cuda")
    T = 2048 if small else 8192
    kv, slots = _llama_cache(T, dev)
    lay = PagedKVLayout(kv)
    cs = 256
    n = (T + cs - 1) // cs
    chunks = [torch.empty(lay.chunk_shape(cs), dtype=torch.bfloat16, device=dev) for _ in range(n)]
    ptrs = torch.tensor([c.data_ptr() for c in chunks], dtype=torch.int64, device=dev)
    moved = lay.chunk_bytes(T)
    mod = ops.native()
    for mode, name in ((1, "tma"), (2, "simt")):
        for to_chunk, case in ((True, "gather"), (False, "scatter")):
            def fn():
                mod.kv_transfer(lay.native(), None, ptrs, lay.chunk_native(), 0, 0, cs, True,
                                slots, 0, 0, lay.num_layers, to_chunk, mode, None, None, 0, None)
            _emit(f"{case}_{name}", _time(fn), moved, tokens=T, layers=32)


def bench_offload(small: bool):
    from .config import LMCacheEngineConfig
    from .v1.gpu_connector import VLLMPagedMemGPUConnector
    from .v1.memory_management import MemoryFormat, PinnedMemoryAllocator

    dev = torch.device("cuda")
    T = 2048 if small else 8192
    kv, slots = _llama_cache(T, dev)
    cs = 256
    for mode in ("copy_engine", "zero_copy"):
        cfg = LMCacheEngineConfig.from_defaults(chunk_size=cs, cpu_transfer_mode=mode)
        conn = VLLMPagedMemGPUConnector(cfg, kvcaches=kv)
        alloc = PinnedMemoryAllocator(conn.chunk_bytes(T) + (1 << 20))
        starts = list(range(0, T, cs))
        ends = [min(s + cs, T) for s in starts]
        objs = [alloc.allocate(conn.get_shape(e - s), torch.bfloat16, MemoryFormat.KV_2LTD)
                for s, e in zip(starts, ends)]
        moved = conn.chunk_bytes(T)
        ms = _time(lambda: conn.batched_from_gpu(objs, starts, ends, slot_mapping=slots), 5, 2)
        _emit(f"offload_store_{mode}", ms, moved, traffic_bytes=moved, tokens=T,
              note="bound: host link (PCIe) bandwidth")
        ms = _time(lambda: conn.batched_to_gpu(objs, starts, ends, slot_mapping=slots), 5, 2)
        _emit(f"offload_load_{mode}", ms, moved, traffic_bytes=moved, tokens=T,
              note="bound: host link (PCIe) bandwidth")
        for o in objs:
            o.ref_count_down()
        alloc.close()


def bench_cachegen(small: bool):
    from . import ops

    mod = ops.native()
    L, T, C = 64, 256, 1024  # K and V of 32 layers stacked, 8 heads x 128
    bins = 32
    sym = (torch.randn(L, T, C, device="cuda") * 4 + 16).clamp(0, bins - 1).to(torch.uint8)
    cdf = mod.calculate_cdf(sym, bins)
    ms = _time(lambda: mod.calculate_cdf(sym, bins))
    _emit("cachegen_cdf", ms, sym.numel(), traffic_bytes=sym.numel())
    cap = 512
    out = torch.empty(L, C, cap, dtype=torch.uint8, device="cuda")
    lens = torch.empty(L, C, dtype=torch.int32, device="cuda")
    ms = _time(lambda: mod.encode_fast_new(cdf, sym, out, lens))
    _emit("cachegen_encode", ms, sym.numel(), traffic_bytes=sym.numel() + int(lens.sum()),
          symbols=sym.numel(), ratio=round(sym.numel() / int(lens.sum()), 3))
    streams = torch.cat([out[l, c, :lens[l, c]] for l in range(2) for c in range(C)]) \
        if small else None
    flat = out.view(L * C, cap)
    lens_flat = lens.view(-1)
    idx = torch.arange(cap, device="cuda").unsqueeze(0) < lens_flat.unsqueeze(1)
    streams = flat[idx]
    cum = lens_flat.cumsum(0).to(torch.int32).view(L, C)
    dec = torch.empty_like(sym)
    ms = _time(lambda: mod.decode_fast_prefsum(cdf, streams, cum, dec))
    assert torch.equal(dec, sym)
    _emit("cachegen_decode", ms, sym.numel(), traffic_bytes=sym.numel() + streams.numel())


def bench_rope(small: bool):
    from . import ops
    from .ops.reference import make_cos_sin_cache

    T, H, D = 8192, 8, 128
    cache = make_cos_sin_cache(16384, D, 500000.0).cuda()
    k = torch.randn(T, H * D, device="cuda", dtype=torch.bfloat16)
    old = torch.randint(0, 8192, (T,), device="cuda")
    new = old + 100
    ms = _time(lambda: ops.native().rotary_embedding_k_fused(old, new, k, D, cache, True))
    _emit("rope_delta", ms, k.numel() * 2)


def bench_push(small: bool):
    from .parallel.pd_push import PushReceiver, PushSender
    from .v1.kv_format import PagedKVLayout

    T = 4096 if small else 16384
    L, H, D, BS = 64, 2, 128, 128
    nb = 2 * T // BS
    mk = lambda: [(torch.randn(nb, BS, H, D, device="cuda", dtype=torch.bfloat16),
                   torch.randn(nb, BS, H, D, device="cuda", dtype=torch.bfloat16))
                  for _ in range(L)]
    src, dst = mk(), mk()
    g = torch.Generator().manual_seed(1)
    t = torch.arange(T)
    ss = (torch.randperm(nb, generator=g)[: T // BS][t // BS] * BS + t % BS).int().cuda()
    ds = (torch.randperm(nb, generator=g)[: T // BS][t // BS] * BS + t % BS).int().cuda()
    moved = T * L * 2 * H * D * 2
    for engine in ("auto", "push"):
        recv = PushReceiver(PagedKVLayout(dst))
        send = PushSender(PagedKVLayout(src), engine=engine)
        send.connect([recv.desc])
        ms = _time(lambda: send.push(ss, ds))
        _emit("push_loopback_" + ("tma_copy" if engine == "auto" else "push_kernel"), ms,
              moved, tokens=T, layers=L)
        send.check()


CASES = {"gather": bench_gather_scatter, "offload": bench_offload, "cachegen": bench_cachegen,
         "rope": bench_rope, "push": bench_push}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--small", action="store_true")
    a = ap.parse_args()
    for name, fn in CASES.items():
        if a.only and name not in a.only.split(","):
            continue
        fn(a.small)


if __name__ == "__main__":
    main()
