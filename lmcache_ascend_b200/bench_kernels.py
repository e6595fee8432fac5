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
* ``cachegen``: quantise + CDF + encode + decode + dequantise of stacked
  Llama-3-8B 256-token chunks (8-bit early / 4-bit late layers).
* ``rope``: K re-rotation, 65536 tokens x 8 heads x 128.
* ``c8``: DeepSeek-V3.2 indexer C8 cache <-> chunk packets, 61 layers.
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


_ITERS = {"iters": 10, "warmup": 3}


def _time(fn, iters=None, warmup=None):
    iters = _ITERS["iters"] if iters is None else iters
    warmup = _ITERS["warmup"] if warmup is None else warmup
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
    # layerwise: per-layer chunk objects, one transfer per layer (the engine's
    # store_layer / retrieve_layer path)
    from .v1.gpu_connector import VLLMPagedMemLayerwiseGPUConnector

    L = len(kv)
    for mode in ("copy_engine", "zero_copy"):
        cfg = LMCacheEngineConfig.from_defaults(chunk_size=cs, cpu_transfer_mode=mode,
                                                use_layerwise=True)
        conn = VLLMPagedMemLayerwiseGPUConnector(cfg, kvcaches=kv)
        starts = list(range(0, T, cs))
        ends = [min(s + cs, T) for s in starts]
        per_layer_bytes = sum(conn.get_shape(e - s).numel() * 2 for s, e in zip(starts, ends))
        alloc = PinnedMemoryAllocator(L * per_layer_bytes + (4 << 20))
        objs = [[alloc.allocate(conn.get_shape(e - s), torch.bfloat16, MemoryFormat.KV_2LTD)
                 for s, e in zip(starts, ends)] for _ in range(L)]
        moved = L * per_layer_bytes

        def store():
            g = conn.batched_from_gpu(objs, starts, ends, slot_mapping=slots)
            for _ in g:
                pass

        def load():
            g = conn.batched_to_gpu(None, starts, ends, slot_mapping=slots)
            next(g)
            g.send(objs)
            for _ in g:
                pass

        ms = _time(store, 5, 2)
        _emit(f"offload_layerwise_store_{mode}", ms, moved, traffic_bytes=moved, tokens=T,
              layers=L, note="one transfer per layer; bound: host link")
        ms = _time(load, 5, 2)
        _emit(f"offload_layerwise_load_{mode}", ms, moved, traffic_bytes=moved, tokens=T,
              layers=L, note="one transfer per layer; bound: host link")
        for row in objs:
            for o in row:
                o.ref_count_down()
        alloc.close()


def bench_cachegen(small: bool):
    """Llama-3-8B chunks (256 tokens x 32 layers x 8 heads x
    128), bf16 N(0,1) x per-channel U(0.5, 2); 8-bit (256 bins) for the first
    third of the layers, 4-bit (16 bins) after.  ``chunks`` chunks are stacked
    as rows so every stage's input is larger than L2."""
    from .ops import api
    from .v1.cachegen import _group_order

    mod = api.native()
    chunks = 4 if small else 8
    L, T, C = 32, 256, 1024
    g = torch.Generator(device="cuda").manual_seed(0)
    ch_scale = torch.rand(1, 1, C, device="cuda", generator=g) * 1.5 + 0.5
    x = (torch.randn(chunks * 2 * L, T, C, device="cuda", generator=g) * ch_scale).to(
        torch.bfloat16)
    layer_bins = [256 if l < L // 3 else 16 for l in range(L)]
    row_bins = (layer_bins * 2) * chunks
    order, pos = _group_order(row_bins)
    rb = torch.tensor(row_bins, dtype=torch.int32, device="cuda")
    pos_t = torch.tensor(pos, dtype=torch.int32, device="cuda")
    kv_bytes = x.numel() * 2
    n = x.numel()
    sym = torch.empty(x.shape, dtype=torch.uint8, device="cuda")
    scale = torch.empty(x.shape[:2], dtype=torch.float32, device="cuda")
    ms = _time(lambda: mod.cachegen_quantize(x, rb, sym, scale, pos_t))
    _emit("cachegen_quantize", ms, kv_bytes, traffic_bytes=kv_bytes + n, symbols=n)
    slices, off = [], 0
    for bins, rows in order:
        slices.append((bins, sym[off:off + len(rows)]))
        off += len(rows)
    cdfs = [mod.calculate_cdf(sg, bins) for bins, sg in slices]
    ms = _time(lambda: [mod.calculate_cdf(sg, bins) for bins, sg in slices])
    _emit("cachegen_cdf", ms, kv_bytes, traffic_bytes=n, symbols=n)
    cap = ((T * 12 + 7) // 8 + 4) // 4 * 4
    outs = [torch.empty(sg.shape[0], C, cap, dtype=torch.uint8, device="cuda")
            for _, sg in slices]
    lens = [torch.empty(sg.shape[0], C, dtype=torch.int32, device="cuda") for _, sg in slices]
    enc = lambda: [mod.encode_fast_new(cdf, sg, o, ln)
                   for cdf, (_, sg), o, ln in zip(cdfs, slices, outs, lens)]
    enc()
    total = sum(int(ln.sum()) for ln in lens)
    ms = _time(enc)
    _emit("cachegen_encode", ms, kv_bytes, traffic_bytes=n + total, symbols=n,
          bytes_out=total, ratio_vs_bf16=round(kv_bytes / total, 3))
    streams, cums = [], []
    for o, ln in zip(outs, lens):
        flat = o.view(-1, cap)
        mask = torch.arange(cap, device="cuda").unsqueeze(0) < ln.view(-1, 1)
        streams.append(flat[mask])
        cums.append(ln.view(-1).cumsum(0).to(torch.int32).view(ln.shape))
    dsym = torch.empty_like(sym)
    dslices, off = [], 0
    for _, sg in slices:
        dslices.append(dsym[off:off + sg.shape[0]])
        off += sg.shape[0]
    dec = lambda: [mod.decode_fast_prefsum(cdf, st, cu, d)
                   for cdf, st, cu, d in zip(cdfs, streams, cums, dslices)]
    ms = _time(dec)
    assert torch.equal(dsym, sym)
    _emit("cachegen_decode", ms, kv_bytes, traffic_bytes=n + total, symbols=n)
    y = torch.empty_like(x)
    ms = _time(lambda: mod.cachegen_dequantize(dsym, scale, rb, y, pos_t))
    err = (y.float() - x.float())
    _emit("cachegen_dequantize", ms, kv_bytes, traffic_bytes=kv_bytes + n,
          max_abs_err=round(float(err.abs().max()), 4),
          rel_rms_err=round(float(err.pow(2).mean().sqrt() / x.float().pow(2).mean().sqrt()), 4))


def bench_cachegen_serde(small: bool):
    """BASELINE config 4 end to end through the serde API: KV_2LTD chunks of
    256 tokens x 32 layers x 8 heads x 128 (bf16 N(0,1) x per-channel
    U(0.5, 2); 8-bit for the first third of the layers, 4-bit after) encoded
    by ``encode_kv(...).to_bytes()`` on the device (quantise, CDF, encode,
    compaction, one D2H) and decoded by ``decode_kv_bytes`` (one H2D,
    decode, dequantise) back into a device chunk.  Times include the
    host <-> device copies of the payload; GB/s counts bf16 KV bytes."""
    from .v1.cachegen import CacheGenConfig, decode_kv_bytes, encode_kv

    chunks = 2 if small else 8
    L, T, H, D = 32, 256, 8, 128
    C = H * D
    g = torch.Generator(device="cuda").manual_seed(0)
    ch_scale = torch.rand(1, 1, 1, C, device="cuda", generator=g) * 1.5 + 0.5
    kvs = [(torch.randn(2, L, T, C, device="cuda", generator=g) * ch_scale).to(torch.bfloat16)
           for _ in range(chunks)]
    cfg = CacheGenConfig.from_ranges(L, [(0, L // 3, 256), (L // 3, L, 16)],
                                     [(0, L // 3, 256), (L // 3, L, 16)])
    kv_bytes = sum(k.numel() * 2 for k in kvs)
    payloads = []

    def enc():
        payloads.clear()
        for k in kvs:
            payloads.append(encode_kv(k, cfg).to_bytes())

    ms = _time(enc, iters=3, warmup=1)
    wire = sum(len(b) for b in payloads)
    _emit("cachegen_serde_encode", ms, kv_bytes, traffic_bytes=kv_bytes, chunks=chunks,
          payload_bytes=wire, ratio_vs_bf16=round(kv_bytes / wire, 3),
          note="to_bytes included (one D2H per chunk)")
    outs = [torch.empty_like(k) for k in kvs]

    def dec():
        for b, o in zip(payloads, outs):
            decode_kv_bytes(b, "cuda", out=o)

    ms = _time(dec, iters=3, warmup=1)
    err = torch.cat([(o.float() - k.float()).flatten() for o, k in zip(outs, kvs)])
    ref = torch.cat([k.float().flatten() for k in kvs])
    _emit("cachegen_serde_decode", ms, kv_bytes, traffic_bytes=kv_bytes, chunks=chunks,
          payload_bytes=wire, max_abs_err=round(float(err.abs().max()), 4),
          rel_rms_err=round(float(err.pow(2).mean().sqrt() / ref.pow(2).mean().sqrt()), 4),
          note="from bytes: one H2D per chunk")


def bench_rope(small: bool):
    """K re-rotation (BASELINE config 5 pass: theta 10000, deltas 0-8192) on a
    bf16 K of 65536 tokens x 8 heads x 128 (128 MiB, larger than L2)."""
    from . import ops
    from .ops.reference import make_cos_sin_cache

    T, H, D = (8192 if small else 65536), 8, 128
    cache = make_cos_sin_cache(65536 + 8192, D, 10000.0).cuda()
    k = torch.randn(T, H * D, device="cuda", dtype=torch.bfloat16)
    old = torch.randint(0, 65536, (T,), device="cuda")
    new = old + torch.randint(0, 8193, (T,), device="cuda")
    ms = _time(lambda: ops.native().rotary_embedding_k_fused(old, new, k, D, cache, True))
    _emit("rope_delta", ms, k.numel() * 2, tokens=T)


def bench_c8(small: bool):
    """Indexer C8 (DeepSeek-V3.2 lightning indexer: int8 keys 128 B/token +
    fp16 scale) paged cache -> per-chunk device packets, 61 layers, 32k tokens."""
    from .ops import api

    L, T, chunk = 61, (8192 if small else 32768), 256
    nb = 2 * T // 128
    states = [api.IndexerC8State(
        torch.randint(-128, 127, (nb, 128, 1, 128), dtype=torch.int8, device="cuda"),
        torch.randn(nb, 128, 1, 1, device="cuda").half()) for _ in range(L)]
    grp = api.IndexerC8GroupState(states)
    g = torch.Generator().manual_seed(0)
    t = torch.arange(T)
    slots = (torch.randperm(nb, generator=g)[: T // 128][t // 128] * 128 + t % 128).int().cuda()
    packets = [torch.empty(grp.packet_bytes(chunk), dtype=torch.uint8, device="cuda")
               for _ in range(T // chunk)]
    moved = grp.packet_bytes(T)
    ms = _time(lambda: api.indexer_c8_transfer_prepared(grp, packets, slots, chunk, True))
    _emit("indexer_c8_to_packets", ms, moved, tokens=T, layers=L)
    ms = _time(lambda: api.indexer_c8_transfer_prepared(grp, packets, slots, chunk, False))
    _emit("indexer_c8_from_packets", ms, moved, tokens=T, layers=L)


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
    for engine in ("bulk", "simt"):
        recv = PushReceiver(PagedKVLayout(dst))
        send = PushSender(PagedKVLayout(src), engine=engine)
        send.connect([recv.desc])
        ms = _time(lambda: send.push(ss, ds))
        _emit(f"push_loopback_{engine}_kernel", ms, moved, traffic_bytes=2 * moved,
              tokens=T, layers=L)
        send.check()
    # fp8 push kernel alone (into the receiver's staging; local stores here)
    recv = PushReceiver(PagedKVLayout(dst), fp8_staging_tokens=T)
    send = PushSender(PagedKVLayout(src))
    send.connect([recv.desc])
    wire = T * L * 2 * (H * D + (H * D // 128) * 4)
    for tile in (128, 512):
        # the release hands the staging buffer back (no dequant in this case)
        ms = _time(lambda: (send.push(ss, ds, quant="fp8", tile_tokens=tile),
                            recv.release_staging()))
        _emit(f"push_loopback_fp8_kernel_tile{tile}", ms, moved, traffic_bytes=moved + wire,
              tokens=T, layers=L, wire_bytes=wire)
    ms = _time(lambda: recv.dequantize(ds))
    _emit("push_fp8_dequantize", ms, moved, traffic_bytes=moved + wire, tokens=T, layers=L)
    send.check()
    recv.check()


CASES = {"gather": bench_gather_scatter, "offload": bench_offload, "cachegen": bench_cachegen,
         "cachegen_serde": bench_cachegen_serde,
         "rope": bench_rope, "c8": bench_c8, "push": bench_push}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--small", action="store_true")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3,
                    help="untimed launches per case (0 with --iters 1 for a profiler capture)")
    a = ap.parse_args()
    _ITERS.update(iters=max(1, a.iters), warmup=max(0, a.warmup))
    for name, fn in CASES.items():
        if a.only and name not in a.only.split(","):
            continue
        fn(a.small)


if __name__ == "__main__":
    main()
