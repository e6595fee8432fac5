"""DeepSeek-V3.2-shaped disaggregated prefill: MLA latent + C8 indexer push.

Per layer (61 layers) the paged cache holds, per token, the MLA latent
(kv_lora_rank 512 + rope 64 = 576 bf16 = 1152 bytes), the lightning-indexer
key (128 int8) and its fp32 scale (4 bytes); block size 64.  Both caches are
replicated across the TP ranks of an instance, so in 1P(TP4) -> 1D(TP4)
prefill rank r pushes a full copy to decode rank r (N/2 disjoint pairs; N=1
is the same kernel in loopback).  One push launch moves all three planes:
TMA bulk copies for the latent and the indexer keys, per-lane 4-byte copies
for the scales, one flag release per (layer, plane, tile).

Requests: 32768 random tokens each; step i pushes request i mod 16 (16
distinct block tables on both sides).  After each push the decoder
re-positions the request's cached keys for reuse (CacheBlend): the 64 rope
dims of every latent row are re-rotated from their stored positions to
positions shifted by a random delta in [0, 8192) (theta 10000), in place in
the paged cache, addressed by slot.
"""

from __future__ import annotations

import torch

LAYERS, LATENT, ROPE, IDX, BS = 61, 576, 64, 128, 64


def _cache(L, nb, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    out = []
    for _ in range(L):
        lat = torch.randn(nb, BS, LATENT, generator=g, device=dev).to(torch.bfloat16)
        key = torch.randint(-128, 128, (nb, BS, IDX), generator=g, device=dev,
                            dtype=torch.int8)
        sc = torch.rand(nb, BS, 1, generator=g, device=dev)
        out.append((lat, key, sc))
    return out


def _bytes_view(cache):
    """Per layer (latent, key, scale) as uint8 [nb, BS, row bytes] planes."""
    return [tuple(t.view(torch.uint8).view(t.shape[0], BS, -1) for t in layer)
            for layer in cache]


def run_config5(dev, rank: int, world: int, gloo=None, tokens: int = 32768,
                requests: int = 16, steps: int = 16, warmup: int = 3,
                peer_copy_gbps=None) -> dict:
    import torch.distributed as dist

    from .ops.reference import make_cos_sin_cache
    from .parallel.pd_push import PushReceiver, PushSender, ReceiverDesc
    from .v1.kv_format import PagedKVLayout

    from . import ops

    native = ops.native()
    L = LAYERS
    nb = 2 * tokens // BS
    pre = world == 1 or rank < world // 2
    dec = world == 1 or rank >= world // 2
    src = _cache(L, nb, dev, 10 + rank) if pre else None
    dst = _cache(L, nb, dev, 100 + rank) if dec else None
    recv = PushReceiver(PagedKVLayout(_bytes_view(dst))) if dec else None
    send = PushSender(PagedKVLayout(_bytes_view(src))) if pre else None
    if world == 1:
        send.connect([recv.desc])
    else:
        descs = [None] * world
        dist.all_gather_object(descs, recv.desc.to_dict() if recv else None, group=gloo)
        if pre:
            send.connect([ReceiverDesc.from_dict(descs[rank + world // 2])])
        dist.barrier(group=gloo)
    g = torch.Generator().manual_seed(5)
    t = torch.arange(tokens)
    tables = []
    for _ in range(requests):
        sb = torch.randperm(nb, generator=g)[: tokens // BS]
        db = torch.randperm(nb, generator=g)[: tokens // BS]
        tables.append(((sb[t // BS] * BS + t % BS).int().to(dev),
                       (db[t // BS] * BS + t % BS).int().to(dev)))
    rope_cache = make_cos_sin_cache(tokens + 8192, ROPE, 10000.0).to(dev)
    old_pos = torch.arange(tokens, device=dev, dtype=torch.int32)
    deltas = [torch.randint(0, 8192, (tokens,), generator=g).int().to(dev)
              for _ in range(requests)]
    n_total = warmup + steps
    targets = [recv.expect(tokens) for _ in range(n_total)] if dec else [None] * n_total

    def barrier():
        if world > 1:
            dist.barrier(group=gloo)
        torch.cuda.synchronize()

    def push_step(i):
        ss, ds = tables[i % requests]
        if pre:
            send.push(ss, ds)
        if dec:
            recv.wait(targets[i], timeout_s=10.0)

    rope_keys = [layer[0].view(nb * BS, LATENT)[:, 512:] for layer in dst] if dec else []

    def rope_step(i):
        if not dec:
            return
        _, ds = tables[i % requests]
        new_pos = old_pos + deltas[i % requests]
        # every layer's rope columns in one launch
        native.rotary_embedding_k_fused_layers(old_pos, new_pos, rope_keys, ROPE, rope_cache,
                                               True, ds)

    def timed(fn, base):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(base + i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        barrier()
        tt = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    for i in range(warmup):
        push_step(i)
    push_ms = timed(push_step, warmup)
    for o in (send, recv):
        if o is not None:
            o.check()
    for i in range(warmup):
        rope_step(i)
    rope_ms = timed(rope_step, warmup)
    row = LATENT * 2 + IDX + 4
    pair_bytes = tokens * L * row
    pairs = max(1, world // 2)
    per_pair = pair_bytes / (push_ms / 1e3) / 1e9
    rope_bytes = 2 * tokens * L * ROPE * 2  # read + write of the rope dims
    out = {"ms_per_request": round(push_ms, 4), "gbps_per_pair": round(per_pair, 2),
           "aggregate_gbps": round(per_pair * pairs, 2), "bytes_per_pair": pair_bytes,
           "planes": {"latent_bytes": LATENT * 2, "indexer_key_bytes": IDX,
                      "indexer_scale_bytes": 4},
           "layers": L, "tokens": tokens, "block_size": BS, "requests": requests,
           "launches_per_request": 1 + (1 if dec else 0),
           "rope_reposition": {"ms_per_request": round(rope_ms, 4),
                               "gbps": round(rope_bytes / (rope_ms / 1e3) / 1e9, 2),
                               "theta": 10000.0, "delta_range": [0, 8192],
                               "launches_per_request": 1}}
    if peer_copy_gbps:
        out["frac_of_measured_peer_copy"] = round(per_pair / peer_copy_gbps, 4)
    if send is not None:
        send.close()
    barrier()
    return out
