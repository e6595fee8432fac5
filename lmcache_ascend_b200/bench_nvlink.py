"""NVLink peer-bandwidth probe: the roofline denominators of the PD push.

One process drives every visible GPU (peer access enabled between all of
them), so no rank rendezvous is involved.  For each timed case the payload is
1 GiB laid out as the push benchmark's paged KV (64 layers x K/V planes x
16384 tokens x 512-byte rows, Qwen3-32B TP4 shard), moved from GPU i's HBM
into GPU j's HBM:

* ``ce``: the copy engines, one cudaMemcpyAsync per (layer, plane) plane of
  8 MiB (what a peer copy of the same bytes costs without any SM);
* ``push_bulk`` / ``push_simt``: this repo's push kernel (TMA bulk stores or
  16-byte SIMT stores through the peer address), block-table gather on the
  source side included;
* ``pull_bulk`` / ``pull_simt``: the same kernel launched on the receiving
  GPU, loading the sender's rows through the peer address (TMA bulk loads
  without multicast, or 16-byte loads) and storing them locally.

Pairs are timed alone (0 -> 1) and all at once (i -> i + N/2 for every i,
the pairing of ``bench.py``), each with CUDA events on the source GPU's
stream after warm-up, reported as GB/s per pair (max time over pairs).

``python -m lmcache_ascend_b200.bench_nvlink`` (needs 2+ GPUs)
"""

from __future__ import annotations

import argparse
import json

import torch


def _cache(L, nb, bs, H, D, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return [(torch.randn(nb, bs, H, D, generator=g).to(torch.bfloat16).to(dev),
             torch.randn(nb, bs, H, D, generator=g).to(torch.bfloat16).to(dev))
            for _ in range(L)]


def main() -> None:
    from . import ops
    from .v1.kv_format import PagedKVLayout

    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--grid", type=int, default=0, help="push CTAs (0: the kernel's default)")
    ap.add_argument("--kinds", default="ce,push_bulk,push_simt,pull_bulk,pull_simt")
    a = ap.parse_args()
    n = torch.cuda.device_count()
    if n < 2:
        print(json.dumps({"probe": "nvlink", "unavailable": "needs 2+ GPUs"}))
        return
    mod = ops.native()
    for i in range(n):
        for k in range(n):
            if i != k:
                mod.enable_peer_access(i, k)
    L, T, H, D, BS = a.layers, a.tokens, 2, 128, 128
    nb = 2 * T // BS
    moved = T * L * 2 * H * D * 2
    caches, layouts, slots = {}, {}, {}
    for d in range(n):
        dev = torch.device("cuda", d)
        caches[d] = _cache(L, nb, BS, H, D, dev, seed=d)
        layouts[d] = PagedKVLayout(caches[d])
        g = torch.Generator().manual_seed(100 + d)
        blocks = torch.randperm(nb, generator=g)[: T // BS]
        t = torch.arange(T)
        slots[d] = (blocks[t // BS] * BS + t % BS).to(torch.int32).to(dev)

    def layout_seen_from(run_dev: int, owner: int):
        """``owner``'s paged cache described on ``run_dev`` (peer addresses)."""
        lay = layouts[owner]
        es = lay.elem_size
        ptrs = torch.tensor([t.data_ptr() for layer in caches[owner] for t in layer],
                            dtype=torch.int64, device=torch.device("cuda", run_dev))
        nat = mod.PagedLayout(ptrs, [p.views[0].stride(0) * es for p in lay.planes],
                              [p.views[0].stride(1) * es for p in lay.planes], lay.row_bytes,
                              lay.block_size, lay.num_slots, [], [])
        nat.set_bases_aligned(True)
        return nat

    def make_op(kind, i, k):
        """(device that launches, op) moving GPU i's planes into GPU k's."""
        if kind == "ce":
            plane = T * H * D * 2
            dsts = torch.tensor([t.data_ptr() for layer in caches[k] for t in layer],
                                dtype=torch.int64)
            srcs = torch.tensor([t.data_ptr() for layer in caches[i] for t in layer],
                                dtype=torch.int64)
            sizes = torch.full((dsts.numel(),), plane, dtype=torch.int64)
            return i, lambda: mod.layerwise_prefill_dma_copy(dsts, srcs, sizes)
        mode = 1 if kind.endswith("bulk") else 2
        if kind.startswith("pull"):
            # the receiver's SMs load the sender's rows through the peer
            # mapping and store them locally
            src, dst, run_dev = layout_seen_from(k, i), layouts[k].native(), k
            ss = slots[i].to(torch.device("cuda", k))
            ds = slots[k]
        else:
            src, dst, run_dev = layouts[i].native(), layout_seen_from(i, k), i
            ss, ds = slots[i], slots[k].to(torch.device("cuda", i))
        cnt = torch.zeros(1 << 16, dtype=torch.int32, device=torch.device("cuda", run_dev))
        return run_dev, lambda: mod.pd_push(src, dst, ss, ds, 0, L, 1, [], 512, a.grid, None,
                                            mode, cnt)

    def run(kind, pairs):
        ops_ = [make_op(kind, i, k) for i, k in pairs]
        for _ in range(a.warmup):
            for i, f in ops_:
                with torch.cuda.device(i):
                    f()
        for d in range(n):
            torch.cuda.synchronize(d)
        ev = {}
        for i, f in ops_:
            with torch.cuda.device(i):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev[i] = (e0, e1)
        for i, _ in ops_:
            with torch.cuda.device(i):
                ev[i][0].record()
        for _ in range(a.iters):
            for i, f in ops_:
                with torch.cuda.device(i):
                    f()
        for i, _ in ops_:
            with torch.cuda.device(i):
                ev[i][1].record()
        for d in range(n):
            torch.cuda.synchronize(d)
        ms = max(ev[i][0].elapsed_time(ev[i][1]) / a.iters for i, _ in ops_)
        return ms

    half = n // 2
    cases = [("pair_0_to_1", [(0, 1)])]
    if n >= 4:
        cases.append((f"all_{half}_pairs", [(i, i + half) for i in range(half)]))
    for name, pairs in cases:
        for kind in a.kinds.split(","):
            ms = run(kind, pairs)
            print(json.dumps({"probe": "nvlink", "case": name, "kind": kind, "gpus": n,
                              "grid": a.grid,
                              "pairs": len(pairs), "ms": round(ms, 4),
                              "gbps_per_pair": round(moved / ms / 1e6, 1),
                              "bytes_per_pair": moved}), flush=True)


if __name__ == "__main__":
    main()
