#!/usr/bin/env python
"""Headline benchmark: prefill->decode KV push (GB/s), Qwen3-32B-shaped.

1 prefiller at TP4 -> 1 decoder at TP4 on 8 GPUs,
Qwen3-32B KV (64 layers, 8 KV heads split over TP4 = 2 heads per rank,
head_dim 128, block_size 128, bf16), 16384-token requests pushed layer by
layer from the prefiller's paged blocks into the decoder's paged blocks.

Scaling (weak): each GPU pair carries one TP4 shard (2 KV heads) of one
16k-token request per step.  N GPUs = N/2 pairs (rank r -> rank r + N/2);
N=1 runs the same push kernel in loopback (prefiller and decoder caches on
one GPU, bound by HBM instead of NVLink).  ``value`` is the whole-job
aggregate GB/s over all pairs; ``e2e`` repeats the measurement through the
public engine API with per-step host->device slot-mapping copies and a
device->host completion-status read.

Roofline: at N>1 every prefiller also times a copy-engine copy of the same
bytes into its decoder's memory (one cudaMemcpyAsync per plane, through the
same peer mapping) in this run, and the push is reported as a fraction of
that measured peer bandwidth; at N=1 the bound is HBM (read + write) from
MEASURED_PEAKS.json.

Baseline arm (same invocation, after ours): per step the prefiller gathers
every layer with ``index_select``, sends all layers with ONE
``batch_isend_irecv`` on a process group of its own pair, and the decoder
``index_copy_``s them into its paged cache; ``vs_baseline`` is ours / that.

Launch: ``python bench.py`` (N=1) or
``torchrun --nproc-per-node N bench.py --gpus N``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

NVLINK_NOMINAL_GBPS = 900.0  # NVLink 5, per direction per GPU (context only)
HBM_FALLBACK_GBPS = 6650.0   # used only when MEASURED_PEAKS.json is absent
HERE = os.path.dirname(os.path.abspath(__file__))


def measured_hbm_gbps() -> float:
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except Exception:
        return HBM_FALLBACK_GBPS


def reference_arm() -> dict:
    """The reference's own public API, installed unmodified under
    baseline/_ref (its setup.py needs an Ascend NPU and CANN to build)."""
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(ref):
        return {"impl": "reference", "unavailable":
                "LMCache-Ascend is not installed: its setup.py stops with 'No available NPU "
                "found' (it builds AscendC kernels against CANN/torch_npu); nothing to import"}
    sys.path.insert(0, ref)
    try:
        import lmcache_ascend  # noqa: F401
    except Exception as e:  # the actual import error, one line
        return {"impl": "reference",
                "unavailable": f"import lmcache_ascend failed: {type(e).__name__}: {e}"[:400]}
    return {"impl": "reference", "unavailable":
            "lmcache_ascend imported, but its KV push runs on Ascend NPUs (hccl/hixl "
            "channels); there is no CUDA device path to time"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--engine", default="auto", choices=["auto", "bulk", "simt"],
                    help="push kernel (auto: TMA bulk copies when rows allow)")
    ap.add_argument("--no-baseline", action="store_true",
                    help="skip the NCCL + index_copy baseline arm")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--layers", type=int, default=64)
    ap.add_argument("--heads", type=int, default=2, help="KV heads per rank (TP4 shard)")
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--block-size", type=int, default=128)
    ap.add_argument("--grid", type=int, default=0)
    ap.add_argument("--tile", type=int, default=512)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-ttft", action="store_true",
                    help="skip the TTFT-on-prefix-hit measurement (Qwen3-32B, 16k hit)")
    ap.add_argument("--ttft-requests", type=int, default=8)
    ap.add_argument("--no-fp8", action="store_true",
                    help="skip the block-scaled fp8 push measurement")
    ap.add_argument("--multicast", action="store_true",
                    help="also time the NVLS fan-out (rank 0 -> every other rank), N > 1")
    ap.add_argument("--no-overlap", action="store_true",
                    help="skip the prefill-forward + layer-by-layer push overlap measurement")
    ap.add_argument("--overlap-iters", type=int, default=2)
    ap.add_argument("--no-config5", action="store_true",
                    help="skip the DeepSeek-V3.2 MLA latent + C8 indexer push (config 5)")
    ap.add_argument("--no-config2", action="store_true",
                    help="skip the Llama-3-8B local offload per DP replica (config 2)")
    ap.add_argument("--config2-requests", type=int, default=64)
    ap.add_argument("--fp8-tile", type=int, default=512,
                    help="tokens per fp8 push unit (one flag release per unit)")
    return ap.parse_args()


def out(d):
    print(json.dumps(d), flush=True)


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index
        self.path = f"/tmp/lmc_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def block_table_slots(T, block_size, num_blocks, seed, device):
    g = torch.Generator().manual_seed(seed)
    nblk = (T + block_size - 1) // block_size
    blocks = torch.randperm(num_blocks, generator=g)[:nblk]
    t = torch.arange(T)
    return (blocks[t // block_size] * block_size + t % block_size).to(torch.int32).to(device)


def make_cache(L, num_blocks, block_size, H, D, device, seed):
    """vLLM SEPARATE_KV layout: per layer (K, V) each [NB, BS, H, D] bf16."""
    torch.manual_seed(seed)
    kv = []
    for _ in range(L):
        k = torch.randn(num_blocks, block_size, H, D, device=device, dtype=torch.bfloat16)
        v = torch.randn(num_blocks, block_size, H, D, device=device, dtype=torch.bfloat16)
        kv.append((k, v))
    return kv


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = {"model": "Qwen3-32B (KV shape: 64 layers, 8 KV heads, head_dim 128)",
           "global_batch": max(1, world // 2), "seq_len": a.tokens,
           "parallelism": ("pd-loopback-1gpu" if world == 1 else
                           f"1P(TP{world // 2})->1D(TP{world // 2})"),
           "kv_heads_per_rank": a.heads, "block_size": a.block_size, "layers": a.layers,
           "l2": "inputs larger than L2 (1 GiB of KV read per rank per step)"}
    if a.impl == "reference":
        if rank == 0:
            out(reference_arm())
        return
    if not torch.cuda.is_available():
        if rank == 0:
            out({"metric": "kv_push_gbps", "unavailable": "no CUDA device"})
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch.distributed as dist

    gloo = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=120))
        if world % 2:
            raise SystemExit("bench needs an even number of GPUs (prefiller/decoder pairs)")

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from lmcache_ascend_b200 import ops
    from lmcache_ascend_b200.parallel.pd_push import PushReceiver, PushSender, ReceiverDesc
    from lmcache_ascend_b200.v1.kv_format import PagedKVLayout

    ops.native()
    L, T, H, D, BS = a.layers, a.tokens, a.heads, a.head_dim, a.block_size
    nblocks = 2 * ((T + BS - 1) // BS)
    pairs = 1 if world == 1 else world // 2
    role_p = world == 1 or rank < world // 2
    role_d = world == 1 or rank >= world // 2
    bytes_per_pair = T * L * 2 * H * D * 2  # K and V rows, bf16

    src_cache = make_cache(L, nblocks, BS, H, D, dev, 1 + rank) if role_p else None
    dst_cache = make_cache(L, nblocks, BS, H, D, dev, 1000 + rank) if role_d else None
    src_slots = block_table_slots(T, BS, nblocks, 11, dev)
    dst_slots = block_table_slots(T, BS, nblocks, 22, dev)

    sender = receiver = None
    if role_d:
        receiver = PushReceiver(PagedKVLayout(dst_cache))
    if role_p:
        sender = PushSender(PagedKVLayout(src_cache), engine=a.engine)
    if world == 1:
        sender.connect([receiver.desc])
    else:
        descs = [None] * world
        dist.all_gather_object(descs, receiver.desc.to_dict() if receiver else None, group=gloo)
        if role_p:
            sender.connect([ReceiverDesc.from_dict(descs[rank + world // 2])])
        dist.barrier(group=gloo)

    # ------------------------------------------------------------ our push
    def step(targets):
        if sender is not None:
            sender.push(src_slots, dst_slots, tile_tokens=a.tile, grid=a.grid)
        if receiver is not None:
            receiver.wait(targets, timeout_s=5.0)

    n_targets = a.warmup + a.steps
    targets = ([receiver.expect(T, tile_tokens=a.tile) for _ in range(n_targets)]
               if receiver is not None else [None] * n_targets)
    ti = 0

    def barrier():
        if world > 1:
            dist.barrier(group=gloo)
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        t = torch.tensor([x], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, steps):
        """CUDA-event time of `steps` calls on this rank's stream (ms/step),
        bracketed by a barrier + synchronize on both sides; max over ranks."""
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        ms_ = e0.elapsed_time(e1) / steps
        barrier()
        return max_over_ranks(ms_)

    for _ in range(a.warmup):
        step(targets[ti]); ti += 1
    barrier()
    for o in (receiver, sender):
        if o is not None:
            o.check()

    clocks = ClockSampler(local)
    if rank == 0:
        clocks.start()
    base_ti = ti
    ms = timed(lambda i: step(targets[base_ti + i]), a.steps)
    ck = clocks.stop() if rank == 0 else None
    for o in (receiver, sender):
        if o is not None:
            o.check()
    value = bytes_per_pair * pairs / (ms / 1e3) / 1e9

    # ---------------------------------------- measured peer-copy roofline
    # The copy engines' rate into the same decoder memory through the same
    # peer mapping: one cudaMemcpyAsync per (layer, plane) of the pushed
    # rows' size, timed like the push.  N=1 uses the HBM figure instead.
    peer_copy = None
    if world > 1:
        plane_bytes = T * H * D * 2
        dsts = srcs = sizes = None
        if role_p:
            dptrs = sender._dst.ptrs.cpu().tolist()  # receiver's plane bases, mapped here
            sptrs = [t.data_ptr() for layer in src_cache for t in layer]
            dsts = torch.tensor(dptrs, dtype=torch.int64)
            srcs = torch.tensor(sptrs, dtype=torch.int64)
            sizes = torch.full((len(sptrs),), plane_bytes, dtype=torch.int64)

        def ce_copy(_i):
            if role_p:
                ops.native().layerwise_prefill_dma_copy(dsts, srcs, sizes)

        for i in range(a.warmup):
            ce_copy(i)
        ce_ms = timed(ce_copy, a.steps)
        peer_copy = {"gbps_per_pair": round(bytes_per_pair / (ce_ms / 1e3) / 1e9, 2),
                     "ms_per_step": round(ce_ms, 4),
                     "how": "cudaMemcpyAsync per (layer, plane) into the decoder's planes "
                            "through the push's peer mapping, max over ranks"}

    # --------------------------------------- baseline: NCCL + index_copy_
    baseline = None
    if not a.no_baseline:
        pair_groups = {}
        if world > 1:
            for r0 in range(world // 2):  # every rank creates every group, same order
                pair_groups[r0] = dist.new_group([r0, r0 + world // 2], backend="nccl")
        my_pair = pair_groups.get(rank % (world // 2)) if world > 1 else None
        peer = (rank + world // 2) % world if world > 1 else 0
        ls, ld = src_slots.long(), dst_slots.long()
        bufs = [torch.empty(2, T, H * D, device=dev, dtype=torch.bfloat16) for _ in range(L)]

        def step_nccl(_i):
            if role_p:
                for l in range(L):
                    k, v = src_cache[l]
                    torch.index_select(k.view(-1, H * D), 0, ls, out=bufs[l][0])
                    torch.index_select(v.view(-1, H * D), 0, ls, out=bufs[l][1])
            if world > 1:
                op = dist.isend if role_p else dist.irecv
                reqs = dist.batch_isend_irecv([dist.P2POp(op, bufs[l], peer, group=my_pair)
                                               for l in range(L)])
                for r_ in reqs:
                    r_.wait()
            if role_d:
                for l in range(L):
                    k, v = dst_cache[l]
                    k.view(-1, H * D).index_copy_(0, ld, bufs[l][0])
                    v.view(-1, H * D).index_copy_(0, ld, bufs[l][1])

        for i in range(a.warmup):
            step_nccl(i)
        b_ms = timed(step_nccl, a.steps)
        b_val = bytes_per_pair * pairs / (b_ms / 1e3) / 1e9
        baseline = {"value": round(b_val, 2), "ms_per_step": round(b_ms, 4),
                    "impl": ("index_select -> one batch_isend_irecv of all layers on a "
                             "per-pair NCCL group -> index_copy_" if world > 1 else
                             "index_select -> index_copy_ (loopback, no NCCL)")}
        del bufs
        for g_ in pair_groups.values():
            dist.destroy_process_group(g_)
        barrier()

    # ------------------------------------------------- fp8 push (lossy)
    # The same push with block-scaled fp8 on the wire: the prefiller's kernel
    # quantises (128-element groups, fp32 scales) into the decoder's staging,
    # the decoder dequantises into its bf16 cache after the layer flags.
    # Reported as bf16-equivalent GB/s per pair, receiver dequant included.
    fp8 = None
    if not a.no_fp8:
        recv8 = PushReceiver(PagedKVLayout(dst_cache), fp8_staging_tokens=T) if role_d else None
        send8 = PushSender(PagedKVLayout(src_cache)) if role_p else None
        if world == 1:
            send8.connect([recv8.desc])
        else:
            d8 = [None] * world
            dist.all_gather_object(d8, recv8.desc.to_dict() if recv8 else None, group=gloo)
            if role_p:
                send8.connect([ReceiverDesc.from_dict(d8[rank + world // 2])])
            dist.barrier(group=gloo)
        tg8 = ([recv8.expect(T, tile_tokens=a.fp8_tile) for _ in range(a.warmup + a.steps)]
               if recv8 is not None else [None] * (a.warmup + a.steps))

        def step8(i):
            if send8 is not None:
                send8.push(src_slots, dst_slots, tile_tokens=a.fp8_tile, grid=a.grid,
                           quant="fp8")
            if recv8 is not None:  # dequantise each 8-layer group as soon as it landed
                for l0 in range(0, L, 8):
                    n8 = min(8, L - l0)
                    recv8.wait(tg8[i][l0:l0 + n8], layer_begin=l0, timeout_s=5.0)
                    recv8.dequantize(dst_slots, layer_begin=l0, num_layers=n8)

        for i in range(a.warmup):
            step8(i)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        for i in range(a.steps):
            step8(a.warmup + i)
        f1.record()
        torch.cuda.synchronize()
        fms = torch.tensor([f0.elapsed_time(f1) / a.steps], device=dev)
        if world > 1:
            dist.all_reduce(fms, op=dist.ReduceOp.MAX)
        fms = float(fms.item())
        barrier()
        for o in (send8, recv8):
            if o is not None:
                o.check()
        wire = T * L * 2 * (H * D + (H * D // 128) * 4)
        fp8 = {"bf16_equiv_gbps_per_pair": round(bytes_per_pair / (fms / 1e3) / 1e9, 2),
               "wire_gbps_per_pair": round(wire / (fms / 1e3) / 1e9, 2),
               "ms_per_step": round(fms, 4), "wire_bytes_per_pair": wire,
               "bf16_bytes_per_pair": bytes_per_pair, "group": 128,
               "note": "lossy (e4m3, one fp32 scale per 128 elements); decoder dequant "
                       "included"}
        if send8 is not None:
            send8.close()

    # ------------------------------------------------ NVLS fan-out (opt-in)
    # Rank 0 writes the whole cache once through the multicast address of a
    # symmetric staging buffer; NVSwitch delivers it to every rank; the
    # decoders scatter each 8-layer group into their paged caches as soon as
    # its flags complete.  Steps are separated by a
    # host barrier (one staging buffer), each timed on its own: receivers
    # measure wait + scatter from before the push starts, rank 0 the push.
    mcast = None
    if a.multicast and world > 1:
        from lmcache_ascend_b200.parallel.pd_multicast import MulticastFanout

        fan = MulticastFanout(dist.group.WORLD, L, 2, H * D * 2, T, dev)
        if fan.has_multicast:
            src_l = PagedKVLayout(src_cache) if rank == 0 else None
            dst_l = PagedKVLayout(dst_cache) if dst_cache is not None else None
            per = []
            for i in range(a.warmup + a.steps):
                tg = fan.expect(T, tile_tokens=a.tile)
                barrier()
                m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                m0.record()
                if rank == 0:
                    fan.push(src_l, src_slots, tile_tokens=a.tile)
                for l0 in range(0, L, 8):  # scatter each 8-layer group as it lands
                    n8 = min(8, L - l0)
                    fan.wait(tg[l0:l0 + n8], timeout_s=5.0, layer_begin=l0)
                    if dst_l is not None:
                        fan.scatter(dst_l, dst_slots, T, layer_begin=l0, num_layers=n8)
                if dst_l is None:
                    fan.release()  # hand the staging back (no-op on rank 0, the root)
                m1.record()
                torch.cuda.synchronize()
                if i >= a.warmup:
                    per.append(m0.elapsed_time(m1))
            fan.check()
            mms = torch.tensor([sum(per) / len(per)], device=dev)
            dist.all_reduce(mms, op=dist.ReduceOp.MAX)
            mms = float(mms.item())
            receivers = world - 1
            mcast = {"ms_per_step": round(mms, 4), "receivers": receivers,
                     "egress_gbps": round(bytes_per_pair / (mms / 1e3) / 1e9, 2),
                     "delivered_gbps": round(bytes_per_pair * receivers / (mms / 1e3) / 1e9, 2),
                     "note": "rank 0 -> all ranks through one multicast store per vector; "
                             "decoder scatter included; host barrier between steps"}
        else:
            mcast = {"unavailable": "no NVLink multicast on this system"}
        barrier()
        del fan

    # ------------------------------------------------------------ e2e arm
    # Same transfer through the engine's public API: the decoder reserves its
    # slots (LMCacheEngine.reserve_direct_prefill), the prefiller calls
    # LMCacheEngine.store_direct_prefill (grant over ZMQ, then the fused
    # push), the decoder LMCacheEngine.wait_direct_prefill (bounded device
    # flag wait).  Every step copies the slot mappings host->device from
    # pinned memory and reads the completion status back.
    e2e = None
    if not a.no_e2e:
        from lmcache_ascend_b200.config import LMCacheEngineConfig, LMCacheEngineMetadata
        from lmcache_ascend_b200.v1.cache_engine import LMCacheEngine
        from lmcache_ascend_b200.v1.gpu_connector import VLLMPagedMemGPUConnector

        base = dict(chunk_size=256, enable_pd=True, transfer_channel="nvlink",
                    pd_buffer_device="cuda", pd_buffer_size=32 << 20, local_cpu=False,
                    max_local_cpu_size=0.01, pd_peer_init_port=[0], pd_peer_alloc_port=[0])
        md = LMCacheEngineMetadata("Qwen3-32B", max(1, world // 2), rank % max(1, world // 2),
                                   "vllm", torch.bfloat16)
        eng_r = eng_s = None
        if role_d:
            rc = LMCacheEngineConfig.from_defaults(pd_role="receiver", **base)
            eng_r = LMCacheEngine(rc, md, VLLMPagedMemGPUConnector(rc, kvcaches=dst_cache))
            eng_r.post_init()
            urls = eng_r.storage_manager.backends["PDBackend"].endpoints()
        else:
            urls = None
        if world > 1:
            allu = [None] * world
            dist.all_gather_object(allu, urls, group=gloo)
        else:
            allu = [urls]
        if role_p:
            iu, au = allu[rank + world // 2] if world > 1 else allu[0]
            sc = LMCacheEngineConfig.from_defaults(pd_role="sender", **base)
            eng_s = LMCacheEngine(sc, md, VLLMPagedMemGPUConnector(sc, kvcaches=src_cache),
                                  peer_init_url=iu, peer_alloc_url=au)
            eng_s.post_init()
        # the step's inputs live in pinned host memory: the engine copies them
        # to the device (and digests the destination slots for the grant)
        h_src = src_slots.cpu().pin_memory()
        h_dst = dst_slots.cpu().pin_memory()
        # each step reads its completion status back (D2H into pinned memory)
        # and the host checks it one step later, so step i+1's grant overlaps
        # step i's push on the device
        h_status = [torch.empty(4, dtype=torch.int64).pin_memory() for _ in range(2)]
        st_ev = [None, None]

        def check_status(b):
            if st_ev[b] is not None:
                st_ev[b].synchronize()
                if int(h_status[b][0]) != 0:
                    raise RuntimeError(f"push reported status {h_status[b].tolist()}")

        def e2e_step(i):
            b = hash(i) & 1
            check_status(b)
            if eng_r is not None:  # the decoder's allocation for this request
                eng_r.reserve_direct_prefill(f"bench-{i}", h_dst)
            if eng_s is not None:
                eng_s.store_direct_prefill(slot_mapping=h_src, dst_slot_mapping=h_dst,
                                           req_id=f"bench-{i}")
                pd = eng_s.storage_manager.backends["PDBackend"]
                h_status[b].copy_(pd.push_sender.status.tensor, non_blocking=True)
            if eng_r is not None:
                if not eng_r.wait_direct_prefill(f"bench-{i}", timeout_s=10.0):
                    raise RuntimeError("decoder never granted the push")
                pd = eng_r.storage_manager.backends["PDBackend"]
                h_status[b].copy_(pd.push_receiver.status.tensor, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            st_ev[b] = ev

        for i in range(a.warmup):
            e2e_step(f"w{i}")
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(a.steps):
            e2e_step(i)
        t1.record()
        torch.cuda.synchronize()
        check_status(0)
        check_status(1)
        ems = torch.tensor([t0.elapsed_time(t1) / a.steps], device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        ems = float(ems.item())
        barrier()
        e2e = {"value": round(bytes_per_pair * pairs / (ems / 1e3) / 1e9, 2), "unit": "GB/s",
               "ms_per_step": round(ems, 4),
               "h2d_bytes_per_step": (src_slots.numel() + dst_slots.numel()) * 4 * pairs,
               "d2h_bytes_per_step": 32 * world,
               "api": "LMCacheEngine.reserve_direct_prefill (decoder) / store_direct_prefill "
                      "(prefiller: grant, then push) / wait_direct_prefill (decoder)"}
        for e in (eng_s, eng_r):
            if e is not None:
                e.close()

    # ------------------------------------------------------ TTFT on a hit
    # Second half of the headline metric: every rank serves a 16k-token
    # prefix hit of Qwen3-32B (TP1, random init) from its own CPU tier
    # through the engine API; p50 over requests, max over ranks.
    ttft = None
    if not a.no_ttft:
        for c in (src_cache, dst_cache):
            if c is not None:
                c.clear()
        torch.cuda.empty_cache()
        barrier()
        from lmcache_ascend_b200.bench_ttft import run_ttft

        ttft = run_ttft(dev, tokens=a.tokens, requests=a.ttft_requests, warmup=3)
        p50 = torch.tensor([ttft["p50_ms"]], device=dev)
        if world > 1:
            dist.all_reduce(p50, op=dist.ReduceOp.MAX)
        ttft["p50_ms_max_over_ranks"] = round(float(p50.item()), 3)
        barrier()
        # the same hit served from the HBM tier (the prefix kept on the GPU)
        ttft_hbm = run_ttft(dev, tokens=a.tokens, requests=a.ttft_requests, warmup=3,
                            tier="hbm")
        p50 = torch.tensor([ttft_hbm["p50_ms"]], device=dev)
        if world > 1:
            dist.all_reduce(p50, op=dist.ReduceOp.MAX)
        ttft_hbm["p50_ms_max_over_ranks"] = round(float(p50.item()), 3)
        ttft["hbm_tier"] = ttft_hbm
        barrier()

    # ------------------------------------ push hidden under the prefill
    # The serving path: a Qwen3-32B TP4-shard prefill forward of the prompt,
    # the vLLM connector's save_kv_layer pushing each layer behind its KV
    # write; (forward + push) / forward, max over ranks.
    overlap = None
    if not a.no_overlap:
        for c_ in (src_cache, dst_cache):
            if c_ is not None:
                c_.clear()
        torch.cuda.empty_cache()
        barrier()
        from lmcache_ascend_b200.bench_overlap import run_prefill_overlap

        overlap = run_prefill_overlap(dev, rank, world, gloo, tokens=a.tokens,
                                      iters=a.overlap_iters, warmup=1)
        barrier()

    # ------------------- config 5: DeepSeek-V3.2 latent + C8 indexer push
    config5 = None
    if not a.no_config5:
        torch.cuda.empty_cache()
        barrier()
        from lmcache_ascend_b200.bench_config5 import run_config5

        config5 = run_config5(dev, rank, world, gloo, warmup=max(3, a.warmup),
                              peer_copy_gbps=peer_copy["gbps_per_pair"] if peer_copy else None)
        barrier()

    # ------------------- config 2: local offload, one replica per GPU
    config2 = None
    if not a.no_config2:
        torch.cuda.empty_cache()
        barrier()
        from lmcache_ascend_b200.bench_config2 import run_config2

        config2 = run_config2(dev, rank, world, gloo, requests=a.config2_requests)
        barrier()

    if rank == 0:
        per_pair = value / pairs
        if world == 1:
            hbm = measured_hbm_gbps()
            roof = {"bound": "HBM (loopback: read + write)",
                    "frac_of_measured_hbm": round(2 * per_pair / hbm, 4),
                    "measured_hbm_gbps": hbm}
        else:
            roof = {"bound": "NVLink per direction per pair",
                    "frac_of_measured_peer_copy": (round(per_pair / peer_copy["gbps_per_pair"], 4)
                                                   if peer_copy else None),
                    "frac_of_nominal_900": round(per_pair / NVLINK_NOMINAL_GBPS, 4),
                    "peer_copy": peer_copy}
        # this repo's kernels per timed step: one push per prefiller (it also
        # releases the flags) and one bounded flag wait per decoder
        launches = a.steps * (2 if world == 1 else world)
        out({"metric": "kv_push_gbps", "value": round(value, 2), "unit": "GB/s",
             "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
             "higher_is_better": True, "scaling": "weak",
             "vs_baseline": round(value / baseline["value"], 3) if baseline else None,
             "vs_baseline_of": "the NCCL + index_copy_ arm of this run (no published "
                               "reference number exists for this metric)",
             "impl": a.impl, "engine": a.engine, "dtype": "bf16",
             "data": "synthetic (random-init bf16 KV of the Qwen3-32B TP4 shard shape, "
                     "random block tables)",
             "config": cfg, "bytes_per_pair_per_step": bytes_per_pair,
             "per_pair_gbps": round(per_pair, 2), "roofline": roof, "baseline": baseline,
             "clocks": ck, "e2e": e2e, "gpu_launches": launches, "ttft": ttft,
             "push_fp8": fp8, "prefill_overlap": overlap, "config5_dsv32_mla_c8": config5,
             "config2_llama3_8b_offload": config2,
             **({"multicast": mcast} if mcast is not None else {})})
    if sender is not None:
        sender.close()
    if world > 1:
        dist.barrier(group=gloo)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
