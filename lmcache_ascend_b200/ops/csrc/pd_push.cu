// K9: fused disaggregated-prefill KV push over NVLink peer memory.
//
// The reference moves prefill KV to the decoder in two steps: a connector
// gather into registered chunk buffers, then one RDMA write per chunk page
// (`HcclAgent::WriteBatch`, reference csrc/hccl/hccl_agent.cpp:297-326, driven
// by lmcache_ascend/v1/storage_backend/pd/sender_mixin.py:339-423).  On B200
// every GPU of the box reaches every other GPU's HBM through NVSwitch, so the
// push is one kernel: it reads the prefiller's paged rows (its own HBM) and
// stores them straight into the decoder's paged blocks through peer-mapped
// addresses, with no staging buffer, no NCCL call and no TMA multicast.
//
// Completion protocol (per layer, so the decoder can start layer l while the
// prefiller still pushes l+1):
//   * each CTA finishing a unit (layer, plane, token tile) runs
//     __syncthreads(); fence.acq_rel.sys; red.release.sys.add(flag[l], 1)
//     on the decoder's flag word for layer l (the flag lives in decoder HBM);
//   * the decoder waits with `pd_wait_flags`, a bounded acquire spin that
//     reports kStatusFlagTimeout instead of hanging.
// Flags are cumulative counters: the receiver knows how many units each push
// adds (`push_units_per_layer`) and waits for base + units.
//
// Fan-out: one launch may store the same rows to up to kMaxReplicas decoder
// caches (TP-replicated MLA latent cache); loads happen once.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "kv_copy.cuh"
#include "mem_kernels.h"

namespace lmc {

constexpr int kMaxReplicas = 4;
constexpr int kPushWarps = 4;

struct PushJob {
  PagedDesc src;
  PagedDesc dst;  // dst.ptrs: [replicas][num_layers * num_planes] peer VAs
  const void *src_slots;
  const void *dst_slots;
  int32_t slot_is_i64;
  int32_t num_tokens;
  int32_t layer_begin;
  int32_t num_layers;
  int32_t tile_tokens;
  int32_t replicas;
  unsigned *flags[kMaxReplicas];  // per replica: flag array [num_layers_total]
  DeviceStatus *status;
};

__device__ __forceinline__ int64_t push_slot(const void *p, int is64, int t) {
  return is64 ? static_cast<const int64_t *>(p)[t]
              : static_cast<int64_t>(static_cast<const int32_t *>(p)[t]);
}

// One CTA (kPushWarps warps) per unit = (layer, plane, tile of tokens).
// The CTA streams the unit's rows as a flat array of 16-byte vectors: each
// thread resolves the rows of its vectors directly (slot loads are warp
// broadcasts; 32-bit slot arithmetic), keeps kVecPerThread independent loads
// in flight and then stores them to every replica.  One barrier + one
// system-scope release per unit publishes the unit to the decoder.  Small
// CTAs keep several units per SM in flight so one CTA's release latency is
// hidden behind the others' copies.
constexpr int kMaxTile = 1024;
constexpr int kVecPerThread = 8;

__device__ __forceinline__ unsigned row_off(const PagedDesc &pd, const PlaneDesc &pl,
                                            unsigned slot) {
  const unsigned bs = static_cast<unsigned>(pd.block_size);
  const unsigned b = slot / bs;
  return static_cast<unsigned>(static_cast<int64_t>(b) * pl.block_stride +
                               static_cast<int64_t>(slot - b * bs) * pl.slot_stride);
}

// Byte offset of row byte `vb` inside the paged row: identity for
// contiguous rows, (vb / seg) * seg_stride + vb % seg for head-major rows.
__device__ __forceinline__ unsigned seg_off(const PlaneDesc &pl, unsigned vb) {
  if (pl.seg_bytes <= 0 || pl.seg_bytes >= pl.row_bytes) return vb;
  const unsigned sb = static_cast<unsigned>(pl.seg_bytes);
  const unsigned q = vb / sb;
  return static_cast<unsigned>(q * pl.seg_stride) + (vb - q * sb);
}

__global__ void __launch_bounds__(kPushWarps * 32)
    pd_push_kernel(PushJob j) {
  const int np = j.src.num_planes;
  const int tiles = (j.num_tokens + j.tile_tokens - 1) / j.tile_tokens;
  const int units_per_layer = np * tiles;
  const int total = units_per_layer * j.num_layers;
  const int tid = threadIdx.x;
  constexpr int kThreads = kPushWarps * 32;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    const int li = u / units_per_layer;
    const int rem = u - li * units_per_layer;
    const int p = rem / tiles;
    const int tile = rem - p * tiles;
    const int layer = j.layer_begin + li;
    const PlaneDesc spl = j.src.plane[p];
    const PlaneDesc dpl = j.dst.plane[p];
    const int rb = spl.row_bytes;
    const int t0 = tile * j.tile_tokens;
    const int n = min(j.num_tokens - t0, j.tile_tokens);
    const char *sbase = reinterpret_cast<const char *>(j.src.ptrs[layer * np + p]);
    if ((rb & 15) == 0) {
      const int vpr = rb >> 4;  // vectors per row
      const int nv = n * vpr;
      for (int base = 0; base < nv; base += kThreads * kVecPerThread) {
        int4 v[kVecPerThread];
        unsigned so[kVecPerThread], dp[kVecPerThread];
#pragma unroll
        for (int k = 0; k < kVecPerThread; ++k) {
          const int g = base + k * kThreads + tid;
          so[k] = ~0u;
          if (g < nv) {
            const int ti = g / vpr;
            const unsigned vb = static_cast<unsigned>(g - ti * vpr) * 16u;
            const int64_t ss = push_slot(j.src_slots, j.slot_is_i64, t0 + ti);
            const int64_t dd = push_slot(j.dst_slots, j.slot_is_i64, t0 + ti);
            if (ss >= 0 && dd >= 0) {
              if (ss >= j.src.num_slots || dd >= j.dst.num_slots) {
                if (vb == 0) report_status(j.status, kStatusBadSlot, t0 + ti, ss, dd);
              } else {
                so[k] = row_off(j.src, spl, static_cast<unsigned>(ss)) + seg_off(spl, vb);
                dp[k] = row_off(j.dst, dpl, static_cast<unsigned>(dd)) + seg_off(dpl, vb);
              }
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kVecPerThread; ++k)
          if (so[k] != ~0u) v[k] = ld_nc_v4(sbase + so[k]);
        for (int r = 0; r < j.replicas; ++r) {
          char *db = reinterpret_cast<char *>(
              j.dst.ptrs[(static_cast<int64_t>(r) * j.dst.num_layers + layer) * np + p]);
#pragma unroll
          for (int k = 0; k < kVecPerThread; ++k)
            if (so[k] != ~0u) st_cs_v4(db + dp[k], v[k]);
        }
      }
    } else {
      for (int g = tid; g < n * rb; g += kThreads) {
        const int ti = g / rb;
        const int bi = g - ti * rb;
        const int64_t ss = push_slot(j.src_slots, j.slot_is_i64, t0 + ti);
        const int64_t dd = push_slot(j.dst_slots, j.slot_is_i64, t0 + ti);
        if (ss < 0 || dd < 0 || ss >= j.src.num_slots || dd >= j.dst.num_slots) continue;
        const unsigned so = row_off(j.src, spl, static_cast<unsigned>(ss));
        const unsigned dof = row_off(j.dst, dpl, static_cast<unsigned>(dd));
        for (int r = 0; r < j.replicas; ++r) {
          char *db = reinterpret_cast<char *>(
              j.dst.ptrs[(static_cast<int64_t>(r) * j.dst.num_layers + layer) * np + p]);
          db[dof + seg_off(dpl, bi)] = sbase[so + seg_off(spl, bi)];
        }
      }
    }
    // publish this unit: every thread's stores are ordered before the release
    __syncthreads();
    if (tid == 0) {
      fence_acq_rel_sys();
      for (int r = 0; r < j.replicas; ++r)
        if (j.flags[r]) red_release_sys_add(j.flags[r] + layer, 1u);
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk (TMA) push: the default engine for 16-byte aligned, contiguous rows.
//
// Work: every unit (layer, plane, tile of `tile_tokens` tokens; the units and
// flag counts of pd_push_kernel) is cut into pieces of at most 64 tokens that
// fit one shared-memory stage, with the same number of pieces for every tile
// of a plane (the last tile's surplus pieces are empty).  The pieces of the
// launch are numbered layer-major and each warp takes one contiguous range
// of them, so every warp moves the same amount whatever the tile size, and
// consecutive pieces of a warp are neighbours in memory.
//
// Per piece the warp's lanes plan runs of tokens contiguous on both sides
// (plan_runs), load them from this GPU's paged cache with
// `cp.async.bulk.shared::cta.global` (mbarrier completion; never multicast)
// and write them to the destination's paged blocks -- local or peer memory
// -- with `cp.async.bulk.global.shared::cta`, one bulk group per piece.
// Stage reuse waits for `cp.async.bulk.wait_group.read 1` only.
//
// Flags: a unit may be shared by two warps.  When a warp is done with its
// part of a unit and those writes have completed (`cp.async.bulk.wait_group
// kLag`, kLag pieces later, which by then costs nothing), lane 0 adds its
// piece count to the unit's counter in this GPU's memory (acq_rel, GPU
// scope); the warp that brings the count to the unit's piece total resets
// the counter for the next launch and publishes the unit: system fence, then
// red.release.sys.add on the decoder's layer flag.  The counters therefore
// start and end every launch at zero.
// ---------------------------------------------------------------------------
constexpr int kBulkWarps = 2;
constexpr int kBulkStages = 2;
constexpr int kBulkStageBytes = 8192;
constexpr int kBulkLag = 4;       // pieces between the end of a unit part and its release
constexpr int kBulkPending = 4;   // unit parts that may wait for their release
constexpr int kTmaRingOffset = 128;  // mbarriers (warps * stages * 8 bytes) come first
static_assert(kBulkWarps * kBulkStages * 8 <= kTmaRingOffset, "mbarrier area too small");

__device__ __forceinline__ unsigned warp_sum_u32(unsigned v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct BulkPushJob {
  CopyJob c;                       // src paged + replica-0 dst paged + slots
  const int64_t *dst_ptrs;         // [replicas][dst_layers * planes] destination bases
  int32_t dst_layers;              // layers per replica in dst_ptrs
  int32_t replicas;
  int32_t tile_tokens;             // flag unit
  int32_t stage_bytes;
  unsigned *flags[kMaxReplicas];   // per replica: layer flag array (or null)
  unsigned long long budget_ns;    // bound on each mbarrier wait
  uint32_t bulk_planes;            // bit p: plane p moves by TMA bulk copies, else by
                                   // per-lane loads/stores (rows not 16-byte aligned)
  unsigned *counters;              // [units of this launch], zero between launches
  bool gpu_scope;                  // every destination (and its waiter) on this GPU
};

// Publish a finished unit: order this thread's earlier writes (and, through
// the counters' acq_rel, the other warps' writes of the unit) before the
// flag increments.  System scope when a destination is a peer GPU.
__device__ __forceinline__ void bulk_publish(const BulkPushJob &j, int layer) {
  if (j.gpu_scope) {
    fence_acq_rel_gpu();
    for (int r = 0; r < j.replicas; ++r)
      if (j.flags[r]) red_release_gpu_add(j.flags[r] + layer, 1u);
  } else {
    fence_acq_rel_sys();
    for (int r = 0; r < j.replicas; ++r)
      if (j.flags[r]) red_release_sys_add(j.flags[r] + layer, 1u);
  }
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_complete() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned *p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

// One row of `rb` bytes with the widest granule both addresses allow.
__device__ __forceinline__ void copy_row_granules(char *dst, const char *src, int rb) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                      static_cast<uintptr_t>(rb);
  if ((a & 15) == 0) {
    for (int o = 0; o < rb; o += 16)
      *reinterpret_cast<int4 *>(dst + o) = *reinterpret_cast<const int4 *>(src + o);
  } else if ((a & 7) == 0) {
    for (int o = 0; o < rb; o += 8)
      *reinterpret_cast<long long *>(dst + o) = *reinterpret_cast<const long long *>(src + o);
  } else if ((a & 3) == 0) {
    for (int o = 0; o < rb; o += 4)
      *reinterpret_cast<int *>(dst + o) = *reinterpret_cast<const int *>(src + o);
  } else {
    for (int o = 0; o < rb; ++o) dst[o] = src[o];
  }
}

// A piece, decoded from its index in the launch.
struct PieceAt {
  int unit;    // unit index in the launch: (layer * planes + plane) * tiles + tile
  int layer;   // layer index in the launch
  int plane;
  int ppu;     // pieces of this unit
  bool last;   // last piece of its unit
  Unit u;      // tokens of the piece (u.n <= 0: an empty trailing piece)
};

__global__ void __launch_bounds__(kBulkWarps * 32, 6)
    pd_push_bulk_kernel(BulkPushJob j) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int S = kBulkStages;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * S;
  unsigned char *ring =
      smem + kTmaRingOffset + static_cast<size_t>(warp) * S * j.stage_bytes;
  const CopyJob &c = j.c;
  const int np = c.paged.num_planes;
  const int tiles = (c.num_tokens + j.tile_tokens - 1) / j.tile_tokens;
  const int gw = blockIdx.x * kBulkWarps + warp;
  const int nw = gridDim.x * kBulkWarps;
  // pieces per unit and tokens per piece of each plane (0 pieces: not bulk)
  auto piece_tokens = [&](int p) {
    const int t = j.stage_bytes / plane_of(c.paged, p).row_bytes;
    return t > 64 ? 64 : (t < 1 ? 1 : t);
  };
  auto ppu_of = [&](int p) {
    if (p >= np || !((j.bulk_planes >> p) & 1u)) return 0;
    return (j.tile_tokens + piece_tokens(p) - 1) / piece_tokens(p);
  };
  const int ppu0 = ppu_of(0), ppu1 = ppu_of(1), ppu2 = ppu_of(2);
  const long long per_layer = static_cast<long long>(tiles) * (ppu0 + ppu1 + ppu2);
  const long long total = per_layer * c.num_layers;
  const long long base = total / nw, extra = total % nw;
  const long long first = gw * base + min(static_cast<long long>(gw), extra);
  const long long count = base + (gw < extra ? 1 : 0);

  // Position of a piece, advanced one piece at a time (a warp's pieces are
  // consecutive): layer in launch, plane, tile, piece in the unit.
  struct Cur {
    int li, p, tile, pc;
  };
  auto ppu_p = [&](int p) { return p == 0 ? ppu0 : (p == 1 ? ppu1 : ppu2); };
  auto seek = [&](long long q) {  // one division-based decode per warp
    Cur r;
    r.li = static_cast<int>(q / per_layer);
    long long rem = q - r.li * per_layer;
    r.p = 0;
    while (r.p < 2 && rem >= static_cast<long long>(tiles) * ppu_p(r.p)) {
      rem -= static_cast<long long>(tiles) * ppu_p(r.p);
      ++r.p;
    }
    const int ppu = ppu_p(r.p);
    r.tile = static_cast<int>(rem / ppu);
    r.pc = static_cast<int>(rem - static_cast<long long>(r.tile) * ppu);
    return r;
  };
  auto step_cur = [&](Cur &r) {
    if (++r.pc < ppu_p(r.p)) return;
    r.pc = 0;
    if (++r.tile < tiles) return;
    r.tile = 0;
    do {  // next plane with pieces, else the next layer's first one
      if (++r.p >= np) {
        r.p = 0;
        ++r.li;
      }
    } while (ppu_p(r.p) == 0);
  };
  auto piece_of = [&](const Cur &r) {
    PieceAt a;
    const int per = piece_tokens(r.p);
    const int tend = min(c.num_tokens, (r.tile + 1) * j.tile_tokens);
    a.unit = (r.li * np + r.p) * tiles + r.tile;
    a.layer = r.li;
    a.plane = r.p;
    a.ppu = ppu_p(r.p);
    a.last = r.pc == a.ppu - 1;
    a.u.layer = r.li;
    a.u.plane = r.p;
    a.u.t0 = r.tile * j.tile_tokens + r.pc * per;
    a.u.n = min(per, tend - a.u.t0);
    return a;
  };

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  Cur lcur = seek(first), scur = lcur;  // load and store cursors
  auto issue_loads = [&](long long k) {
    const PieceAt pa = piece_of(lcur);
    step_cur(lcur);
    const int s = static_cast<int>(k % S);
    unsigned bytes = 0;
    LaneRuns r;
    r.len[0] = r.len[1] = 0;
    if (pa.u.n > 0) {
      r = plan_runs(c, pa.u, lane, c.num_tokens);
      bytes = warp_sum_u32((r.len[0] + r.len[1]) * plane_of(c.paged, pa.plane).row_bytes);
    }
    if (lane == 0) mbar_arrive_expect_tx(&bars[s], bytes);
    __syncwarp();
    const unsigned rb = plane_of(c.paged, pa.plane).row_bytes;
    unsigned char *buf = ring + static_cast<size_t>(s) * j.stage_bytes;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (r.len[h]) bulk_g2s(buf + (h * 32 + lane) * rb, r.src[h], r.len[h] * rb, &bars[s]);
  };

  // Unit parts waiting for their writes, oldest first: unit (-1: empty slot),
  // pieces done by this warp, layer, index of the part's last piece.
  // Constant indices only, so the queue lives in registers.
  int qu[kBulkPending], qc[kBulkPending], ql[kBulkPending];
  long long qk[kBulkPending];
#pragma unroll
  for (int i = 0; i < kBulkPending; ++i) qu[i] = -1, qc[i] = 0, ql[i] = 0, qk[i] = 0;
  auto settle_front = [&](int ppu_front) {
    if (lane == 0) {
      const unsigned before = atom_add_acq_rel_gpu(j.counters + qu[0],
                                                   static_cast<unsigned>(qc[0]));
      if (before + static_cast<unsigned>(qc[0]) == static_cast<unsigned>(ppu_front)) {
        j.counters[qu[0]] = 0u;  // ready for the next launch
        bulk_publish(j, c.layer_begin + ql[0]);
      }
    }
#pragma unroll
    for (int i = 0; i + 1 < kBulkPending; ++i)
      qu[i] = qu[i + 1], qc[i] = qc[i + 1], ql[i] = ql[i + 1], qk[i] = qk[i + 1];
    qu[kBulkPending - 1] = -1;
  };
  auto ppu_unit = [&](int unit) {
    const int p = (unit / tiles) % np;
    return p == 0 ? ppu0 : (p == 1 ? ppu1 : ppu2);
  };
  // settle every queued part whose last piece is <= kdone (its writes are done)
  auto settle_upto = [&](long long kdone) {
    if (qu[0] < 0 || qk[0] > kdone) return;
    fence_proxy_async_global();  // completed bulk writes before the generic atomics
    __syncwarp();
#pragma unroll
    for (int i = 0; i < kBulkPending; ++i)
      if (qu[0] >= 0 && qk[0] <= kdone) settle_front(ppu_unit(qu[0]));
  };
  auto enqueue = [&](int unit, int cnt, int layer, long long k) {
    if (qu[kBulkPending - 1] >= 0) {  // full: drain every outstanding write
      bulk_wait_complete<0>();
      settle_upto(0x7fffffffffffffffll);
    }
    bool placed = false;
#pragma unroll
    for (int i = 0; i < kBulkPending; ++i)
      if (!placed && qu[i] < 0) qu[i] = unit, qc[i] = cnt, ql[i] = layer, qk[i] = k,
                                placed = true;
  };

  long long kl = 0;
  for (; kl < S - 1 && kl < count; ++kl) issue_loads(kl);
  int cur_unit = -1, cur_cnt = 0, cur_layer = 0;
  for (long long k = 0; k < count; ++k) {
    const int s = static_cast<int>(k % S);
    const unsigned parity = static_cast<unsigned>((k / S) & 1);
    if (!mbar_wait_bounded(&bars[s], parity, j.budget_ns)) {
      if (lane == 0) report_status(c.status, kStatusMbarTimeout, gw, static_cast<long long>(k),
                                   0);
      break;
    }
    const PieceAt pa = piece_of(scur);
    step_cur(scur);
    if (pa.u.n > 0) {
      const LaneRuns r = plan_runs(c, pa.u, lane, c.num_tokens);
      const unsigned rb = plane_of(c.paged, pa.plane).row_bytes;
      const unsigned char *buf = ring + static_cast<size_t>(s) * j.stage_bytes;
      const int layer = c.layer_begin + pa.layer;
      const int64_t slot0 = static_cast<int64_t>(layer) * np + pa.plane;
      const char *base0 = reinterpret_cast<const char *>(j.dst_ptrs[slot0]);
      for (int rep = 0; rep < j.replicas; ++rep) {
        const char *dbase = reinterpret_cast<const char *>(
            j.dst_ptrs[static_cast<int64_t>(rep) * j.dst_layers * np + slot0]);
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (r.len[h])
            bulk_s2g(const_cast<char *>(dbase) + (r.dst[h] - base0),
                     buf + (h * 32 + lane) * rb, r.len[h] * rb);
      }
    }
    bulk_commit();
    if (pa.unit != cur_unit) {
      cur_unit = pa.unit;
      cur_cnt = 0;
      cur_layer = pa.layer;
    }
    ++cur_cnt;
    if (pa.last || k == count - 1) {  // this warp is done with its part of the unit
      enqueue(cur_unit, cur_cnt, cur_layer, k);
      cur_unit = -1;
    }
    if (qu[0] >= 0 && qk[0] <= k - kBulkLag) {
      bulk_wait_complete<kBulkLag>();  // pieces <= k - kBulkLag written
      settle_upto(k - kBulkLag);
    }
    if (kl < count) {
      bulk_wait_read<1>();  // piece k - 1 has read its stage
      __syncwarp();
      issue_loads(kl);
      ++kl;
    }
  }
  bulk_wait_complete<0>();
  settle_upto(0x7fffffffffffffffll);

  // Units of planes whose rows are not 16-byte aligned (the 4-byte scale
  // plane of a C8 indexer, say): one token per lane, widest aligned granule,
  // published right after the warp's stores (generic proxy only).
  if (j.bulk_planes == (1u << np) - 1u) return;
  const int units = np * tiles * c.num_layers;
  for (int u = gw; u < units; u += nw) {
    const int li = u / (np * tiles);
    const int p = (u - li * np * tiles) / tiles;
    if ((j.bulk_planes >> p) & 1u) continue;
    const int t0 = (u - li * np * tiles - p * tiles) * j.tile_tokens;
    const int n = min(c.num_tokens - t0, j.tile_tokens);
    const int layer = c.layer_begin + li;
    const PlaneDesc sp = plane_of(c.paged, p);
    const PlaneDesc dp = plane_of(c.dst_paged, p);
    const char *sb = reinterpret_cast<const char *>(c.paged.ptrs[layer * np + p]);
    for (int t = lane; t < n; t += 32) {
      const int64_t ss = push_slot(c.slots, c.slot_is_i64, t0 + t);
      const int64_t dd = push_slot(c.dst_slots, c.slot_is_i64, t0 + t);
      if (ss < 0 || dd < 0) continue;
      if (ss >= c.paged.num_slots || dd >= c.dst_paged.num_slots) {
        report_status(c.status, kStatusBadSlot, t0 + t, ss, dd);
        continue;
      }
      const char *src = sb + (ss / c.paged.block_size) * sp.block_stride +
                        (ss % c.paged.block_size) * sp.slot_stride;
      const int64_t doff = (dd / c.dst_paged.block_size) * dp.block_stride +
                           (dd % c.dst_paged.block_size) * dp.slot_stride;
      for (int rep = 0; rep < j.replicas; ++rep) {
        char *db = reinterpret_cast<char *>(
            j.dst_ptrs[static_cast<int64_t>(rep) * j.dst_layers * np + layer * np + p]);
        copy_row_granules(db + doff, src, sp.row_bytes);
      }
    }
    __syncwarp();
    if (lane == 0) bulk_publish(j, layer);
  }
}

// ---------------------------------------------------------------------------
// Block-scaled fp8 push.  The prefiller reads bf16 paged rows, quantises
// every group of G consecutive elements (G = 128: one head of head_dim 128)
// to e4m3 with scale = amax / 448, and stores the fp8 bytes plus the fp32
// scales into a staging area in the decoder's HBM (through peer addresses),
// halving the bytes that cross NVLink.  Staging is laid out by push token
// order: q[(layer * planes + plane) * T + t][row_elems], scales
// [(layer * planes + plane) * T + t][row_elems / G].  The per-layer flags are
// released exactly as in pd_push_kernel; the decoder then runs
// pd_dequant_scatter_kernel from its staging into its bf16 paged cache.
// ---------------------------------------------------------------------------
struct PushQJob {
  PagedDesc src;
  const void *src_slots;
  int32_t slot_is_i64;
  int32_t num_tokens;     // tokens in this push (staging rows per layer plane)
  int32_t layer_begin;
  int32_t num_layers;
  int32_t tile_tokens;
  int32_t group;          // elements per scale group (multiple of 128 / 16 lanes)
  uint8_t *q;             // peer staging, fp8
  float *scales;          // peer staging, fp32
  unsigned *flags;
  DeviceStatus *status;
  int32_t gpu_scope;      // the staging (and its waiter) is on this GPU
};

__device__ __forceinline__ float bf16x2_lo(uint32_t w) {
  return __uint_as_float(w << 16);
}
__device__ __forceinline__ float bf16x2_hi(uint32_t w) {
  return __uint_as_float(w & 0xFFFF0000u);
}

constexpr int kQVec = 4;  // groups (half-warp items) per thread in flight

// An 8-lane quarter-warp owns one 128-element segment of a group: lane i
// holds elements 16i .. 16i+15 (two 16-byte loads, one 16-byte fp8 store).
template <int SPG>  // 128-element segments per scale group (group = 128 * SPG)
__global__ void __launch_bounds__(kPushWarps * 32) pd_push_fp8_kernel(PushQJob j) {
  const int np = j.src.num_planes;
  const int tiles = (j.num_tokens + j.tile_tokens - 1) / j.tile_tokens;
  const int units_per_layer = np * tiles;
  const int total = units_per_layer * j.num_layers;
  const int tid = threadIdx.x;
  const int quarter = tid >> 3;    // quarter-warp index in the CTA
  const int ql = tid & 7;          // lane within the quarter-warp
  constexpr int kQuarters = kPushWarps * 4;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    const int li = u / units_per_layer;
    const int rem = u - li * units_per_layer;
    const int p = rem / tiles;
    const int tile = rem - p * tiles;
    const int layer = j.layer_begin + li;
    const PlaneDesc spl = j.src.plane[p];
    const int row_elems = spl.row_bytes >> 1;
    const int gpr = row_elems / j.group;       // groups per row
    const int t0 = tile * j.tile_tokens;
    const int n = min(j.num_tokens - t0, j.tile_tokens);
    const char *sbase = reinterpret_cast<const char *>(j.src.ptrs[layer * np + p]);
    const int64_t rowq0 = (static_cast<int64_t>(layer) * np + p) * j.num_tokens;
    const int items = n * gpr;                 // (token, group) pairs of this unit
    for (int base = 0; base < items; base += kQuarters * kQVec) {
      uint4 v[kQVec][SPG][2];
      int ti_[kQVec], gi_[kQVec];
      bool ok[kQVec];
#pragma unroll
      for (int k = 0; k < kQVec; ++k) {
        const int it = base + k * kQuarters + quarter;
        ok[k] = false;
        ti_[k] = gi_[k] = 0;
        if (it < items) {
          const int ti = it / gpr;
          const int gi = it - ti * gpr;
          ti_[k] = ti;
          gi_[k] = gi;
          const int64_t ss = push_slot(j.src_slots, j.slot_is_i64, t0 + ti);
          if (ss >= 0 && ss < j.src.num_slots) {
            ok[k] = true;
            const unsigned ro = row_off(j.src, spl, static_cast<unsigned>(ss));
#pragma unroll
            for (int sgi = 0; sgi < SPG; ++sgi) {
#pragma unroll
              for (int hv = 0; hv < 2; ++hv) {
                const unsigned vb =
                    static_cast<unsigned>(gi * j.group + sgi * 128 + ql * 16 + hv * 8) * 2u;
                const int4 x = ld_nc_v4(sbase + ro + seg_off(spl, vb));
                v[k][sgi][hv] = make_uint4(static_cast<unsigned>(x.x), static_cast<unsigned>(x.y),
                                           static_cast<unsigned>(x.z), static_cast<unsigned>(x.w));
              }
            }
          } else if (ss >= j.src.num_slots && ql == 0 && gi == 0) {
            report_status(j.status, kStatusBadSlot, t0 + ti, ss, j.src.num_slots);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kQVec; ++k) {
        float amax = 0.f;
        if (ok[k]) {
#pragma unroll
          for (int sgi = 0; sgi < SPG; ++sgi) {
#pragma unroll
            for (int hv = 0; hv < 2; ++hv) {
              const uint32_t w[4] = {v[k][sgi][hv].x, v[k][sgi][hv].y, v[k][sgi][hv].z,
                                     v[k][sgi][hv].w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                amax = fmaxf(amax, fmaxf(fabsf(bf16x2_lo(w[e])), fabsf(bf16x2_hi(w[e]))));
            }
          }
        }
#pragma unroll
        for (int o = 4; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (!ok[k]) continue;
        // A group whose largest magnitude is below 448 / FLT_MAX (bf16
        // subnormals) would get an infinite inverse scale and turn its zeros
        // into NaN (0 * inf): such a group is sent as zeros with scale 0.
        float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
        const bool tiny = !(inv <= 3.402823466e38f);
        if (tiny) inv = 0.f;
        const int64_t row = rowq0 + t0 + ti_[k];
        uint8_t *qrow = j.q + row * row_elems + static_cast<int64_t>(gi_[k]) * j.group;
#pragma unroll
        for (int sgi = 0; sgi < SPG; ++sgi) {
          uint32_t packed[4];
#pragma unroll
          for (int hv = 0; hv < 2; ++hv) {
            const uint32_t w[4] = {v[k][sgi][hv].x, v[k][sgi][hv].y, v[k][sgi][hv].z,
                                   v[k][sgi][hv].w};
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
              const __nv_fp8x2_storage_t a = __nv_cvt_float2_to_fp8x2(
                  make_float2(bf16x2_lo(w[e]) * inv, bf16x2_hi(w[e]) * inv), __NV_SATFINITE,
                  __NV_E4M3);
              const __nv_fp8x2_storage_t b = __nv_cvt_float2_to_fp8x2(
                  make_float2(bf16x2_lo(w[e + 1]) * inv, bf16x2_hi(w[e + 1]) * inv),
                  __NV_SATFINITE, __NV_E4M3);
              packed[hv * 2 + (e >> 1)] =
                  static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
            }
          }
          *reinterpret_cast<uint4 *>(qrow + sgi * 128 + ql * 16) =
              make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
        if (ql == 0) j.scales[row * gpr + gi_[k]] = tiny ? 0.f : __fdiv_rn(amax, 448.f);
      }
    }
    __syncthreads();
    if (tid == 0 && j.flags) {
      if (j.gpu_scope) {
        fence_acq_rel_gpu();
        red_release_gpu_add(j.flags + layer, 1u);
      } else {
        fence_acq_rel_sys();
        red_release_sys_add(j.flags + layer, 1u);
      }
    }
  }
}

// Decoder side of the fp8 push: staging (fp8 rows + per-group scales) ->
// bf16 paged rows at dst_slots.  Same shape as the quantising push kernel run
// backwards: a CTA takes (layer, plane, tile of tokens) units, so the index
// math is per unit; an 8-lane quarter-warp owns one token's 128-element
// segments (lane i: elements 16i .. 16i+15, one 16-byte fp8 load and two
// 16-byte bf16 stores), and each lane keeps kDqSegs segments of loads in
// flight.  SPR: 128-element segments per row (upper bound; `spr` is exact).
constexpr int kDqWarps = 8;
constexpr int kDqSegs = 4;
constexpr int kDqTile = 256;

template <int SPR>
__global__ void __launch_bounds__(kDqWarps * 32) pd_dequant_scatter_kernel(
    PagedDesc dst, const uint8_t *__restrict__ q, const float *__restrict__ scales,
    const void *dst_slots, int slot_is_i64, int num_tokens, int layer_begin, int num_layers,
    int group, DeviceStatus *status) {
  constexpr int kTok = SPR >= kDqSegs ? 1 : kDqSegs / SPR;  // tokens per quarter in flight
  constexpr int kQuarters = kDqWarps * 4;
  const int np = dst.num_planes;
  const int row_elems = dst.plane[0].row_bytes >> 1;  // every plane has the same rows
  const int spr = row_elems >> 7;
  const int gpr = row_elems / group;
  const int tiles = (num_tokens + kDqTile - 1) / kDqTile;
  const int units_per_layer = np * tiles;
  const int total = units_per_layer * num_layers;
  const int quarter = threadIdx.x >> 3;
  const int ql = threadIdx.x & 7;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    const int li = u / units_per_layer;
    const int rem = u - li * units_per_layer;
    const int p = rem / tiles;
    const int tile = rem - p * tiles;
    const int layer = layer_begin + li;
    const PlaneDesc pl = plane_of(dst, p);
    char *dbase = reinterpret_cast<char *>(dst.ptrs[layer * np + p]);
    const int t0 = tile * kDqTile;
    const int n = min(num_tokens - t0, kDqTile);
    const int64_t row0 = (static_cast<int64_t>(layer) * np + p) * num_tokens + t0;
    for (int base = 0; base < n; base += kQuarters * kTok) {
      uint4 w[kTok][SPR];
      float sc[kTok][SPR];
      int64_t ds[kTok];
#pragma unroll
      for (int k = 0; k < kTok; ++k) {
        const int ti = base + k * kQuarters + quarter;
        ds[k] = -1;
        if (ti < n) {
          ds[k] = push_slot(dst_slots, slot_is_i64, t0 + ti);
          const int64_t row = row0 + ti;
#pragma unroll
          for (int s = 0; s < SPR; ++s) {
            if (s < spr) {
              w[k][s] = __ldg(reinterpret_cast<const uint4 *>(q + row * row_elems + s * 128 +
                                                              ql * 16));
              sc[k][s] = __ldg(scales + row * gpr + (s * 128) / group);
            }
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kTok; ++k) {
        if (ds[k] < 0) continue;
        if (ds[k] >= dst.num_slots) {
          if (ql == 0) report_status(status, kStatusBadSlot, t0 + base + k * kQuarters + quarter,
                                     ds[k], dst.num_slots);
          continue;
        }
        char *prow = dbase + row_off(dst, pl, static_cast<unsigned>(ds[k]));
#pragma unroll
        for (int s = 0; s < SPR; ++s) {
          if (s >= spr) continue;
          const uint32_t ww[4] = {w[k][s].x, w[k][s].y, w[k][s].z, w[k][s].w};
          uint32_t out[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
                  static_cast<__nv_fp8x2_storage_t>((ww[e] >> (16 * h)) & 0xFFFFu), __NV_E4M3);
              const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&hr));
              const __nv_bfloat162 bv = __floats2bfloat162_rn(f.x * sc[k][s], f.y * sc[k][s]);
              out[e * 2 + h] = *reinterpret_cast<const uint32_t *>(&bv);
            }
          }
          const unsigned vb = static_cast<unsigned>(s * 128 + ql * 16) * 2u;
          *reinterpret_cast<uint4 *>(prow + seg_off(pl, vb)) =
              make_uint4(out[0], out[1], out[2], out[3]);
          *reinterpret_cast<uint4 *>(prow + seg_off(pl, vb + 16)) =
              make_uint4(out[4], out[5], out[6], out[7]);
        }
      }
    }
  }
}

// Decoder side: one thread per layer waits (bounded) until
// flags[layer] - targets[i] >= 0.  Writes kStatusFlagTimeout on expiry.
__global__ void pd_wait_flags_kernel(const unsigned *flags,
                                     const unsigned *targets, int layer_begin,
                                     int num_layers,
                                     unsigned long long budget_ns,
                                     DeviceStatus *status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= num_layers) return;
  unsigned seen = 0;
  if (!wait_flag_geq(flags + layer_begin + i, targets[i], budget_ns, &seen))
    report_status(status, kStatusFlagTimeout, layer_begin + i, seen, targets[i]);
}

// One thread: bounded wait until *flag - target >= 0 (local or peer flag).
__global__ void pd_wait_value_kernel(const unsigned *flag, unsigned target,
                                     unsigned long long budget_ns, DeviceStatus *status) {
  unsigned seen = 0;
  if (!wait_flag_geq(flag, target, budget_ns, &seen))
    report_status(status, kStatusFlagTimeout, -1, seen, target);
}

// One thread: *flag += inc with release semantics, after the stream's
// earlier work (hands a staging buffer back to its writer).
__global__ void pd_flag_add_kernel(unsigned *flag, unsigned inc) {
  fence_acq_rel_sys();
  red_release_sys_add(flag, inc);
}

int64_t push_units_per_layer(int64_t num_tokens, int64_t num_planes,
                             int64_t tile_tokens) {
  return num_planes * ((num_tokens + tile_tokens - 1) / tile_tokens);
}

void pd_push(const PagedLayout &src, const PagedLayout &dst,
             const at::Tensor &src_slots, const at::Tensor &dst_slots,
             int64_t layer_begin, int64_t num_layers, int64_t replicas,
             const std::vector<int64_t> &flag_ptrs, int64_t tile_tokens,
             int64_t grid, const c10::optional<at::Tensor> &status, int64_t mode,
             const c10::optional<at::Tensor> &counters, bool local_dst) {
  TORCH_CHECK(src_slots.is_cuda() && dst_slots.is_cuda(),
              "slot mappings must live on the device");
  TORCH_CHECK(src_slots.scalar_type() == dst_slots.scalar_type(),
              "src/dst slot mappings must share a dtype");
  TORCH_CHECK(src_slots.numel() == dst_slots.numel(),
              "src/dst slot mappings must have the same length");
  TORCH_CHECK(src_slots.is_contiguous() && dst_slots.is_contiguous(),
              "slot mappings must be contiguous");
  TORCH_CHECK(replicas >= 1 && replicas <= kMaxReplicas, "1..4 replicas");
  TORCH_CHECK(src.desc().num_planes == dst.desc().num_planes,
              "src/dst plane count mismatch");
  TORCH_CHECK(dst.desc().num_layers % replicas == 0,
              "dst table must hold replicas * layers entries");
  const int dst_layers = dst.desc().num_layers / static_cast<int>(replicas);
  TORCH_CHECK(layer_begin >= 0 && layer_begin + num_layers <= src.desc().num_layers &&
                  layer_begin + num_layers <= dst_layers,
              "layer range out of the caches");
  for (int p = 0; p < src.desc().num_planes; ++p) {
    TORCH_CHECK(src.desc().plane[p].row_bytes == dst.desc().plane[p].row_bytes,
                "src/dst row size mismatch on plane ", p);
    for (const PlaneDesc *pl : {&src.desc().plane[p], &dst.desc().plane[p]})
      TORCH_CHECK(pl->seg_bytes == 0 || pl->seg_bytes % 16 == 0,
                  "pd_push: row segments must be 16-byte multiples");
  }
  TORCH_CHECK(flag_ptrs.empty() || static_cast<int64_t>(flag_ptrs.size()) == replicas,
              "flag_ptrs: one per replica (or none)");
  if (src_slots.numel() == 0 || num_layers == 0) return;
  const c10::cuda::CUDAGuard guard(src_slots.device());
  PushJob j;
  std::memset(&j, 0, sizeof(j));
  j.src = src.desc();
  j.dst = dst.desc();
  j.dst.num_layers = dst_layers;
  j.src_slots = src_slots.data_ptr();
  j.dst_slots = dst_slots.data_ptr();
  j.slot_is_i64 = src_slots.scalar_type() == at::kLong;
  j.num_tokens = static_cast<int32_t>(src_slots.numel());
  j.layer_begin = static_cast<int32_t>(layer_begin);
  j.num_layers = static_cast<int32_t>(num_layers);
  j.tile_tokens = static_cast<int32_t>(tile_tokens > 0 ? tile_tokens : 128);
  TORCH_CHECK(j.tile_tokens <= kMaxTile, "tile_tokens must be <= ", kMaxTile);
  for (int p = 0; p < src.desc().num_planes; ++p) {
    const auto &sp = src.desc().plane[p];
    const auto &dp = dst.desc().plane[p];
    const int64_t sblk = (src.desc().num_slots + src.desc().block_size - 1) / src.desc().block_size;
    const int64_t dblk = (dst.desc().num_slots + dst.desc().block_size - 1) / dst.desc().block_size;
    TORCH_CHECK(sblk * sp.block_stride < (1LL << 32) - 1 &&
                    dblk * dp.block_stride < (1LL << 32) - 1,
                "pd_push: each layer plane must span less than 4 GiB");
  }
  j.replicas = static_cast<int32_t>(replicas);
  for (size_t r = 0; r < flag_ptrs.size(); ++r)
    j.flags[r] = reinterpret_cast<unsigned *>(flag_ptrs[r]);
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->nbytes() >= sizeof(DeviceStatus),
                "status must be a device tensor of >= 24 bytes");
    j.status = reinterpret_cast<DeviceStatus *>(status->data_ptr());
  }
  const int dev = src_slots.device().index();
  const long long units =
      push_units_per_layer(j.num_tokens, j.src.num_planes, j.tile_tokens) *
      static_cast<long long>(num_layers);
  const auto stream = at::cuda::getCurrentCUDAStream(dev).stream();
  TORCH_CHECK(mode >= 0 && mode <= 2, "pd_push: mode 0 (auto), 1 (bulk) or 2 (simt)");
  // planes that move by TMA bulk copies: 16-byte aligned rows, strides and
  // bases on both sides, rows that fit a stage; the others go per lane inside
  // the same kernel (at least one bulk plane is needed to pick this engine)
  uint32_t bulk_planes = 0;
  for (int p = 0; p < j.src.num_planes; ++p)
    if (src.plane_aligned(p) && dst.plane_aligned(p) &&
        j.src.plane[p].row_bytes <= kBulkStageBytes)
      bulk_planes |= 1u << p;
  const bool bulk_ok = bulk_planes != 0 && !src.segmented() && !dst.segmented();
  TORCH_CHECK(mode != 1 || bulk_ok,
              "pd_push: the bulk engine needs 16-byte aligned, contiguous rows of at most ",
              kBulkStageBytes, " bytes on both sides");
  if (mode != 2 && bulk_ok) {
    BulkPushJob b;
    std::memset(&b, 0, sizeof(b));
    b.c.paged = j.src;
    b.c.dst_paged = j.dst;
    b.c.slots = j.src_slots;
    b.c.dst_slots = j.dst_slots;
    b.c.slot_is_i64 = j.slot_is_i64;
    b.c.num_tokens = j.num_tokens;
    b.c.layer_begin = j.layer_begin;
    b.c.chunk_layer_begin = j.layer_begin;
    b.c.num_layers = j.num_layers;
    b.c.to_chunk = 1;
    b.c.status = j.status;
    b.dst_ptrs = j.dst.ptrs;
    b.dst_layers = dst_layers;
    b.replicas = j.replicas;
    b.tile_tokens = j.tile_tokens;
    b.stage_bytes = kBulkStageBytes;
    for (int r = 0; r < kMaxReplicas; ++r) b.flags[r] = j.flags[r];
    b.budget_ns = 2000000000ull;  // 2 s per mbarrier wait
    b.bulk_planes = bulk_planes;
    // per-unit completion counters, zero between launches: the caller's
    // (reused across its launches on one stream), else a fresh zeroed one
    at::Tensor cnt;
    if (counters.has_value()) {
      TORCH_CHECK(counters->is_cuda() && counters->scalar_type() == at::kInt &&
                      counters->is_contiguous() && counters->numel() >= units &&
                      counters->device() == src_slots.device(),
                  "pd_push: counters must be a contiguous device int32 tensor with one "
                  "entry per unit (", units, ")");
      cnt = *counters;
    } else {
      cnt = at::zeros({std::max<long long>(1, units)}, src_slots.options().dtype(at::kInt));
    }
    b.counters = reinterpret_cast<unsigned *>(cnt.data_ptr());
    b.gpu_scope = local_dst;
    const size_t smem = kTmaRingOffset +
                        static_cast<size_t>(kBulkWarps) * kBulkStages * kBulkStageBytes;
    static bool attr_set[64] = {false};
    if (!attr_set[dev & 63]) {
      C10_CUDA_CHECK(cudaFuncSetAttribute(pd_push_bulk_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
      attr_set[dev & 63] = true;
    }
    // as many CTAs as fit an SM's shared memory, on every SM (each warp takes
    // an equal range of pieces, so the grid is not bounded by the units)
    const int per_sm = std::max(1, static_cast<int>((228 * 1024) / (smem + 1024)));
    const long long ctas = num_sms(dev) * static_cast<long long>(per_sm);
    int g = grid > 0 ? static_cast<int>(grid) : num_sms(dev) * per_sm;
    g = static_cast<int>(std::max(1LL, std::min<long long>(ctas, g)));
    pd_push_bulk_kernel<<<g, kBulkWarps * 32, smem, stream>>>(b);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  int g = grid > 0 ? static_cast<int>(grid) : num_sms(dev) * 16;
  g = static_cast<int>(std::max(1LL, std::min<long long>(units, g)));
  pd_push_kernel<<<g, kPushWarps * 32, 0, stream>>>(j);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void pd_wait_flags(int64_t flags_ptr, const at::Tensor &targets,
                   int64_t layer_begin, double timeout_s,
                   const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(targets.is_cuda() && targets.scalar_type() == at::kInt,
              "targets must be a device int32 tensor");
  const c10::cuda::CUDAGuard guard(targets.device());
  const int n = static_cast<int>(targets.numel());
  if (n == 0) return;
  DeviceStatus *st = nullptr;
  if (status.has_value())
    st = reinterpret_cast<DeviceStatus *>(status->data_ptr());
  const unsigned long long budget =
      static_cast<unsigned long long>(std::max(0.0, timeout_s) * 1e9);
  pd_wait_flags_kernel<<<(n + 127) / 128, 128, 0,
                         at::cuda::getCurrentCUDAStream(targets.device().index())
                             .stream()>>>(
      reinterpret_cast<const unsigned *>(flags_ptr),
      reinterpret_cast<const unsigned *>(targets.data_ptr()),
      static_cast<int>(layer_begin), n, budget, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t fp8_staging_bytes(const PagedLayout &layout, int64_t num_tokens, int64_t num_layers,
                          int64_t group, bool scales) {
  int64_t q = 0, sc = 0;
  for (int p = 0; p < layout.desc().num_planes; ++p) {
    const int64_t re = layout.desc().plane[p].row_bytes / 2;
    q += re;
    sc += re / group;
  }
  return scales ? num_layers * num_tokens * sc * 4 : num_layers * num_tokens * q;
}

void pd_push_fp8(const PagedLayout &src, int64_t q_ptr, int64_t scale_ptr,
                 const at::Tensor &src_slots, int64_t layer_begin, int64_t num_layers,
                 int64_t flag_ptr, int64_t tile_tokens, int64_t grid, int64_t group,
                 const c10::optional<at::Tensor> &status, bool local_dst) {
  TORCH_CHECK(src_slots.is_cuda() && src_slots.is_contiguous() &&
                  (src_slots.scalar_type() == at::kInt || src_slots.scalar_type() == at::kLong),
              "src_slots: contiguous device int32/int64");
  TORCH_CHECK(group == 128 || group == 256 || group == 512,
              "fp8 push: group of 128, 256 or 512 elements");
  TORCH_CHECK(layer_begin >= 0 && layer_begin + num_layers <= src.desc().num_layers,
              "layer range out of the cache");
  for (int p = 0; p < src.desc().num_planes; ++p) {
    const auto &pl = src.desc().plane[p];
    TORCH_CHECK((pl.row_bytes / 2) % group == 0, "fp8 push: row elements must be a multiple "
                "of the group (bf16 rows)");
    TORCH_CHECK(pl.row_bytes == src.desc().plane[0].row_bytes,
                "fp8 push: every plane must have the same row size");
    TORCH_CHECK(pl.seg_bytes == 0 || pl.seg_bytes % 256 == 0,
                "fp8 push: head-major segments must hold whole 128-element pieces");
  }
  TORCH_CHECK(q_ptr % 16 == 0 && scale_ptr % 4 == 0, "fp8 push: staging alignment");
  // row_off() computes 32-bit byte offsets inside one layer plane
  for (int p = 0; p < src.desc().num_planes; ++p) {
    const int64_t nblk = (src.desc().num_slots + src.desc().block_size - 1) / src.desc().block_size;
    TORCH_CHECK(nblk * src.desc().plane[p].block_stride < (1LL << 32) - 1,
                "fp8 push: each layer plane must span less than 4 GiB");
  }
  if (src_slots.numel() == 0 || num_layers == 0) return;
  const c10::cuda::CUDAGuard guard(src_slots.device());
  PushQJob j;
  std::memset(&j, 0, sizeof(j));
  j.src = src.desc();
  j.src_slots = src_slots.data_ptr();
  j.slot_is_i64 = src_slots.scalar_type() == at::kLong;
  j.num_tokens = static_cast<int32_t>(src_slots.numel());
  j.layer_begin = static_cast<int32_t>(layer_begin);
  j.num_layers = static_cast<int32_t>(num_layers);
  j.tile_tokens = static_cast<int32_t>(tile_tokens > 0 ? tile_tokens : 128);
  j.group = static_cast<int32_t>(group);
  j.q = reinterpret_cast<uint8_t *>(q_ptr);
  j.scales = reinterpret_cast<float *>(scale_ptr);
  j.flags = reinterpret_cast<unsigned *>(flag_ptr);
  j.gpu_scope = local_dst ? 1 : 0;
  if (status.has_value()) j.status = reinterpret_cast<DeviceStatus *>(status->data_ptr());
  const int dev = src_slots.device().index();
  const long long units =
      push_units_per_layer(j.num_tokens, j.src.num_planes, j.tile_tokens) * num_layers;
  int g = grid > 0 ? static_cast<int>(grid) : num_sms(dev) * 16;
  g = static_cast<int>(std::max(1LL, std::min<long long>(units, g)));
  auto stream = at::cuda::getCurrentCUDAStream(dev).stream();
  if (group == 128)
    pd_push_fp8_kernel<1><<<g, kPushWarps * 32, 0, stream>>>(j);
  else if (group == 256)
    pd_push_fp8_kernel<2><<<g, kPushWarps * 32, 0, stream>>>(j);
  else
    pd_push_fp8_kernel<4><<<g, kPushWarps * 32, 0, stream>>>(j);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void pd_dequant_scatter(const PagedLayout &dst, int64_t q_ptr, int64_t scale_ptr,
                        const at::Tensor &dst_slots, int64_t layer_begin, int64_t num_layers,
                        int64_t group, const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(dst_slots.is_cuda() && dst_slots.is_contiguous() &&
                  (dst_slots.scalar_type() == at::kInt || dst_slots.scalar_type() == at::kLong),
              "dst_slots: contiguous device int32/int64");
  for (int p = 0; p < dst.desc().num_planes; ++p) {
    const auto &pl = dst.desc().plane[p];
    TORCH_CHECK(pl.row_bytes == dst.desc().plane[0].row_bytes && pl.row_bytes % 16 == 0 &&
                    (pl.row_bytes / 2) % group == 0 && pl.block_stride % 16 == 0 &&
                    pl.slot_stride % 16 == 0 && (pl.seg_bytes == 0 || pl.seg_bytes % 16 == 0),
                "dequant scatter: equal, 16-byte aligned bf16 rows");
  }
  if (dst_slots.numel() == 0 || num_layers == 0) return;
  const c10::cuda::CUDAGuard guard(dst_slots.device());
  const int dev = dst_slots.device().index();
  DeviceStatus *st = status.has_value() ? reinterpret_cast<DeviceStatus *>(status->data_ptr())
                                        : nullptr;
  TORCH_CHECK(num_layers * dst.desc().num_planes * dst_slots.numel() < (1LL << 31),
              "dequant scatter: too many rows for one launch");
  const int rb = dst.desc().plane[0].row_bytes;
  TORCH_CHECK(rb % 256 == 0 && rb <= 8 * 256,
              "dequant scatter: rows of 128 .. 1024 bf16 elements, in 128-element pieces");
  for (int p = 0; p < dst.desc().num_planes; ++p) {
    const int64_t nblk = (dst.desc().num_slots + dst.desc().block_size - 1) / dst.desc().block_size;
    TORCH_CHECK(nblk * dst.desc().plane[p].block_stride < (1LL << 32) - 1,
                "dequant scatter: each layer plane must span less than 4 GiB");
  }
  const auto stream = at::cuda::getCurrentCUDAStream(dev).stream();
  const auto *qp = reinterpret_cast<const uint8_t *>(q_ptr);
  const auto *sp = reinterpret_cast<const float *>(scale_ptr);
  const int is64 = dst_slots.scalar_type() == at::kLong;
  const int n = static_cast<int>(dst_slots.numel());
  const long long units = static_cast<long long>(dst.desc().num_planes) *
                          ((n + kDqTile - 1) / kDqTile) * num_layers;
  const int g = static_cast<int>(std::max(1LL, std::min<long long>(units, num_sms(dev) * 8)));
  auto go = [&](auto spr) {
    constexpr int V = decltype(spr)::value;
    pd_dequant_scatter_kernel<V><<<g, kDqWarps * 32, 0, stream>>>(
        dst.desc(), qp, sp, dst_slots.data_ptr(), is64, n, static_cast<int>(layer_begin),
        static_cast<int>(num_layers), static_cast<int>(group), st);
  };
  const int spr = rb / 256;
  if (spr <= 1)
    go(std::integral_constant<int, 1>());
  else if (spr <= 2)
    go(std::integral_constant<int, 2>());
  else if (spr <= 4)
    go(std::integral_constant<int, 4>());
  else
    go(std::integral_constant<int, 8>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void pd_wait_value(int64_t flag_ptr, int64_t target, double timeout_s,
                   const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(flag_ptr % 4 == 0, "flag must be 4-byte aligned");
  DeviceStatus *st = status.has_value() ? reinterpret_cast<DeviceStatus *>(status->data_ptr())
                                        : nullptr;
  const unsigned long long budget =
      static_cast<unsigned long long>(std::max(0.0, timeout_s) * 1e9);
  pd_wait_value_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const unsigned *>(flag_ptr), static_cast<unsigned>(target), budget, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void pd_flag_add(int64_t flag_ptr, int64_t inc) {
  TORCH_CHECK(flag_ptr % 4 == 0, "flag must be 4-byte aligned");
  pd_flag_add_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<unsigned *>(flag_ptr), static_cast<unsigned>(inc));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
