// Paged <-> chunk row-copy engines shared by the gather/scatter kernels
// (mem_kernels.cu) and the PD push (pd_push.cu).
//
// Two engines:
//  * `tma_rows_kernel`: one warp per CTA drives a ring of shared-memory
//    stages with TMA bulk copies (`cp.async.bulk`, non-multicast).  Runs of
//    tokens that are contiguous on BOTH sides are merged into one bulk copy
//    (a vLLM block of 16 tokens x 2 KiB is one 32 KiB copy).  Used when both
//    sides are this GPU's own memory and rows are 16-byte multiples.
//  * `simt_rows_kernel`: warp-per-row 16-byte vector copy.  Used for
//    host-mapped pinned memory, peer memory (NVLink stores), and rows that are
//    not 16-byte multiples (falls back to 4- or 1-byte granules).
#pragma once

#include "common.cuh"
#include "layout.h"

namespace lmc {

struct CopyJob {
  PagedDesc paged;
  ChunkView chunk;
  const void *slots;  // [num_tokens] int32 or int64, -1 = skip
  int32_t slot_is_i64;
  int32_t num_tokens;
  int32_t layer_begin;  // first paged layer
  int32_t chunk_layer_begin;
  int32_t num_layers;   // layers moved by this launch
  int32_t to_chunk;     // 1: paged -> chunk (store), 0: chunk -> paged
  DeviceStatus *status;
  // Sparse: chunk token of slot entry t is chunk_idx[t] (int32 or int64,
  // same dtype as the slots), bounded by chunk_idx_limit.  nullptr = t.
  const void *chunk_idx;
  int64_t chunk_idx_limit;
  // Graph-capturable: when set, only the first min(*num_tokens_dev,
  // num_tokens) entries are processed (device-side count).
  const int32_t *num_tokens_dev;
  // Paged -> paged (same-GPU push / block copy): when dst_slots is set the
  // destination is dst_paged at dst_slots[t] instead of the chunk view.
  PagedDesc dst_paged;
  const void *dst_slots;
  // Planes moved by this launch (bit p = plane p); 0 = every plane.  Lets one
  // transfer run its 16-byte-aligned planes on the TMA engine and the others
  // (e.g. 2-byte scale rows) on the SIMT engine.
  uint32_t plane_mask;
};

__device__ __forceinline__ bool plane_selected(const CopyJob &j, int p) {
  return j.plane_mask == 0 || ((j.plane_mask >> p) & 1u);
}

// Effective token count (reads the device-side count when present).
__device__ __forceinline__ int effective_tokens(const CopyJob &j) {
  if (j.num_tokens_dev == nullptr) return j.num_tokens;
  const int n = *j.num_tokens_dev;
  return n < 0 ? 0 : (n < j.num_tokens ? n : j.num_tokens);
}

// Tokens of the chunk sequence a chunk-pointer table addresses: the slot count
// for dense transfers, the index bound for sparse ones (the last chunk may be
// partial, so its token count is derived from this total).
__device__ __forceinline__ int chunk_seq_tokens(const CopyJob &j) {
  return j.chunk_idx != nullptr ? static_cast<int>(j.chunk_idx_limit) : j.num_tokens;
}

__device__ __forceinline__ int64_t load_idx(const CopyJob &j, int t) {
  if (j.chunk_idx == nullptr) return t;
  return j.slot_is_i64 ? static_cast<const int64_t *>(j.chunk_idx)[t]
                       : static_cast<int64_t>(static_cast<const int32_t *>(j.chunk_idx)[t]);
}

// Select element p (0..2) of a 3-array with constant indices: runtime
// indexing of kernel-parameter arrays would copy the whole struct to local
// memory.
template <typename T>
__device__ __forceinline__ T sel3(const T (&a)[kMaxPlanes], int p) {
  return p == 0 ? a[0] : (p == 1 ? a[1] : a[2]);
}

__device__ __forceinline__ PlaneDesc plane_of(const PagedDesc &pd, int p) {
  return p == 0 ? pd.plane[0] : (p == 1 ? pd.plane[1] : pd.plane[2]);
}

__device__ __forceinline__ int64_t load_slot(const CopyJob &j, int t) {
  return j.slot_is_i64 ? static_cast<const int64_t *>(j.slots)[t]
                       : static_cast<int64_t>(static_cast<const int32_t *>(j.slots)[t]);
}

__device__ __forceinline__ char *paged_addr(const PagedDesc &pd, int layer,
                                            int p, int64_t slot) {
  const int64_t blk = slot / pd.block_size;
  const int64_t off = slot - blk * pd.block_size;
  char *base = reinterpret_cast<char *>(pd.ptrs[layer * pd.num_planes + p]);
  const PlaneDesc pl = plane_of(pd, p);
  return base + blk * pl.block_stride + off * pl.slot_stride;
}

__device__ __forceinline__ char *chunk_addr(const ChunkView &cv, int layer,
                                            int p, int64_t t, int total_tokens) {
  char *base;
  int64_t tl, tc;
  if (cv.chunk_ptrs != nullptr) {
    const int c = static_cast<int>(t / cv.chunk_tokens);
    tl = t - static_cast<int64_t>(c) * cv.chunk_tokens;
    tc = min(cv.chunk_tokens, total_tokens - c * cv.chunk_tokens);
    base = reinterpret_cast<char *>(cv.chunk_ptrs[c]);
  } else {
    tl = t + cv.tok_off;
    tc = cv.ntok;
    base = cv.base;
  }
  return base + p * sel3(cv.plane_stride_t, p) * tc + layer * cv.layer_stride_t * tc +
         tl * sel3(cv.token_stride, p) + sel3(cv.col_off, p);
}

// Work decomposition: unit = (layer, plane, tile of tokens).  Tile size per
// plane is stage_bytes / row_bytes (capped at 64 tokens = 2 per lane).
struct UnitMap {
  int tile[kMaxPlanes];
  int ntiles[kMaxPlanes];
  int units_per_layer;
};

__device__ __forceinline__ UnitMap make_unit_map(const CopyJob &j,
                                                 int stage_bytes) {
  UnitMap m;
  m.units_per_layer = 0;
  for (int p = 0; p < kMaxPlanes; ++p) {
    if (p < j.paged.num_planes && plane_selected(j, p)) {
      int tt = stage_bytes / plane_of(j.paged, p).row_bytes;
      tt = tt > 64 ? 64 : (tt < 1 ? 1 : tt);
      m.tile[p] = tt;
      m.ntiles[p] = (j.num_tokens + tt - 1) / tt;
    } else {
      m.tile[p] = 1;
      m.ntiles[p] = 0;
    }
    m.units_per_layer += m.ntiles[p];
  }
  return m;
}

struct Unit {
  int layer;  // index within this launch [0, num_layers)
  int plane;
  int t0;
  int n;
};

__device__ __forceinline__ Unit decode_unit(const CopyJob &j, const UnitMap &m,
                                            int u) {
  Unit r;
  r.layer = u / m.units_per_layer;
  int rem = u - r.layer * m.units_per_layer;
  int p = 0;
  if (rem >= m.ntiles[0]) {
    rem -= m.ntiles[0];
    ++p;
    if (rem >= m.ntiles[1]) {
      rem -= m.ntiles[1];
      ++p;
    }
  }
  r.plane = p;
  const int tile = sel3(m.tile, p);
  r.t0 = rem * tile;
  r.n = min(tile, j.num_tokens - r.t0);
  return r;
}

// Per-lane view of the (up to two) tokens a lane owns in a unit, with
// run-start detection across the warp.
struct LaneRuns {
  char *src[2];
  char *dst[2];
  unsigned len[2];  // run length in tokens if this token starts a run, else 0
};

__device__ __forceinline__ LaneRuns plan_runs(const CopyJob &j, const Unit &u,
                                              int lane, int total_tokens) {
  LaneRuns r;
  const int rb = plane_of(j.paged, u.plane).row_bytes;
  bool valid[2];
  for (int h = 0; h < 2; ++h) {
    const int i = h * 32 + lane;
    valid[h] = false;
    r.src[h] = r.dst[h] = nullptr;
    if (i < u.n) {
      const int t = u.t0 + i;
      const int64_t slot = load_slot(j, t);
      if (slot >= 0) {
        if (slot >= j.paged.num_slots) {
          report_status(j.status, kStatusBadSlot, t, slot, j.paged.num_slots);
        } else {
          const int64_t ct = j.dst_slots != nullptr
                                 ? (j.slot_is_i64 ? static_cast<const int64_t *>(j.dst_slots)[t]
                                                  : static_cast<const int32_t *>(j.dst_slots)[t])
                                 : load_idx(j, t);
          const int64_t limit = j.dst_slots != nullptr ? j.dst_paged.num_slots
                                                       : j.chunk_idx_limit;
          if (ct < 0 && j.dst_slots != nullptr) {
            // destination slot -1: skip the token
          } else if (ct < 0 || ((j.chunk_idx != nullptr || j.dst_slots != nullptr) &&
                                ct >= limit)) {
            report_status(j.status, kStatusBadIndex, t, ct, limit);
          } else if (j.dst_slots != nullptr) {
            r.src[h] = paged_addr(j.paged, j.layer_begin + u.layer, u.plane, slot);
            r.dst[h] = paged_addr(j.dst_paged, j.chunk_layer_begin + u.layer, u.plane, ct);
            valid[h] = true;
          } else {
            char *pa = paged_addr(j.paged, j.layer_begin + u.layer, u.plane, slot);
            char *ca = chunk_addr(j.chunk, j.chunk_layer_begin + u.layer, u.plane,
                                  ct, total_tokens);
            r.src[h] = j.to_chunk ? pa : ca;
            r.dst[h] = j.to_chunk ? ca : pa;
            valid[h] = true;
          }
        }
      }
    }
  }
  // A token starts a run unless the previous token is valid and both of its
  // addresses continue exactly where the previous row ends.  All shuffles are
  // executed by the full warp.
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(r.src[0]);
  const uintptr_t d0 = reinterpret_cast<uintptr_t>(r.dst[0]);
  const uintptr_t s1 = reinterpret_cast<uintptr_t>(r.src[1]);
  const uintptr_t d1 = reinterpret_cast<uintptr_t>(r.dst[1]);
  uintptr_t ps0 = __shfl_up_sync(0xffffffffu, s0, 1);
  uintptr_t pd0 = __shfl_up_sync(0xffffffffu, d0, 1);
  uintptr_t ps1 = __shfl_up_sync(0xffffffffu, s1, 1);
  uintptr_t pd1 = __shfl_up_sync(0xffffffffu, d1, 1);
  const uintptr_t ls0 = __shfl_sync(0xffffffffu, s0, 31);
  const uintptr_t ld0 = __shfl_sync(0xffffffffu, d0, 31);
  if (lane == 0) {
    ps0 = 0;
    pd0 = 0;
    ps1 = ls0;
    pd1 = ld0;
  }
  const bool cont0 = valid[0] && ps0 != 0 && s0 == ps0 + rb && d0 == pd0 + rb;
  const bool cont1 = valid[1] && ps1 != 0 && s1 == ps1 + rb && d1 == pd1 + rb;
  // Every token that does not continue a run is a break point; invalid
  // tokens are break points that start nothing.
  const unsigned long long breaks =
      (static_cast<unsigned long long>(__ballot_sync(0xffffffffu, !cont1)) << 32) |
      __ballot_sync(0xffffffffu, !cont0);
  for (int h = 0; h < 2; ++h) {
    const int i = h * 32 + lane;
    const bool cont = h ? cont1 : cont0;
    r.len[h] = 0;
    if (valid[h] && !cont) {
      const unsigned long long after =
          (i == 63) ? 0ull : ((breaks >> (i + 1)) << (i + 1));
      int end = after ? (__ffsll(static_cast<long long>(after)) - 1) : u.n;
      if (end > u.n) end = u.n;
      r.len[h] = static_cast<unsigned>(end - i);
    }
  }
  return r;
}

}  // namespace lmc
