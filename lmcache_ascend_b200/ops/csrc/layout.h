// Layout descriptors for the paged KV cache and for LMCache chunk objects.
//
// The reference computes per-format strides and plane offsets in its host
// utilities (reference csrc/utils.h:53-346, csrc/mem_kernels.cpp:142-165).
// Here every format is reduced to the same two descriptors, so one kernel
// family serves MERGED (flash and flashinfer orders), SEPARATE, MLA and DSA
// caches in both token-major and plane-major chunk orders:
//
//   paged address(layer l, plane p, slot s) =
//       ptrs[l * num_planes + p] + (s / block_size) * block_stride[p]
//                                + (s % block_size) * slot_stride[p]
//   chunk address(layer l, plane p, token t) =
//       base + p * plane_stride[p] + l * layer_stride + t * token_stride
//            + col_off[p]
//
// A "plane" is one tensor component of a layer's cache: K and V for
// MERGED/SEPARATE, k_nope and k_pe for MLA, plus the lightning-indexer key
// for DSA.
#pragma once

#include <cstdint>

namespace lmc {

constexpr int kMaxPlanes = 3;

struct PlaneDesc {
  int64_t block_stride;  // bytes between consecutive blocks of this plane
  int64_t slot_stride;   // bytes between consecutive slots inside a block
  int32_t row_bytes;     // bytes moved per token for this plane
  // Segmented rows (head-major "HND" caches): a token's row is
  // row_bytes / seg_bytes segments of seg_bytes, seg_stride bytes apart in
  // the paged cache (contiguous in chunks).  seg_bytes == 0: contiguous row.
  int32_t seg_bytes;
  int64_t seg_stride;
};

struct PagedDesc {
  const int64_t *ptrs;  // device table [num_layers * num_planes] of base VAs
  PlaneDesc plane[kMaxPlanes];
  int32_t num_layers;
  int32_t num_planes;
  int32_t block_size;
  int32_t pad_;
  int64_t num_slots;  // num_blocks * block_size, for bounds checks
};

struct ChunkDesc {
  char *base;
  int64_t plane_stride[kMaxPlanes];
  int64_t layer_stride;
  int64_t token_stride;
  int64_t col_off[kMaxPlanes];
};

// A chunk-side view that is either one buffer or a table of chunk objects.
struct ChunkView {
  char *base;                 // single chunk (when chunk_ptrs == nullptr)
  const int64_t *chunk_ptrs;  // multi-chunk: base VA of each chunk object
  int32_t chunk_tokens;       // multi-chunk: tokens per full chunk
  int32_t ntok;               // single chunk: token dim of the chunk tensor
  int32_t tok_off;            // single chunk: first chunk token to use
  int32_t pad_;
  int64_t plane_stride_t[kMaxPlanes];  // bytes per (plane) per chunk token
  int64_t layer_stride_t;              // bytes per (layer) per chunk token
  int64_t token_stride[kMaxPlanes];    // bytes between consecutive tokens
  int64_t col_off[kMaxPlanes];         // byte offset of the plane in a row
};

}  // namespace lmc
