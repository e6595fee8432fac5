// Host-side declarations of the paged <-> chunk transfer ops.
#pragma once

#include <torch/extension.h>

#include <vector>

#include <cuda_runtime.h>

#include "layout.h"

namespace lmc {

struct CopyJob;  // kv_copy.cuh (device-side definition)

// Paged-cache layout of every layer, built once per registered KV cache.
// `ptrs` is a device int64 table [num_layers * num_planes] of plane bases.
class PagedLayout {
 public:
  PagedLayout(at::Tensor ptrs, std::vector<int64_t> block_stride,
              std::vector<int64_t> slot_stride, std::vector<int64_t> row_bytes,
              int64_t block_size, int64_t num_slots,
              std::vector<int64_t> seg_bytes = {}, std::vector<int64_t> seg_stride = {});
  bool segmented() const { return segmented_; }
  const PagedDesc &desc() const { return desc_; }
  // TMA bulk copies need 16-byte aligned, contiguous rows on the paged side
  bool aligned() const { return aligned16_ && bases_aligned_ && !segmented_; }
  // the same condition for one plane
  bool plane_aligned(int p) const { return plane16_[p] && bases_aligned_; }
  void set_bases_aligned(bool v) { bases_aligned_ = v; }
  int64_t num_layers() const { return desc_.num_layers; }
  int64_t num_planes() const { return desc_.num_planes; }
  at::Tensor ptrs() const { return ptrs_; }

 private:
  at::Tensor ptrs_;
  PagedDesc desc_;
  bool aligned16_ = true;
  bool plane16_[kMaxPlanes] = {false, false, false};
  bool bases_aligned_ = true;
  bool segmented_ = false;
};

// Chunk-object layout (strides are per chunk token, see kv_copy.cuh).
class ChunkLayout {
 public:
  ChunkLayout(std::vector<int64_t> plane_stride_t, int64_t layer_stride_t,
              std::vector<int64_t> token_stride, std::vector<int64_t> col_off);
  const ChunkView &view() const { return view_; }

 private:
  ChunkView view_;
};

int num_sms(int device);

void launch_copy(const CopyJob &j, bool chunk_on_device, bool aligned,
                 int64_t mode, cudaStream_t stream, int device);

// Generic paged <-> chunk transfer.  `mode`: 0 auto, 1 TMA bulk, 2 SIMT.
void kv_transfer(const PagedLayout &paged, const c10::optional<at::Tensor> &chunk,
                 const c10::optional<at::Tensor> &chunk_ptrs,
                 const ChunkLayout &layout, int64_t chunk_ntok,
                 int64_t chunk_tok_off, int64_t chunk_tokens,
                 bool chunk_on_device, const at::Tensor &slots,
                 int64_t layer_begin, int64_t chunk_layer_begin,
                 int64_t num_layers, bool to_chunk, int64_t mode,
                 const c10::optional<at::Tensor> &status,
                 const c10::optional<at::Tensor> &chunk_idx,
                 int64_t chunk_idx_limit,
                 const c10::optional<at::Tensor> &num_tokens_dev);

void paged_copy(const PagedLayout &src, const PagedLayout &dst, const at::Tensor &src_slots,
                const at::Tensor &dst_slots, int64_t layer_begin, int64_t dst_layer_begin,
                int64_t num_layers, int64_t mode, const c10::optional<at::Tensor> &status,
                int64_t flags_ptr, int64_t flag_inc);

void fused_multi_layer_kv_transfer(at::Tensor &host_chunk, at::Tensor &staging,
                                   const PagedLayout &paged, const ChunkLayout &layout,
                                   const at::Tensor &slots, bool from_gpu, int64_t mode,
                                   const c10::optional<at::Tensor> &status);

}  // namespace lmc
