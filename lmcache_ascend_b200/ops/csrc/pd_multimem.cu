// K9 fan-out through NVSwitch multicast (NVLS): one prefiller pushes the same
// KV to several decoders while its NVLink egress carries the bytes once.
//
// The group's members (the prefiller and its decoders) share a symmetric
// staging buffer bound to one NVLink multicast object.  The prefiller reads
// its own paged rows (plain loads from its HBM) and writes each 16-byte vector
// once with `multimem.st` to the multicast address: NVSwitch delivers it to
// every member's copy of the staging buffer.  After a unit's stores, one
// `multimem.red.release` adds 1 to the layer's flag in every member's copy.
// Each decoder waits on its own copy of the flags (bounded acquire spin) and
// then scatters the staging rows into its paged cache with a local copy.
//
// Loads never come from another GPU's memory, and there is no TMA here: the
// multicast object is only ever the target of multimem stores and reductions.
//
// Staging layout: row ((layer * planes + plane) * T + t), `row_bytes` each
// (every plane has the same row size), then the flag words at `flags_off`.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <cstring>

#include "kv_copy.cuh"
#include "mem_kernels.h"

namespace lmc {

constexpr int kMcWarps = 4;
constexpr int kMcVec = 8;

struct McJob {
  PagedDesc src;
  const void *src_slots;
  int32_t slot_is_i64;
  int32_t num_tokens;
  int32_t layer_begin;
  int32_t num_layers;
  int32_t tile_tokens;
  char *mc_rows;       // multicast address of the staging rows
  unsigned *mc_flags;  // multicast address of the flag words [num_layers_total]
  DeviceStatus *status;
};

__device__ __forceinline__ void multimem_st_v4(void *mc, int4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(__int_as_float(v.x)), "f"(__int_as_float(v.y)), "f"(__int_as_float(v.z)),
               "f"(__int_as_float(v.w))
               : "memory");
}

__device__ __forceinline__ void multimem_red_release_add(unsigned *mc, unsigned v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc), "r"(v)
               : "memory");
}

__device__ __forceinline__ int64_t mc_slot(const void *p, int is64, int t) {
  return is64 ? static_cast<const int64_t *>(p)[t]
              : static_cast<int64_t>(static_cast<const int32_t *>(p)[t]);
}

__global__ void __launch_bounds__(kMcWarps * 32) pd_push_multimem_kernel(McJob j) {
  const int np = j.src.num_planes;
  const int tiles = (j.num_tokens + j.tile_tokens - 1) / j.tile_tokens;
  const int units_per_layer = np * tiles;
  const int total = units_per_layer * j.num_layers;
  const int tid = threadIdx.x;
  constexpr int kThreads = kMcWarps * 32;
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    const int li = u / units_per_layer;
    const int rem = u - li * units_per_layer;
    const int p = rem / tiles;
    const int tile = rem - p * tiles;
    const int layer = j.layer_begin + li;
    const PlaneDesc spl = plane_of(j.src, p);
    const int rb = spl.row_bytes;
    const int vpr = rb >> 4;
    const int t0 = tile * j.tile_tokens;
    const int n = min(j.num_tokens - t0, j.tile_tokens);
    const int nv = n * vpr;
    char *mrow0 = j.mc_rows + ((static_cast<int64_t>(layer) * np + p) * j.num_tokens + t0) * rb;
    for (int base = 0; base < nv; base += kThreads * kMcVec) {
      int4 v[kMcVec];
      bool ok[kMcVec];
#pragma unroll
      for (int k = 0; k < kMcVec; ++k) {
        const int g = base + k * kThreads + tid;
        ok[k] = false;
        if (g < nv) {
          const int ti = g / vpr;
          const int vb = (g - ti * vpr) * 16;
          const int64_t ss = mc_slot(j.src_slots, j.slot_is_i64, t0 + ti);
          if (ss >= 0 && ss < j.src.num_slots) {
            ok[k] = true;
            v[k] = ld_nc_v4(paged_addr(j.src, layer, p, ss) + vb);
          } else if (ss >= j.src.num_slots && vb == 0) {
            report_status(j.status, kStatusBadSlot, t0 + ti, ss, j.src.num_slots);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < kMcVec; ++k) {
        const int g = base + k * kThreads + tid;
        if (ok[k]) multimem_st_v4(mrow0 + static_cast<int64_t>(g) * 16, v[k]);
      }
    }
    __syncthreads();
    if (tid == 0) {
      fence_acq_rel_sys();
      multimem_red_release_add(j.mc_flags + layer, 1u);
    }
  }
}

// src paged cache -> every group member's staging (through the multicast
// address); flags at mc_flags (multicast address) count finished units.
void pd_push_multimem(const PagedLayout &src, int64_t mc_rows, int64_t mc_flags,
                      const at::Tensor &src_slots, int64_t layer_begin, int64_t num_layers,
                      int64_t tile_tokens, int64_t grid,
                      const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(src_slots.is_cuda() && src_slots.is_contiguous() &&
                  (src_slots.scalar_type() == at::kInt || src_slots.scalar_type() == at::kLong),
              "src_slots: contiguous device int32/int64");
  TORCH_CHECK(src.aligned(), "multimem push: 16-byte aligned, contiguous paged rows");
  for (int p = 0; p < src.desc().num_planes; ++p)
    TORCH_CHECK(src.desc().plane[p].row_bytes == src.desc().plane[0].row_bytes,
                "multimem push: every plane must have the same row size");
  TORCH_CHECK(layer_begin >= 0 && layer_begin + num_layers <= src.desc().num_layers,
              "layer range out of the cache");
  TORCH_CHECK(mc_rows % 16 == 0 && mc_flags % 4 == 0, "multimem push: staging alignment");
  if (src_slots.numel() == 0 || num_layers == 0) return;
  const c10::cuda::CUDAGuard guard(src_slots.device());
  McJob j;
  std::memset(&j, 0, sizeof(j));
  j.src = src.desc();
  j.src_slots = src_slots.data_ptr();
  j.slot_is_i64 = src_slots.scalar_type() == at::kLong;
  j.num_tokens = static_cast<int32_t>(src_slots.numel());
  j.layer_begin = static_cast<int32_t>(layer_begin);
  j.num_layers = static_cast<int32_t>(num_layers);
  j.tile_tokens = static_cast<int32_t>(tile_tokens > 0 ? tile_tokens : 128);
  j.mc_rows = reinterpret_cast<char *>(mc_rows);
  j.mc_flags = reinterpret_cast<unsigned *>(mc_flags);
  if (status.has_value()) j.status = reinterpret_cast<DeviceStatus *>(status->data_ptr());
  const int dev = src_slots.device().index();
  const long long units =
      static_cast<long long>(j.src.num_planes) *
      ((j.num_tokens + j.tile_tokens - 1) / j.tile_tokens) * num_layers;
  const int g = static_cast<int>(
      std::max(1LL, std::min<long long>(units, grid > 0 ? grid : num_sms(dev) * 16)));
  pd_push_multimem_kernel<<<g, kMcWarps * 32, 0, at::cuda::getCurrentCUDAStream(dev).stream()>>>(
      j);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
