// N14: batched (dst, src, bytes) copies for the layerwise prefill pipeline.
//
// Reference: `layerwise_prefill_dma_copy` and its timed diagnostic variant
// (csrc/pybind.cpp:264-311), a loop of async H2D/D2H copies on the current
// stream.  Two forms here:
//  * `dma_copy_batch`: one cudaMemcpyAsync per entry on the current stream
//    (copy engines; right for few, large, host<->device copies);
//  * `gather_copy`: one kernel over a device table of entries, warp per
//    16-byte-aligned run (right for many small device/host-mapped copies,
//    one launch instead of thousands of API calls).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <chrono>

#include "common.cuh"

namespace lmc {

void dma_copy_batch(const at::Tensor &dsts, const at::Tensor &srcs,
                    const at::Tensor &sizes) {
  TORCH_CHECK(dsts.device().is_cpu() && srcs.device().is_cpu() && sizes.device().is_cpu(),
              "dma_copy_batch: pointer tables must be host int64 tensors");
  TORCH_CHECK(dsts.scalar_type() == at::kLong && srcs.scalar_type() == at::kLong &&
                  sizes.scalar_type() == at::kLong,
              "dma_copy_batch: int64 tables");
  const int64_t n = dsts.numel();
  TORCH_CHECK(srcs.numel() == n && sizes.numel() == n, "dma_copy_batch: length mismatch");
  auto d = dsts.contiguous(), s = srcs.contiguous(), z = sizes.contiguous();
  const int64_t *dp = d.data_ptr<int64_t>(), *sp = s.data_ptr<int64_t>(),
                *zp = z.data_ptr<int64_t>();
  cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
  // entries that continue the previous one on both sides merge into one copy
  // (per-layer chunk objects allocated back to back land in adjacent staging
  // slots: a layer of a long prompt becomes one large DMA)
  int64_t i = 0;
  while (i < n) {
    if (zp[i] <= 0) {
      ++i;
      continue;
    }
    const int64_t d0 = dp[i], s0 = sp[i];
    int64_t len = zp[i];
    int64_t j = i + 1;
    while (j < n && zp[j] > 0 && dp[j] == d0 + len && sp[j] == s0 + len) len += zp[j++];
    cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void *>(d0),
                                    reinterpret_cast<const void *>(s0),
                                    static_cast<size_t>(len), cudaMemcpyDefault, st);
    TORCH_CHECK(e == cudaSuccess, "cudaMemcpyAsync failed at entry ", i, ": ",
                cudaGetErrorString(e));
    i = j;
  }
}

// Same as dma_copy_batch, synchronising the stream and returning the wall
// time in milliseconds (diagnostic variant).
double dma_copy_batch_timed(const at::Tensor &dsts, const at::Tensor &srcs,
                            const at::Tensor &sizes) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
  cudaStreamSynchronize(st);
  const auto t0 = std::chrono::steady_clock::now();
  dma_copy_batch(dsts, srcs, sizes);
  cudaStreamSynchronize(st);
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0)
      .count();
}

__global__ void gather_copy_kernel(const int64_t *__restrict__ table, int n) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int i = warp; i < n; i += nwarps) {
    char *dst = reinterpret_cast<char *>(table[3 * i]);
    const char *src = reinterpret_cast<const char *>(table[3 * i + 1]);
    const int64_t bytes = table[3 * i + 2];
    const bool v16 = ((reinterpret_cast<uintptr_t>(dst) |
                       reinterpret_cast<uintptr_t>(src) | bytes) & 15) == 0;
    if (v16) {
      for (int64_t off = lane * 16; off < bytes; off += 512)
        st_v4(dst + off, ld_v4(src + off));
    } else {
      for (int64_t off = lane; off < bytes; off += 32) dst[off] = src[off];
    }
  }
}

// table: device int64 [n, 3] of (dst, src, bytes)
void gather_copy(const at::Tensor &table) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == at::kLong &&
                  table.dim() == 2 && table.size(1) == 3 && table.is_contiguous(),
              "gather_copy: device int64 [n, 3] table");
  const int n = static_cast<int>(table.size(0));
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(table.device());
  const int threads = 256;
  const int blocks = std::min((n * 32 + threads - 1) / threads, 148 * 8);
  gather_copy_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      table.data_ptr<int64_t>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
