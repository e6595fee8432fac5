// K6: DSA lightning-indexer (C8) cache <-> per-chunk packets.
//
// Reference: csrc/indexer_c8/kernel.cpp:28-150 (copy loop) and
// csrc/indexer_c8.cpp:126-185 (launcher): per layer, int8 keys of 128 bytes a
// token plus one fp16 scale a token move between the paged cache and a
// packet laid out [keys of `cap` tokens | scales of `cap` tokens] per layer.
//
// Rows are 128 bytes (keys) and 2 bytes (scales), so per-token work must be a
// few instructions: a CTA takes one chunk (packet) and a group of layers,
// stages the chunk's physical slots in shared memory once, and then for
// every layer moves the key plane as a flat range of 16-byte vectors (vector
// v is part of token v / (key_bytes / 16); consecutive lanes touch
// consecutive 16 bytes whenever the slots run contiguously, which paged
// blocks do) and the scale plane as one 2-byte copy per token.  Loads are
// issued in batches of kC8Unroll before their stores.  A short last packet
// whose layers are not 16-byte aligned moves in 2-byte units.  A slot of -1 (invalid
// or out of range, mapped on the host) is skipped.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace lmc {

namespace {

constexpr int kC8Threads = 256;
constexpr int kC8Unroll = 8;

// One layer's key plane of one chunk in units of V (uint4, or 2 bytes for a
// chunk whose packet layers are not 16-byte aligned): unit u belongs to token
// u / (key_bytes / sizeof(V)).
template <typename V>
__device__ __forceinline__ void c8_keys(uint8_t *kc, uint8_t *kp, const int64_t *slots, int cnt,
                                        int key_bytes, bool to_packet) {
  constexpr int W = sizeof(V);
  const int upt = key_bytes / W;
  const int nu = cnt * upt;
  for (int u0 = threadIdx.x; u0 < nu; u0 += kC8Threads * kC8Unroll) {
    V val[kC8Unroll];
    V *dst[kC8Unroll];
#pragma unroll
    for (int k = 0; k < kC8Unroll; ++k) {
      const int u = u0 + k * kC8Threads;
      dst[k] = nullptr;
      if (u < nu) {
        const int t = u / upt;
        const int64_t p = slots[t];
        if (p >= 0) {
          const size_t co = static_cast<size_t>(p) * key_bytes + static_cast<size_t>(u - t * upt) * W;
          const size_t po = static_cast<size_t>(u) * W;
          const V *src = reinterpret_cast<const V *>(to_packet ? kc + co : kp + po);
          dst[k] = reinterpret_cast<V *>(to_packet ? kp + po : kc + co);
          val[k] = *src;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kC8Unroll; ++k)
      if (dst[k] != nullptr) *dst[k] = val[k];
  }
}

__global__ void __launch_bounds__(kC8Threads) c8_copy_kernel(
    const int64_t *__restrict__ planes,   // [L][P] cache base pointers (keys, scales)
    const int64_t *__restrict__ phys,     // [n] physical slot per token, -1 = skip
    const int64_t *__restrict__ packets,  // [chunks] packet base pointers
    int n, int cap, int L, int layers_per_cta, int key_bytes, int P, int64_t phys_limit,
    bool to_packet) {
  extern __shared__ int64_t c8_slots[];
  const int chunk = blockIdx.x;
  const int t0 = chunk * cap;
  const int cnt = min(cap, n - t0);  // a packet holds its own token count
  if (cnt <= 0) return;
  for (int t = threadIdx.x; t < cnt; t += blockDim.x) {
    const int64_t p = phys[t0 + t];
    c8_slots[t] = (p >= 0 && p < phys_limit) ? p : -1;  // bad slots are skipped
  }
  __syncthreads();
  const int l0 = blockIdx.y * layers_per_cta;
  const int l1 = min(L, l0 + layers_per_cta);
  const size_t row_sum = static_cast<size_t>(key_bytes) + (P > 1 ? 2 : 0);
  const size_t layer_bytes = static_cast<size_t>(cnt) * row_sum;
  const bool vec = (layer_bytes & 15) == 0;  // every layer of the packet 16-byte aligned
  uint8_t *pkt = reinterpret_cast<uint8_t *>(packets[chunk]);
  for (int l = l0; l < l1; ++l) {
    uint8_t *kc = reinterpret_cast<uint8_t *>(planes[static_cast<size_t>(l) * P]);
    uint8_t *kp = pkt + static_cast<size_t>(l) * layer_bytes;
    if (vec) c8_keys<uint4>(kc, kp, c8_slots, cnt, key_bytes, to_packet);
    else c8_keys<unsigned short>(kc, kp, c8_slots, cnt, key_bytes, to_packet);
    if (P > 1) {
      uint8_t *sc = reinterpret_cast<uint8_t *>(planes[static_cast<size_t>(l) * P + 1]);
      uint8_t *sp = kp + static_cast<size_t>(cnt) * key_bytes;
      for (int t = threadIdx.x; t < cnt; t += kC8Threads) {
        const int64_t p = c8_slots[t];
        if (p < 0) continue;
        unsigned short *a = reinterpret_cast<unsigned short *>(sc + p * 2);
        unsigned short *b = reinterpret_cast<unsigned short *>(sp + static_cast<size_t>(t) * 2);
        if (to_packet) *b = *a;
        else *a = *b;
      }
    }
  }
}

}  // namespace

// planes: device int64 [L * P] (P = 2: keys and scales of each layer, P = 1:
// keys only); phys: device int64 [n]; packets: device int64 [ceil(n / cap)];
// phys_limit: physical slots of the cache (larger slots are skipped).  Every
// base pointer must be 16-byte aligned (the caller checks and otherwise takes
// the general copy engine); packet p holds min(cap, n - p cap) tokens.
void c8_copy(const at::Tensor &planes, const at::Tensor &phys, const at::Tensor &packets,
             int64_t cap, int64_t num_layers, int64_t key_bytes, int64_t phys_limit,
             bool to_packet) {
  TORCH_CHECK(planes.is_cuda() && phys.is_cuda() && packets.is_cuda(),
              "c8_copy: pointer tables and slots must be device tensors");
  TORCH_CHECK(planes.scalar_type() == at::kLong && phys.scalar_type() == at::kLong &&
                  packets.scalar_type() == at::kLong,
              "c8_copy: int64 tables");
  TORCH_CHECK(key_bytes > 0 && key_bytes % 16 == 0, "c8_copy: key rows of 16-byte multiples");
  TORCH_CHECK(cap > 0 && cap <= 8192, "c8_copy: 1 <= capacity <= 8192 tokens");
  TORCH_CHECK(num_layers > 0 && planes.numel() % num_layers == 0, "c8_copy: plane table");
  const int P = static_cast<int>(planes.numel() / num_layers);
  TORCH_CHECK(P == 1 || P == 2, "c8_copy: one or two planes per layer");
  const int64_t n = phys.numel();
  const int64_t chunks = (n + cap - 1) / cap;
  TORCH_CHECK(packets.numel() >= chunks, "c8_copy: fewer packets than chunks");
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(phys.device());
  auto pl = planes.contiguous(), ph = phys.contiguous(), pk = packets.contiguous();
  int dev = 0, sms = 148;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  // about eight CTAs per SM in all: layer groups per chunk fill what the
  // chunks alone do not
  const int64_t want = static_cast<int64_t>(sms) * 8;
  const int groups = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(num_layers, (want + chunks - 1) / chunks)));
  const int lpc = static_cast<int>((num_layers + groups - 1) / groups);
  const int gy = static_cast<int>((num_layers + lpc - 1) / lpc);
  const size_t smem = static_cast<size_t>(cap) * sizeof(int64_t);
  if (smem > 48 * 1024)
    C10_CUDA_CHECK(cudaFuncSetAttribute(c8_copy_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(gy));
  c8_copy_kernel<<<grid, kC8Threads, smem, at::cuda::getCurrentCUDAStream().stream()>>>(
      pl.data_ptr<int64_t>(), ph.data_ptr<int64_t>(), pk.data_ptr<int64_t>(),
      static_cast<int>(n), static_cast<int>(cap), static_cast<int>(num_layers), lpc,
      static_cast<int>(key_bytes), P, phys_limit, to_packet);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
