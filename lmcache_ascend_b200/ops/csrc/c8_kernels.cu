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
constexpr int64_t kC8Block = 128;  // tokens per C8 cache block
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

// Logical slot -> physical slot of the C8 cache (reference
// csrc/indexer_c8.cpp:12-45): with a block map, block b lives at physical
// block map[b]; otherwise at b * factor.  Slots outside the logical capacity,
// or mapped outside the physical cache, give -1 (skipped).
struct C8SlotMap {
  const int32_t *block_map;  // [logical blocks] or null
  int64_t cache_slots;       // logical capacity
  int64_t phys_limit;        // physical slots
  int factor;                // 1 or 2
  __device__ __forceinline__ int64_t operator()(int64_t s) const {
    if (s < 0 || s >= cache_slots) return -1;
    const int64_t b = s / kC8Block, r = s - b * kC8Block;
    const int64_t p = block_map != nullptr ? static_cast<int64_t>(block_map[b]) * kC8Block + r
                                           : b * factor * kC8Block + r;
    return (p >= 0 && p < phys_limit) ? p : -1;
  }
};

template <typename ST>
__global__ void __launch_bounds__(kC8Threads) c8_copy_kernel(
    const int64_t *__restrict__ planes,   // [L][P] cache base pointers (keys, scales)
    const ST *__restrict__ slots,         // [n] logical slot per token
    const int64_t *__restrict__ packets,  // [chunks] packet base pointers
    C8SlotMap map, int n, int cap, int L, int layers_per_cta, int key_bytes, int P,
    bool to_packet) {
  extern __shared__ int64_t c8_slots[];
  const int chunk = blockIdx.x;
  const int t0 = chunk * cap;
  const int cnt = min(cap, n - t0);  // a packet holds its own token count
  if (cnt <= 0) return;
  for (int t = threadIdx.x; t < cnt; t += blockDim.x)
    c8_slots[t] = map(static_cast<int64_t>(slots[t0 + t]));
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
// keys only); slots: device int32/int64 [n] logical slots; packets: device
// int64 [ceil(n / cap)]; block_map: optional device int32 [logical blocks];
// cache_slots: logical capacity; phys_limit: physical slots.  Every base
// pointer must be 16-byte aligned (the caller checks and otherwise takes the
// general copy engine); packet p holds min(cap, n - p cap) tokens.
void c8_copy(const at::Tensor &planes, const at::Tensor &slots, const at::Tensor &packets,
             int64_t cap, int64_t num_layers, int64_t key_bytes, int64_t factor,
             const c10::optional<at::Tensor> &block_map, int64_t cache_slots,
             int64_t phys_limit, bool to_packet) {
  TORCH_CHECK(planes.is_cuda() && slots.is_cuda() && packets.is_cuda(),
              "c8_copy: pointer tables and slots must be device tensors");
  TORCH_CHECK(planes.scalar_type() == at::kLong && packets.scalar_type() == at::kLong,
              "c8_copy: int64 pointer tables");
  TORCH_CHECK(slots.scalar_type() == at::kLong || slots.scalar_type() == at::kInt,
              "c8_copy: int32 or int64 slots");
  TORCH_CHECK(key_bytes > 0 && key_bytes % 16 == 0, "c8_copy: key rows of 16-byte multiples");
  TORCH_CHECK(cap > 0 && cap <= 8192, "c8_copy: 1 <= capacity <= 8192 tokens");
  TORCH_CHECK(factor == 1 || factor == 2, "c8_copy: block factor 1 or 2");
  TORCH_CHECK(num_layers > 0 && planes.numel() % num_layers == 0, "c8_copy: plane table");
  const int P = static_cast<int>(planes.numel() / num_layers);
  TORCH_CHECK(P == 1 || P == 2, "c8_copy: one or two planes per layer");
  const int64_t n = slots.numel();
  const int64_t chunks = (n + cap - 1) / cap;
  TORCH_CHECK(packets.numel() >= chunks, "c8_copy: fewer packets than chunks");
  C8SlotMap map{nullptr, cache_slots, phys_limit, static_cast<int>(factor)};
  at::Tensor bm;
  if (block_map.has_value()) {
    bm = block_map->contiguous();
    TORCH_CHECK(bm.is_cuda() && bm.scalar_type() == at::kInt &&
                    bm.numel() * kC8Block >= cache_slots,
                "c8_copy: block map must be device int32 covering the logical blocks");
    map.block_map = bm.data_ptr<int32_t>();
  }
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(slots.device());
  auto pl = planes.contiguous(), sl = slots.contiguous(), pk = packets.contiguous();
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
  dim3 grid(static_cast<unsigned>(chunks), static_cast<unsigned>(gy));
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  auto launch = [&](auto *kernel, const auto *sp) {
    if (smem > 48 * 1024)
      C10_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    kernel<<<grid, kC8Threads, smem, stream>>>(
        pl.data_ptr<int64_t>(), sp, pk.data_ptr<int64_t>(), map, static_cast<int>(n),
        static_cast<int>(cap), static_cast<int>(num_layers), lpc, static_cast<int>(key_bytes),
        P, to_packet);
  };
  if (sl.scalar_type() == at::kLong) launch(c8_copy_kernel<int64_t>, sl.data_ptr<int64_t>());
  else launch(c8_copy_kernel<int32_t>, sl.data_ptr<int32_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
