// K8: fused RoPE re-rotation of cached keys (CacheBlend re-positioning).
//
// Semantics of the reference op `rotary_embedding_k_fused(old_positions,
// new_positions, key, head_size, cos_sin_cache, is_neox)`
// (csrc/pos_kernels.cpp:164-196, Python wrapper
// lmcache_ascend/v1/blend/positional_encoding.py:95-118): K was rotated for
// positions `old`; rewrite it in place as if it had been rotated for `new`.
//
// Instead of undoing and redoing the rotation (two roundings), the kernel
// rotates once by the angle difference, using the angle-difference identities
//   cos(a - b) = cos a cos b + sin a sin b,  sin(a - b) = sin a cos b - cos a sin b
// on the cached cos/sin values in fp32, and rounds once to the key dtype.
// cos_sin_cache is vLLM's layout: [max_position, rot_dim], first half cos,
// second half sin.  neox pairs (i, i + rot/2); GPT-J pairs (2i, 2i + 1).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

namespace lmc {

template <typename T>
__device__ __forceinline__ float to_f(T v) { return static_cast<float>(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v) { return static_cast<T>(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// grid.x = tokens (grid-stride), block threads cover heads * rot/2 pairs
// Row of token t: t itself, or rows[t] when the keys live in a paged cache
// (rows = slot mapping; a negative slot skips the token).
template <typename PT>
__device__ __forceinline__ int64_t key_row(const PT *rows, int t) {
  return rows == nullptr ? static_cast<int64_t>(t) : static_cast<int64_t>(rows[t]);
}

// Rotation by the angle difference, with the contractions fixed so every
// path (scalar, vector, head-grouped) rounds identically:
//   cos(n - o) = cn co + sn so,  sin(n - o) = sn co - cn so,
//   y1 = x1 cd - x2 sd,          y2 = x2 cd + x1 sd.
__device__ __forceinline__ void rot_delta(float ca, float sa, float cb, float sb, float &cd,
                                          float &sd) {
  cd = __fmaf_rn(ca, cb, __fmul_rn(sa, sb));
  sd = __fmaf_rn(sa, cb, -__fmul_rn(ca, sb));
}
__device__ __forceinline__ void rot_apply(float x1, float x2, float cd, float sd, float &y1,
                                          float &y2) {
  y1 = __fmaf_rn(x1, cd, -__fmul_rn(x2, sd));
  y2 = __fmaf_rn(x2, cd, __fmul_rn(x1, sd));
}

template <typename KT, typename CT, typename PT>
__global__ void rope_delta_kernel(const PT *__restrict__ old_pos,
                                  const PT *__restrict__ new_pos, KT *key,
                                  const CT *__restrict__ cache, int num_tokens,
                                  int num_heads, int head_size, int rot_dim,
                                  int64_t key_stride, bool neox, const PT *rows) {
  const int half = rot_dim / 2;
  const int pairs = num_heads * half;
  for (int t = blockIdx.x; t < num_tokens; t += gridDim.x) {
    const int64_t row = key_row(rows, t);
    if (row < 0) continue;
    const int64_t po = static_cast<int64_t>(old_pos[t]);
    const int64_t pn = static_cast<int64_t>(new_pos[t]);
    const CT *co = cache + po * rot_dim;
    const CT *cn = cache + pn * rot_dim;
    KT *kt = key + row * key_stride;
    for (int q = threadIdx.x; q < pairs; q += blockDim.x) {
      const int h = q / half;
      const int i = q - h * half;
      const float ca = to_f(cn[i]), sa = to_f(cn[half + i]);
      const float cb = to_f(co[i]), sb = to_f(co[half + i]);
      float cd, sd;  // cos / sin (new - old)
      rot_delta(ca, sa, cb, sb, cd, sd);
      KT *kh = kt + static_cast<int64_t>(h) * head_size;
      const int i1 = neox ? i : 2 * i;
      const int i2 = neox ? i + half : 2 * i + 1;
      const float x1 = to_f(kh[i1]);
      const float x2 = to_f(kh[i2]);
      float y1, y2;
      rot_apply(x1, x2, cd, sd, y1, y2);
      kh[i1] = from_f<KT>(y1);
      kh[i2] = from_f<KT>(y2);
    }
  }
}

// N consecutive cos/sin values as fp32: 16-byte loads for an fp32 cache
// (the caller's offsets keep them 16-byte aligned), element loads otherwise.
template <typename CT, int N>
__device__ __forceinline__ void load_cs(const CT *p, float (&o)[N]) {
  if constexpr (std::is_same<CT, float>::value && N % 4 == 0) {
#pragma unroll
    for (int k = 0; k < N / 4; ++k) {
      const float4 v = reinterpret_cast<const float4 *>(p)[k];
      o[4 * k] = v.x;
      o[4 * k + 1] = v.y;
      o[4 * k + 2] = v.z;
      o[4 * k + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < N; ++k) o[k] = to_f(p[k]);
  }
}

// Vector path: one warp per token (grid-stride); a unit is VE = 16 / sizeof(KT)
// consecutive rotary dims of one head, moved with 16-byte loads and stores,
// and its cos/sin rows read as vectors too.  neox: the unit's first halves at
// [i0, i0 + VE) and partners at half + i0; GPT-J: the unit holds VE / 2
// adjacent (2p, 2p + 1) pairs.  Same arithmetic as rope_delta_kernel, so both
// paths give identical results.
template <typename KT, typename CT, typename PT, bool kNeox>
__global__ void __launch_bounds__(128) rope_delta_vec_kernel(
    const PT *__restrict__ old_pos, const PT *__restrict__ new_pos, KT *key,
    const CT *__restrict__ cache, int num_tokens, int num_heads, int head_size, int rot_dim,
    int64_t key_stride, const PT *rows, const int64_t *__restrict__ layer_keys) {
  constexpr int VE = 16 / sizeof(KT);
  constexpr int NP = kNeox ? VE : VE / 2;  // rotation pairs per unit
  // several layers in one launch: blockIdx.y picks the layer's key view
  if (layer_keys != nullptr) key = reinterpret_cast<KT *>(layer_keys[blockIdx.y]);
  const int half = rot_dim / 2;
  const int per_head = kNeox ? half / VE : rot_dim / VE;
  const int units = num_heads * per_head;
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  if (units <= 16 && (32 % units) == 0) {
    // few units per token (e.g. MLA's single 64-dim rope head: 4 units):
    // a warp takes 32 / units tokens at once, one unit per lane
    const int tpw = 32 / units;
    const int u = lane % units;
    const int h = u / per_head;
    const int g = u - h * per_head;
    const int i0 = kNeox ? g * VE : g * VE / 2;
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    for (int64_t tb = wid * tpw; tb < num_tokens; tb += static_cast<int64_t>(nw) * tpw) {
      const int64_t t = tb + lane / units;
      if (t >= num_tokens) continue;
      const int64_t row = key_row(rows, t);
      if (row < 0) continue;
      const CT *co = cache + static_cast<int64_t>(old_pos[t]) * rot_dim;
      const CT *cn = cache + static_cast<int64_t>(new_pos[t]) * rot_dim;
      KT *kh = key + row * key_stride + static_cast<int64_t>(h) * head_size;
      float ca[NP], sa[NP], cb[NP], sb[NP];
      load_cs<CT, NP>(cn + i0, ca);
      load_cs<CT, NP>(cn + half + i0, sa);
      load_cs<CT, NP>(co + i0, cb);
      load_cs<CT, NP>(co + half + i0, sb);
      if (kNeox) {
        uint4 a = *reinterpret_cast<const uint4 *>(kh + i0);
        uint4 b = *reinterpret_cast<const uint4 *>(kh + half + i0);
        KT *x1 = reinterpret_cast<KT *>(&a);
        KT *x2 = reinterpret_cast<KT *>(&b);
#pragma unroll
        for (int j = 0; j < VE; ++j) {
          float cd, sd, y1, y2;
          rot_delta(ca[j], sa[j], cb[j], sb[j], cd, sd);
          rot_apply(to_f(x1[j]), to_f(x2[j]), cd, sd, y1, y2);
          x1[j] = from_f<KT>(y1);
          x2[j] = from_f<KT>(y2);
        }
        *reinterpret_cast<uint4 *>(kh + i0) = a;
        *reinterpret_cast<uint4 *>(kh + half + i0) = b;
      } else {
        uint4 a = *reinterpret_cast<const uint4 *>(kh + g * VE);
        KT *x = reinterpret_cast<KT *>(&a);
#pragma unroll
        for (int j = 0; j < VE / 2; ++j) {
          float cd, sd, y1, y2;
          rot_delta(ca[j], sa[j], cb[j], sb[j], cd, sd);
          rot_apply(to_f(x[2 * j]), to_f(x[2 * j + 1]), cd, sd, y1, y2);
          x[2 * j] = from_f<KT>(y1);
          x[2 * j + 1] = from_f<KT>(y2);
        }
        *reinterpret_cast<uint4 *>(kh + g * VE) = a;
      }
    }
    return;
  }
  // the warp's next 32 tokens' rows and positions are read one per lane and
  // handed out by shuffles, so a token's cos/sin loads do not wait on its own
  // position loads
  int64_t pf_row = -1, pf_po = 0, pf_pn = 0;
  int it = 0;
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < num_tokens;
       t += nw, ++it) {
    if ((it & 31) == 0) {
      const long long tl = static_cast<long long>(t) + static_cast<long long>(lane) * nw;
      pf_row = -1;
      if (tl < num_tokens) {
        pf_row = key_row(rows, static_cast<int>(tl));
        pf_po = static_cast<int64_t>(old_pos[tl]);
        pf_pn = static_cast<int64_t>(new_pos[tl]);
      }
    }
    const int src = it & 31;
    const int64_t row = __shfl_sync(0xffffffffu, pf_row, src);
    if (row < 0) continue;
    const int64_t po = __shfl_sync(0xffffffffu, pf_po, src);
    const int64_t pn = __shfl_sync(0xffffffffu, pf_pn, src);
    const CT *co = cache + po * rot_dim;
    const CT *cn = cache + pn * rot_dim;
    KT *kt = key + row * key_stride;
    if (per_head <= 32 && (32 % per_head) == 0) {
      // Lane = (unit g of a head, head group): the rotation by the angle
      // difference of unit g is formed once and applied to every head of the
      // lane's group, whose key loads are all issued before the first use.
      const int g = lane % per_head;
      const int hg = 32 / per_head;
      const int i0 = kNeox ? g * VE : g * VE / 2;
      // two heads of the lane's group at a time: their four key loads are in
      // flight together (the first pair's before the cos/sin loads), and the
      // register count leaves room for 3 CTAs/SM
      uint4 a[2], b[2];
      KT *kh[2];
      auto load_pair = [&](int hb) {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int h = hb + k * hg;
          kh[k] = h < num_heads ? kt + static_cast<int64_t>(h) * head_size : nullptr;
          if (kh[k] == nullptr) continue;
          if (kNeox) {
            a[k] = *reinterpret_cast<const uint4 *>(kh[k] + i0);
            b[k] = *reinterpret_cast<const uint4 *>(kh[k] + half + i0);
          } else {
            a[k] = *reinterpret_cast<const uint4 *>(kh[k] + g * VE);
          }
        }
      };
      const int hb0 = lane / per_head;
      if (hb0 < num_heads) load_pair(hb0);
      float ca[NP], sa[NP], cb[NP], sb[NP], cd[NP], sd[NP];
      load_cs<CT, NP>(cn + i0, ca);
      load_cs<CT, NP>(cn + half + i0, sa);
      load_cs<CT, NP>(co + i0, cb);
      load_cs<CT, NP>(co + half + i0, sb);
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        rot_delta(ca[j], sa[j], cb[j], sb[j], cd[j], sd[j]);
      }
      for (int hb = hb0; hb < num_heads; hb += 2 * hg) {
        if (hb != hb0) load_pair(hb);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (kh[k] == nullptr) continue;
          if (kNeox) {
            KT *x1 = reinterpret_cast<KT *>(&a[k]);
            KT *x2 = reinterpret_cast<KT *>(&b[k]);
#pragma unroll
            for (int j = 0; j < VE; ++j) {
              float y1, y2;
              rot_apply(to_f(x1[j]), to_f(x2[j]), cd[j], sd[j], y1, y2);
              x1[j] = from_f<KT>(y1);
              x2[j] = from_f<KT>(y2);
            }
            *reinterpret_cast<uint4 *>(kh[k] + i0) = a[k];
            *reinterpret_cast<uint4 *>(kh[k] + half + i0) = b[k];
          } else {
            KT *x = reinterpret_cast<KT *>(&a[k]);
#pragma unroll
            for (int j = 0; j < VE / 2; ++j) {
              float y1, y2;
              rot_apply(to_f(x[2 * j]), to_f(x[2 * j + 1]), cd[j], sd[j], y1, y2);
              x[2 * j] = from_f<KT>(y1);
              x[2 * j + 1] = from_f<KT>(y2);
            }
            *reinterpret_cast<uint4 *>(kh[k] + g * VE) = a[k];
          }
        }
      }
      continue;
    }
    for (int u = lane; u < units; u += 32) {
      const int h = u / per_head;
      const int g = u - h * per_head;
      KT *kh = kt + static_cast<int64_t>(h) * head_size;
      const int i0 = kNeox ? g * VE : g * VE / 2;  // first rotation pair of the unit
      float ca[NP], sa[NP], cb[NP], sb[NP];
      load_cs<CT, NP>(cn + i0, ca);
      load_cs<CT, NP>(cn + half + i0, sa);
      load_cs<CT, NP>(co + i0, cb);
      load_cs<CT, NP>(co + half + i0, sb);
      if (kNeox) {
        uint4 a = *reinterpret_cast<const uint4 *>(kh + i0);
        uint4 b = *reinterpret_cast<const uint4 *>(kh + half + i0);
        KT *x1 = reinterpret_cast<KT *>(&a);
        KT *x2 = reinterpret_cast<KT *>(&b);
#pragma unroll
        for (int j = 0; j < VE; ++j) {
          float cd, sd, y1, y2;
          rot_delta(ca[j], sa[j], cb[j], sb[j], cd, sd);
          rot_apply(to_f(x1[j]), to_f(x2[j]), cd, sd, y1, y2);
          x1[j] = from_f<KT>(y1);
          x2[j] = from_f<KT>(y2);
        }
        *reinterpret_cast<uint4 *>(kh + i0) = a;
        *reinterpret_cast<uint4 *>(kh + half + i0) = b;
      } else {
        const int e0 = g * VE;
        uint4 a = *reinterpret_cast<const uint4 *>(kh + e0);
        KT *x = reinterpret_cast<KT *>(&a);
#pragma unroll
        for (int j = 0; j < VE / 2; ++j) {
          float cd, sd, y1, y2;
          rot_delta(ca[j], sa[j], cb[j], sb[j], cd, sd);
          rot_apply(to_f(x[2 * j]), to_f(x[2 * j + 1]), cd, sd, y1, y2);
          x[2 * j] = from_f<KT>(y1);
          x[2 * j + 1] = from_f<KT>(y2);
        }
        *reinterpret_cast<uint4 *>(kh + e0) = a;
      }
    }
  }
}

template <typename KT, typename CT, typename PT>
static void launch_rope_t(const PT *op, const PT *np, at::Tensor &key, const at::Tensor &cache,
                          int T, int H, int D, int rot, int64_t stride, bool neox,
                          cudaStream_t s, const PT *rows, const int64_t *layer_keys = nullptr,
                          int num_layers = 1) {
  constexpr int VE = 16 / sizeof(KT);
  const int half = rot / 2;
  const bool vec = (reinterpret_cast<uintptr_t>(key.data_ptr()) % 16 == 0) &&
                   (stride * static_cast<int64_t>(sizeof(KT))) % 16 == 0 &&
                   (D * static_cast<int>(sizeof(KT))) % 16 == 0 &&
                   (neox ? half % VE == 0 : rot % VE == 0) &&
                   reinterpret_cast<uintptr_t>(cache.data_ptr()) % 16 == 0 &&
                   (rot * static_cast<int>(sizeof(CT))) % 16 == 0;
  auto *kp = reinterpret_cast<KT *>(key.data_ptr());
  const auto *cp = reinterpret_cast<const CT *>(cache.data_ptr());
  if (vec) {
    int dev = 0, sms = 148;
    C10_CUDA_CHECK(cudaGetDevice(&dev));
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // 4 warps per block; about 16 blocks per SM in all, over the layers
    const int per_layer =
        std::max(1, std::min((T + 3) / 4, sms * 16 / std::max(1, num_layers)));
    const dim3 grid(per_layer, num_layers);
    if (neox)
      rope_delta_vec_kernel<KT, CT, PT, true><<<grid, 128, 0, s>>>(op, np, kp, cp, T, H, D,
                                                                   rot, stride, rows,
                                                                   layer_keys);
    else
      rope_delta_vec_kernel<KT, CT, PT, false><<<grid, 128, 0, s>>>(op, np, kp, cp, T, H, D,
                                                                    rot, stride, rows,
                                                                    layer_keys);
    return;
  }
  TORCH_CHECK(layer_keys == nullptr, "rope: several layers need 16-byte aligned key rows");
  const int threads = std::min(1024, std::max(32, ((H * rot / 2) + 31) / 32 * 32));
  const int blocks = std::min(T, 148 * 16);
  rope_delta_kernel<KT, CT, PT><<<blocks, threads, 0, s>>>(op, np, kp, cp, T, H, D, rot, stride,
                                                           neox, rows);
}

template <typename KT, typename CT>
static void launch_rope(const at::Tensor &op, const at::Tensor &np, at::Tensor &key,
                        const at::Tensor &cache, int T, int H, int D, int rot,
                        int64_t stride, bool neox, cudaStream_t s,
                        const c10::optional<at::Tensor> &rows,
                        const int64_t *layer_keys = nullptr, int num_layers = 1) {
  if (op.scalar_type() == at::kLong)
    launch_rope_t<KT, CT, int64_t>(op.data_ptr<int64_t>(), np.data_ptr<int64_t>(), key, cache,
                                   T, H, D, rot, stride, neox, s,
                                   rows.has_value() ? rows->data_ptr<int64_t>() : nullptr,
                                   layer_keys, num_layers);
  else
    launch_rope_t<KT, CT, int32_t>(op.data_ptr<int32_t>(), np.data_ptr<int32_t>(), key, cache,
                                   T, H, D, rot, stride, neox, s,
                                   rows.has_value() ? rows->data_ptr<int32_t>() : nullptr,
                                   layer_keys, num_layers);
}

// `slot_mapping` (optional, the positions' dtype): token t's key row is
// key[slot_mapping[t]] -- key is then a [cache rows, H*D] view of a paged
// cache plane -- and tokens with a negative slot are skipped.
static void rope_impl(const at::Tensor &old_positions, const at::Tensor &new_positions,
                      at::Tensor &key, int64_t head_size, const at::Tensor &cos_sin_cache,
                      bool is_neox, const c10::optional<at::Tensor> &slot_mapping,
                      const int64_t *layer_keys, int num_layers) {
  TORCH_CHECK(key.is_cuda() && old_positions.is_cuda() && new_positions.is_cuda() &&
                  cos_sin_cache.is_cuda(),
              "rope: all tensors must be on the device");
  TORCH_CHECK(old_positions.scalar_type() == new_positions.scalar_type() &&
                  (old_positions.scalar_type() == at::kLong ||
                   old_positions.scalar_type() == at::kInt),
              "rope: positions must both be int32 or int64");
  const int T = static_cast<int>(old_positions.numel());
  TORCH_CHECK(new_positions.numel() == T, "rope: position length mismatch");
  const bool mapped = slot_mapping.has_value();
  if (mapped) {
    TORCH_CHECK(slot_mapping->is_cuda() && slot_mapping->is_contiguous() &&
                    slot_mapping->scalar_type() == old_positions.scalar_type() &&
                    slot_mapping->numel() == T,
                "rope: slot_mapping must be a contiguous device tensor of the positions' "
                "dtype and length");
    TORCH_CHECK(key.dim() == 2, "rope: with a slot mapping, key is [cache rows, H*D]");
  } else {
    TORCH_CHECK(key.dim() >= 2 && key.size(0) == T, "rope: key must be [T, H*D]");
  }
  TORCH_CHECK(key.stride(-1) == 1, "rope: key rows must be contiguous");
  const int64_t rows_in_key = key.size(0);
  const int64_t hidden = rows_in_key > 0 ? key.numel() / rows_in_key : 0;
  TORCH_CHECK(hidden % head_size == 0, "rope: hidden not a multiple of head_size");
  const int H = static_cast<int>(hidden / head_size);
  const int rot = static_cast<int>(cos_sin_cache.size(1));
  TORCH_CHECK(rot <= head_size && rot % 2 == 0, "rope: bad rot_dim");
  TORCH_CHECK(cos_sin_cache.is_contiguous(), "rope: cos_sin_cache must be contiguous");
  const int64_t stride = key.dim() == 2 ? key.stride(0) : hidden;
  if (key.dim() != 2) TORCH_CHECK(key.is_contiguous(), "rope: key must be contiguous");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(key.device());
  auto op = old_positions.contiguous();
  auto np = new_positions.contiguous();
  cudaStream_t s = at::cuda::getCurrentCUDAStream().stream();
  const auto kt = key.scalar_type();
  const auto ct = cos_sin_cache.scalar_type();
  const int D = static_cast<int>(head_size);
#define LMC_ROPE_CASE(KTYPE, KCT)                                                  \
  if (ct == at::kFloat)                                                            \
    launch_rope<KTYPE, float>(op, np, key, cos_sin_cache, T, H, D, rot, stride,    \
                              is_neox, s, slot_mapping, layer_keys, num_layers);   \
  else if (ct == at::kBFloat16)                                                    \
    launch_rope<KTYPE, __nv_bfloat16>(op, np, key, cos_sin_cache, T, H, D, rot,    \
                                      stride, is_neox, s, slot_mapping,            \
                                      layer_keys, num_layers);                     \
  else if (ct == at::kHalf)                                                        \
    launch_rope<KTYPE, __half>(op, np, key, cos_sin_cache, T, H, D, rot, stride,   \
                               is_neox, s, slot_mapping, layer_keys, num_layers);  \
  else                                                                             \
    TORCH_CHECK(false, "rope: unsupported cos_sin_cache dtype");
  if (kt == at::kBFloat16) {
    LMC_ROPE_CASE(__nv_bfloat16, 0)
  } else if (kt == at::kHalf) {
    LMC_ROPE_CASE(__half, 0)
  } else if (kt == at::kFloat) {
    LMC_ROPE_CASE(float, 0)
  } else {
    TORCH_CHECK(false, "rope: unsupported key dtype");
  }
#undef LMC_ROPE_CASE
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rotary_embedding_k_fused(const at::Tensor &old_positions,
                              const at::Tensor &new_positions, at::Tensor &key,
                              int64_t head_size, const at::Tensor &cos_sin_cache,
                              bool is_neox, const c10::optional<at::Tensor> &slot_mapping) {
  rope_impl(old_positions, new_positions, key, head_size, cos_sin_cache, is_neox, slot_mapping,
            nullptr, 1);
}

// The same re-rotation applied to the key views of several layers (same
// shape, strides and dtype: e.g. the rope columns of every layer of an MLA
// cache) in one launch; blockIdx.y picks the layer.  Layers whose views are
// not 16-byte aligned run one launch each.
void rotary_embedding_k_fused_layers(const at::Tensor &old_positions,
                                     const at::Tensor &new_positions,
                                     const std::vector<at::Tensor> &keys, int64_t head_size,
                                     const at::Tensor &cos_sin_cache, bool is_neox,
                                     const c10::optional<at::Tensor> &slot_mapping) {
  TORCH_CHECK(!keys.empty(), "rope: no layers");
  const at::Tensor &k0 = keys[0];
  bool aligned = true;
  for (const auto &k : keys) {
    TORCH_CHECK(k.device() == k0.device() && k.scalar_type() == k0.scalar_type() &&
                    k.sizes() == k0.sizes() && k.strides() == k0.strides(),
                "rope: every layer's key view needs the same shape, strides and dtype");
    aligned = aligned && reinterpret_cast<uintptr_t>(k.data_ptr()) % 16 == 0;
  }
  if (!aligned || keys.size() == 1) {
    for (const auto &k : keys) {
      at::Tensor kk = k;
      rope_impl(old_positions, new_positions, kk, head_size, cos_sin_cache, is_neox,
                slot_mapping, nullptr, 1);
    }
    return;
  }
  const c10::cuda::CUDAGuard guard(k0.device());
  auto host = at::empty({static_cast<int64_t>(keys.size())},
                        at::TensorOptions().dtype(at::kLong).pinned_memory(true));
  for (size_t i = 0; i < keys.size(); ++i)
    host.data_ptr<int64_t>()[i] = reinterpret_cast<int64_t>(keys[i].data_ptr());
  auto table = host.to(k0.device(), /*non_blocking=*/true);
  at::Tensor kk = k0;
  rope_impl(old_positions, new_positions, kk, head_size, cos_sin_cache, is_neox, slot_mapping,
            table.data_ptr<int64_t>(), static_cast<int>(keys.size()));
}

}  // namespace lmc
