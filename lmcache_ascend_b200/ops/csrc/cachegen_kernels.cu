// K7: CacheGen entropy coding -- CDF construction, encode and decode.
//
// Format (kept compatible with the reference's kernel tests,
// tests/v1/test_cachegen_kernels.py, and its description in
// docs/cachegen/Cachegen.md:34-41): every (layer, channel) stream has a
// 16-bit CDF whose symbol intervals are powers of two aligned to their size,
// so a symbol always maps to the same prefix code = the top `len` bits of the
// interval start, len = 16 - log2(width).  Bits are packed MSB-first; a
// stream's byte length is ceil(bits / 8) with zero padding.
//
// CDF tensor: int16 [L, C, bins + 1].  Entry s (s < bins) holds
// (start_s & 0xFFF0) | len_s: starts are multiples of 16 (max code length
// 12 bits) so the low 4 bits carry the code length for the decoder.  The last
// entry stands for 0x10000 and is ignored.  Encode derives lengths from the
// interval widths, so it also accepts CDFs without length bits (as the
// reference tests pass).  Decode requires non-decreasing starts.
//
// calculate_cdf builds the aligned CDF from a histogram with an exact integer
// procedure (cdf_assign below); the same procedure is mirrored in Python for
// the CPU path, so both produce identical tables.
//
// Decode inputs follow the reference's `decode_fast_prefsum`
// (csrc/cachegen_kernels.cpp:64-107): stream byte lengths are given as an
// inclusive prefix sum over the row-major (layer, channel) order and the
// streams are concatenated in that order.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace lmc {

constexpr int kCgMaxBins = 256;
constexpr int kCgChanPerBlock = 32;

// ---------------------------------------------------------------------------
// Aligned CDF assignment for one channel (runs on one thread).
//   counts[bins] -> start[bins], len[bins]
// ---------------------------------------------------------------------------
__host__ __device__ inline int cg_popcount(unsigned x) {
#ifdef __CUDA_ARCH__
  return __popc(x);
#else
  return __builtin_popcount(x);
#endif
}

__host__ __device__ inline int cg_log2(unsigned w) {  // w is a power of two
  int e = 0;
  while ((1u << e) < w) ++e;
  return e;
}

__host__ __device__ inline void cdf_assign(const unsigned *counts, int bins,
                                           unsigned short *out /* [bins+1] */) {
  if (bins == 1) {
    out[0] = 0;  // start 0, len 0: the only symbol costs no bits
    out[1] = 0;
    return;
  }
  unsigned long long total = 0;
  for (int s = 0; s < bins; ++s) total += counts[s];
  // smoothed probability p_s = (2 c_s + 1) / (2 N + bins)
  const unsigned long long den = 2ull * total + static_cast<unsigned>(bins);
  unsigned pos = 0;
  for (int s = 0; s < bins; ++s) {
    const int k = bins - s;  // symbols left, including s
    const unsigned R = 65536u - pos;
    unsigned w;
    if (k == 1) {
      w = R;
    } else {
      // desired width: power of two nearest (linearly) to p * 65536
      const unsigned long long x = (2ull * counts[s] + 1ull) * 65536ull;
      unsigned wd = 16;
      while (wd < 32768u && den * (2ull * wd) <= x) wd <<= 1;
      if (wd < 32768u && 2ull * x >= 3ull * den * wd) wd <<= 1;
      const int ed = cg_log2(wd);
      const unsigned maxw = pos == 0 ? 32768u : (pos & (~pos + 1u));
      int best_e = -1, best_d = 1 << 30;
      for (int e = 4; (1u << e) <= maxw; ++e) {
        const unsigned cand = 1u << e;
        if (cand >= R) break;
        const unsigned rem = R - cand;
        if (cg_popcount(rem) > k - 1) continue;
        if (static_cast<unsigned>(k - 1) > rem / 16u) continue;
        const int d = e > ed ? e - ed : ed - e;
        if (d < best_d || (d == best_d && e > best_e)) {
          best_d = d;
          best_e = e;
        }
      }
      w = best_e >= 0 ? (1u << best_e) : 16u;  // unreachable fallback
    }
    const int len = 16 - cg_log2(w);
    out[s] = static_cast<unsigned short>((pos & 0xFFF0u) | static_cast<unsigned>(len));
    pos += w;
  }
  out[bins] = 0;  // stands for 0x10000
}

// ---------------------------------------------------------------------------
// calculate_cdf: block per (layer, 32-channel tile); histogram in shared mem.
// ---------------------------------------------------------------------------
__global__ void cg_cdf_kernel(const uint8_t *__restrict__ in, int16_t *out,
                              int L, int T, int C, int bins) {
  extern __shared__ unsigned hist[];  // [32][bins]
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCgChanPerBlock;
  const int nc = min(kCgChanPerBlock, C - c0);
  for (int i = threadIdx.x; i < kCgChanPerBlock * bins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const uint8_t *base = in + static_cast<size_t>(l) * T * C + c0;
  if (lane < nc) {
    for (int t = warp; t < T; t += nwarps) {
      int s = base[static_cast<size_t>(t) * C + lane];
      if (s >= bins) s = bins - 1;
      atomicAdd(&hist[lane * bins + s], 1u);
    }
  }
  __syncthreads();
  if (threadIdx.x < nc) {
    unsigned short tmp[kCgMaxBins + 1];
    cdf_assign(&hist[threadIdx.x * bins], bins, tmp);
    int16_t *o = out + (static_cast<size_t>(l) * C + c0 + threadIdx.x) * (bins + 1);
    for (int s = 0; s <= bins; ++s) o[s] = static_cast<int16_t>(tmp[s]);
  }
}

// ---------------------------------------------------------------------------
// encode: one lane per (layer, channel) stream; lanes of a warp take 32
// consecutive channels so symbol reads are coalesced.
// ---------------------------------------------------------------------------
__global__ void cg_encode_kernel(const int16_t *__restrict__ cdf,
                                 const uint8_t *__restrict__ sym, uint8_t *out,
                                 int32_t *out_len, int L, int T, int C, int bins,
                                 int cap, DeviceStatus *status) {
  extern __shared__ unsigned short tab[];  // [32][2][bins]: code, len
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCgChanPerBlock;
  const int lane = threadIdx.x;
  const int nc = min(kCgChanPerBlock, C - c0);
  // build code tables for the 32 channels (one channel per thread)
  if (lane < nc) {
    const int16_t *cd = cdf + (static_cast<size_t>(l) * C + c0 + lane) * (bins + 1);
    unsigned short *code = tab + lane * 2 * bins;
    unsigned short *len = code + bins;
    for (int s = 0; s < bins; ++s) {
      const unsigned st = static_cast<unsigned short>(cd[s]) & 0xFFF0u;
      const unsigned en =
          (s + 1 == bins) ? 65536u : (static_cast<unsigned short>(cd[s + 1]) & 0xFFF0u);
      const unsigned w = en > st ? en - st : 0u;
      if (w == 0) {
        code[s] = 0;
        len[s] = 0xFFFF;  // not encodable
      } else {
        int e = 31 - __clz(w);  // floor(log2 w)
        const int ln = 16 - e;
        len[s] = static_cast<unsigned short>(ln);
        code[s] = static_cast<unsigned short>(ln == 0 ? 0 : (st >> (16 - ln)));
      }
    }
  }
  __syncwarp();
  if (lane >= nc) return;
  const unsigned short *code = tab + lane * 2 * bins;
  const unsigned short *len = code + bins;
  const int c = c0 + lane;
  const uint8_t *sp = sym + static_cast<size_t>(l) * T * C + c;
  uint8_t *op = out + (static_cast<size_t>(l) * C + c) * cap;
  unsigned long long acc = 0;  // bits, MSB-first, `nb` valid bits at the top
  int nb = 0;
  int nbytes = 0;
  bool overflow = false;
  for (int t = 0; t < T; ++t) {
    int s = sp[static_cast<size_t>(t) * C];
    if (s >= bins) s = bins - 1;
    const unsigned ln = len[s];
    if (ln == 0xFFFF) {
      report_status(status, kStatusBadIndex, l * C + c, t, s);
      continue;
    }
    if (ln) {
      acc |= static_cast<unsigned long long>(code[s]) << (64 - nb - ln);
      nb += ln;
    }
    while (nb >= 8) {
      if (nbytes < cap)
        op[nbytes] = static_cast<uint8_t>(acc >> 56);
      else
        overflow = true;
      ++nbytes;
      acc <<= 8;
      nb -= 8;
    }
  }
  if (nb > 0) {
    if (nbytes < cap)
      op[nbytes] = static_cast<uint8_t>(acc >> 56);
    else
      overflow = true;
    ++nbytes;
  }
  if (overflow) {
    report_status(status, kStatusBadIndex, l * C + c, nbytes, cap);
    nbytes = cap;
  }
  out_len[static_cast<size_t>(l) * C + c] = nbytes;
}

// ---------------------------------------------------------------------------
// decode (prefix-summed lengths): one lane per stream, binary search of the
// 16-bit window in the channel's interval starts.
// ---------------------------------------------------------------------------
__global__ void cg_decode_kernel(const int16_t *__restrict__ cdf,
                                 const uint8_t *__restrict__ bytes,
                                 const int32_t *__restrict__ cum_len,
                                 uint8_t *out, int L, int T, int C, int bins) {
  extern __shared__ unsigned short st_tab[];  // [32][bins] starts, [32][bins] lens
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCgChanPerBlock;
  const int lane = threadIdx.x;
  const int nc = min(kCgChanPerBlock, C - c0);
  unsigned short *starts = st_tab + lane * bins;
  unsigned short *lens = st_tab + kCgChanPerBlock * bins + lane * bins;
  if (lane < nc) {
    const int16_t *cd = cdf + (static_cast<size_t>(l) * C + c0 + lane) * (bins + 1);
    for (int s = 0; s < bins; ++s) {
      const unsigned short v = static_cast<unsigned short>(cd[s]);
      starts[s] = v & 0xFFF0u;
      lens[s] = v & 0xFu;
    }
  }
  __syncwarp();
  if (lane >= nc) return;
  const int c = c0 + lane;
  const size_t idx = static_cast<size_t>(l) * C + c;
  const int32_t b0 = idx == 0 ? 0 : cum_len[idx - 1];
  const int32_t b1 = cum_len[idx];
  const uint8_t *p = bytes + b0;
  const int n = b1 - b0;
  int rd = 0;                  // next byte to load
  unsigned long long win = 0;  // MSB-aligned bit window
  int nb = 0;
  uint8_t *op = out + static_cast<size_t>(l) * T * C + c;
  for (int t = 0; t < T; ++t) {
    while (nb <= 56) {
      const unsigned long long byte = rd < n ? __ldg(p + rd) : 0ull;
      ++rd;
      win |= byte << (56 - nb);
      nb += 8;
    }
    const unsigned v = static_cast<unsigned>(win >> 48);
    // largest s with starts[s] <= v
    int lo = 0, hi = bins - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (starts[mid] <= v) lo = mid; else hi = mid - 1;
    }
    const int ln = lens[lo];
    win <<= ln;
    nb -= ln;
    op[static_cast<size_t>(t) * C] = static_cast<uint8_t>(lo);
  }
}

// ---------------------------------------------------------------------------
// Host launchers (op names of the reference's pybind module).
// ---------------------------------------------------------------------------
at::Tensor calculate_cdf(const at::Tensor &input, int64_t n_bins) {
  TORCH_CHECK(input.is_cuda() && input.dim() == 3, "input: device [L, T, C]");
  TORCH_CHECK(input.scalar_type() == at::kByte || input.scalar_type() == at::kChar,
              "input must be uint8/int8 symbols");
  TORCH_CHECK(n_bins >= 1 && n_bins <= kCgMaxBins, "1 <= n_bins <= 256");
  auto in = input.contiguous();
  const int L = in.size(0), T = in.size(1), C = in.size(2);
  const c10::cuda::CUDAGuard guard(in.device());
  auto out = at::zeros({L, C, n_bins + 1}, in.options().dtype(at::kShort));
  if (L == 0 || C == 0) return out;
  dim3 grid((C + kCgChanPerBlock - 1) / kCgChanPerBlock, L);
  const size_t smem = sizeof(unsigned) * kCgChanPerBlock * n_bins;
  cg_cdf_kernel<<<grid, 256, smem, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const uint8_t *>(in.data_ptr()), out.data_ptr<int16_t>(),
      L, T, C, static_cast<int>(n_bins));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void encode_fast_new(const at::Tensor &cdf, const at::Tensor &input_sym,
                     at::Tensor &output_buffer, at::Tensor &output_lengths,
                     const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(cdf.is_cuda() && input_sym.is_cuda() && output_buffer.is_cuda() &&
                  output_lengths.is_cuda(),
              "encode: all tensors must be on the device");
  TORCH_CHECK(input_sym.dim() == 3 && cdf.dim() == 3 && output_buffer.dim() == 3,
              "encode: sym [L,T,C], cdf [L,C,bins+1], out [L,C,cap]");
  const int L = input_sym.size(0), T = input_sym.size(1), C = input_sym.size(2);
  const int bins = static_cast<int>(cdf.size(2)) - 1;
  TORCH_CHECK(bins >= 1 && bins <= kCgMaxBins, "encode: 1 <= bins <= 256");
  TORCH_CHECK(cdf.size(0) == L && cdf.size(1) == C, "encode: cdf shape mismatch");
  TORCH_CHECK(C <= (1 << 15), "encode: at most 32768 channels");
  TORCH_CHECK(output_buffer.size(0) == L && output_buffer.size(1) == C,
              "encode: output buffer shape mismatch");
  TORCH_CHECK(output_lengths.scalar_type() == at::kInt &&
                  output_lengths.numel() == static_cast<int64_t>(L) * C,
              "encode: output_lengths must be int32 [L, C]");
  TORCH_CHECK(output_buffer.is_contiguous() && output_lengths.is_contiguous(),
              "encode: outputs must be contiguous");
  auto c = cdf.to(at::kShort).contiguous();
  auto s = input_sym.contiguous();
  const c10::cuda::CUDAGuard guard(s.device());
  if (L == 0 || C == 0) return;
  dim3 grid((C + kCgChanPerBlock - 1) / kCgChanPerBlock, L);
  const size_t smem = sizeof(unsigned short) * kCgChanPerBlock * 2 * bins;
  DeviceStatus *st = status.has_value()
                         ? reinterpret_cast<DeviceStatus *>(status->data_ptr())
                         : nullptr;
  cg_encode_kernel<<<grid, kCgChanPerBlock, smem,
                     at::cuda::getCurrentCUDAStream().stream()>>>(
      c.data_ptr<int16_t>(), reinterpret_cast<const uint8_t *>(s.data_ptr()),
      reinterpret_cast<uint8_t *>(output_buffer.data_ptr()),
      output_lengths.data_ptr<int32_t>(), L, T, C, bins,
      static_cast<int>(output_buffer.size(2)), st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void decode_fast_prefsum(const at::Tensor &cdf, const at::Tensor &bytestreams,
                         const at::Tensor &lengths, at::Tensor &output) {
  TORCH_CHECK(cdf.is_cuda() && bytestreams.is_cuda() && lengths.is_cuda() &&
                  output.is_cuda(),
              "decode: all tensors must be on the device");
  TORCH_CHECK(cdf.dim() == 3 && output.dim() == 3, "decode: cdf [L,C,bins+1], out [L,T,C]");
  const int L = cdf.size(0), C = cdf.size(1);
  const int bins = static_cast<int>(cdf.size(2)) - 1;
  TORCH_CHECK(bins >= 1 && bins <= kCgMaxBins, "decode: 1 <= bins <= 256");
  TORCH_CHECK(output.size(0) == L && output.size(2) == C, "decode: output shape");
  TORCH_CHECK(lengths.numel() == static_cast<int64_t>(L) * C &&
                  lengths.scalar_type() == at::kInt,
              "decode: lengths must be int32 [L, C] (inclusive prefix sum)");
  TORCH_CHECK(output.is_contiguous(), "decode: output must be contiguous");
  const int T = output.size(1);
  auto c = cdf.to(at::kShort).contiguous();
  auto b = bytestreams.contiguous();
  auto len = lengths.contiguous();
  const c10::cuda::CUDAGuard guard(c.device());
  if (L == 0 || C == 0 || T == 0) return;
  dim3 grid((C + kCgChanPerBlock - 1) / kCgChanPerBlock, L);
  const size_t smem = sizeof(unsigned short) * kCgChanPerBlock * 2 * bins;
  cg_decode_kernel<<<grid, kCgChanPerBlock, smem,
                     at::cuda::getCurrentCUDAStream().stream()>>>(
      c.data_ptr<int16_t>(), reinterpret_cast<const uint8_t *>(b.data_ptr()),
      len.data_ptr<int32_t>(), reinterpret_cast<uint8_t *>(output.data_ptr()),
      L, T, C, bins);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
