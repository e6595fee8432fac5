// K7: CacheGen quantisation and entropy coding -- quantise / dequantise,
// CDF construction, encode and decode.
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
//
// Work decomposition (B200): a stream is inherently serial, so the kernels
// keep one thread per (layer, channel) stream and keep everything else off
// its critical path, with straight-line code so that the 32 lanes of a warp
// (each at its own bit position) do not serialise on divergent branches.
// Encode stages [64 tokens x CH channels] symbol tiles in shared memory with
// 16-byte loads (double buffered: the next tile's loads are in flight while
// the current one is coded) and emits 32-bit big-endian words.  Decode
// keeps no tables in shared memory (they bounded the resident streams): up
// to 16 symbols it compares the window against the whole CDF held in
// registers; above that, against every 16th entry in registers and then a
// 4-step binary search over the chosen group's entries in the stream's own
// (L1-resident) CDF row.  The window is refilled once per two symbols from
// 16-byte loads issued well ahead.  Shared tables elsewhere are laid out
// [entry][channel] so that a warp's lanes hit 32 different banks.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace lmc {

constexpr int kCgMaxBins = 256;
constexpr int kCgChan = 128;     // channels per histogram block
constexpr int kCgExpTab = 8192;  // counts with a precomputed width exponent (split CDF)
constexpr int kCgTile = 64;      // tokens per encode shared-memory tile

__host__ __device__ inline int cg_popcount(unsigned x) {
#ifdef __CUDA_ARCH__
  return __popc(x);
#else
  return __builtin_popcount(x);
#endif
}

__host__ __device__ inline int cg_log2_floor(unsigned v) {  // v >= 1
#ifdef __CUDA_ARCH__
  return 31 - __clz(v);
#else
  return 31 - __builtin_clz(v);
#endif
}

// Smallest e with 2^e >= w (the exponent of a power-of-two width; a last
// symbol's remainder width rounds up).
__host__ __device__ inline int cg_log2(unsigned w) {
  if (w <= 1) return 0;
  const int e = cg_log2_floor(w);
  return (1u << e) < w ? e + 1 : e;
}

__host__ __device__ inline int cg_msb64(unsigned long long v) {  // v >= 1
#ifdef __CUDA_ARCH__
  return 63 - __clzll(static_cast<long long>(v));
#else
  return 63 - __builtin_clzll(v);
#endif
}

// ---------------------------------------------------------------------------
// Aligned CDF assignment for one channel (runs on one thread).
//   counts(s) -> count of symbol s; put(s, entry) stores CDF entry s.
// Widths are powers of two >= 16 summing to 65536, each as close (in log2)
// to the smoothed probability as the alignment of the running start allows,
// with enough room left for the remaining symbols.
// ---------------------------------------------------------------------------
// Desired width exponent of a symbol with `count` occurrences: the largest
// power of two wd in [16, 32768] with den * 2 wd <= x, x = (2 count + 1) 65536
// (a monotone condition: start from an msb estimate and step to it), doubled
// when p * 65536 is nearer the next power.  It depends on the symbol alone,
// so it can be computed for every symbol at once.
__host__ __device__ inline int cg_desired_exp(unsigned count, unsigned long long den) {
  const unsigned long long x = (2ull * count + 1ull) * 65536ull;
  int g = cg_msb64(x) - cg_msb64(den) - 1;
  g = g < 4 ? 4 : (g > 15 ? 15 : g);
  unsigned wd = 1u << g;
  while (wd > 16u && den * (2ull * wd) > x) wd >>= 1;
  while (wd < 32768u && den * (2ull * wd) <= x) wd <<= 1;
  if (wd < 32768u && 2ull * x >= 3ull * den * wd) wd <<= 1;
  return cg_log2(wd);
}

// The serial placement: ed_of(s) -> desired exponent of symbol s.
template <class Ed, class Put>
__host__ __device__ inline void cdf_place(Ed ed_of, int bins, Put put) {
  unsigned pos = 0;
  for (int s = 0; s < bins; ++s) {
    const int k = bins - s;  // symbols left, including s
    const unsigned R = 65536u - pos;
    unsigned w;
    if (k == 1) {
      w = R;
    } else {
      const int ed = ed_of(s);
      const unsigned maxw = pos == 0 ? 32768u : (pos & (~pos + 1u));
      // feasible widths 2^e: aligned at pos, leave room (a sum of at most k-1
      // powers of two >= 16) for the remaining symbols.  Take the feasible e
      // closest to ed, the larger one on a tie.
      int best_e = -1;
      if (k - 1 >= 16) {
        // popcount(R - 2^e) <= 16 <= k - 1 always holds, so the feasible e
        // are the interval [4, emax]: clamp ed into it
        const long long room = static_cast<long long>(R) - 16ll * (k - 1);
        if (room >= 16 && R >= 17) {
          int emax = cg_log2_floor(maxw);
          emax = min(emax, cg_log2_floor(R - 1));
          emax = min(emax, cg_log2_floor(static_cast<unsigned>(room)));
          emax = min(emax, 15);
          if (emax >= 4) best_e = ed < 4 ? 4 : (ed > emax ? emax : ed);
        }
      } else {
        auto feasible = [&](int e) {
          if (e < 4 || e > 15) return false;
          const unsigned cand = 1u << e;
          if (cand > maxw || cand >= R) return false;
          const unsigned rem = R - cand;
          return cg_popcount(rem) <= k - 1 && static_cast<unsigned>(k - 1) <= rem / 16u;
        };
        for (int d = 0; d <= 11 && best_e < 0; ++d) {  // outward from ed
          if (feasible(ed + d)) best_e = ed + d;
          else if (d > 0 && feasible(ed - d)) best_e = ed - d;
        }
      }
      w = best_e >= 0 ? (1u << best_e) : 16u;  // unreachable fallback
    }
    const int len = 16 - cg_log2(w);
    put(s, static_cast<unsigned short>((pos & 0xFFF0u) | static_cast<unsigned>(len)));
    pos += w;
  }
  put(bins, 0);  // stands for 0x10000
}

// smoothed probability p_s = (2 c_s + 1) / (2 N + bins), N = total count
template <class Counts, class Put>
__host__ __device__ inline void cdf_assign(Counts counts, int bins, Put put) {
  if (bins == 1) {
    put(0, 0);  // start 0, len 0: the only symbol costs no bits
    put(1, 0);
    return;
  }
  unsigned long long total = 0;
  for (int s = 0; s < bins; ++s) total += counts(s);
  const unsigned long long den = 2ull * total + static_cast<unsigned>(bins);
  cdf_place([&](int s) { return cg_desired_exp(counts(s), den); }, bins, put);
}

// ---------------------------------------------------------------------------
// calculate_cdf: block per (layer, 128-channel tile).  Each warp takes whole
// token rows (lane = 4 consecutive channels, one 32-bit load); the shared
// histogram column of channel c is (c / 4) + 32 * (c % 4), so the 32 lanes'
// atomics of one step land in 32 different banks.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int cg_hcol(int c) { return (c >> 2) | ((c & 3) << 5); }

// Counters: 16-bit halves of 32-bit words, [bins / 2][kCgChan] words, when
// T < 65536 (half the shared memory: 256 bins fit 3 blocks per SM); 32-bit
// counters [bins][kCgChan] otherwise (kWide).
// Histogram of one (layer, 128-channel tile) into shared memory.
template <bool kWide>
__device__ __forceinline__ void cg_histogram(const uint8_t *__restrict__ in, unsigned *hist,
                                             int l, int T, int C, int c0, int nc, int bins,
                                             bool vec4) {
  const int words = (kWide ? bins : (bins + 1) >> 1) * kCgChan;
  for (int i = threadIdx.x; i < words; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const uint8_t *base = in + static_cast<size_t>(l) * T * C + c0;
  const int cl = lane * 4;
  if (cl < nc) {
    for (int t = warp; t < T; t += nwarps) {
      const uint8_t *rp = base + static_cast<size_t>(t) * C + cl;
      uint32_t v;
      if (vec4) {
        v = __ldg(reinterpret_cast<const uint32_t *>(rp));
      } else {
        v = 0;
        for (int j = 0; j < 4 && cl + j < nc; ++j) v |= static_cast<uint32_t>(__ldg(rp + j)) << (8 * j);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (cl + j < nc) {
          int s = (v >> (8 * j)) & 0xFF;
          if (s >= bins) s = bins - 1;
          if (kWide)
            atomicAdd(&hist[s * kCgChan + cg_hcol(cl + j)], 1u);
          else
            atomicAdd(&hist[(s >> 1) * kCgChan + cg_hcol(cl + j)], 1u << ((s & 1) * 16));
        }
      }
    }
  }
  __syncthreads();
}

template <bool kWide>
__device__ __forceinline__ unsigned cg_hist_count(const unsigned *hist, int s, int col) {
  return kWide ? hist[s * kCgChan + col]
               : (hist[(s >> 1) * kCgChan + col] >> ((s & 1) * 16)) & 0xFFFFu;
}

// Fused form (few bins): histogram, then the assignment by one thread per
// channel from shared memory.
template <bool kWide>
__global__ void __launch_bounds__(256) cg_cdf_kernel(const uint8_t *__restrict__ in,
                                                     int16_t *out, int L, int T, int C,
                                                     int bins, bool vec4) {
  extern __shared__ unsigned hist[];
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCgChan;
  const int nc = min(kCgChan, C - c0);
  cg_histogram<kWide>(in, hist, l, T, C, c0, nc, bins, vec4);
  if (threadIdx.x < nc) {
    const int col = cg_hcol(threadIdx.x);
    int16_t *o = out + (static_cast<size_t>(l) * C + c0 + threadIdx.x) * (bins + 1);
    cdf_assign([&](int s) { return cg_hist_count<kWide>(hist, s, col); }, bins,
               [&](int s, unsigned short v) { o[s] = static_cast<int16_t>(v); });
  }
}

// Split form (many bins): the histogram tables of 256 bins leave room for
// only 3 blocks per SM, and the serial assignment then runs on 12 warps per
// SM.  Here the histogram kernel turns each (symbol, channel) count into its
// desired width exponent at once (it depends on that count and on
// den = 2 T + bins only: every token adds one symbol to every channel) and
// writes them as exps[L][bins][C] bytes; the serial placement then runs as
// its own kernel, one thread per (layer, channel), with no shared memory.
template <bool kWide>
__global__ void __launch_bounds__(256) cg_hist_kernel(const uint8_t *__restrict__ in,
                                                      uint8_t *exps, int L, int T, int C,
                                                      int bins, bool vec4) {
  extern __shared__ unsigned hist[];
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * kCgChan;
  const int nc = min(kCgChan, C - c0);
  const unsigned long long den = 2ull * static_cast<unsigned>(T) + static_cast<unsigned>(bins);
  // the exponent depends on the count alone (den is fixed), so short chunks
  // (T < kCgExpTab) look it up in a table of every count 0..T built once
  uint8_t *tab = reinterpret_cast<uint8_t *>(hist + (kWide ? bins : (bins + 1) / 2) * kCgChan);
  const bool use_tab = T < kCgExpTab;
  if (use_tab)
    for (int v = threadIdx.x; v <= T; v += blockDim.x)
      tab[v] = static_cast<uint8_t>(cg_desired_exp(static_cast<unsigned>(v), den));
  cg_histogram<kWide>(in, hist, l, T, C, c0, nc, bins, vec4);  // synchronises
  uint8_t *el = exps + static_cast<size_t>(l) * bins * C + c0;
  for (int i = threadIdx.x; i < bins * kCgChan; i += blockDim.x) {
    const int s = i / kCgChan, c = i - s * kCgChan;
    if (c < nc) {
      const unsigned cnt = cg_hist_count<kWide>(hist, s, cg_hcol(c));
      el[static_cast<size_t>(s) * C + c] =
          use_tab ? tab[cnt] : static_cast<uint8_t>(cg_desired_exp(cnt, den));
    }
  }
}

// Exponents read kBatch at a time (the placement asks for them in order).
struct CgExpBatch {
  static constexpr int kBatch = 16;
  const uint8_t *p;
  size_t stride;
  int bins;
  int base;
  uint8_t buf[kBatch];
  __device__ int operator()(int s) {
    if (s < base || s >= base + kBatch) {
      base = s;
#pragma unroll
      for (int k = 0; k < kBatch; ++k)
        buf[k] = s + k < bins ? __ldg(p + static_cast<size_t>(s + k) * stride) : 0;
    }
    return buf[s - base];
  }
};

// Placement, one thread per (layer, channel), kPlaceCh channels per block.
// Entries are collected kPlaceRun symbols at a time in shared memory and
// then written as one contiguous 2 kPlaceRun-byte piece per channel: written
// one by one, each 2-byte entry would be its own sector write (the lanes'
// rows are 2 (bins + 1) bytes apart).  Every thread runs the same number of
// steps (threads past the last channel repeat it and store nothing), so the
// block can synchronise at every flush.
constexpr int kPlaceCh = 128;
constexpr int kPlaceRun = 16;

__global__ void __launch_bounds__(kPlaceCh) cg_place_kernel(const uint8_t *__restrict__ exps,
                                                            int16_t *out, int L, int C,
                                                            int bins) {
  __shared__ int16_t run[kPlaceCh][kPlaceRun + 1];
  const int row = bins + 1;
  const long long n = static_cast<long long>(L) * C;
  const long long i0 = static_cast<long long>(blockIdx.x) * kPlaceCh;
  const long long i = min(i0 + threadIdx.x, n - 1);
  const int nrows = static_cast<int>(n - i0 < kPlaceCh ? n - i0 : kPlaceCh);
  const int l = static_cast<int>(i / C);
  const int c = static_cast<int>(i - static_cast<long long>(l) * C);
  CgExpBatch eb{exps + static_cast<size_t>(l) * bins * C + c, static_cast<size_t>(C), bins,
                -CgExpBatch::kBatch, {}};
  int16_t *base = out + static_cast<size_t>(i0) * row;
  cdf_place(eb, bins, [&](int s, unsigned short v) {
    run[threadIdx.x][s % kPlaceRun] = static_cast<int16_t>(v);
    if (s % kPlaceRun == kPlaceRun - 1 || s == bins) {
      const int s0 = s - s % kPlaceRun;
      const int cnt = s - s0 + 1;
      __syncthreads();
      // flush entries s0 .. s of every channel, lanes over (channel, entry)
      for (int e = threadIdx.x; e < nrows * cnt; e += kPlaceCh) {
        const int ch = e / cnt, k = e - ch * cnt;
        base[static_cast<size_t>(ch) * row + s0 + k] = run[ch][k];
      }
      __syncthreads();
    }
  });
}

// ---------------------------------------------------------------------------
// encode: block per (layer, 128-channel tile), thread per stream.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cg_bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// Append `n` bytes (the top bytes of big-endian word `w`) at op[nbytes..].
__device__ __forceinline__ void cg_put_bytes(uint8_t *op, int nbytes, int cap, uint32_t w,
                                             int n, bool &overflow) {
  for (int j = 0; j < n; ++j) {
    if (nbytes + j < cap)
      op[nbytes + j] = static_cast<uint8_t>(w >> (24 - 8 * j));
    else
      overflow = true;
  }
}

template <int CH>
__global__ void __launch_bounds__(CH) cg_encode_kernel(
    const int16_t *__restrict__ cdf, const uint8_t *__restrict__ sym, uint8_t *out,
    int32_t *out_len, int L, int T, int C, int bins, int cap, bool vec16, bool word_out,
    DeviceStatus *status) {
  extern __shared__ __align__(16) uint8_t cg_smem[];
  const int tab_words = ((bins + 1) >> 1) * CH;
  uint32_t *tab = reinterpret_cast<uint32_t *>(cg_smem);  // (code << 4) | len, 0xF = invalid
  uint8_t *tile = cg_smem + ((tab_words * 4 + 15) & ~15);  // [2][kCgTile][CH]
  constexpr int kTileBytes = kCgTile * CH;
  constexpr int kRowVecs = CH / 16;  // 16-byte vectors per tile row
  const int l = blockIdx.y;
  const int c0 = blockIdx.x * CH;
  const int tid = threadIdx.x;
  const int nc = min(CH, C - c0);
  if (tid < nc) {
    // the channel's CDF entries are read 16 at a time, so the loads of a
    // 256-symbol table are in flight together instead of one per step
    const unsigned short *cd = reinterpret_cast<const unsigned short *>(cdf) +
                               (static_cast<size_t>(l) * C + c0 + tid) * (bins + 1);
    unsigned st = __ldg(cd) & 0xFFF0u;
    for (int s0 = 0; s0 < bins; s0 += 16) {
      unsigned nxt[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int s = s0 + k;
        nxt[k] = s + 1 < bins ? (__ldg(cd + s + 1) & 0xFFF0u) : 65536u;
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int s = s0 + k;
        if (s >= bins) break;
        const unsigned en = nxt[k];
        const unsigned w = en > st ? en - st : 0u;
        unsigned e = 0xFu;  // not encodable
        if (w != 0) {
          const int ln = 16 - (31 - __clz(w));  // 16 - floor(log2 w)
          e = (static_cast<unsigned>(ln == 0 ? 0 : (st >> (16 - ln))) << 4) |
              static_cast<unsigned>(ln);
        }
        uint32_t &tw = tab[(s >> 1) * CH + tid];
        tw = (s & 1) ? ((tw & 0xFFFFu) | (e << 16)) : ((tw & 0xFFFF0000u) | e);
        st = en;
      }
    }
  }
  const uint8_t *base = sym + static_cast<size_t>(l) * T * C + c0;
  // tile loader: kCgTile * CH / 16 vectors per tile, 4 per thread
  uint4 r[4];
  auto gload = [&](int t0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = tid + k * CH;
      const int row = i / kRowVecs, vc = (i % kRowVecs) * 16;
      const int t = t0 + row;
      r[k] = (t < T && vc < nc)
                 ? __ldg(reinterpret_cast<const uint4 *>(base + static_cast<size_t>(t) * C + vc))
                 : make_uint4(0, 0, 0, 0);
    }
  };
  auto sstore = [&](int b) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = tid + k * CH;
      *reinterpret_cast<uint4 *>(tile + b * kTileBytes + (i / kRowVecs) * CH +
                                 (i % kRowVecs) * 16) = r[k];
    }
  };
  auto bload = [&](int b, int t0) {  // unaligned rows: byte loads straight into the tile
    for (int i = tid; i < kTileBytes; i += CH) {
      const int row = i / CH, c = i % CH;
      const int t = t0 + row;
      tile[b * kTileBytes + i] = (t < T && c < nc) ? __ldg(base + static_cast<size_t>(t) * C + c) : 0;
    }
  };
  if (vec16) {
    gload(0);
    sstore(0);
  } else {
    bload(0, 0);
  }
  __syncthreads();

  const int c = c0 + tid;
  uint8_t *op = out + (static_cast<size_t>(l) * C + c) * cap;
  uint32_t acc = 0;  // MSB-first, `nb` valid bits at the top, nb < 32
  int nb = 0;
  int nbytes = 0;
  bool overflow = false;
  auto emit = [&](uint32_t w) {
    if (word_out && nbytes + 4 <= cap)
      *reinterpret_cast<uint32_t *>(op + nbytes) = cg_bswap(w);
    else
      cg_put_bytes(op, nbytes, cap, w, 4, overflow);
    nbytes += 4;
  };
  auto append = [&](unsigned e, int t) {
    const int ln = static_cast<int>(e & 0xFu);
    if (ln == 0xF) {
      report_status(status, kStatusBadIndex, l * C + c, t, -1);
      return;
    }
    if (ln == 0) return;
    const uint32_t code = e >> 4;
    const int tot = nb + ln;
    if (tot < 32) {
      acc |= code << (32 - tot);
      nb = tot;
    } else {
      emit(acc | (code >> (tot - 32)));
      nb = tot - 32;
      acc = nb ? (code << (32 - nb)) : 0u;
    }
  };
  auto entry = [&](int sym) {
    const int q = sym >= bins ? bins - 1 : sym;
    const uint32_t w = tab[(q >> 1) * CH + tid];
    return (q & 1) ? (w >> 16) : (w & 0xFFFFu);
  };
  const int ntiles = (T + kCgTile - 1) / kCgTile;
  for (int k = 0; k < ntiles; ++k) {
    const int b = k & 1;
    const bool more = k + 1 < ntiles;
    if (more && vec16) gload((k + 1) * kCgTile);
    if (tid < nc) {
      const int rows = min(kCgTile, T - k * kCgTile);
      const uint8_t *tp = tile + b * kTileBytes + tid;
      constexpr int kCgChanT = CH;
      const int t0 = k * kCgTile;
      int row = 0;
      for (; row + 4 <= rows; row += 4) {  // four independent lookups, then the chain
        const unsigned e0 = entry(tp[(row + 0) * kCgChanT]);
        const unsigned e1 = entry(tp[(row + 1) * kCgChanT]);
        const unsigned e2 = entry(tp[(row + 2) * kCgChanT]);
        const unsigned e3 = entry(tp[(row + 3) * kCgChanT]);
        append(e0, t0 + row);
        append(e1, t0 + row + 1);
        append(e2, t0 + row + 2);
        append(e3, t0 + row + 3);
      }
      for (; row < rows; ++row) append(entry(tp[row * kCgChanT]), t0 + row);
    }
    if (more) {
      if (vec16)
        sstore(b ^ 1);
      else
        bload(b ^ 1, (k + 1) * kCgTile);
    }
    __syncthreads();
  }
  if (tid >= nc) return;
  if (nb > 0) {
    const int n = (nb + 7) >> 3;
    cg_put_bytes(op, nbytes, cap, acc, n, overflow);
    nbytes += n;
  }
  if (overflow) {
    report_status(status, kStatusBadIndex, l * C + c, nbytes, cap);
    nbytes = cap;
  }
  out_len[static_cast<size_t>(l) * C + c] = nbytes;
}

// ---------------------------------------------------------------------------
// decode (prefix-summed stream lengths): bit reader shared by the decoders.
// ---------------------------------------------------------------------------
// 16 bytes at `pos` (a multiple of 16 counted from the 16-aligned `abase`);
// the buffer is the byte range [lo, hi), bytes outside it read as 0.
__device__ __forceinline__ uint4 cg_fetch16(const uint8_t *abase, long long pos, long long lo,
                                            long long hi) {
  if (pos >= lo && pos + 16 <= hi) return __ldg(reinterpret_cast<const uint4 *>(abase + pos));
  uint4 v = make_uint4(0, 0, 0, 0);
  uint8_t *vb = reinterpret_cast<uint8_t *>(&v);
  for (int j = 0; j < 16; ++j) {
    const long long q = pos + j;
    if (q >= lo && q < hi) vb[j] = __ldg(abase + q);
  }
  return v;
}

__device__ __forceinline__ uint32_t cg_word(const uint4 &v, int j) {
  const uint32_t w = j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
  return cg_bswap(w);
}

// ---------------------------------------------------------------------------
// decode, at most 16 symbols: the stream's CDF fits in registers (interval
// starts and code lengths), so no table is built and no shared memory is
// used; a thread per (layer, channel) stream at full occupancy.  A symbol is
// the last interval whose start is <= the window's top 16 bits (the starts
// increase; unused entries start at 0x10000, past every window value).
// The bit reader: a ring of three 16-byte loads, refilled once per two
// symbols (a code is at most 12 bits).
// ---------------------------------------------------------------------------
constexpr int kDecSmallBins = 16;
constexpr int kDecSmallThreads = 128;

__global__ void __launch_bounds__(kDecSmallThreads) cg_decode_small_kernel(
    const int16_t *__restrict__ cdf, const uint8_t *__restrict__ bytes,
    const int32_t *__restrict__ cum_len, long long total_bytes, uint8_t *out, int L, int T,
    int C, int bins) {
  const long long idx = static_cast<long long>(blockIdx.x) * kDecSmallThreads + threadIdx.x;
  if (idx >= static_cast<long long>(L) * C) return;
  const int l = static_cast<int>(idx / C);
  const int c = static_cast<int>(idx - static_cast<long long>(l) * C);
  const int16_t *cd = cdf + idx * (bins + 1);
  unsigned st[kDecSmallBins], ln_of[kDecSmallBins];
#pragma unroll
  for (int k = 0; k < kDecSmallBins; ++k) {
    const unsigned e = k < bins ? static_cast<unsigned short>(__ldg(cd + k)) : 0u;
    st[k] = k < bins ? (e & 0xFFF0u) : 0x10000u;
    ln_of[k] = e & 0xFu;
  }
  const long long b0 = idx == 0 ? 0 : cum_len[idx - 1];
  const uint8_t *abase =
      reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(bytes) & ~uintptr_t(15));
  const long long lo = bytes - abase;  // 0..15
  const long long hi = lo + total_bytes;
  const long long start = lo + b0;
  long long pos = start & ~15ll;
  uint4 A = cg_fetch16(abase, pos, lo, hi);
  uint4 B = cg_fetch16(abase, pos + 16, lo, hi);
  uint4 D = cg_fetch16(abase, pos + 32, lo, hi);
  pos += 48;
  int j = static_cast<int>((start - (start & ~15ll)) >> 2);  // next word of A
  const int skip = static_cast<int>(start & 3) * 8;
  unsigned long long win = static_cast<unsigned long long>(cg_word(A, j)) << 32;
  win <<= skip;
  int nb = 32 - skip;  // valid bits at the top of win
  auto next_word = [&]() {
    if (++j == 4) {
      A = B;
      B = D;
      D = cg_fetch16(abase, pos, lo, hi);
      pos += 16;
      j = 0;
    }
  };
  next_word();
  auto decode1 = [&]() -> unsigned {
    const unsigned v = static_cast<unsigned>(win >> 48);
    unsigned sym = 0, ln = ln_of[0];
#pragma unroll
    for (int k = 1; k < kDecSmallBins; ++k) {
      const bool ge = v >= st[k];
      sym = ge ? static_cast<unsigned>(k) : sym;
      ln = ge ? ln_of[k] : ln;
    }
    win <<= ln;
    nb -= static_cast<int>(ln);
    return sym;
  };
  uint8_t *op = out + static_cast<size_t>(l) * T * C + c;
  const size_t step = static_cast<size_t>(C);
  int t = 0;
  for (; t + 2 <= T; t += 2) {
    if (nb <= 32) {  // two codes need at most 24 bits
      win |= static_cast<unsigned long long>(cg_word(A, j)) << (32 - nb);
      nb += 32;
      next_word();
    }
    const unsigned s0 = decode1();
    const unsigned s1 = decode1();
    op[0] = static_cast<uint8_t>(s0);
    op[step] = static_cast<uint8_t>(s1);
    op += 2 * step;
  }
  if (t < T) {
    if (nb <= 32) win |= static_cast<unsigned long long>(cg_word(A, j)) << (32 - nb);
    op[0] = static_cast<uint8_t>(decode1());
  }
}

// ---------------------------------------------------------------------------
// decode, 17..256 symbols: a two-level search of the stream's CDF instead of
// a per-stream lookup table in shared memory (the 1 KB tables of 256-symbol
// streams left room for 7 warps per SM).  Registers hold every 16th entry;
// the last of those <= the window's top 16 bits picks a group of 16 symbols,
// and a 4-step binary search over that group's entries (L1-resident global
// loads of the stream's own 2 (bins + 1)-byte CDF row) picks the symbol.  An
// entry is start | code length with start a multiple of 16, so
// "start <= v" is "entry <= v | 15".
// ---------------------------------------------------------------------------
constexpr int kDecWideThreads = 128;

__global__ void __launch_bounds__(kDecWideThreads) cg_decode_wide_kernel(
    const int16_t *__restrict__ cdf, const uint8_t *__restrict__ bytes,
    const int32_t *__restrict__ cum_len, long long total_bytes, uint8_t *out, int L, int T,
    int C, int bins) {
  const long long idx = static_cast<long long>(blockIdx.x) * kDecWideThreads + threadIdx.x;
  if (idx >= static_cast<long long>(L) * C) return;
  const int l = static_cast<int>(idx / C);
  const int c = static_cast<int>(idx - static_cast<long long>(l) * C);
  const unsigned short *cd = reinterpret_cast<const unsigned short *>(cdf) + idx * (bins + 1);
  unsigned coarse[16];
#pragma unroll
  for (int g = 0; g < 16; ++g)
    coarse[g] = 16 * g < bins ? static_cast<unsigned>(__ldg(cd + 16 * g)) : 0x10000u;
  const long long b0 = idx == 0 ? 0 : cum_len[idx - 1];
  const uint8_t *abase =
      reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(bytes) & ~uintptr_t(15));
  const long long lo = bytes - abase;  // 0..15
  const long long hi = lo + total_bytes;
  const long long start = lo + b0;
  long long pos = start & ~15ll;
  uint4 A = cg_fetch16(abase, pos, lo, hi);
  uint4 B = cg_fetch16(abase, pos + 16, lo, hi);
  uint4 D = cg_fetch16(abase, pos + 32, lo, hi);
  pos += 48;
  int j = static_cast<int>((start - (start & ~15ll)) >> 2);  // next word of A
  const int skip = static_cast<int>(start & 3) * 8;
  unsigned long long win = static_cast<unsigned long long>(cg_word(A, j)) << 32;
  win <<= skip;
  int nb = 32 - skip;  // valid bits at the top of win
  auto next_word = [&]() {
    if (++j == 4) {
      A = B;
      B = D;
      D = cg_fetch16(abase, pos, lo, hi);
      pos += 16;
      j = 0;
    }
  };
  next_word();
  auto decode1 = [&]() -> unsigned {
    const unsigned vv = static_cast<unsigned>(win >> 48) | 15u;
    int k = 0;
    unsigned e = coarse[0];
#pragma unroll
    for (int g = 1; g < 16; ++g) {
      const bool ge = vv >= coarse[g];
      k = ge ? 16 * g : k;
      e = ge ? coarse[g] : e;
    }
#pragma unroll
    for (int step = 8; step >= 1; step >>= 1) {
      const int m = k + step;
      if (m < bins) {
        const unsigned em = __ldg(cd + m);
        if (vv >= em) {
          k = m;
          e = em;
        }
      }
    }
    const unsigned ln = e & 0xFu;
    win <<= ln;
    nb -= static_cast<int>(ln);
    return static_cast<unsigned>(k);
  };
  uint8_t *op = out + static_cast<size_t>(l) * T * C + c;
  const size_t step = static_cast<size_t>(C);
  int t = 0;
  for (; t + 2 <= T; t += 2) {
    if (nb <= 32) {  // two codes need at most 24 bits
      win |= static_cast<unsigned long long>(cg_word(A, j)) << (32 - nb);
      nb += 32;
      next_word();
    }
    const unsigned s0 = decode1();
    const unsigned s1 = decode1();
    op[0] = static_cast<uint8_t>(s0);
    op[step] = static_cast<uint8_t>(s1);
    op += 2 * step;
  }
  if (t < T) {
    if (nb <= 32) win |= static_cast<unsigned long long>(cg_word(A, j)) << (32 - nb);
    op[0] = static_cast<uint8_t>(decode1());
  }
}

// ---------------------------------------------------------------------------
// CDF rows from the stored code lengths (the serialised form keeps 4-bit
// lengths, two per byte, first in the high nibble): a thread per (row,
// channel) walks its bins, start_s = sum over r < s of 2^(16 - len_r), entry
// = (start & 0xFFF0) | len, and a closing 0 entry.  One launch in place of the
// unpack / power / scan / pack sequence of tensor ops.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) cg_cdf_from_lengths_kernel(
    const uint8_t *__restrict__ packed, int16_t *out, long long streams, int bins) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= streams) return;
  unsigned short *o = reinterpret_cast<unsigned short *>(out) + i * (bins + 1);
  unsigned pos = 0;
  const long long e0 = i * bins;
  for (int s = 0; s < bins; ++s) {
    const long long e = e0 + s;
    const unsigned b = __ldg(packed + (e >> 1));
    const unsigned ln = (e & 1) ? (b & 0xFu) : (b >> 4);
    o[s] = static_cast<unsigned short>((pos & 0xFFF0u) | ln);
    pos += 1u << (16 - ln);
  }
  o[bins] = 0;
}

// ---------------------------------------------------------------------------
// quantise: x [R, T, C] (rows = K layers then V layers of a KV_2LTD chunk) ->
// symbols [R, T, C] uint8 and scale [R, T] fp32, warp per (row, token):
//   half = bins / 2 - 1, scale = max(amax |x|, 1e-8) / half,
//   q = clamp(rint(x / scale) + half, 0, 2 half)
// with IEEE round-to-nearest division, so it matches the PyTorch expression
// bit for bit.  Symbol row r goes to row_dst[r] (grouping rows that share a
// bin count), scales stay in source order.
// dequantise is the inverse: y = (q - half) * scale, rounded to the dtype.
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float cg_to_f(T v);
template <> __device__ __forceinline__ float cg_to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float cg_to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float cg_to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T cg_from_f(float v);
template <> __device__ __forceinline__ float cg_from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half cg_from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 cg_from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// rint(x / s) with the quotient rounded to nearest (IEEE), computed as x * (1/s)
// and redone with the exact division only when the product lies within
// 1e-6 relative of a rounding tie (k + 0.5): the product is within 2.5 ulp
// (< 1e-6 relative) of the rounded quotient, so away from a tie both round to
// the same integer.
__device__ __forceinline__ float cg_rint_div(float x, float s, float r) {
  float a = x * r;
  const float frac = a - floorf(a);
  if (fabsf(frac - 0.5f) <= fabsf(a) * 1e-6f) a = __fdiv_rn(x, s);
  return rintf(a);
}

template <typename T, int kKeep>  // kKeep: vectors per lane kept in registers between passes
__global__ void __launch_bounds__(256) cg_quantize_kernel(
    const T *__restrict__ x, const int32_t *__restrict__ bins, const int32_t *__restrict__ row_dst,
    uint8_t *__restrict__ sym, float *__restrict__ scale, int R, int Tn, int C, bool vec) {
  constexpr int kV = 16 / sizeof(T);  // elements per 16-byte vector
  const int lane = threadIdx.x & 31;
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int nvec = C / kV;
  const bool keep = vec && nvec <= 32 * kKeep;
  for (long long gw = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       gw < static_cast<long long>(R) * Tn; gw += nwarps) {
    const int r = static_cast<int>(gw / Tn), t = static_cast<int>(gw % Tn);
    const T *row = x + (static_cast<size_t>(r) * Tn + t) * C;
    float amax = 0.f;
    uint4 held[kKeep];
    if (keep) {
#pragma unroll
      for (int k = 0; k < kKeep; ++k) {
        const int v = lane + 32 * k;
        held[k] = v < nvec ? __ldg(reinterpret_cast<const uint4 *>(row) + v)
                           : make_uint4(0, 0, 0, 0);
        const T *e = reinterpret_cast<const T *>(&held[k]);
#pragma unroll
        for (int j = 0; j < kV; ++j) amax = fmaxf(amax, fabsf(cg_to_f(e[j])));
      }
    } else if (vec) {
      for (int v = lane; v < nvec; v += 32) {
        const uint4 u = __ldg(reinterpret_cast<const uint4 *>(row) + v);
        const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
        for (int j = 0; j < kV; ++j) amax = fmaxf(amax, fabsf(cg_to_f(e[j])));
      }
    } else {
      for (int i = lane; i < C; i += 32) amax = fmaxf(amax, fabsf(cg_to_f(row[i])));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float half = static_cast<float>(bins[r] / 2 - 1);
    const float sc = __fdiv_rn(fmaxf(amax, 1e-8f), half);
    const float rc = __frcp_rn(sc);
    const float top = 2.f * half;
    const int dr = row_dst ? row_dst[r] : r;
    uint8_t *orow = sym + (static_cast<size_t>(dr) * Tn + t) * C;
    auto q = [&](float f) {
      const float v = cg_rint_div(f, sc, rc) + half;
      return static_cast<uint8_t>(static_cast<int>(fminf(fmaxf(v, 0.f), top)));
    };
    auto put = [&](int v, const uint4 &u) {
      const T *e = reinterpret_cast<const T *>(&u);
      uint8_t b[kV];
#pragma unroll
      for (int j = 0; j < kV; ++j) b[j] = q(cg_to_f(e[j]));
      if constexpr (kV == 8) {
        *reinterpret_cast<uint2 *>(orow + v * kV) = *reinterpret_cast<const uint2 *>(b);
      } else {
        *reinterpret_cast<uint32_t *>(orow + v * kV) = *reinterpret_cast<const uint32_t *>(b);
      }
    };
    if (keep) {
#pragma unroll
      for (int k = 0; k < kKeep; ++k) {
        const int v = lane + 32 * k;
        if (v < nvec) put(v, held[k]);
      }
    } else if (vec) {
      for (int v = lane; v < nvec; v += 32) put(v, __ldg(reinterpret_cast<const uint4 *>(row) + v));
    } else {
      for (int i = lane; i < C; i += 32) orow[i] = q(cg_to_f(row[i]));
    }
    if (lane == 0) scale[static_cast<size_t>(r) * Tn + t] = sc;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) cg_dequantize_kernel(
    const uint8_t *__restrict__ sym, const float *__restrict__ scale,
    const int32_t *__restrict__ bins, const int32_t *__restrict__ row_src, T *__restrict__ y,
    int R, int Tn, int C, bool vec) {
  constexpr int kV = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long gw = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       gw < static_cast<long long>(R) * Tn; gw += nwarps) {
    const int r = static_cast<int>(gw / Tn), t = static_cast<int>(gw % Tn);
    const float half = static_cast<float>(bins[r] / 2 - 1);
    const float sc = scale[static_cast<size_t>(r) * Tn + t];
    const int sr = row_src ? row_src[r] : r;
    const uint8_t *irow = sym + (static_cast<size_t>(sr) * Tn + t) * C;
    T *orow = y + (static_cast<size_t>(r) * Tn + t) * C;
    if (vec) {
      for (int v = lane; v < C / kV; v += 32) {
        uint8_t b[kV];
        if constexpr (kV == 8) {
          *reinterpret_cast<uint2 *>(b) = *reinterpret_cast<const uint2 *>(irow + v * kV);
        } else {
          *reinterpret_cast<uint32_t *>(b) = *reinterpret_cast<const uint32_t *>(irow + v * kV);
        }
        uint4 u;
        T *e = reinterpret_cast<T *>(&u);
#pragma unroll
        for (int j = 0; j < kV; ++j)
          e[j] = cg_from_f<T>(__fmul_rn(static_cast<float>(b[j]) - half, sc));
        reinterpret_cast<uint4 *>(orow)[v] = u;
      }
    } else {
      for (int i = lane; i < C; i += 32)
        orow[i] = cg_from_f<T>(__fmul_rn(static_cast<float>(irow[i]) - half, sc));
    }
  }
}

// ---------------------------------------------------------------------------
// Host launchers (op names of the reference's pybind module, plus the fused
// quantise / dequantise pair).
// ---------------------------------------------------------------------------
static bool cg_aligned(const void *p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

static void cg_smem_attr(const void *fn, size_t smem) {
  if (smem > 48 * 1024) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
  }
}

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
  dim3 grid((C + kCgChan - 1) / kCgChan, L);
  const bool wide = T >= 65536;
  const size_t smem = sizeof(unsigned) * kCgChan * (wide ? n_bins : (n_bins + 1) / 2);
  const bool vec4 = C % 4 == 0 && cg_aligned(in.data_ptr(), 4);
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const auto *ip = reinterpret_cast<const uint8_t *>(in.data_ptr());
  if (n_bins > 64) {
    auto exps = at::empty({L, n_bins, C}, in.options().dtype(at::kByte));
    auto *cp = exps.data_ptr<uint8_t>();
    const size_t hsmem = smem + (T < kCgExpTab ? static_cast<size_t>(T) + 1 : 0);
    if (wide) {
      cg_smem_attr(reinterpret_cast<const void *>(cg_hist_kernel<true>), hsmem);
      cg_hist_kernel<true><<<grid, 256, hsmem, stream>>>(ip, cp, L, T, C,
                                                        static_cast<int>(n_bins), vec4);
    } else {
      cg_smem_attr(reinterpret_cast<const void *>(cg_hist_kernel<false>), hsmem);
      cg_hist_kernel<false><<<grid, 256, hsmem, stream>>>(ip, cp, L, T, C,
                                                         static_cast<int>(n_bins), vec4);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    const long long n = static_cast<long long>(L) * C;
    cg_place_kernel<<<static_cast<unsigned>((n + kPlaceCh - 1) / kPlaceCh), kPlaceCh, 0,
                      stream>>>(
        cp, out.data_ptr<int16_t>(), L, C, static_cast<int>(n_bins));
  } else if (wide) {
    cg_smem_attr(reinterpret_cast<const void *>(cg_cdf_kernel<true>), smem);
    cg_cdf_kernel<true><<<grid, 256, smem, stream>>>(ip, out.data_ptr<int16_t>(), L, T, C,
                                                    static_cast<int>(n_bins), vec4);
  } else {
    cg_smem_attr(reinterpret_cast<const void *>(cg_cdf_kernel<false>), smem);
    cg_cdf_kernel<false><<<grid, 256, smem, stream>>>(ip, out.data_ptr<int16_t>(), L, T, C,
                                                     static_cast<int>(n_bins), vec4);
  }
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
  const int cap = static_cast<int>(output_buffer.size(2));
  const bool vec16 = C % 16 == 0 && cg_aligned(s.data_ptr(), 16);
  const bool word_out = cap % 4 == 0 && cg_aligned(output_buffer.data_ptr(), 4);
  DeviceStatus *st = status.has_value()
                         ? reinterpret_cast<DeviceStatus *>(status->data_ptr())
                         : nullptr;
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  auto launch = [&](auto ch) {
    constexpr int CH = decltype(ch)::value;
    dim3 grid((C + CH - 1) / CH, L);
    const size_t tab = ((static_cast<size_t>(bins + 1) / 2) * CH * 4 + 15) & ~size_t(15);
    const size_t smem = tab + 2 * kCgTile * CH;
    cg_smem_attr(reinterpret_cast<const void *>(cg_encode_kernel<CH>), smem);
    cg_encode_kernel<CH><<<grid, CH, smem, stream>>>(
        c.data_ptr<int16_t>(), reinterpret_cast<const uint8_t *>(s.data_ptr()),
        reinterpret_cast<uint8_t *>(output_buffer.data_ptr()),
        output_lengths.data_ptr<int32_t>(), L, T, C, bins, cap, vec16, word_out, st);
  };
  // 32 channels per block for large code tables keeps several blocks per SM
  if (bins > 64)
    launch(std::integral_constant<int, 32>());
  else
    launch(std::integral_constant<int, 128>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

at::Tensor cachegen_cdf_from_lengths(const at::Tensor &packed, int64_t rows, int64_t channels,
                                     int64_t bins) {
  TORCH_CHECK(packed.is_cuda() && packed.scalar_type() == at::kByte && packed.is_contiguous(),
              "cdf_from_lengths: packed lengths must be a contiguous device uint8 tensor");
  TORCH_CHECK(bins >= 1 && bins <= kCgMaxBins, "cdf_from_lengths: 1 <= bins <= 256");
  const long long streams = rows * channels;
  TORCH_CHECK(packed.numel() * 2 >= streams * bins, "cdf_from_lengths: too few lengths");
  const c10::cuda::CUDAGuard guard(packed.device());
  auto out = at::empty({rows, channels, bins + 1}, packed.options().dtype(at::kShort));
  if (streams == 0) return out;
  cg_cdf_from_lengths_kernel<<<static_cast<unsigned>((streams + 127) / 128), 128, 0,
                               at::cuda::getCurrentCUDAStream().stream()>>>(
      packed.data_ptr<uint8_t>(), out.data_ptr<int16_t>(), streams, static_cast<int>(bins));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
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
  TORCH_CHECK(bytestreams.scalar_type() == at::kByte || bytestreams.scalar_type() == at::kChar,
              "decode: bytestreams must be uint8");
  const int T = output.size(1);
  auto c = cdf.to(at::kShort).contiguous();
  auto b = bytestreams.contiguous();
  auto len = lengths.contiguous();
  const c10::cuda::CUDAGuard guard(c.device());
  if (L == 0 || C == 0 || T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const auto *bp = reinterpret_cast<const uint8_t *>(b.data_ptr());
  auto *op8 = reinterpret_cast<uint8_t *>(output.data_ptr());
  const long long nbytes = static_cast<long long>(b.numel());
  const long long nstreams = static_cast<long long>(L) * C;
  if (bins <= kDecSmallBins) {
    cg_decode_small_kernel<<<static_cast<unsigned>((nstreams + kDecSmallThreads - 1) /
                                                   kDecSmallThreads),
                             kDecSmallThreads, 0, stream>>>(
        c.data_ptr<int16_t>(), bp, len.data_ptr<int32_t>(), nbytes, op8, L, T, C, bins);
  } else {
    cg_decode_wide_kernel<<<static_cast<unsigned>((nstreams + kDecWideThreads - 1) /
                                                  kDecWideThreads),
                            kDecWideThreads, 0, stream>>>(
        c.data_ptr<int16_t>(), bp, len.data_ptr<int32_t>(), nbytes, op8, L, T, C, bins);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static int cg_rows_grid(int64_t rows) {
  int dev = 0, sms = 148;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t blocks = (rows + 7) / 8;  // 8 warps per block
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, sms * 16)));
}

// x [R, T, C] float -> sym [R, T, C] uint8 (row r written at row_dst[r]),
// scale [R, T] fp32.
void cachegen_quantize(const at::Tensor &x, const at::Tensor &bins, at::Tensor &sym,
                       at::Tensor &scale, const c10::optional<at::Tensor> &row_dst) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3 && x.is_contiguous(), "quantize: x device [R, T, C]");
  const int R = x.size(0), Tn = x.size(1), C = x.size(2);
  TORCH_CHECK(bins.is_cuda() && bins.scalar_type() == at::kInt && bins.numel() == R,
              "quantize: bins int32 [R] on the device");
  TORCH_CHECK(sym.is_cuda() && sym.scalar_type() == at::kByte && sym.is_contiguous() &&
                  sym.numel() == x.numel(),
              "quantize: sym uint8 [R, T, C]");
  TORCH_CHECK(scale.is_cuda() && scale.scalar_type() == at::kFloat && scale.is_contiguous() &&
                  scale.numel() == static_cast<int64_t>(R) * Tn,
              "quantize: scale fp32 [R, T]");
  const int32_t *rd = nullptr;
  if (row_dst.has_value()) {
    TORCH_CHECK(row_dst->is_cuda() && row_dst->scalar_type() == at::kInt &&
                    row_dst->numel() == R,
                "quantize: row_dst int32 [R]");
    rd = row_dst->data_ptr<int32_t>();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  if (x.numel() == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const int grid = cg_rows_grid(static_cast<int64_t>(R) * Tn);
  const int kV = 16 / static_cast<int>(x.element_size());
  const bool vec = C % kV == 0 && cg_aligned(x.data_ptr(), 16) && cg_aligned(sym.data_ptr(), 8);
  auto *sp = reinterpret_cast<uint8_t *>(sym.data_ptr());
  // hold the row in registers with as few as cover it (occupancy)
  const bool four = C / kV <= 32 * 4;
  auto go = [&](auto tag, auto keep) {
    using T = decltype(tag);
    constexpr int K = decltype(keep)::value;
    cg_quantize_kernel<T, K><<<grid, 256, 0, stream>>>(
        reinterpret_cast<const T *>(x.data_ptr()), bins.data_ptr<int32_t>(), rd, sp,
        scale.data_ptr<float>(), R, Tn, C, vec);
  };
  auto by_keep = [&](auto tag) {
    if (four)
      go(tag, std::integral_constant<int, 4>());
    else
      go(tag, std::integral_constant<int, 8>());
  };
  if (x.scalar_type() == at::kBFloat16) {
    by_keep(__nv_bfloat16());
  } else if (x.scalar_type() == at::kHalf) {
    by_keep(__half());
  } else {
    TORCH_CHECK(x.scalar_type() == at::kFloat, "quantize: bf16, fp16 or fp32 input");
    by_keep(float());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// sym (row r read from row_src[r]) + scale [R, T] -> y [R, T, C] in y's dtype.
void cachegen_dequantize(const at::Tensor &sym, const at::Tensor &scale, const at::Tensor &bins,
                         at::Tensor &y, const c10::optional<at::Tensor> &row_src) {
  TORCH_CHECK(y.is_cuda() && y.dim() == 3 && y.is_contiguous(), "dequantize: y device [R, T, C]");
  const int R = y.size(0), Tn = y.size(1), C = y.size(2);
  TORCH_CHECK(sym.is_cuda() && sym.scalar_type() == at::kByte && sym.is_contiguous() &&
                  sym.numel() == y.numel(),
              "dequantize: sym uint8 [R, T, C]");
  TORCH_CHECK(scale.is_cuda() && scale.scalar_type() == at::kFloat && scale.is_contiguous() &&
                  scale.numel() == static_cast<int64_t>(R) * Tn,
              "dequantize: scale fp32 [R, T]");
  TORCH_CHECK(bins.is_cuda() && bins.scalar_type() == at::kInt && bins.numel() == R,
              "dequantize: bins int32 [R]");
  const int32_t *rs = nullptr;
  if (row_src.has_value()) {
    TORCH_CHECK(row_src->is_cuda() && row_src->scalar_type() == at::kInt &&
                    row_src->numel() == R,
                "dequantize: row_src int32 [R]");
    rs = row_src->data_ptr<int32_t>();
  }
  const c10::cuda::CUDAGuard guard(y.device());
  if (y.numel() == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const int grid = cg_rows_grid(static_cast<int64_t>(R) * Tn);
  const int kV = 16 / static_cast<int>(y.element_size());
  const bool vec = C % kV == 0 && cg_aligned(y.data_ptr(), 16) && cg_aligned(sym.data_ptr(), 8);
  const auto *sp = reinterpret_cast<const uint8_t *>(sym.data_ptr());
  if (y.scalar_type() == at::kBFloat16) {
    cg_dequantize_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        sp, scale.data_ptr<float>(), bins.data_ptr<int32_t>(), rs,
        reinterpret_cast<__nv_bfloat16 *>(y.data_ptr()), R, Tn, C, vec);
  } else if (y.scalar_type() == at::kHalf) {
    cg_dequantize_kernel<__half><<<grid, 256, 0, stream>>>(
        sp, scale.data_ptr<float>(), bins.data_ptr<int32_t>(), rs,
        reinterpret_cast<__half *>(y.data_ptr()), R, Tn, C, vec);
  } else {
    TORCH_CHECK(y.scalar_type() == at::kFloat, "dequantize: bf16, fp16 or fp32 output");
    cg_dequantize_kernel<float><<<grid, 256, 0, stream>>>(
        sp, scale.data_ptr<float>(), bins.data_ptr<int32_t>(), rs, y.data_ptr<float>(), R, Tn,
        C, vec);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// Stream compaction for the serialised payload: the encoder writes each
// stream into a fixed-capacity slot; this packs them back to back on the
// device (warp per stream), so a chunk's payload leaves the GPU in one copy
// instead of a masked select plus one transfer per bin group.
//   dst[off[s] .. off[s] + len[s]) = src_base[slot_of(s)][0 .. len[s])
// where stream s of group g (streams [first[g], first[g + 1])) lives at
// src[g] + (s - first[g]) * cap[g].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) cg_compact_kernel(
    const int64_t *__restrict__ src, const int64_t *__restrict__ cap,
    const int64_t *__restrict__ first, int groups, const int32_t *__restrict__ len,
    const int64_t *__restrict__ off, uint8_t *__restrict__ dst, int64_t n) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t s = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; s < n;
       s += nw) {
    int g = 0;
    while (g + 1 < groups && s >= first[g + 1]) ++g;
    const uint8_t *a = reinterpret_cast<const uint8_t *>(src[g]) + (s - first[g]) * cap[g];
    uint8_t *d = dst + off[s];
    const int m = len[s];
    for (int i = lane; i < m; i += 32) d[i] = a[i];
  }
}

void cachegen_compact(const at::Tensor &src, const at::Tensor &cap, const at::Tensor &first,
                      const at::Tensor &lengths, const at::Tensor &offsets, at::Tensor &dst) {
  TORCH_CHECK(src.is_cuda() && cap.is_cuda() && first.is_cuda() && lengths.is_cuda() &&
                  offsets.is_cuda() && dst.is_cuda(),
              "compact: device tensors");
  TORCH_CHECK(src.scalar_type() == at::kLong && cap.scalar_type() == at::kLong &&
                  first.scalar_type() == at::kLong && offsets.scalar_type() == at::kLong &&
                  lengths.scalar_type() == at::kInt && dst.scalar_type() == at::kByte,
              "compact: int64 tables, int32 lengths, uint8 destination");
  TORCH_CHECK(src.numel() == cap.numel() && first.numel() == src.numel() &&
                  lengths.numel() == offsets.numel() && lengths.is_contiguous() &&
                  offsets.is_contiguous() && dst.is_contiguous(),
              "compact: table sizes");
  const int64_t n = lengths.numel();
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(dst.device());
  const int64_t blocks = std::min<int64_t>((n * 32 + 255) / 256, 148 * 16);
  cg_compact_kernel<<<static_cast<int>(blocks), 256, 0,
                      at::cuda::getCurrentCUDAStream().stream()>>>(
      src.data_ptr<int64_t>(), cap.data_ptr<int64_t>(), first.data_ptr<int64_t>(),
      static_cast<int>(src.numel()), lengths.data_ptr<int32_t>(), offsets.data_ptr<int64_t>(),
      dst.data_ptr<uint8_t>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lmc
