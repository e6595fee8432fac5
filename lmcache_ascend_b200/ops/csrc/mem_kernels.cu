// K1/K2/K4 + flash-layout ops: paged KV cache <-> LMCache chunk objects.
//
// Semantics follow the reference launchers (csrc/mem_kernels.cpp:75-111
// `multi_layer_kv_transfer`, :113-213 `fused_multi_layer_kv_transfer`,
// :265-334 `single_layer_kv_transfer`, :1036-1307 dense multi-chunk direct
// transfer, :1341-1440 `load_and_reshape_flash`):
//   for every layer l, plane p and token t with slot = slot_mapping[t] >= 0
//     chunk[p, l, t, :]  <->  paged[l][p][slot, :]
// The implementation is new: every format is described by PagedDesc/ChunkView
// (layout.h, kv_copy.cuh) and moved by one of two engines, TMA bulk copies
// through a shared-memory ring (device<->device) or 16-byte SIMT vectors
// (host-mapped pinned memory, unaligned rows).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <c10/cuda/CUDAGuard.h>

#include "kv_copy.cuh"
#include "mem_kernels.h"

namespace lmc {

// ---------------------------------------------------------------------------
// TMA engine: one warp per CTA, ring of `stages` shared-memory buffers.
// ---------------------------------------------------------------------------
constexpr int kTmaBarBytes = 1024;  // mbarrier area at the start of smem

__device__ __forceinline__ unsigned warp_sum(unsigned v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Each warp of the CTA is an independent pipeline with its own ring of
// `stages` buffers and mbarriers, so instruction latency of one warp's
// address planning overlaps the others' copies.
__global__ void __launch_bounds__(256)
    tma_rows_kernel(CopyJob j, int stage_bytes, int stages,
                    unsigned long long budget_ns) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * stages;
  unsigned char *ring = smem + kTmaBarBytes + static_cast<size_t>(warp) * stages * stage_bytes;

  j.num_tokens = effective_tokens(j);
  const UnitMap m = make_unit_map(j, stage_bytes);
  const int total_units = m.units_per_layer * j.num_layers;
  const int gw = blockIdx.x * nwarps + warp;
  const int nw = gridDim.x * nwarps;
  if (gw >= total_units) return;
  const int n_iter = (total_units - gw + nw - 1) / nw;

  if (lane == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto issue_loads = [&](int k) {
    const Unit u = decode_unit(j, m, gw + k * nw);
    const int s = k % stages;
    const LaneRuns r = plan_runs(j, u, lane, chunk_seq_tokens(j));
    const unsigned rb = plane_of(j.paged, u.plane).row_bytes;
    const unsigned total = warp_sum((r.len[0] + r.len[1]) * rb);
    if (lane == 0) mbar_arrive_expect_tx(&bars[s], total);
    __syncwarp();
    unsigned char *buf = ring + static_cast<size_t>(s) * stage_bytes;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (r.len[h])
        bulk_g2s(buf + (h * 32 + lane) * rb, r.src[h], r.len[h] * rb, &bars[s]);
  };

  auto issue_stores = [&](int k) {
    const Unit u = decode_unit(j, m, gw + k * nw);
    const int s = k % stages;
    const LaneRuns r = plan_runs(j, u, lane, chunk_seq_tokens(j));
    const unsigned rb = plane_of(j.paged, u.plane).row_bytes;
    unsigned char *buf = ring + static_cast<size_t>(s) * stage_bytes;
#pragma unroll
    for (int h = 0; h < 2; ++h)
      if (r.len[h]) bulk_s2g(r.dst[h], buf + (h * 32 + lane) * rb, r.len[h] * rb);
    bulk_commit();
  };

  const int prologue = n_iter < stages - 1 ? n_iter : stages - 1;
  for (int k = 0; k < prologue; ++k) issue_loads(k);
  for (int k = 0; k < n_iter; ++k) {
    const int s = k % stages;
    const unsigned parity = (k / stages) & 1;
    if (!mbar_wait_bounded(&bars[s], parity, budget_ns)) {
      if (lane == 0)
        report_status(j.status, kStatusMbarTimeout, gw, k, n_iter);
      break;
    }
    issue_stores(k);
    const int kn = k + stages - 1;
    if (kn < n_iter) {
      bulk_wait_read<1>();
      __syncwarp();
      issue_loads(kn);
    }
  }
  bulk_wait_all();
}

// ---------------------------------------------------------------------------
// Planes chosen by the job's plane mask, without runtime-indexed arrays (which
// would live in local memory).
__device__ __forceinline__ int num_selected_planes(const CopyJob &j) {
  int n = 0;
#pragma unroll
  for (int q = 0; q < kMaxPlanes; ++q) n += (q < j.paged.num_planes && plane_selected(j, q));
  return n;
}
__device__ __forceinline__ int kth_selected_plane(const CopyJob &j, int k) {
  int c = -1, p = 0;
#pragma unroll
  for (int q = 0; q < kMaxPlanes; ++q) {
    if (q < j.paged.num_planes && plane_selected(j, q)) {
      ++c;
      if (c == k) p = q;
    }
  }
  return p;
}

// SIMT engine: warp per (layer, plane, token) row, 16 B vectors when aligned.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void warp_copy_row(char *dst, const char *src,
                                              int rb, int lane) {
  const bool v16 = ((reinterpret_cast<uintptr_t>(dst) |
                     reinterpret_cast<uintptr_t>(src) | rb) & 15) == 0;
  if (v16) {
    // up to 4 independent 16 B loads in flight per lane before the stores
    int off = lane * 16;
    for (; off + 3 * 512 < rb; off += 4 * 512) {
      int4 a = ld_v4(src + off), b = ld_v4(src + off + 512),
           c = ld_v4(src + off + 1024), d = ld_v4(src + off + 1536);
      st_v4(dst + off, a);
      st_v4(dst + off + 512, b);
      st_v4(dst + off + 1024, c);
      st_v4(dst + off + 1536, d);
    }
    for (; off < rb; off += 512) st_v4(dst + off, ld_v4(src + off));
    return;
  }
  const bool v4 = ((reinterpret_cast<uintptr_t>(dst) |
                    reinterpret_cast<uintptr_t>(src) | rb) & 3) == 0;
  if (v4) {
    for (int off = lane * 4; off < rb; off += 128)
      *reinterpret_cast<int *>(dst + off) =
          *reinterpret_cast<const volatile int *>(src + off);
    return;
  }
  for (int off = lane; off < rb; off += 32) dst[off] = src[off];
}

__global__ void __launch_bounds__(256) simt_rows_kernel(CopyJob j) {
  j.num_tokens = effective_tokens(j);
  if (j.num_tokens == 0) return;
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x +
                          threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const int nsel = num_selected_planes(j);
  const long long rows = static_cast<long long>(j.num_layers) * nsel * j.num_tokens;
  for (long long r = warp; r < rows; r += nwarps) {
    const int t = static_cast<int>(r % j.num_tokens);
    const long long lp = r / j.num_tokens;
    const int k = static_cast<int>(lp % nsel);
    const int p = kth_selected_plane(j, k);
    const int l = static_cast<int>(lp / nsel);
    const int64_t slot = load_slot(j, t);
    if (slot < 0) continue;
    if (slot >= j.paged.num_slots) {
      if (lane == 0)
        report_status(j.status, kStatusBadSlot, t, slot, j.paged.num_slots);
      continue;
    }
    if (j.dst_slots != nullptr) {
      const int64_t ds = j.slot_is_i64 ? static_cast<const int64_t *>(j.dst_slots)[t]
                                       : static_cast<const int32_t *>(j.dst_slots)[t];
      if (ds < 0) continue;
      if (ds >= j.dst_paged.num_slots) {
        if (lane == 0) report_status(j.status, kStatusBadIndex, t, ds, j.dst_paged.num_slots);
        continue;
      }
      const PlaneDesc sp = plane_of(j.paged, p);
      const PlaneDesc dp = plane_of(j.dst_paged, p);
      char *sa = paged_addr(j.paged, j.layer_begin + l, p, slot);
      char *da = paged_addr(j.dst_paged, j.chunk_layer_begin + l, p, ds);
      const bool sseg = sp.seg_bytes > 0 && sp.seg_bytes < sp.row_bytes;
      const bool dseg = dp.seg_bytes > 0 && dp.seg_bytes < dp.row_bytes;
      if (!sseg && !dseg) {
        warp_copy_row(da, sa, sp.row_bytes, lane);
      } else {
        // copy in units that never straddle a segment on either side
        const int u = sseg && dseg ? min(sp.seg_bytes, dp.seg_bytes)
                                   : (sseg ? sp.seg_bytes : dp.seg_bytes);
        for (int off = 0; off < sp.row_bytes; off += u) {
          const int64_t so = sseg ? (off / sp.seg_bytes) * sp.seg_stride + off % sp.seg_bytes
                                  : off;
          const int64_t doff = dseg ? (off / dp.seg_bytes) * dp.seg_stride +
                                          off % dp.seg_bytes
                                    : off;
          warp_copy_row(da + doff, sa + so, u, lane);
        }
      }
      continue;
    }
    const int64_t ct = load_idx(j, t);
    if (ct < 0 || (j.chunk_idx != nullptr && ct >= j.chunk_idx_limit)) {
      if (lane == 0)
        report_status(j.status, kStatusBadIndex, t, ct, j.chunk_idx_limit);
      continue;
    }
    char *pa = paged_addr(j.paged, j.layer_begin + l, p, slot);
    char *ca = chunk_addr(j.chunk, j.chunk_layer_begin + l, p, ct, chunk_seq_tokens(j));
    const PlaneDesc pl = plane_of(j.paged, p);
    const int rb = pl.row_bytes;
    if (pl.seg_bytes > 0 && pl.seg_bytes < rb) {
      // head-major cache: the row is strided segments on the paged side
      for (int off = 0, sg = 0; off < rb; off += pl.seg_bytes, ++sg) {
        char *ps = pa + static_cast<int64_t>(sg) * pl.seg_stride;
        if (j.to_chunk)
          warp_copy_row(ca + off, ps, pl.seg_bytes, lane);
        else
          warp_copy_row(ps, ca + off, pl.seg_bytes, lane);
      }
    } else if (j.to_chunk) {
      warp_copy_row(ca, pa, rb, lane);
    } else {
      warp_copy_row(pa, ca, rb, lane);
    }
  }
}

// SIMT engine for rows of at most 16 bytes (fp16 scale planes and the like):
// one thread per (layer, plane, token) row instead of one warp.
__device__ __forceinline__ void thread_copy_small(char *dst, const char *src, int rb) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                      static_cast<uintptr_t>(rb);
  if ((a & 7) == 0) {
    for (int o = 0; o < rb; o += 8)
      *reinterpret_cast<long long *>(dst + o) = *reinterpret_cast<const long long *>(src + o);
  } else if ((a & 3) == 0) {
    for (int o = 0; o < rb; o += 4)
      *reinterpret_cast<int *>(dst + o) = *reinterpret_cast<const int *>(src + o);
  } else if ((a & 1) == 0) {
    for (int o = 0; o < rb; o += 2)
      *reinterpret_cast<short *>(dst + o) = *reinterpret_cast<const short *>(src + o);
  } else {
    for (int o = 0; o < rb; ++o) dst[o] = src[o];
  }
}

__global__ void __launch_bounds__(256) simt_small_rows_kernel(CopyJob j) {
  j.num_tokens = effective_tokens(j);
  if (j.num_tokens == 0) return;
  const int nsel = num_selected_planes(j);
  const long long rows = static_cast<long long>(j.num_layers) * nsel * j.num_tokens;
  const long long nth = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long r = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows;
       r += nth) {
    const int t = static_cast<int>(r % j.num_tokens);
    const long long lp = r / j.num_tokens;
    const int k = static_cast<int>(lp % nsel);
    const int p = kth_selected_plane(j, k);
    const int l = static_cast<int>(lp / nsel);
    const int64_t slot = load_slot(j, t);
    if (slot < 0) continue;
    if (slot >= j.paged.num_slots) {
      report_status(j.status, kStatusBadSlot, t, slot, j.paged.num_slots);
      continue;
    }
    const int64_t ct = load_idx(j, t);
    if (ct < 0 || (j.chunk_idx != nullptr && ct >= j.chunk_idx_limit)) {
      report_status(j.status, kStatusBadIndex, t, ct, j.chunk_idx_limit);
      continue;
    }
    char *pa = paged_addr(j.paged, j.layer_begin + l, p, slot);
    char *ca = chunk_addr(j.chunk, j.chunk_layer_begin + l, p, ct, chunk_seq_tokens(j));
    const int rb = plane_of(j.paged, p).row_bytes;
    if (j.to_chunk)
      thread_copy_small(ca, pa, rb);
    else
      thread_copy_small(pa, ca, rb);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (cached[device] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cached[device] = v > 0 ? v : 148;
  }
  return cached[device];
}

PagedLayout::PagedLayout(at::Tensor ptrs, std::vector<int64_t> block_stride,
                         std::vector<int64_t> slot_stride,
                         std::vector<int64_t> row_bytes, int64_t block_size,
                         int64_t num_slots, std::vector<int64_t> seg_bytes,
                         std::vector<int64_t> seg_stride)
    : ptrs_(ptrs) {
  TORCH_CHECK(ptrs.scalar_type() == at::kLong && ptrs.is_contiguous(),
              "PagedLayout: ptrs must be a contiguous int64 tensor");
  const int np = static_cast<int>(row_bytes.size());
  TORCH_CHECK(np >= 1 && np <= kMaxPlanes, "PagedLayout: 1..3 planes");
  TORCH_CHECK(block_stride.size() == row_bytes.size() &&
                  slot_stride.size() == row_bytes.size(),
              "PagedLayout: stride lists must match row_bytes");
  TORCH_CHECK(ptrs.numel() % np == 0, "PagedLayout: ptrs not [L * planes]");
  std::memset(&desc_, 0, sizeof(desc_));
  desc_.ptrs = ptrs.data_ptr<int64_t>();
  desc_.num_planes = np;
  desc_.num_layers = static_cast<int32_t>(ptrs.numel() / np);
  desc_.block_size = static_cast<int32_t>(block_size);
  desc_.num_slots = num_slots;
  aligned16_ = true;
  for (int p = 0; p < np; ++p) {
    desc_.plane[p].block_stride = block_stride[p];
    desc_.plane[p].slot_stride = slot_stride[p];
    desc_.plane[p].row_bytes = static_cast<int32_t>(row_bytes[p]);
    TORCH_CHECK(row_bytes[p] > 0, "PagedLayout: row_bytes must be > 0");
    plane16_[p] = ((block_stride[p] | slot_stride[p] | row_bytes[p]) & 15) == 0;
    if (!plane16_[p]) aligned16_ = false;
    if (p < static_cast<int>(seg_bytes.size()) && seg_bytes[p] > 0 &&
        seg_bytes[p] < row_bytes[p]) {
      plane16_[p] = false;
      TORCH_CHECK(row_bytes[p] % seg_bytes[p] == 0 &&
                      p < static_cast<int>(seg_stride.size()),
                  "PagedLayout: row must be a whole number of segments");
      desc_.plane[p].seg_bytes = static_cast<int32_t>(seg_bytes[p]);
      desc_.plane[p].seg_stride = seg_stride[p];
      segmented_ = true;
    }
  }
  TORCH_CHECK(ptrs.is_cuda(), "PagedLayout: ptrs table must live on the device");
  // Alignment of the plane base pointers is checked by the Python layer,
  // which knows them, and recorded with set_bases_aligned().
}

ChunkLayout::ChunkLayout(std::vector<int64_t> plane_stride_t,
                         int64_t layer_stride_t, std::vector<int64_t> token_stride,
                         std::vector<int64_t> col_off) {
  std::memset(&view_, 0, sizeof(view_));
  TORCH_CHECK(plane_stride_t.size() <= kMaxPlanes && col_off.size() <= kMaxPlanes,
              "ChunkLayout: at most 3 planes");
  for (size_t p = 0; p < plane_stride_t.size(); ++p)
    view_.plane_stride_t[p] = plane_stride_t[p];
  for (size_t p = 0; p < col_off.size(); ++p) view_.col_off[p] = col_off[p];
  view_.layer_stride_t = layer_stride_t;
  TORCH_CHECK(token_stride.size() >= 1 && token_stride.size() <= kMaxPlanes,
              "ChunkLayout: 1..3 token strides");
  for (int p = 0; p < kMaxPlanes; ++p)
    view_.token_stride[p] =
        token_stride[std::min<size_t>(p, token_stride.size() - 1)];
}

static DeviceStatus *status_ptr(const c10::optional<at::Tensor> &status) {
  if (!status.has_value()) return nullptr;
  TORCH_CHECK(status->is_cuda() && status->nbytes() >= sizeof(DeviceStatus),
              "status must be a device tensor of >= 24 bytes");
  return reinterpret_cast<DeviceStatus *>(status->data_ptr());
}

void launch_copy(const CopyJob &j, bool chunk_on_device, bool aligned,
                 int64_t mode, cudaStream_t stream, int device) {
  if (j.num_tokens <= 0 || j.num_layers <= 0) return;
  bool use_tma = (mode == 1) || (mode == 0 && chunk_on_device && aligned);
  if (mode == 1) TORCH_CHECK(aligned, "TMA mode needs 16-byte aligned rows");
  if (use_tma) {
    // 2 warps x 2 stages x 8 KiB per CTA: several CTAs per SM, each warp an
    // independent load/store pipeline (measured best on B200 for 0.5-2 KiB rows)
    constexpr int stage_bytes = 8192;
    constexpr int stages = 2;
    constexpr int warps = 2;
    int max_rb = 0;
    for (int p = 0; p < j.paged.num_planes; ++p)
      max_rb = std::max(max_rb, static_cast<int>(j.paged.plane[p].row_bytes));
    const int sb = std::max(stage_bytes, max_rb);
    TORCH_CHECK(warps * stages * 8 <= kTmaBarBytes, "too many TMA stages");
    const size_t smem = kTmaBarBytes + static_cast<size_t>(sb) * stages * warps;
    TORCH_CHECK(smem <= 227 * 1024, "TMA ring too large: ", smem);
    static bool attr_set[64] = {false};
    if (!attr_set[device & 63]) {
      cudaFuncSetAttribute(tma_rows_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           227 * 1024);
      attr_set[device & 63] = true;
    }
    long long units = 0;
    for (int p = 0; p < j.paged.num_planes; ++p) {
      if (j.plane_mask != 0 && !((j.plane_mask >> p) & 1u)) continue;
      int tt = sb / j.paged.plane[p].row_bytes;
      tt = std::min(64, std::max(1, tt));
      units += (j.num_tokens + tt - 1) / tt;
    }
    units *= j.num_layers;
    const int per_sm = std::max(1, static_cast<int>((228 * 1024) / (smem + 1024)));
    const int grid_cap = num_sms(device) * per_sm;
    const long long ctas = (units + warps - 1) / warps;
    const int grid = static_cast<int>(std::max(1LL, std::min<long long>(ctas, grid_cap)));
    const unsigned long long budget_ns = 2000000000ull;  // 2 s
    tma_rows_kernel<<<grid, 32 * warps, smem, stream>>>(j, sb, stages, budget_ns);
  } else {
    int nsel = 0;
    bool small = j.dst_slots == nullptr;
    for (int p = 0; p < j.paged.num_planes; ++p) {
      if (j.plane_mask != 0 && !((j.plane_mask >> p) & 1u)) continue;
      ++nsel;
      const PlaneDesc &pl = j.paged.plane[p];
      if (pl.row_bytes > 16 || (pl.seg_bytes > 0 && pl.seg_bytes < pl.row_bytes)) small = false;
    }
    const long long rows = static_cast<long long>(j.num_layers) * nsel * j.num_tokens;
    const int threads = 256;
    const long long cap = static_cast<long long>(num_sms(device)) * 8;
    if (small) {  // thread per row
      long long blocks = (rows + threads - 1) / threads;
      blocks = std::max(1LL, std::min(blocks, cap));
      simt_small_rows_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(j);
    } else {  // warp per row
      long long blocks = (rows * 32 + threads - 1) / threads;
      blocks = std::max(1LL, std::min(blocks, cap));
      simt_rows_kernel<<<static_cast<int>(blocks), threads, 0, stream>>>(j);
    }
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

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
                 const c10::optional<at::Tensor> &num_tokens_dev) {
  TORCH_CHECK(slots.is_cuda(), "slot_mapping must be on the device");
  TORCH_CHECK(slots.scalar_type() == at::kLong || slots.scalar_type() == at::kInt,
              "slot_mapping must be int32 or int64");
  TORCH_CHECK(slots.is_contiguous(), "slot_mapping must be contiguous");
  TORCH_CHECK(layer_begin >= 0 && num_layers >= 0 &&
                  layer_begin + num_layers <= paged.desc().num_layers,
              "layer range out of the paged cache");
  const c10::cuda::CUDAGuard guard(slots.device());
  CopyJob j;
  std::memset(&j, 0, sizeof(j));
  j.paged = paged.desc();
  j.chunk = layout.view();
  bool aligned = paged.aligned();
  if (chunk_ptrs.has_value()) {
    TORCH_CHECK(chunk_ptrs->is_cuda() && chunk_ptrs->scalar_type() == at::kLong,
                "chunk_ptrs must be a device int64 tensor");
    TORCH_CHECK(chunk_tokens > 0, "chunk_tokens must be > 0");
    j.chunk.chunk_ptrs = chunk_ptrs->data_ptr<int64_t>();
    j.chunk.chunk_tokens = static_cast<int32_t>(chunk_tokens);
  } else {
    TORCH_CHECK(chunk.has_value(), "either chunk or chunk_ptrs is required");
    j.chunk.base = static_cast<char *>(chunk->data_ptr());
    j.chunk.ntok = static_cast<int32_t>(chunk_ntok);
    j.chunk.tok_off = static_cast<int32_t>(chunk_tok_off);
    if (!chunk_idx.has_value())
      TORCH_CHECK(chunk_tok_off + slots.numel() <= chunk_ntok,
                  "token range exceeds the chunk");
    chunk_on_device = chunk->is_cuda();
    if (reinterpret_cast<uintptr_t>(j.chunk.base) & 15) aligned = false;
  }
  // Chunk-side alignment of plane p: layer and plane offsets scale with the
  // chunk's token count, so check them at every count this launch uses (the
  // full chunk and a partial last one), plus the per-token stride and column.
  int64_t tcs[2] = {0, 0};
  int ntc = 0;
  if (chunk_ptrs.has_value()) {
    const int64_t total = chunk_idx.has_value() ? chunk_idx_limit : slots.numel();
    tcs[ntc++] = chunk_tokens;
    if (total % chunk_tokens) tcs[ntc++] = total % chunk_tokens;
  } else {
    tcs[ntc++] = chunk_ntok;
  }
  auto chunk_plane_ok = [&](int p) {
    if ((j.chunk.col_off[p] | j.chunk.token_stride[p]) & 15) return false;
    for (int i = 0; i < ntc; ++i)
      if (((j.chunk.layer_stride_t | j.chunk.plane_stride_t[p]) * tcs[i]) & 15) return false;
    return true;
  };
  for (int p = 0; p < j.paged.num_planes; ++p)
    if (!chunk_plane_ok(p)) aligned = false;
  j.slots = slots.data_ptr();
  j.slot_is_i64 = slots.scalar_type() == at::kLong;
  j.num_tokens = static_cast<int32_t>(slots.numel());
  j.layer_begin = static_cast<int32_t>(layer_begin);
  j.chunk_layer_begin = static_cast<int32_t>(chunk_layer_begin);
  j.num_layers = static_cast<int32_t>(num_layers);
  j.to_chunk = to_chunk ? 1 : 0;
  j.status = status_ptr(status);
  if (chunk_idx.has_value()) {
    TORCH_CHECK(chunk_idx->is_cuda() && chunk_idx->is_contiguous() &&
                    chunk_idx->scalar_type() == slots.scalar_type() &&
                    chunk_idx->numel() == slots.numel(),
                "chunk_idx: device tensor with the slot mapping's dtype/length");
    j.chunk_idx = chunk_idx->data_ptr();
    j.chunk_idx_limit = chunk_idx_limit;
  }
  if (num_tokens_dev.has_value()) {
    TORCH_CHECK(num_tokens_dev->is_cuda() &&
                    num_tokens_dev->scalar_type() == at::kInt,
                "num_tokens_dev: device int32 tensor");
    j.num_tokens_dev = num_tokens_dev->data_ptr<int32_t>();
  }
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream(slots.device().index()).stream();
  const int dev = slots.device().index();
  if (mode == 0 && chunk_on_device && !aligned) {
    // split by plane: aligned planes on the TMA engine, the rest on SIMT
    const bool base_ok = chunk_ptrs.has_value() ||
                         (reinterpret_cast<uintptr_t>(j.chunk.base) & 15) == 0;
    uint32_t tma_mask = 0, simt_mask = 0;
    for (int p = 0; p < j.paged.num_planes; ++p) {
      const bool ok = base_ok && paged.plane_aligned(p) && chunk_plane_ok(p);
      (ok ? tma_mask : simt_mask) |= 1u << p;
    }
    if (tma_mask != 0 && simt_mask != 0) {
      CopyJob a = j;
      a.plane_mask = tma_mask;
      launch_copy(a, true, true, 0, stream, dev);
      CopyJob b = j;
      b.plane_mask = simt_mask;
      launch_copy(b, true, false, 2, stream, dev);
      return;
    }
  }
  launch_copy(j, chunk_on_device, aligned, mode, stream, dev);
}

// Adds `inc` to flags[layer_begin .. layer_begin + n) with release semantics
// (stream-ordered after the copy kernel that precedes it).
__global__ void bump_flags_kernel(unsigned *flags, int layer_begin, int n, unsigned inc) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    fence_acq_rel_sys();
    red_release_sys_add(flags + layer_begin + i, inc);
  }
}

// Paged -> paged copy on this GPU (same-device PD push, block copies):
//   dst[l'][p][dst_slots[t]] = src[l][p][src_slots[t]]
// optionally followed by a per-layer flag release (`flags_ptr`, `flag_inc`).
void paged_copy(const PagedLayout &src, const PagedLayout &dst, const at::Tensor &src_slots,
                const at::Tensor &dst_slots, int64_t layer_begin, int64_t dst_layer_begin,
                int64_t num_layers, int64_t mode, const c10::optional<at::Tensor> &status,
                int64_t flags_ptr, int64_t flag_inc) {
  TORCH_CHECK(src_slots.is_cuda() && dst_slots.is_cuda(), "slot mappings must be on the device");
  TORCH_CHECK(src_slots.scalar_type() == dst_slots.scalar_type() &&
                  src_slots.numel() == dst_slots.numel(),
              "src/dst slot mappings must match in dtype and length");
  TORCH_CHECK(src_slots.is_contiguous() && dst_slots.is_contiguous(), "contiguous slots");
  TORCH_CHECK(src.desc().num_planes == dst.desc().num_planes, "plane count mismatch");
  for (int p = 0; p < src.desc().num_planes; ++p)
    TORCH_CHECK(src.desc().plane[p].row_bytes == dst.desc().plane[p].row_bytes,
                "row size mismatch on plane ", p);
  TORCH_CHECK(layer_begin >= 0 && layer_begin + num_layers <= src.desc().num_layers &&
                  dst_layer_begin >= 0 && dst_layer_begin + num_layers <= dst.desc().num_layers,
              "layer range out of the caches");
  const c10::cuda::CUDAGuard guard(src_slots.device());
  CopyJob j;
  std::memset(&j, 0, sizeof(j));
  j.paged = src.desc();
  j.dst_paged = dst.desc();
  j.slots = src_slots.data_ptr();
  j.dst_slots = dst_slots.data_ptr();
  j.slot_is_i64 = src_slots.scalar_type() == at::kLong;
  j.num_tokens = static_cast<int32_t>(src_slots.numel());
  j.layer_begin = static_cast<int32_t>(layer_begin);
  j.chunk_layer_begin = static_cast<int32_t>(dst_layer_begin);
  j.num_layers = static_cast<int32_t>(num_layers);
  j.to_chunk = 1;
  j.status = status_ptr(status);
  const int dev = src_slots.device().index();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(dev).stream();
  launch_copy(j, true, src.aligned() && dst.aligned(), mode, stream, dev);
  if (flags_ptr != 0 && num_layers > 0) {
    bump_flags_kernel<<<(static_cast<int>(num_layers) + 127) / 128, 128, 0, stream>>>(
        reinterpret_cast<unsigned *>(flags_ptr), static_cast<int>(dst_layer_begin),
        static_cast<int>(num_layers), static_cast<unsigned>(flag_inc));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// N2 `fused_multi_layer_kv_transfer` (reference csrc/mem_kernels.cpp:113-213):
// all layers between the paged cache and ONE pinned host chunk through a
// caller-provided device staging buffer, on the current stream.
//   from_gpu: TMA gather paged -> staging, then D2H copy staging -> host
//   to_gpu:   H2D copy host -> staging, then TMA scatter staging -> paged
void fused_multi_layer_kv_transfer(at::Tensor &host_chunk, at::Tensor &staging,
                                   const PagedLayout &paged, const ChunkLayout &layout,
                                   const at::Tensor &slots, bool from_gpu, int64_t mode,
                                   const c10::optional<at::Tensor> &status) {
  TORCH_CHECK(!host_chunk.is_cuda() && host_chunk.is_contiguous(),
              "host_chunk must be a contiguous host tensor");
  TORCH_CHECK(host_chunk.dim() == 4, "host_chunk must be a 4-D chunk [P, L, T, E]");
  TORCH_CHECK(staging.is_cuda() && staging.is_contiguous(), "staging must be on the device");
  const size_t nbytes = host_chunk.nbytes();
  TORCH_CHECK(staging.nbytes() >= nbytes, "staging buffer too small: need ", nbytes,
              " bytes, got ", staging.nbytes());
  TORCH_CHECK(slots.numel() <= host_chunk.size(2), "more slots than chunk tokens");
  const c10::cuda::CUDAGuard guard(slots.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(slots.device().index()).stream();
  auto stage = at::from_blob(staging.data_ptr(), host_chunk.sizes(),
                             host_chunk.options().device(staging.device()));
  if (!from_gpu) {
    cudaError_t e = cudaMemcpyAsync(staging.data_ptr(), host_chunk.data_ptr(), nbytes,
                                    cudaMemcpyHostToDevice, stream);
    TORCH_CHECK(e == cudaSuccess, "H2D copy failed: ", cudaGetErrorString(e));
  }
  kv_transfer(paged, stage, c10::nullopt, layout, host_chunk.size(2), 0, 0, true, slots, 0, 0,
              paged.desc().num_layers, from_gpu, mode, status, c10::nullopt, 0, c10::nullopt);
  if (from_gpu) {
    cudaError_t e = cudaMemcpyAsync(host_chunk.data_ptr(), staging.data_ptr(), nbytes,
                                    cudaMemcpyDeviceToHost, stream);
    TORCH_CHECK(e == cudaSuccess, "D2H copy failed: ", cudaGetErrorString(e));
  }
}

}  // namespace lmc
