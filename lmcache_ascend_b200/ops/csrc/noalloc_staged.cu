// Allocation-free variant of the staged paged <-> host chunk transfer
// (`fused_multi_layer_kv_transfer` in mem_kernels.cu): the staging buffer is a
// file-scope device array instead of a caller-provided tensor.  See noalloc.h
// for who needs this, the size limit and the calling rules.  This entry point
// has no counterpart in the reference (LMCache-Ascend).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <exception>

#include "kv_copy.cuh"
#include "mem_kernels.h"
#include "noalloc.h"

namespace {

// The staging array: LMC_NOALLOC_STAGING_BYTES on every device that loads
// the library, for the life of the process.  Host code must not pass this
// symbol to a kernel (on the host it names a host-side stand-in); it uses the
// device address that cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) unsigned char lmc_noalloc_staging[LMC_NOALLOC_STAGING_BYTES];

constexpr int kMaxDevices = 64;

// With the target device current: the array's device address on that device.
// Looked up on every call (a symbol lookup, no allocation), so a device reset
// or a re-created primary context never leaves a stale address behind.  The
// first lookup on a device loads the library's module there.
cudaError_t staging_address(void **out) {
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, lmc_noalloc_staging);
  if (e != cudaSuccess) return e;
  *out = p;
  return cudaSuccess;
}

int fail(char *err, size_t err_len, int code, const char *fmt, ...) {
  if (err != nullptr && err_len > 0) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(err, err_len, fmt, ap);
    va_end(ap);
  }
  return code;
}

}  // namespace

extern "C" size_t lmc_noalloc_staging_capacity(void) { return LMC_NOALLOC_STAGING_BYTES; }

extern "C" int lmc_staged_kv_transfer_noalloc(
    const int64_t *d_plane_ptrs, int num_layers, int num_planes, const int64_t *block_stride,
    const int64_t *slot_stride, const int32_t *row_bytes, int block_size, int64_t num_slots,
    const void *d_slots, int slots_are_int64, int num_tokens, void *host_chunk,
    size_t host_chunk_bytes, int from_gpu, int device, cudaStream_t stream, char *err,
    size_t err_len) {
  if (err != nullptr && err_len > 0) err[0] = '\0';
  if (num_planes < 1 || num_planes > lmc::kMaxPlanes)
    return fail(err, err_len, 1, "num_planes must be 1..3 (got %d)", num_planes);
  if (num_layers < 1 || num_tokens < 0 || block_size < 1 || num_slots < 1)
    return fail(err, err_len, 1, "bad sizes: layers=%d tokens=%d block_size=%d slots=%lld",
                num_layers, num_tokens, block_size, static_cast<long long>(num_slots));
  if (d_plane_ptrs == nullptr || block_stride == nullptr || slot_stride == nullptr ||
      row_bytes == nullptr || host_chunk == nullptr || (num_tokens > 0 && d_slots == nullptr))
    return fail(err, err_len, 1, "null pointer argument");
  if (device < 0 || device >= kMaxDevices)
    return fail(err, err_len, 1, "device %d out of range", device);
  int64_t row_sum = 0;
  for (int p = 0; p < num_planes; ++p) {
    if (row_bytes[p] <= 0) return fail(err, err_len, 1, "row_bytes[%d] must be > 0", p);
    row_sum += row_bytes[p];
  }
  const size_t chunk_bytes =
      static_cast<size_t>(num_layers) * static_cast<size_t>(num_tokens) * row_sum;
  if (host_chunk_bytes != chunk_bytes)
    return fail(err, err_len, 2, "host chunk is %zu bytes, the transfer needs %zu",
                host_chunk_bytes, chunk_bytes);
  if (chunk_bytes > LMC_NOALLOC_STAGING_BYTES)
    return fail(err, err_len, 3,
                "transfer of %zu bytes exceeds the %u-byte static staging array; "
                "split it into calls of fewer tokens",
                chunk_bytes, static_cast<unsigned>(LMC_NOALLOC_STAGING_BYTES));
  if (num_tokens == 0) return 0;

  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != device) {
    const cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess)
      return fail(err, err_len, 4, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  }
  auto restore = [&]() {
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
  };
  void *stage = nullptr;
  cudaError_t e = staging_address(&stage);
  if (e != cudaSuccess) {
    restore();
    return fail(err, err_len, 4, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  }

  lmc::CopyJob j;
  std::memset(&j, 0, sizeof(j));
  j.paged.ptrs = d_plane_ptrs;
  j.paged.num_layers = num_layers;
  j.paged.num_planes = num_planes;
  j.paged.block_size = block_size;
  j.paged.num_slots = num_slots;
  for (int p = 0; p < num_planes; ++p) {
    j.paged.plane[p].block_stride = block_stride[p];
    j.paged.plane[p].slot_stride = slot_stride[p];
    j.paged.plane[p].row_bytes = row_bytes[p];
  }
  const bool two_ltd = num_planes == 2 && row_bytes[0] == row_bytes[1];
  j.chunk.base = static_cast<char *>(stage);
  j.chunk.ntok = num_tokens;
  if (two_ltd) {
    for (int p = 0; p < 2; ++p) {
      j.chunk.plane_stride_t[p] = static_cast<int64_t>(num_layers) * row_bytes[0];
      j.chunk.token_stride[p] = row_bytes[0];
    }
    j.chunk.layer_stride_t = row_bytes[0];
  } else {
    int64_t off = 0;
    for (int p = 0; p < num_planes; ++p) {
      j.chunk.token_stride[p] = row_sum;
      j.chunk.col_off[p] = off;
      off += row_bytes[p];
    }
    j.chunk.layer_stride_t = row_sum;
  }
  j.slots = d_slots;
  j.slot_is_i64 = slots_are_int64 ? 1 : 0;
  j.num_tokens = num_tokens;
  j.num_layers = num_layers;
  j.to_chunk = from_gpu ? 1 : 0;

  int code = 0;
  try {
    if (from_gpu) {
      // Tokens with slot -1 are not written by the gather; clear the used
      // part of the shared array so they read as zeros, not as the previous
      // call's data.
      e = cudaMemsetAsync(stage, 0, chunk_bytes, stream);
      if (e == cudaSuccess) {
        // SIMT engine: it checks alignment per row, so any plane base works.
        lmc::launch_copy(j, true, false, 2, stream, device);
        e = cudaMemcpyAsync(host_chunk, stage, chunk_bytes, cudaMemcpyDeviceToHost, stream);
      }
    } else {
      e = cudaMemcpyAsync(stage, host_chunk, chunk_bytes, cudaMemcpyHostToDevice, stream);
      if (e == cudaSuccess) lmc::launch_copy(j, true, false, 2, stream, device);
    }
    // launch_copy checks its own launch (and throws); only the return codes of
    // this call's memset/memcpy are read here, so errors left by unrelated
    // work in the process are neither reported nor cleared
    if (e != cudaSuccess)
      code = fail(err, err_len, 5, "CUDA error: %s", cudaGetErrorString(e));
  } catch (const std::exception &ex) {
    code = fail(err, err_len, 6, "launch failed: %s", ex.what());
  }
  restore();
  return code;
}
