// Allocation-free C entry point for the staged paged <-> host chunk transfer.
//
// This entry point has no counterpart in the reference (LMCache-Ascend); it is
// an addition of this library.
//
// Who needs it: callers that cannot allocate device memory at the time they
// move KV -- a serving runtime that has handed all free HBM to its KV cache
// and forbids cudaMalloc afterwards, code running under a memory budget that
// must not grow, or a plain C host program that does not link torch and
// so has neither torch's allocator nor a tensor to pass as staging.  Those
// callers pass only their inputs and outputs; the staging buffer this
// transfer needs lives in a fixed device array inside the library.
//
// Limits and rules:
//  * the staging array holds LMC_NOALLOC_STAGING_BYTES (16 MiB) per device;
//    every GPU that loads the library reserves it until the process exits.
//    A transfer whose chunk is larger is rejected with an error, not split;
//  * every call looks up the array's device address on its device (a symbol
//    lookup, no allocation), so the entry point stays valid across a device
//    reset; the first call on a device also loads the library's module there,
//    so make that first call before any stream capture;
//  * all calls share the one array: calls that overlap on the GPU (two
//    streams, two threads) race on it.  Serialise them;
//  * nothing is allocated: no cudaMalloc, cudaFree or allocating library
//    routine is called.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#define LMC_NOALLOC_STAGING_BYTES (16u << 20)

#ifdef __cplusplus
extern "C" {
#endif

// Moves every layer of `num_tokens` tokens between a paged KV cache and one
// pinned host chunk, through the library's static staging array, on `stream`.
//
//   from_gpu != 0: paged -> staging (gather kernel) -> host chunk (D2H copy)
//   from_gpu == 0: host chunk -> staging (H2D copy) -> paged (scatter kernel)
//
// Paged cache: `d_plane_ptrs` is a DEVICE array of num_layers * num_planes
// base addresses (layer-major); per plane p, block_stride[p], slot_stride[p]
// and row_bytes[p] (host arrays) give the byte layout; slot s of a plane lives
// at base + (s / block_size) * block_stride + (s % block_size) * slot_stride.
// `d_slots` is a DEVICE array of num_tokens slot indices (int32, or int64 when
// slots_are_int64); -1 skips a token.
// Host chunk: when num_planes == 2 and both rows match it is [2, L, T, row]
// (K plane then V plane); otherwise [1, L, T, sum(rows)] (planes side by
// side in each token row).  `host_chunk_bytes` must equal that size.
// Returns 0 on success; otherwise a nonzero code and a message in `err`.
__attribute__((visibility("default"))) int lmc_staged_kv_transfer_noalloc(
    const int64_t *d_plane_ptrs, int num_layers, int num_planes,
    const int64_t *block_stride, const int64_t *slot_stride, const int32_t *row_bytes,
    int block_size, int64_t num_slots, const void *d_slots, int slots_are_int64,
    int num_tokens, void *host_chunk, size_t host_chunk_bytes, int from_gpu, int device,
    cudaStream_t stream, char *err, size_t err_len);

// Capacity of the staging array in bytes.
__attribute__((visibility("default"))) size_t lmc_noalloc_staging_capacity(void);

#ifdef __cplusplus
}
#endif
