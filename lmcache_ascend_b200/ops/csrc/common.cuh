// Device-side building blocks shared by every kernel of the extension.
//
// All kernels here are bandwidth or latency bound (no GEMM-shaped work), so
// the Blackwell features that matter are: 16-byte vector loads/stores, the
// TMA bulk engine (`cp.async.bulk`, NON-multicast only) completing on an
// mbarrier, and system-scope release/acquire operations for flags that cross
// NVLink.  Every spin-wait in this file takes an iteration budget and reports
// failure instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace lmc {

// ---------------------------------------------------------------------------
// Error status shared between device and host.  Kernels that can time out or
// detect bad input write a code here (first writer wins) and return early.
// ---------------------------------------------------------------------------
enum StatusCode : int {
  kStatusOk = 0,
  kStatusMbarTimeout = 1,    // a TMA load never completed within budget
  kStatusFlagTimeout = 2,    // a peer flag never reached its target
  kStatusBadSlot = 3,        // slot index out of the paged cache's range
  kStatusBadAlignment = 4,   // pointer/size not 16-byte aligned for TMA
  kStatusBadIndex = 5,       // selected-token / chunk index out of range
};

struct DeviceStatus {
  int code;     // StatusCode
  int where;    // kernel-specific location id (layer, tile, ...)
  long long a;  // detail (offending index, observed value, ...)
  long long b;
};

__device__ __forceinline__ void report_status(DeviceStatus *st, int code,
                                              int where, long long a,
                                              long long b) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->a = a;
    st->b = b;
    __threadfence_system();
  }
}

// ---------------------------------------------------------------------------
// Vector memory ops
// ---------------------------------------------------------------------------
__device__ __forceinline__ int4 ld_nc_v4(const void *p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Plain (coherent) 16 B load: used where the source may be written by another
// agent during the kernel's lifetime (peer pulls, host-mapped memory).
__device__ __forceinline__ int4 ld_v4(const void *p) {
  int4 v;
  asm volatile("ld.global.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void *p, int4 v) {
  asm volatile("st.global.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Streaming store: the destination is not re-read by this kernel, keep it out
// of L2 where possible (peer memory and host memory bypass L2 anyway).
__device__ __forceinline__ void st_cs_v4(void *p, int4 v) {
  asm volatile("st.global.cs.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------
// System-scope synchronisation (flags that cross NVLink / PCIe)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void red_release_sys_add(unsigned *p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v)
               : "memory");
}

// GPU-scope forms, for a flag whose waiter runs on this same GPU (its
// acquire, system-scoped, synchronises with a release of GPU scope: both
// threads are inside that scope).
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ void red_release_gpu_add(unsigned *p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v)
               : "memory");
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v)
               : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];"
               : "=r"(v)
               : "l"(p)
               : "memory");
  return v;
}

// Bounded spin until *flag - target >= 0 (wrap-safe signed compare).  Returns
// true on success.  `budget_ns` is measured with the global nanosecond timer,
// so the bound holds whatever the SM clock is.
__device__ __forceinline__ bool wait_flag_geq(const unsigned *flag,
                                              unsigned target,
                                              unsigned long long budget_ns,
                                              unsigned *observed) {
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  unsigned v = 0;
  for (;;) {
    v = ld_acquire_sys(flag);
    if (static_cast<int>(v - target) >= 0) {
      if (observed) *observed = v;
      return true;
    }
    unsigned long long t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > budget_ns) break;
    __nanosleep(256);
  }
  if (observed) *observed = v;
  return false;
}

// ---------------------------------------------------------------------------
// mbarrier + TMA bulk copies (cp.async.bulk, never with .multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      unsigned bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_parity(uint64_t *bar,
                                                     unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false after `budget_ns`.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar,
                                                  unsigned parity,
                                                  unsigned long long budget_ns) {
  if (mbar_try_wait_parity(bar, parity)) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    if (mbar_try_wait_parity(bar, parity)) return true;
    unsigned long long t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > budget_ns) return false;
  }
}

// global -> shared::cta bulk copy completing on `bar` (byte count in tx).
// Non-multicast form: the source is always this GPU's own memory.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gsrc,
                                         unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// shared::cta -> global bulk copy, tracked by the issuing thread's bulk group.
__device__ __forceinline__ void bulk_s2g(void *gdst, const void *smem_src,
                                         unsigned bytes) {
  asm volatile(
      "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
      "r"(smem_u32(smem_src)), "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N of this thread's bulk groups still READ shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until all of this thread's bulk groups have fully completed (writes
// visible in global memory).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Make generic-proxy shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace lmc
