// N12/N13: pinned, NUMA-bound and shared-memory host allocators plus the
// host-pointer registry.
//
// Reference: csrc/common/mem_alloc.cpp:19-410 (alloc_pinned_ptr,
// alloc_pinned_numa_ptr, alloc_shm_pinned_ptr / attach / detach / unlink) and
// csrc/common/managed_mem.cpp:50-423 (host ptr -> device VA registry).  On B200
// with UVA a host page registered with cudaHostRegister(Mapped|Portable) has
// the same address on the device, so the registry only keeps ranges for
// validation and reports the device alias from cudaHostGetDevicePointer.
#include <torch/extension.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "slow_path.h"

namespace lmc {

namespace {

constexpr int kMpolBind = 2;
constexpr int kMpolInterleave = 3;

bool cuda_present() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

struct Range {
  size_t size;
  uintptr_t dev;
  int kind;  // 0 cudaHostAlloc, 1 mmap+register, 2 shm, 3 external register
  std::string shm_name;
};

std::mutex g_mu;
std::map<uintptr_t, Range> g_ranges;

void record(void *p, size_t size, int kind, const std::string &name = "") {
  uintptr_t dev = reinterpret_cast<uintptr_t>(p);
  if (cuda_present()) {
    void *d = nullptr;
    if (cudaHostGetDevicePointer(&d, p, 0) == cudaSuccess)
      dev = reinterpret_cast<uintptr_t>(d);
    else
      cudaGetLastError();
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_ranges[reinterpret_cast<uintptr_t>(p)] = Range{size, dev, kind, name};
}

bool bind_numa(void *p, size_t size, int node, bool interleave) {
  if (node < 0) return true;
  unsigned long mask[16];
  std::memset(mask, 0, sizeof(mask));
  if (node >= 64 * 16) return false;
  mask[node / 64] |= 1ul << (node % 64);
  long rc = syscall(SYS_mbind, p, size, interleave ? kMpolInterleave : kMpolBind,
                    mask, 64 * 16, 0);
  return rc == 0;
}

void first_touch(void *p, size_t size) {
  const long page = sysconf(_SC_PAGESIZE);
  volatile char *c = static_cast<volatile char *>(p);
  for (size_t off = 0; off < size; off += page) c[off] = 0;
}

void host_register(void *p, size_t size) {
  if (!cuda_present()) return;
  SlowPathScope scope("cudaHostRegister", static_cast<long long>(size));
  cudaError_t e = cudaHostRegister(p, size, cudaHostRegisterPortable | cudaHostRegisterMapped);
  TORCH_CHECK(e == cudaSuccess || e == cudaErrorHostMemoryAlreadyRegistered,
              "cudaHostRegister failed: ", cudaGetErrorString(e));
  if (e != cudaSuccess) cudaGetLastError();
}

}  // namespace

int64_t alloc_pinned_ptr(int64_t size, int64_t device) {
  TORCH_CHECK(size > 0, "size must be > 0");
  void *p = nullptr;
  if (cuda_present()) {
    SlowPathScope scope("cudaHostAlloc", size);
    if (device >= 0) cudaSetDevice(static_cast<int>(device));
    cudaError_t e = cudaHostAlloc(&p, static_cast<size_t>(size),
                                  cudaHostAllocPortable | cudaHostAllocMapped);
    TORCH_CHECK(e == cudaSuccess, "cudaHostAlloc(", size, ") failed: ",
                cudaGetErrorString(e));
    record(p, size, 0);
  } else {
    // no GPU: plain page-aligned memory keeps the CPU-only paths working
    p = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    TORCH_CHECK(p != MAP_FAILED, "mmap failed");
    record(p, size, 1);
  }
  return reinterpret_cast<int64_t>(p);
}

void free_pinned_ptr(int64_t ptr) {
  void *p = reinterpret_cast<void *>(ptr);
  Range r{};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_ranges.find(reinterpret_cast<uintptr_t>(p));
    TORCH_CHECK(it != g_ranges.end(), "free_pinned_ptr: unknown pointer");
    r = it->second;
    g_ranges.erase(it);
  }
  if (r.kind == 0) {
    cudaFreeHost(p);
  } else {
    if (cuda_present()) {
      cudaHostUnregister(p);
      cudaGetLastError();
    }
    munmap(p, r.size);
  }
}

int64_t alloc_pinned_numa_ptr(int64_t size, int64_t numa_node) {
  TORCH_CHECK(size > 0, "size must be > 0");
  void *p = mmap(nullptr, size, PROT_READ | PROT_WRITE,
                 MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  TORCH_CHECK(p != MAP_FAILED, "mmap(", size, ") failed");
  if (!bind_numa(p, size, static_cast<int>(numa_node), false)) {
    // NUMA policy is an optimisation: keep going unbound (sanitised node)
  }
  first_touch(p, size);
  host_register(p, size);
  record(p, size, 1);
  return reinterpret_cast<int64_t>(p);
}

void free_pinned_numa_ptr(int64_t ptr) { free_pinned_ptr(ptr); }

static void *map_shm(const std::string &name, size_t size, bool create) {
  const int flags = create ? (O_CREAT | O_EXCL | O_RDWR) : O_RDWR;
  int fd = shm_open(name.c_str(), flags, 0600);
  TORCH_CHECK(fd >= 0, "shm_open(", name, ") failed: ", std::strerror(errno));
  if (create) {
    if (ftruncate(fd, static_cast<off_t>(size)) != 0) {
      close(fd);
      shm_unlink(name.c_str());
      TORCH_CHECK(false, "ftruncate failed for ", name);
    }
  } else {
    struct stat st;
    fstat(fd, &st);
    TORCH_CHECK(static_cast<size_t>(st.st_size) >= size, "shm segment ", name,
                " is smaller (", st.st_size, ") than requested ", size);
  }
  void *p = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  TORCH_CHECK(p != MAP_FAILED, "mmap of shm ", name, " failed");
  return p;
}

int64_t alloc_shm_pinned_ptr(int64_t size, const std::string &name,
                             int64_t numa_node) {
  TORCH_CHECK(size > 0, "size must be > 0");
  void *p = map_shm(name, size, true);
  bind_numa(p, size, static_cast<int>(numa_node), true);
  first_touch(p, size);
  host_register(p, size);
  record(p, size, 2, name);
  return reinterpret_cast<int64_t>(p);
}

int64_t attach_shm_pinned_ptr(int64_t size, const std::string &name) {
  void *p = map_shm(name, size, false);
  host_register(p, size);
  record(p, size, 2, name);
  return reinterpret_cast<int64_t>(p);
}

void detach_shm_pinned_ptr(int64_t ptr) { free_pinned_ptr(ptr); }

void free_shm_pinned_ptr(int64_t ptr) {
  std::string name;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_ranges.find(static_cast<uintptr_t>(ptr));
    TORCH_CHECK(it != g_ranges.end(), "free_shm_pinned_ptr: unknown pointer");
    name = it->second.shm_name;
  }
  free_pinned_ptr(ptr);
  if (!name.empty()) shm_unlink(name.c_str());
}

void unlink_shm(const std::string &name) { shm_unlink(name.c_str()); }

// Register memory that somebody else allocated (e.g. a torch CPU tensor).
int64_t register_mapping(int64_t ptr, int64_t size) {
  void *p = reinterpret_cast<void *>(ptr);
  host_register(p, size);
  record(p, size, 3);
  std::lock_guard<std::mutex> lk(g_mu);
  return static_cast<int64_t>(g_ranges[reinterpret_cast<uintptr_t>(p)].dev);
}

void unregister_ptr(int64_t ptr) {
  void *p = reinterpret_cast<void *>(ptr);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_ranges.find(reinterpret_cast<uintptr_t>(p));
    if (it == g_ranges.end()) return;
    TORCH_CHECK(it->second.kind == 3, "unregister_ptr: pointer owned by an allocator");
    g_ranges.erase(it);
  }
  if (cuda_present()) {
    cudaHostUnregister(p);
    cudaGetLastError();
  }
}

// Device alias of any address inside a registered range; -1 if unknown.
int64_t get_device_ptr(int64_t ptr) {
  const uintptr_t a = static_cast<uintptr_t>(ptr);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_ranges.upper_bound(a);
  if (it == g_ranges.begin()) return -1;
  --it;
  if (a >= it->first + it->second.size) return -1;
  return static_cast<int64_t>(it->second.dev + (a - it->first));
}

// Wrap a registered range as a uint8 tensor view (no ownership).
at::Tensor host_tensor_view(int64_t ptr, int64_t size) {
  TORCH_CHECK(get_device_ptr(ptr) != -1 || size == 0,
              "host_tensor_view: pointer is not in a registered range");
  return torch::from_blob(reinterpret_cast<void *>(ptr), {size},
                          torch::TensorOptions().dtype(torch::kUInt8));
}

int64_t registered_bytes() {
  std::lock_guard<std::mutex> lk(g_mu);
  int64_t s = 0;
  for (auto &kv : g_ranges) s += static_cast<int64_t>(kv.second.size);
  return s;
}

}  // namespace lmc
