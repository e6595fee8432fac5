// T1 NVLink transport primitives: export/import of device memory between
// processes, raw device buffers outside the torch caching allocator, peer
// access, and the PCI bus id (reference N15 get_gpu_pci_bus_id,
// csrc/common/dcmi_management.cpp).
//
// The reference registers buffers with HCCL/HIXL and ships RMA descriptors to
// the peer (csrc/hccl/hccl_agent.cpp:25-397, RegisterMem/ImportMem).  Here a
// buffer is exported as a CUDA IPC handle plus the byte offset of the pointer
// inside its allocation; the peer maps it with cudaIpcOpenMemHandle and the
// resulting VA is used directly by the K9 push kernel's peer stores.
#include <torch/extension.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>
#include <string>
#include <tuple>

namespace lmc {

namespace {

using GetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &f, 12000,
                                         cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<GetAddressRangeFn>(f);
  }();
  return fn;
}

struct Imported {
  void *base;
  int refs;
};

std::mutex g_mu;
std::map<std::string, Imported> g_imports;    // handle bytes -> mapping
std::map<uintptr_t, std::string> g_by_base;   // base -> handle bytes

}  // namespace

// Returns (handle bytes, offset of ptr in its allocation, allocation size).
// Binds the device's primary context to the calling thread.  Driver-API
// calls (cuMemGetAddressRange) need a current context, and a thread that
// made no CUDA runtime call yet (e.g. a control-plane server thread) has none.
static void bind_device(int64_t device) {
  cudaError_t e = cudaSetDevice(static_cast<int>(device));
  TORCH_CHECK(e == cudaSuccess, "cudaSetDevice(", device, ") failed: ", cudaGetErrorString(e));
}

std::tuple<pybind11::bytes, int64_t, int64_t> ipc_export(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  bind_device(device);
  auto fn = address_range_fn();
  TORCH_CHECK(fn != nullptr, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  TORCH_CHECK(fn(&base, &size, static_cast<CUdeviceptr>(ptr)) == CUDA_SUCCESS,
              "cuMemGetAddressRange failed for ", ptr);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  TORCH_CHECK(e == cudaSuccess, "cudaIpcGetMemHandle failed: ", cudaGetErrorString(e));
  return std::make_tuple(
      pybind11::bytes(reinterpret_cast<const char *>(&h), sizeof(h)),
      static_cast<int64_t>(ptr - static_cast<int64_t>(base)),
      static_cast<int64_t>(size));
}

// Maps an exported allocation into this process (once per handle, ref
// counted) and returns the VA of `offset` inside it.
int64_t ipc_import(const std::string &handle, int64_t offset, int64_t device) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  bind_device(device);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_imports.find(handle);
  if (it == g_imports.end()) {
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle.data(), sizeof(h));
    void *base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    TORCH_CHECK(e == cudaSuccess, "cudaIpcOpenMemHandle failed: ", cudaGetErrorString(e));
    it = g_imports.emplace(handle, Imported{base, 0}).first;
    g_by_base[reinterpret_cast<uintptr_t>(base)] = handle;
  }
  it->second.refs += 1;
  return reinterpret_cast<int64_t>(it->second.base) + offset;
}

// Drops one reference of the mapping that contains `handle`.
void ipc_close(const std::string &handle) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_imports.find(handle);
  if (it == g_imports.end()) return;
  if (--it->second.refs > 0) return;
  cudaIpcCloseMemHandle(it->second.base);
  cudaGetLastError();
  g_by_base.erase(reinterpret_cast<uintptr_t>(it->second.base));
  g_imports.erase(it);
}

int64_t ipc_open_count() {
  std::lock_guard<std::mutex> lk(g_mu);
  return static_cast<int64_t>(g_imports.size());
}

// A device buffer from cudaMalloc (its own allocation, so an IPC export
// covers exactly this buffer).  Zero-initialised.  Freed with the tensor.
at::Tensor device_buffer(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "nbytes must be > 0");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(nbytes));
  TORCH_CHECK(e == cudaSuccess, "cudaMalloc(", nbytes, ") failed: ", cudaGetErrorString(e));
  cudaMemset(p, 0, static_cast<size_t>(nbytes));
  cudaDeviceSynchronize();
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(
      p, {nbytes}, [](void *q) { cudaFree(q); }, opts);
}

bool enable_peer_access(int64_t device, int64_t peer) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  int can = 0;
  cudaDeviceCanAccessPeer(&can, static_cast<int>(device), static_cast<int>(peer));
  if (!can) return false;
  cudaError_t e = cudaDeviceEnablePeerAccess(static_cast<int>(peer), 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return true;
  }
  return e == cudaSuccess;
}

std::string get_gpu_pci_bus_id(int64_t device) {
  char buf[64] = {0};
  cudaError_t e = cudaDeviceGetPCIBusId(buf, sizeof(buf), static_cast<int>(device));
  TORCH_CHECK(e == cudaSuccess, "cudaDeviceGetPCIBusId failed: ", cudaGetErrorString(e));
  return std::string(buf);
}

}  // namespace lmc
