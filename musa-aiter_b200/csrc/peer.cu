// Peer mappings for paged-block migration between GPUs of one node.
//
// A receiving process exports each destination cache plane as a CUDA IPC
// handle (of the allocation holding it) plus the plane's offset inside that
// allocation; the sending process opens the handles once and then moves blocks
// with the ordinary row engine, its stores landing in the peer's HBM over
// NVLink / NVSwitch (plain 16-byte stores, no waits on peers).
#include <cuda.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "common.cuh"

namespace mak {
namespace {

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn address_range_fn() {
  static GetRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(p);
    cudaGetLastError();
  });
  return fn;
}

// Opened allocations, keyed by (device, handle bytes): a handle is opened once per
// process and device, and closed when its last user releases it.
struct Opened {
  void* base;
  int refs;
};
std::mutex g_ipc_mu;
std::map<std::string, Opened> g_opened;

std::string key_of(int dev, const void* handle) {
  std::string k(reinterpret_cast<const char*>(&dev), sizeof(dev));
  k.append(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
  return k;
}

}  // namespace
}  // namespace mak

using namespace mak;

extern "C" {

int mak_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int mak_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(MAK_E_INVALID, "mak_ipc_export: NULL argument");
  GetRangeFn range = address_range_fn();
  if (range == nullptr) return fail(MAK_E_UNSUPPORTED, "mak_ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(MAK_E_INVALID, "mak_ipc_export: pointer is not device memory of this context");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "mak_ipc_export: cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MAK_OK;
}

int mak_ipc_import(const void* handle, int64_t offset, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr || offset < 0) return fail(MAK_E_INVALID, "mak_ipc_import: bad argument");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "mak_ipc_import: cudaGetDevice");
  const std::string k = key_of(dev, handle);
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  auto it = g_opened.find(k);
  if (it == g_opened.end()) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "mak_ipc_import: cudaIpcOpenMemHandle");
    it = g_opened.emplace(k, Opened{base, 0}).first;
  }
  it->second.refs += 1;
  *ptr_out = static_cast<char*>(it->second.base) + offset;
  return MAK_OK;
}

int mak_ipc_release(const void* handle) {
  if (handle == nullptr) return fail(MAK_E_INVALID, "mak_ipc_release: NULL handle");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "mak_ipc_release: cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  auto it = g_opened.find(key_of(dev, handle));
  if (it == g_opened.end()) return fail(MAK_E_INVALID, "mak_ipc_release: handle is not open");
  if (--it->second.refs > 0) return MAK_OK;
  e = cudaIpcCloseMemHandle(it->second.base);
  g_opened.erase(it);
  if (e != cudaSuccess) return cuda_fail(e, "mak_ipc_release: cudaIpcCloseMemHandle");
  return MAK_OK;
}

}  // extern "C"
