// Allocation-free variant of the row scatter (mak_rows_scatter_static).
//
// Some callers cannot call cudaMalloc, not even through a caching allocator:
// a serving engine that reserved nearly all HBM for its KV-cache pool up front
// and runs the KV copy inside its step loop (a new device allocation there can
// fail or break the engine's memory budget), or a foreign-language caller that
// only holds raw device pointers handed over by another framework's allocator
// and has no allocator of its own.  The regular scatter needs a caller-provided
// workspace for its duplicate-slot hash table; this variant keeps that scratch
// in a file-scope device array instead, so the caller passes only inputs and
// outputs.
//
// The array has a fixed size (enough for MAK_STATIC_SCATTER_MAX_SLOTS slots)
// and lives on every GPU that loads the library until the process exits.  Its
// device address is looked up on the first call in each (device, CUDA context)
// pair and cached; a context destroyed and re-created at the same handle (a
// cudaDeviceReset after the first call) is not detected, so callers that reset
// a device must not use this entry point on it afterwards.
#include <cuda.h>  // CUcontext / CUresult types only: cuCtxGetCurrent is fetched through the runtime

#include <mutex>

#include "common.cuh"

namespace mak {

// Same layout as mak_scatter_workspace_bytes(MAK_STATIC_SCATTER_MAX_SLOTS):
// hash keys and values (capacity = 2 * max slots, a power of two), then the
// resolved slot vector, plus alignment slack.
constexpr int64_t kStaticCapacity = 2 * static_cast<int64_t>(MAK_STATIC_SCATTER_MAX_SLOTS);
constexpr size_t kStaticScratchBytes = (static_cast<size_t>(kStaticCapacity) * 8 + 255) / 256 * 256 * 2 +
                                       (static_cast<size_t>(MAK_STATIC_SCATTER_MAX_SLOTS) * 8 + 255) / 256 * 256 + 256;

static __device__ __align__(256) unsigned char g_static_scatter_scratch[kStaticScratchBytes];

namespace {
// One cached address per (device, CUDA context): the array has its own copy, at its own
// address, in every context that loads the library's module -- the runtime's primary context
// and any context a caller created with the driver API and made current.
constexpr int kMaxScratchEntries = 64;
struct ScratchEntry {
  int device;
  CUcontext ctx;
  void* addr;
};
ScratchEntry g_scratch[kMaxScratchEntries];
int g_scratch_used = 0;
std::mutex g_scratch_mu;
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
}  // namespace

// Device address of the scratch array in the current context.  The name
// g_static_scatter_scratch in host code is only a host-side stand-in, so the
// address is looked up once per (device, context), with that device current, and cached.
static int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "mak_rows_scatter_static: cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_ctx_get_current == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return fail(MAK_E_CUDA, "mak_rows_scatter_static: cuCtxGetCurrent entry point unavailable");
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS)
    return fail(MAK_E_CUDA, "mak_rows_scatter_static: cuCtxGetCurrent failed");
  for (int i = 0; i < g_scratch_used; ++i) {
    if (g_scratch[i].device == dev && g_scratch[i].ctx == ctx) {
      *out = g_scratch[i].addr;
      return MAK_OK;
    }
  }
  // Miss (or no context current on this thread yet: the lookup binds the device's primary
  // context, and the entry is stored under the context that is current afterwards).
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_static_scatter_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "mak_rows_scatter_static: cudaGetSymbolAddress");
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return fail(MAK_E_CUDA, "mak_rows_scatter_static: no CUDA context current after the symbol lookup");
  for (int i = 0; i < g_scratch_used; ++i) {
    if (g_scratch[i].device == dev && g_scratch[i].ctx == ctx) {
      g_scratch[i].addr = p;
      *out = p;
      return MAK_OK;
    }
  }
  // A full table drops its oldest entry (a context beyond the 64th seen is looked up again later).
  if (g_scratch_used == kMaxScratchEntries) {
    for (int i = 1; i < kMaxScratchEntries; ++i) g_scratch[i - 1] = g_scratch[i];
    --g_scratch_used;
  }
  g_scratch[g_scratch_used++] = ScratchEntry{dev, ctx, p};
  *out = p;
  return MAK_OK;
}

}  // namespace mak

using namespace mak;

extern "C" {

int mak_rows_scatter_static(const mak_rows_desc* linear, const mak_rows_desc* paged, const int64_t* row_bytes,
                            int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots,
                            int64_t skip_prefix, void* stream) {
  if (n_slots > MAK_STATIC_SCATTER_MAX_SLOTS)
    return fail(MAK_E_UNSUPPORTED,
                "mak_rows_scatter_static: %lld slots exceed the static scratch limit of %d slots per call; "
                "use mak_rows_scatter with a workspace or split the call",
                (long long)n_slots, MAK_STATIC_SCATTER_MAX_SLOTS);
  if (n_slots <= 0) return mak_rows_scatter(linear, paged, row_bytes, row_bytes0, slots, slot_dtype, n_slots, skip_prefix,
                                            nullptr, 0, stream);
  void* scratch = nullptr;
  int rc = static_scratch_address(&scratch);
  if (rc) return rc;
  return mak_rows_scatter(linear, paged, row_bytes, row_bytes0, slots, slot_dtype, n_slots, skip_prefix, scratch,
                          kStaticScratchBytes, stream);
}

}  // extern "C"
