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
// and lives on every GPU that loads the library until the process exits.
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
constexpr int kMaxScratchDevices = 64;
void* g_scratch_addr[kMaxScratchDevices] = {nullptr};
std::mutex g_scratch_mu;
}  // namespace

// Device address of the scratch array on the current device.  The name
// g_static_scatter_scratch in host code is only a host-side stand-in, so the
// address is looked up once per device (with that device current) and cached.
static int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "mak_rows_scatter_static: cudaGetDevice");
  if (dev < 0 || dev >= kMaxScratchDevices) return fail(MAK_E_UNSUPPORTED, "mak_rows_scatter_static: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scatter_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "mak_rows_scatter_static: cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
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
