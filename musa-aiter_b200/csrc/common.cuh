// Shared device/host helpers of libmak_kvcache (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstddef>

#include "mak_kvcache.h"

namespace mak {

// ---- host-side status helpers (abi_util.cu) --------------------------------
int fail(int status, const char* fmt, ...);            // records message, returns status
int cuda_fail(cudaError_t e, const char* what);        // MAK_E_CUDA with cudaGetErrorString
int launch_status(const char* what);                   // checks cudaGetLastError after a launch; counts it
int sm_count();                                        // SMs of the current device (cached)
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool valid_index_dtype(int32_t dt) { return dt == MAK_DT_I32 || dt == MAK_DT_I64; }
inline int dtype_bytes(int32_t dt) {
  switch (dt) {
    case MAK_DT_U8: return 1;
    case MAK_DT_F16: return 2;
    case MAK_DT_BF16: return 2;
    case MAK_DT_F32: return 4;
    case MAK_DT_I32: return 4;
    case MAK_DT_I64: return 8;
    default: return 0;
  }
}

// Grid size for a grid-stride kernel: enough CTAs for `work_ctas` units of
// work, capped at the number of CTAs that fit on the device at once.
int grid_for(const void* kernel, int threads, size_t smem, int64_t work_ctas);
// Resident CTAs per SM for a kernel launch shape (queried once, then cached).
int blocks_per_sm(const void* kernel, int threads, size_t smem);

// Scatter workspace layout: [hash keys C x u64][hash vals C x i64][eff n x i64]
struct ScatterWs {
  unsigned long long* keys;
  long long* vals;
  int64_t* eff;
  int64_t capacity;  // power of two
};
int64_t hash_capacity(int64_t n);
int carve_scatter_ws(void* ws, size_t ws_bytes, int64_t n, ScatterWs* out);
// Resolves duplicates of `slots` into ws.eff (last index wins).  Returns MAK_OK or error.
int resolve_last_writer(const void* slots, int32_t slot_dtype, int64_t n, const ScatterWs& ws, cudaStream_t st);
// Owner-table last-writer marking: owner[slot] = max(owner[slot], epoch << 32 | i)
// for every in-range slot i < n (n < 2^32, epoch >= 1).  The consuming kernel
// lets item i write only while owner[slot] still equals its own tag.
int mark_owners(const void* slots, int32_t slot_dtype, int64_t n, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                cudaStream_t st, const char* name);

// ---- programmatic dependent launch -------------------------------------------
// Kernels of this library that are launched with launch_pdl() may start while
// the previous kernel of the stream is still draining: their CTAs become
// resident early and block in pdl_wait() (griddepcontrol.wait) until every
// prerequisite grid has completed and its memory is visible.  pdl_wait() must
// therefore come before the kernel's first global-memory access (read or
// write); pdl_trigger() (griddepcontrol.launch_dependents) then lets the next
// launch of the stream be scheduled in the same way.  Both are no-ops for a
// grid launched without the attribute, and the wait is a hardware dependency,
// not a spin on memory.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with cudaLaunchAttributeProgrammaticStreamSerialization (the kernel
// must call pdl_wait() before touching global memory).  Counts the launch and
// returns MAK_OK or the CUDA error as a status.
template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return cuda_fail(e, what);
  }
  return launch_status(what);
}

// ---- device helpers -----------------------------------------------------------
__device__ __forceinline__ int64_t load_index(const void* p, int is64, int64_t i) {
  return is64 ? __ldg(reinterpret_cast<const long long*>(p) + i)
              : static_cast<int64_t>(__ldg(reinterpret_cast<const int*>(p) + i));
}

// Block/offset split of a slot; 32-bit division whenever the operands allow it.
__device__ __forceinline__ void split_slot(int64_t s, int64_t bs, int64_t* b, int64_t* o) {
  if (((s | bs) >> 31) == 0) {
    const uint32_t q = static_cast<uint32_t>(s) / static_cast<uint32_t>(bs);
    *b = q;
    *o = s - static_cast<int64_t>(q) * bs;
  } else {
    *b = s / bs;
    *o = s - (*b) * bs;
  }
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  // SplitMix64 finaliser (Steele, Lea, Flood 2014): spreads consecutive slots.
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

}  // namespace mak
