// Status reporting, device queries and the plan builder of libmak_kvcache:
// slot validation reduction, last-writer-wins duplicate resolution and the
// block-table -> slot-mapping builder.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>

#include "common.cuh"

namespace mak {

static thread_local char g_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MAK_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static std::atomic<uint64_t> g_launches{0};

int launch_status(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return MAK_OK;
}

namespace {
constexpr int kMaxDevices = 64;
int g_sm[kMaxDevices] = {0};
std::mutex g_sm_mu;
}  // namespace

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  {
    std::lock_guard<std::mutex> lk(g_sm_mu);
    if (g_sm[dev] > 0) return g_sm[dev];
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  g_sm[dev] = n;
  return n;
}

namespace {
struct OccKey {
  const void* kernel;
  int threads;
  size_t smem;
  bool operator<(const OccKey& o) const {
    if (kernel != o.kernel) return kernel < o.kernel;
    if (threads != o.threads) return threads < o.threads;
    return smem < o.smem;
  }
};
std::map<OccKey, int> g_occ;
std::mutex g_occ_mu;
}  // namespace

int blocks_per_sm(const void* kernel, int threads, size_t smem) {
  const OccKey key{kernel, threads, smem};
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm <= 0)
    per_sm = 1;
  std::lock_guard<std::mutex> lk(g_occ_mu);
  g_occ[key] = per_sm;
  return per_sm;
}

int grid_for(const void* kernel, int threads, size_t smem, int64_t work_ctas) {
  if (work_ctas <= 0) return 0;
  const int64_t cap = static_cast<int64_t>(blocks_per_sm(kernel, threads, smem)) * sm_count();
  return static_cast<int>(work_ctas < cap ? work_ctas : cap);
}

// ---------------------------------------------------------------------------
// Slot validation: max over the slot vector (negative entries included, so the
// result is -1 when nothing is valid; the caller compares it with NB*BS).
// ---------------------------------------------------------------------------
__global__ void slot_max_kernel(const void* slots, int is64, int64_t n, long long* out) {
  long long m = -1;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const long long s = load_index(slots, is64, i);
    m = s > m ? s : m;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const long long v = __shfl_xor_sync(0xffffffffu, m, o);
    m = v > m ? v : m;
  }
  __shared__ long long warp_max[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) warp_max[wid] = m;
  __syncthreads();
  if (wid == 0) {
    m = lane < (int)(blockDim.x >> 5) ? warp_max[lane] : -1;
    for (int o = 16; o > 0; o >>= 1) {
      const long long v = __shfl_xor_sync(0xffffffffu, m, o);
      m = v > m ? v : m;
    }
    if (lane == 0 && m >= 0) atomicMax(out, m);
  }
}

// ---------------------------------------------------------------------------
// Last-writer-wins resolution through an open-addressing hash table keyed by
// slot.  Insert keeps the largest token index per slot; resolve keeps a token
// only if it is that index.  Load factor <= 1/2, so probing always ends.
// ---------------------------------------------------------------------------
constexpr unsigned long long kEmpty = ~0ull;

__global__ void hash_insert_kernel(const void* slots, int is64, int64_t n, unsigned long long* keys, long long* vals,
                                   int64_t mask) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = load_index(slots, is64, i);
    if (s < 0) continue;
    uint64_t h = mix64(static_cast<uint64_t>(s)) & static_cast<uint64_t>(mask);
    for (int64_t probe = 0; probe <= mask; ++probe) {
      const unsigned long long prev = atomicCAS(keys + h, kEmpty, static_cast<unsigned long long>(s));
      if (prev == kEmpty || prev == static_cast<unsigned long long>(s)) {
        atomicMax(vals + h, static_cast<long long>(i));
        break;
      }
      h = (h + 1) & static_cast<uint64_t>(mask);
    }
  }
}

__global__ void hash_resolve_kernel(const void* slots, int is64, int64_t n, const unsigned long long* keys,
                                    const long long* vals, int64_t mask, int64_t* eff) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = load_index(slots, is64, i);
    int64_t out = -1;
    if (s >= 0) {
      uint64_t h = mix64(static_cast<uint64_t>(s)) & static_cast<uint64_t>(mask);
      for (int64_t probe = 0; probe <= mask; ++probe) {
        const unsigned long long k = keys[h];
        if (k == static_cast<unsigned long long>(s)) {
          out = (vals[h] == i) ? s : -1;
          break;
        }
        if (k == kEmpty) break;
        h = (h + 1) & static_cast<uint64_t>(mask);
      }
    }
    eff[i] = out;
  }
}

__global__ void owner_mark_kernel(const void* slots, int is64, int64_t n, unsigned long long* owner, int64_t rows,
                                  unsigned long long tag_hi) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = load_index(slots, is64, i);
    if (s >= 0 && s < rows) atomicMax(owner + s, tag_hi | static_cast<unsigned long long>(i));
  }
}

int mark_owners(const void* slots, int32_t slot_dtype, int64_t n, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                cudaStream_t st, const char* name) {
  if (owner == nullptr || owner_rows < 0) return fail(MAK_E_INVALID, "%s: owner table is NULL", name);
  if ((reinterpret_cast<uintptr_t>(owner) & 7u) != 0) return fail(MAK_E_INVALID, "%s: owner table must be 8-byte aligned", name);
  if (epoch == 0) return fail(MAK_E_INVALID, "%s: epoch must be at least 1", name);
  if (n >= (int64_t{1} << 32)) return fail(MAK_E_UNSUPPORTED, "%s: owner tables take fewer than 2^32 items", name);
  if (n == 0) return MAK_OK;
  const int threads = 256;
  const int grid = grid_for(reinterpret_cast<const void*>(owner_mark_kernel), threads, 0, (n + threads - 1) / threads);
  return launch_pdl("owner_mark_kernel", owner_mark_kernel, dim3(grid), dim3(threads), 0, st, slots,
                    static_cast<int>(slot_dtype == MAK_DT_I64), n, reinterpret_cast<unsigned long long*>(owner),
                    owner_rows, static_cast<unsigned long long>(epoch) << 32);
}

int64_t hash_capacity(int64_t n) {
  int64_t c = 64;
  while (c < 2 * n) c <<= 1;
  return c;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int carve_scatter_ws(void* ws, size_t ws_bytes, int64_t n, ScatterWs* out) {
  const int64_t cap = hash_capacity(n);
  const size_t need = mak_scatter_workspace_bytes(n);
  if (ws == nullptr || ws_bytes < need)
    return fail(MAK_E_WORKSPACE, "scatter workspace too small: need %zu bytes, got %zu", need, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 15u) != 0) return fail(MAK_E_WORKSPACE, "scatter workspace must be 16-byte aligned");
  char* p = static_cast<char*>(ws);
  out->keys = reinterpret_cast<unsigned long long*>(p);
  p += align_up(cap * sizeof(unsigned long long), 256);
  out->vals = reinterpret_cast<long long*>(p);
  p += align_up(cap * sizeof(long long), 256);
  out->eff = reinterpret_cast<int64_t*>(p);
  out->capacity = cap;
  return MAK_OK;
}

int resolve_last_writer(const void* slots, int32_t slot_dtype, int64_t n, const ScatterWs& ws, cudaStream_t st) {
  if (n <= 0) return MAK_OK;
  // keys and vals are adjacent (vals starts 256-aligned after keys): clear both to all-ones (= empty / -1).
  cudaError_t e = cudaMemsetAsync(ws.keys, 0xFF, align_up(ws.capacity * sizeof(unsigned long long), 256) +
                                                   ws.capacity * sizeof(long long), st);
  if (e != cudaSuccess) return cuda_fail(e, "clear scatter hash table");
  const int threads = 256;
  const int is64 = slot_dtype == MAK_DT_I64;
  int grid = grid_for(reinterpret_cast<const void*>(hash_insert_kernel), threads, 0, (n + threads - 1) / threads);
  hash_insert_kernel<<<grid, threads, 0, st>>>(slots, is64, n, ws.keys, ws.vals, ws.capacity - 1);
  int rc = launch_status("hash_insert_kernel");
  if (rc) return rc;
  grid = grid_for(reinterpret_cast<const void*>(hash_resolve_kernel), threads, 0, (n + threads - 1) / threads);
  hash_resolve_kernel<<<grid, threads, 0, st>>>(slots, is64, n, ws.keys, ws.vals, ws.capacity - 1, ws.eff);
  return launch_status("hash_resolve_kernel");
}

// ---------------------------------------------------------------------------
// Slot mapping from block tables (flash-style dense [B, S] token grid).
// ---------------------------------------------------------------------------
__global__ void build_slot_mapping_kernel(const void* bt, int bt64, int64_t bt_stride, const void* lens, int len64,
                                          int64_t batch, int64_t max_seq, int64_t bs, int64_t* slots) {
  const int64_t total = batch * max_seq;
  pdl_wait();
  pdl_trigger();  // the tile launch that follows waits for this grid's completion all the same
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / max_seq, s = i - b * max_seq;
    const int64_t len = load_index(lens, len64, b);
    int64_t out = -1;
    if (s < len) {
      const int64_t blk = load_index(bt, bt64, b * bt_stride + s / bs);
      out = blk < 0 ? -1 : blk * bs + s % bs;
    }
    slots[i] = out;
  }
}

}  // namespace mak

using namespace mak;

extern "C" {

int mak_abi_version(void) { return MAK_ABI_VERSION; }

const char* mak_last_error(void) { return g_last_error; }

int mak_device_sm_count(void) { return sm_count(); }

uint64_t mak_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t mak_scatter_workspace_bytes(int64_t n_items) {
  if (n_items < 0) n_items = 0;
  const int64_t cap = hash_capacity(n_items);
  return align_up(cap * sizeof(unsigned long long), 256) + align_up(cap * sizeof(long long), 256) +
         align_up(static_cast<size_t>(n_items) * sizeof(int64_t), 256) + 256;
}

int mak_slot_max(const void* slots, int32_t slot_dtype, int64_t n, int64_t* out_max, void* stream) {
  if (!valid_index_dtype(slot_dtype)) return fail(MAK_E_INVALID, "mak_slot_max: slot dtype must be int32 or int64");
  if (out_max == nullptr) return fail(MAK_E_INVALID, "mak_slot_max: out_max is NULL");
  if (n < 0 || (n > 0 && slots == nullptr)) return fail(MAK_E_INVALID, "mak_slot_max: bad slot vector");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(out_max, 0xFF, sizeof(int64_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "mak_slot_max: init");
  if (n == 0) return MAK_OK;
  const int threads = 256;
  int grid = grid_for(reinterpret_cast<const void*>(slot_max_kernel), threads, 0, (n + threads - 1) / threads);
  slot_max_kernel<<<grid, threads, 0, st>>>(slots, slot_dtype == MAK_DT_I64, n, reinterpret_cast<long long*>(out_max));
  return launch_status("slot_max_kernel");
}

int mak_resolve_last_writer(const void* slots, int32_t slot_dtype, int64_t n, int64_t* eff, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!valid_index_dtype(slot_dtype)) return fail(MAK_E_INVALID, "mak_resolve_last_writer: slot dtype must be int32 or int64");
  if (n < 0 || (n > 0 && (slots == nullptr || eff == nullptr)))
    return fail(MAK_E_INVALID, "mak_resolve_last_writer: bad arguments");
  ScatterWs ws{};
  int rc = carve_scatter_ws(workspace, workspace_bytes, n, &ws);
  if (rc) return rc;
  ws.eff = eff;
  return resolve_last_writer(slots, slot_dtype, n, ws, as_stream(stream));
}

int mak_build_slot_mapping(const void* block_tables, int32_t bt_dtype, int64_t bt_stride, const void* seq_lens,
                           int32_t len_dtype, int64_t batch, int64_t max_seq, int64_t block_size, int64_t* slots,
                           void* stream) {
  if (!valid_index_dtype(bt_dtype) || !valid_index_dtype(len_dtype))
    return fail(MAK_E_INVALID, "mak_build_slot_mapping: index dtypes must be int32 or int64");
  if (batch < 0 || max_seq < 0 || block_size <= 0 || bt_stride < 0)
    return fail(MAK_E_INVALID, "mak_build_slot_mapping: bad sizes");
  const int64_t total = batch * max_seq;
  if (total == 0) return MAK_OK;
  if (!block_tables || !seq_lens || !slots) return fail(MAK_E_INVALID, "mak_build_slot_mapping: NULL pointer");
  const int threads = 256;
  int grid = grid_for(reinterpret_cast<const void*>(build_slot_mapping_kernel), threads, 0, (total + threads - 1) / threads);
  // programmatic dependent launch: the launch overlaps the previous kernel's drain
  return launch_pdl("build_slot_mapping_kernel", build_slot_mapping_kernel, dim3(grid), dim3(threads), 0,
                    as_stream(stream), block_tables, static_cast<int>(bt_dtype == MAK_DT_I64), bt_stride, seq_lens,
                    static_cast<int>(len_dtype == MAK_DT_I64), batch, max_seq, block_size, slots);
}

}  // extern "C"
