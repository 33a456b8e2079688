// Staging <-> paged byte-block transfer for DSV4 MLA / blocked-scale groups,
// the indptr/indices -> dense slot builder, and the host <-> device byte-copy
// batch (LMCache direct transfer).
//
// Strided block transfer (reference semantics: csrc/kvcache/kv_transfer_float.mu:3281-3405).
// Staging is [NL][staging_tokens][row_bytes]; block p of the batch covers staging
// tokens offset_in_object + p*BS + t and paged block block_ids[idx_start + p]:
//   mode 0: paged row t at  block*stride + t*row_bytes;
//   mode 1: each staging row is [value_bytes | scale_bytes]; the paged page keeps
//           all values first (block*stride + t*value_bytes) then all scales
//           (block*stride + BS*value_bytes + t*scale_bytes).
// direction 0 writes the paged pages, 1 reads them into staging.  Warps move
// pieces of 32 x 8 vectors of one (layer, block) with the widest vector every
// address allows; all layers go in one launch.  Negative block ids are skipped.
#include <algorithm>

#include "common.cuh"

namespace mak {

constexpr int kStridedLayers = 256;

struct StridedLaunch {
  uint64_t layers[kStridedLayers];
  uint8_t* staging;
  const int64_t* block_ids;
  int64_t idx_start, n_valid, offset_in_object, staging_tokens, block_size, row_bytes, block_stride;
  int64_t value_bytes, scale_bytes;
  int32_t direction, mode, num_layers, layer_base;
};

template <int VEC>
struct VecOf;
template <>
struct VecOf<16> { using T = uint4; };
template <>
struct VecOf<8> { using T = uint2; };
template <>
struct VecOf<4> { using T = uint32_t; };

// One warp item = up to 32 x kStridedU vectors of one (layer, block): the block's staging
// rows are contiguous (BS rows at pitch row_bytes), so vector i sits at staging byte i * VEC;
// on the page it sits at the same offset in mode 0, and in mode 1 at row * value_bytes + col *
// VEC (value part) or BS * value_bytes + row * scale_bytes + (col - vv) * VEC (scale part), where
// row / col are i's row and column in vectors of row_bytes.  Lanes carry (row, col) as they step
// by 32 vectors, so one division per item resolves them; every lane keeps kStridedU vectors in
// flight, and the items of a block go to different warps.
constexpr int kStridedU = 8;

template <int VEC>
__global__ void __launch_bounds__(256) strided_block_kernel(const __grid_constant__ StridedLaunch p) {
  using V = typename VecOf<VEC>::T;
  const int lane = threadIdx.x & 31;
  const uint32_t rv = static_cast<uint32_t>(p.row_bytes / VEC);  // vectors per staging row
  const uint32_t vv = static_cast<uint32_t>(p.value_bytes / VEC);
  const uint32_t n = static_cast<uint32_t>(p.block_size) * rv;   // vectors per (layer, block)
  constexpr uint32_t kPer = 32u * kStridedU;
  const uint32_t per_unit = (n + kPer - 1) / kPer;
  const int64_t total = static_cast<int64_t>(p.num_layers) * p.n_valid * per_unit;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int64_t unit = w / per_unit;
    const uint32_t part = static_cast<uint32_t>(w - unit * per_unit);
    const int layer = static_cast<int>(unit / p.n_valid);
    const int64_t blk_i = unit - static_cast<int64_t>(layer) * p.n_valid;
    const int64_t blk = p.block_ids[p.idx_start + blk_i];
    if (blk < 0) continue;
    uint8_t* staged = p.staging + ((static_cast<int64_t>(p.layer_base + layer) * p.staging_tokens) + p.offset_in_object +
                                   blk_i * p.block_size) * p.row_bytes;
    uint8_t* page = reinterpret_cast<uint8_t*>(p.layers[layer]) + blk * p.block_stride;
    const uint32_t i0 = part * kPer + lane;
    uint32_t row = i0 / rv, col = i0 - row * rv;
    int64_t po[kStridedU];
    V r[kStridedU];
#pragma unroll
    for (int u = 0; u < kStridedU; ++u) {
      const uint32_t i = i0 + 32u * u;
      if (p.mode == 0 || col < vv) {
        po[u] = p.mode == 0 ? static_cast<int64_t>(i) * VEC
                            : static_cast<int64_t>(row) * p.value_bytes + static_cast<int64_t>(col) * VEC;
      } else {
        po[u] = p.block_size * p.value_bytes + static_cast<int64_t>(row) * p.scale_bytes +
                static_cast<int64_t>(col - vv) * VEC;
      }
      if (i < n) {
        if (p.direction == 0) r[u] = *reinterpret_cast<const V*>(staged + static_cast<int64_t>(i) * VEC);
        else r[u] = *reinterpret_cast<const V*>(page + po[u]);
      }
      col += 32u;
      while (col >= rv) {
        col -= rv;
        ++row;
      }
    }
#pragma unroll
    for (int u = 0; u < kStridedU; ++u) {
      const uint32_t i = i0 + 32u * u;
      if (i >= n) continue;
      if (p.direction == 0) *reinterpret_cast<V*>(page + po[u]) = r[u];
      else *reinterpret_cast<V*>(staged + static_cast<int64_t>(i) * VEC) = r[u];
    }
  }
}

template <int VEC>
static int launch_strided(const StridedLaunch& p, cudaStream_t st) {
  const int threads = 256;
  const int64_t n = p.block_size * (p.row_bytes / VEC);
  const int64_t items = static_cast<int64_t>(p.num_layers) * p.n_valid * ((n + 32 * kStridedU - 1) / (32 * kStridedU));
  const int grid = grid_for(reinterpret_cast<const void*>(strided_block_kernel<VEC>), threads, 0, (items + 7) / 8);
  if (grid <= 0) return MAK_OK;
  strided_block_kernel<VEC><<<grid, threads, 0, st>>>(p);
  return launch_status("strided_block_kernel");
}

// slot[b*S + s] = s < min(max(indptr[b+1] - indptr[b], 0), S) ? indices[indptr[b] + s] : -1
__global__ void indexed_slots_kernel(const void* indptr, int ip64, const void* indices, int ix64, int64_t n_indices,
                                     int64_t batch, int64_t max_seq, int64_t* slots) {
  const int64_t total = batch * max_seq;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / max_seq, s = i - b * max_seq;
    const int64_t start = load_index(indptr, ip64, b);
    const int64_t end = load_index(indptr, ip64, b + 1);
    const int64_t len = end > start ? end - start : 0;
    int64_t out = -1;
    if (s < len && start + s >= 0 && start + s < n_indices) out = load_index(indices, ix64, start + s);
    slots[i] = out;
  }
}

// ---------------------------------------------------------------------------
// Byte-copy batch.  Small entries go through one kernel that reads/writes the
// pinned host side directly (unified addressing): CTA rows are entries, CTA
// columns split an entry, 4 independent 16-byte vectors per thread in flight.
// Large entries (or every entry when the caller wants the SMs free) go to the
// copy engines with one cudaMemcpyAsync each.
// ---------------------------------------------------------------------------
constexpr int kBatchEntries = 128;

struct BatchLaunch {
  mak_copy_entry e[kBatchEntries];
  int32_t n;
};

__global__ void __launch_bounds__(256) batch_copy_kernel(const __grid_constant__ BatchLaunch p) {
  const mak_copy_entry& e = p.e[blockIdx.y];
  const uint64_t bits = e.dst | e.src | e.size;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthr = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if ((bits & 15u) == 0) {
    const uint4* s = reinterpret_cast<const uint4*>(e.src);
    uint4* d = reinterpret_cast<uint4*>(e.dst);
    const int64_t n = static_cast<int64_t>(e.size / 16);
    for (int64_t i0 = tid; i0 < n; i0 += nthr * 4) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * nthr < n) r[u] = s[i0 + u * nthr];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * nthr < n) d[i0 + u * nthr] = r[u];
    }
  } else {
    const uint8_t* s = reinterpret_cast<const uint8_t*>(e.src);
    uint8_t* d = reinterpret_cast<uint8_t*>(e.dst);
    for (int64_t i = tid; i < static_cast<int64_t>(e.size); i += nthr) d[i] = s[i];
  }
}

}  // namespace mak

using namespace mak;

extern "C" {

int mak_lmcache_strided_block_transfer(void* staging, const uint64_t* paged_ptrs, const int64_t* block_ids,
                                       int64_t direction, int64_t num_layers, int64_t idx_start, int64_t n_valid,
                                       int64_t offset_in_object, int64_t staging_tokens, int64_t block_size,
                                       int64_t row_bytes, int64_t paged_block_stride, int64_t mode, int64_t value_bytes,
                                       int64_t scale_bytes, void* stream) {
  const char* name = "mak_lmcache_strided_block_transfer";
  if (!staging || !paged_ptrs || !block_ids) return fail(MAK_E_INVALID, "%s: NULL pointer", name);
  if (num_layers <= 0 || num_layers > MAK_MAX_PLANES) return fail(MAK_E_INVALID, "%s: bad num_layers %lld", name, (long long)num_layers);
  if (n_valid <= 0 || block_size <= 0 || staging_tokens <= 0 || idx_start < 0)
    return fail(MAK_E_INVALID, "%s: n_valid, block_size and staging_tokens must be positive", name);
  if (row_bytes <= 0 || (row_bytes & 3) != 0) return fail(MAK_E_INVALID, "%s: row_bytes must be a positive multiple of 4", name);
  if (paged_block_stride <= 0) return fail(MAK_E_INVALID, "%s: paged_block_stride must be positive", name);
  if (direction != 0 && direction != 1) return fail(MAK_E_INVALID, "%s: direction must be 0 or 1", name);
  if (mode != 0 && mode != 1) return fail(MAK_E_INVALID, "%s: mode must be 0 or 1", name);
  if (mode == 1 && (value_bytes <= 0 || scale_bytes <= 0 || (value_bytes & 3) || (scale_bytes & 3) ||
                    value_bytes + scale_bytes != row_bytes))
    return fail(MAK_E_INVALID, "%s: mode 1 needs value_bytes + scale_bytes == row_bytes, both multiples of 4", name);
  if (offset_in_object < 0 || offset_in_object + n_valid * block_size > staging_tokens)
    return fail(MAK_E_INVALID, "%s: block range exceeds the staging object", name);
  if (block_size * row_bytes >= (int64_t{1} << 31))
    return fail(MAK_E_UNSUPPORTED, "%s: a block of %lld rows of %lld bytes exceeds 2 GiB", name, (long long)block_size,
                (long long)row_bytes);
  uint64_t bits = reinterpret_cast<uint64_t>(staging) | static_cast<uint64_t>(row_bytes) |
                  static_cast<uint64_t>(paged_block_stride);
  if (mode == 1) bits |= static_cast<uint64_t>(value_bytes) | static_cast<uint64_t>(scale_bytes);
  for (int64_t l = 0; l < num_layers; ++l) {
    if (paged_ptrs[l] == 0) return fail(MAK_E_INVALID, "%s: layer %lld pointer is NULL", name, (long long)l);
    bits |= paged_ptrs[l];
  }
  const int vec = (bits & 15u) == 0 ? 16 : ((bits & 7u) == 0 ? 8 : 4);
  cudaStream_t st = as_stream(stream);
  for (int64_t l0 = 0; l0 < num_layers; l0 += kStridedLayers) {
    StridedLaunch p;
    memset(&p, 0, sizeof(p));
    const int64_t nl = std::min<int64_t>(kStridedLayers, num_layers - l0);
    for (int64_t l = 0; l < nl; ++l) p.layers[l] = paged_ptrs[l0 + l];
    p.staging = static_cast<uint8_t*>(staging);
    p.block_ids = block_ids;
    p.idx_start = idx_start;
    p.n_valid = n_valid;
    p.offset_in_object = offset_in_object;
    p.staging_tokens = staging_tokens;
    p.block_size = block_size;
    p.row_bytes = row_bytes;
    p.block_stride = paged_block_stride;
    p.value_bytes = value_bytes;
    p.scale_bytes = scale_bytes;
    p.direction = static_cast<int32_t>(direction);
    p.mode = static_cast<int32_t>(mode);
    p.num_layers = static_cast<int32_t>(nl);
    p.layer_base = static_cast<int32_t>(l0);
    int rc = vec == 16 ? launch_strided<16>(p, st) : (vec == 8 ? launch_strided<8>(p, st) : launch_strided<4>(p, st));
    if (rc) return rc;
  }
  return MAK_OK;
}

int mak_memcpy_batch(const mak_copy_entry* entries, int64_t n, int32_t mode, int64_t engine_threshold, void* stream) {
  if (n < 0 || (n > 0 && entries == nullptr)) return fail(MAK_E_INVALID, "mak_memcpy_batch: bad entry array");
  if (mode < MAK_COPY_AUTO || mode > MAK_COPY_KERNEL) return fail(MAK_E_INVALID, "mak_memcpy_batch: bad mode %d", mode);
  cudaStream_t st = as_stream(stream);
  if (engine_threshold <= 0) engine_threshold = 4 << 20;
  BatchLaunch L;
  memset(&L, 0, sizeof(L));
  uint64_t largest = 0;
  auto flush = [&]() -> int {
    if (L.n == 0) return MAK_OK;
    const int threads = 256;
    const uint64_t per_cta = static_cast<uint64_t>(threads) * 16 * 4;
    const unsigned gx = static_cast<unsigned>(std::min<uint64_t>(64, (largest + per_cta - 1) / per_cta));
    batch_copy_kernel<<<dim3(std::max(1u, gx), L.n), threads, 0, st>>>(L);
    const int rc = launch_status("batch_copy_kernel");
    L.n = 0;
    largest = 0;
    return rc;
  };
  for (int64_t i = 0; i < n; ++i) {
    const mak_copy_entry& e = entries[i];
    if (e.size == 0) continue;
    if (e.dst == 0 || e.src == 0) return fail(MAK_E_INVALID, "mak_memcpy_batch: entry %lld has a NULL pointer", (long long)i);
    const bool engine = mode == MAK_COPY_ENGINE || (mode == MAK_COPY_AUTO && e.size >= static_cast<uint64_t>(engine_threshold));
    if (engine) {
      cudaError_t err = cudaMemcpyAsync(reinterpret_cast<void*>(e.dst), reinterpret_cast<const void*>(e.src), e.size,
                                        cudaMemcpyDefault, st);
      if (err != cudaSuccess) return cuda_fail(err, "mak_memcpy_batch: cudaMemcpyAsync");
      continue;
    }
    L.e[L.n++] = e;
    largest = std::max<uint64_t>(largest, e.size);
    if (L.n == kBatchEntries) {
      int rc = flush();
      if (rc) return rc;
    }
  }
  return flush();
}

int mak_runtime_versions(int32_t* runtime_version, int32_t* driver_version) {
  int rt = 0, drv = 0;
  cudaError_t e = cudaRuntimeGetVersion(&rt);
  if (e == cudaSuccess) e = cudaDriverGetVersion(&drv);
  if (e != cudaSuccess) return cuda_fail(e, "mak_runtime_versions");
  if (runtime_version) *runtime_version = rt;
  if (driver_version) *driver_version = drv;
  return MAK_OK;
}

int mak_build_indexed_slots(const void* indptr, int32_t indptr_dtype, const void* indices, int32_t indices_dtype,
                            int64_t n_indices, int64_t batch, int64_t max_seq, int64_t* slots, void* stream) {
  if (!valid_index_dtype(indptr_dtype) || !valid_index_dtype(indices_dtype))
    return fail(MAK_E_INVALID, "mak_build_indexed_slots: index dtypes must be int32 or int64");
  if (batch < 0 || max_seq < 0 || n_indices < 0) return fail(MAK_E_INVALID, "mak_build_indexed_slots: bad sizes");
  const int64_t total = batch * max_seq;
  if (total == 0) return MAK_OK;
  if (!indptr || !slots || (n_indices > 0 && !indices)) return fail(MAK_E_INVALID, "mak_build_indexed_slots: NULL pointer");
  const int threads = 256;
  const int grid = grid_for(reinterpret_cast<const void*>(indexed_slots_kernel), threads, 0, (total + threads - 1) / threads);
  indexed_slots_kernel<<<grid, threads, 0, as_stream(stream)>>>(indptr, indptr_dtype == MAK_DT_I64, indices,
                                                                indices_dtype == MAK_DT_I64, n_indices, batch, max_seq,
                                                                slots);
  return launch_status("indexed_slots_kernel");
}

}  // extern "C"
