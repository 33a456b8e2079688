// Row engine: moves whole token rows (a token's hidden vector, an MLA latent
// row, a DSV4 byte row or an entire paged block) between "planes" (one cache
// tensor per (kv, layer)) addressed through optional index vectors.
//
// One warp owns one row at a time and moves it with the widest vector (16 B
// when every pointer, stride and row width allows) using U independent loads
// per lane before the stores, so each SM keeps tens of KB in flight.  All
// planes of a call go in one launch (plane pointers travel in the kernel's
// parameter block); the warp-row index runs token-fastest inside a plane so
// consecutive warps touch consecutive linear rows.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace mak {

constexpr int kRowPlanes = 128;  // planes per launch (parameter block < 4 KB)

struct RowSide {
  int64_t rows_per_block;
  int64_t block_stride;  // bytes
  int64_t row_stride;    // bytes
  int64_t num_rows;      // valid rows are [0, num_rows)
};

struct RowLaunch {
  uint64_t src[kRowPlanes];
  uint64_t dst[kRowPlanes];
  int32_t row_bytes[kRowPlanes];
  RowSide s, d;
  const void* src_idx;  // NULL -> identity (i + src_base)
  const void* dst_idx;  // NULL -> identity (i + dst_base)
  int64_t n_items;      // items that carry an index
  int64_t n_total;      // items processed; [n_items, n_total) are zero-filled tail rows (identity dst)
  int64_t src_base;
  int64_t dst_base;
  int32_t src_idx64;
  int32_t dst_idx64;
  int32_t num_planes;
  int32_t zero_fill;    // write zeros where the source row is missing
};

template <int V>
struct VecT;
template <>
struct VecT<16> { using T = uint4; };
template <>
struct VecT<8> { using T = uint2; };
template <>
struct VecT<4> { using T = uint32_t; };
template <>
struct VecT<2> { using T = uint16_t; };
template <>
struct VecT<1> { using T = uint8_t; };

__device__ __forceinline__ int64_t row_offset(const RowSide& s, int64_t r) {
  if (s.rows_per_block == 1) return r * s.block_stride;
  int64_t b, o;
  split_slot(r, s.rows_per_block, &b, &o);
  return b * s.block_stride + o * s.row_stride;
}

template <int VEC>
__global__ void __launch_bounds__(256) rows_kernel(const __grid_constant__ RowLaunch p) {
  using V = typename VecT<VEC>::T;
  constexpr int U = (VEC >= 8) ? 4 : 8;  // independent vectors in flight per lane
  const int lane = threadIdx.x & 31;
  const int64_t total = p.n_total * p.num_planes;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
    const int plane = static_cast<int>(w / p.n_total);
    const int64_t i = w - static_cast<int64_t>(plane) * p.n_total;
    const bool indexed = i < p.n_items;
    int64_t dr;
    if (p.dst_idx != nullptr) {
      dr = indexed ? load_index(p.dst_idx, p.dst_idx64, i) : -1;
    } else {
      dr = i + p.dst_base;
    }
    if (dr < 0 || dr >= p.d.num_rows) continue;
    int64_t sr = -1;
    if (indexed) sr = (p.src_idx != nullptr) ? load_index(p.src_idx, p.src_idx64, i) : i + p.src_base;
    const bool have_src = sr >= 0 && sr < p.s.num_rows;
    if (!have_src && !p.zero_fill) continue;
    V* dst = reinterpret_cast<V*>(p.dst[plane] + row_offset(p.d, dr));
    const int64_t nv = p.row_bytes[plane] / VEC;
    if (!have_src) {
      V z;
      memset(&z, 0, sizeof(V));
      for (int64_t v = lane; v < nv; v += 32) dst[v] = z;
      continue;
    }
    const V* src = reinterpret_cast<const V*>(p.src[plane] + row_offset(p.s, sr));
    for (int64_t v0 = lane; v0 < nv; v0 += 32 * U) {
      V r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t v = v0 + 32 * u;
        if (v < nv) r[u] = src[v];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t v = v0 + 32 * u;
        if (v < nv) dst[v] = r[u];
      }
    }
  }
}

static int vec_width(uint64_t bits) {
  if ((bits & 15u) == 0) return 16;
  if ((bits & 7u) == 0) return 8;
  if ((bits & 3u) == 0) return 4;
  if ((bits & 1u) == 0) return 2;
  return 1;
}

template <int VEC>
static int launch_rows_vec(const RowLaunch& p, cudaStream_t st) {
  const int threads = 256;
  const int64_t warps = p.n_total * p.num_planes;
  const int64_t ctas = (warps + (threads / 32) - 1) / (threads / 32);
  const int grid = grid_for(reinterpret_cast<const void*>(rows_kernel<VEC>), threads, 0, ctas);
  if (grid <= 0) return MAK_OK;
  rows_kernel<VEC><<<grid, threads, 0, st>>>(p);
  return launch_status("rows_kernel");
}

struct RowCall {
  const mak_rows_desc* src;
  const mak_rows_desc* dst;
  const int64_t* row_bytes;
  int64_t row_bytes0;
  const void* src_idx;
  int32_t src_idx_dtype;
  const void* dst_idx;
  int32_t dst_idx_dtype;
  int64_t n_items;
  int64_t n_total;
  int64_t src_base;
  int64_t dst_base;
  int32_t zero_fill;
};

static int check_side(const mak_rows_desc* s, const char* name) {
  if (s == nullptr) return fail(MAK_E_INVALID, "%s: row descriptor is NULL", name);
  if (s->num_planes < 0 || s->num_planes > MAK_MAX_PLANES)
    return fail(MAK_E_INVALID, "%s: num_planes %lld outside [0, %d]", name, (long long)s->num_planes, MAK_MAX_PLANES);
  if (s->num_planes > 0 && s->plane_ptrs == nullptr) return fail(MAK_E_INVALID, "%s: plane_ptrs is NULL", name);
  if (s->rows_per_block <= 0 || s->num_rows < 0 || s->block_stride < 0 || s->row_stride < 0)
    return fail(MAK_E_INVALID, "%s: bad row geometry", name);
  for (int64_t p = 0; p < s->num_planes; ++p)
    if (s->plane_ptrs[p] == 0 && s->num_rows > 0) return fail(MAK_E_INVALID, "%s: plane %lld pointer is NULL", name, (long long)p);
  return MAK_OK;
}

static int run_rows(const RowCall& c, cudaStream_t st, const char* name) {
  int rc = check_side(c.src, name);
  if (rc) return rc;
  rc = check_side(c.dst, name);
  if (rc) return rc;
  if (c.src->num_planes != c.dst->num_planes)
    return fail(MAK_E_INVALID, "%s: source has %lld planes, destination %lld", name, (long long)c.src->num_planes,
                (long long)c.dst->num_planes);
  if ((c.src_idx && !valid_index_dtype(c.src_idx_dtype)) || (c.dst_idx && !valid_index_dtype(c.dst_idx_dtype)))
    return fail(MAK_E_INVALID, "%s: index dtype must be int32 or int64", name);
  if (c.n_items < 0 || c.n_total < c.n_items) return fail(MAK_E_INVALID, "%s: bad item counts", name);
  const int64_t planes = c.src->num_planes;
  if (planes == 0 || c.n_total == 0) return MAK_OK;
  // Vector width: the largest power of two (<= 16) dividing every address, stride and row width.
  uint64_t bits = static_cast<uint64_t>(c.src->block_stride) | static_cast<uint64_t>(c.dst->block_stride);
  if (c.src->rows_per_block > 1) bits |= static_cast<uint64_t>(c.src->row_stride);
  if (c.dst->rows_per_block > 1) bits |= static_cast<uint64_t>(c.dst->row_stride);
  for (int64_t p = 0; p < planes; ++p) {
    const int64_t rb = c.row_bytes ? c.row_bytes[p] : c.row_bytes0;
    if (rb < 0 || rb > (int64_t)0x7fffffff) return fail(MAK_E_INVALID, "%s: bad row width %lld", name, (long long)rb);
    bits |= static_cast<uint64_t>(rb) | c.src->plane_ptrs[p] | c.dst->plane_ptrs[p];
  }
  const int vec = vec_width(bits);
  for (int64_t p0 = 0; p0 < planes; p0 += kRowPlanes) {
    RowLaunch L;
    memset(&L, 0, sizeof(L));
    const int64_t np = std::min<int64_t>(kRowPlanes, planes - p0);
    for (int64_t q = 0; q < np; ++q) {
      L.src[q] = c.src->plane_ptrs[p0 + q];
      L.dst[q] = c.dst->plane_ptrs[p0 + q];
      L.row_bytes[q] = static_cast<int32_t>(c.row_bytes ? c.row_bytes[p0 + q] : c.row_bytes0);
    }
    L.s = RowSide{c.src->rows_per_block, c.src->block_stride, c.src->row_stride, c.src->num_rows};
    L.d = RowSide{c.dst->rows_per_block, c.dst->block_stride, c.dst->row_stride, c.dst->num_rows};
    L.src_idx = c.src_idx;
    L.dst_idx = c.dst_idx;
    L.src_idx64 = c.src_idx_dtype == MAK_DT_I64;
    L.dst_idx64 = c.dst_idx_dtype == MAK_DT_I64;
    L.n_items = c.n_items;
    L.n_total = c.n_total;
    L.src_base = c.src_base;
    L.dst_base = c.dst_base;
    L.num_planes = static_cast<int32_t>(np);
    L.zero_fill = c.zero_fill;
    switch (vec) {
      case 16: rc = launch_rows_vec<16>(L, st); break;
      case 8: rc = launch_rows_vec<8>(L, st); break;
      case 4: rc = launch_rows_vec<4>(L, st); break;
      case 2: rc = launch_rows_vec<2>(L, st); break;
      default: rc = launch_rows_vec<1>(L, st); break;
    }
    if (rc) return rc;
  }
  return MAK_OK;
}

}  // namespace mak

using namespace mak;

extern "C" {

int mak_rows_gather(const mak_rows_desc* paged, const mak_rows_desc* linear, const int64_t* row_bytes,
                    int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots, int32_t fill_zero,
                    void* stream) {
  if (n_slots < 0 || (n_slots > 0 && slots == nullptr)) return fail(MAK_E_INVALID, "mak_rows_gather: bad slot vector");
  if (n_slots > 0 && !valid_index_dtype(slot_dtype)) return fail(MAK_E_INVALID, "mak_rows_gather: slot dtype must be int32 or int64");
  if (linear == nullptr) return fail(MAK_E_INVALID, "mak_rows_gather: linear descriptor is NULL");
  RowCall c{};
  c.src = paged;
  c.dst = linear;
  c.row_bytes = row_bytes;
  c.row_bytes0 = row_bytes0;
  c.src_idx = slots;
  c.src_idx_dtype = slot_dtype;
  c.n_items = std::min<int64_t>(n_slots, linear->num_rows);
  c.n_total = fill_zero ? linear->num_rows : c.n_items;
  c.zero_fill = fill_zero ? 1 : 0;
  return run_rows(c, as_stream(stream), "mak_rows_gather");
}

int mak_rows_scatter(const mak_rows_desc* linear, const mak_rows_desc* paged, const int64_t* row_bytes,
                     int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots, int64_t skip_prefix,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (n_slots < 0 || (n_slots > 0 && slots == nullptr)) return fail(MAK_E_INVALID, "mak_rows_scatter: bad slot vector");
  if (n_slots == 0) return MAK_OK;
  if (!valid_index_dtype(slot_dtype)) return fail(MAK_E_INVALID, "mak_rows_scatter: slot dtype must be int32 or int64");
  if (skip_prefix < 0) return fail(MAK_E_INVALID, "mak_rows_scatter: skip_prefix must be non-negative");
  cudaStream_t st = as_stream(stream);
  ScatterWs ws{};
  int rc = carve_scatter_ws(workspace, workspace_bytes, n_slots, &ws);
  if (rc) return rc;
  rc = resolve_last_writer(slots, slot_dtype, n_slots, ws, st);
  if (rc) return rc;
  RowCall c{};
  c.src = linear;
  c.dst = paged;
  c.row_bytes = row_bytes;
  c.row_bytes0 = row_bytes0;
  c.dst_idx = ws.eff;
  c.dst_idx_dtype = MAK_DT_I64;
  c.n_items = n_slots;
  c.n_total = n_slots;
  c.src_base = skip_prefix;
  return run_rows(c, st, "mak_rows_scatter");
}

int mak_rows_copy(const mak_rows_desc* src, const mak_rows_desc* dst, const int64_t* row_bytes, int64_t row_bytes0,
                  const void* src_idx, int32_t src_idx_dtype, const void* dst_idx, int32_t dst_idx_dtype, int64_t n,
                  void* workspace, size_t workspace_bytes, void* stream) {
  if (n < 0) return fail(MAK_E_INVALID, "mak_rows_copy: negative item count");
  if (n == 0) return MAK_OK;
  cudaStream_t st = as_stream(stream);
  RowCall c{};
  c.src = src;
  c.dst = dst;
  c.row_bytes = row_bytes;
  c.row_bytes0 = row_bytes0;
  c.src_idx = src_idx;
  c.src_idx_dtype = src_idx_dtype;
  c.dst_idx = dst_idx;
  c.dst_idx_dtype = dst_idx_dtype;
  c.n_items = n;
  c.n_total = n;
  if (dst_idx != nullptr) {
    if (!valid_index_dtype(dst_idx_dtype)) return fail(MAK_E_INVALID, "mak_rows_copy: index dtype must be int32 or int64");
    ScatterWs ws{};
    int rc = carve_scatter_ws(workspace, workspace_bytes, n, &ws);
    if (rc) return rc;
    rc = resolve_last_writer(dst_idx, dst_idx_dtype, n, ws, st);
    if (rc) return rc;
    c.dst_idx = ws.eff;
    c.dst_idx_dtype = MAK_DT_I64;
  }
  return run_rows(c, st, "mak_rows_copy");
}

}  // extern "C"
