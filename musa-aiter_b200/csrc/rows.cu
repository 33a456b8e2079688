// Row engine: moves whole token rows (a token's hidden vector, an MLA latent
// row, a DSV4 byte row or an entire paged block) between "planes" (one cache
// tensor per (kv, layer)) addressed through optional index vectors.
//
// A warp owns a chunk of up to 32 consecutive items of one plane.  Each lane
// resolves one item's source and destination row (one coalesced index load per
// chunk, so the index latency is paid once per chunk, not once per row) and
// parks the two byte offsets in shared memory.  The chunk length is chosen per
// plane group from the row width and the call's size: long enough to amortise
// the index load, short enough (about 1/8 of a warp's share of the bytes) that
// the last wave stays balanced.  The warp then streams the chunk's
// rows with the widest vector (16 B when every pointer, stride and row width
// allows): narrow rows are split over sub-groups of L lanes (L = the power of
// two covering the row's vectors, so a 128-byte row takes 8 lanes and one warp
// instruction moves 4 rows), wide rows over all 32 lanes; every lane keeps U
// independent loads in flight before its stores.  All planes of a call go in
// one launch (plane pointers travel in the kernel's parameter block).
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace mak {

constexpr int kRowPlanes = 128;  // planes per launch (parameter block < 4 KB)
constexpr int kRowGroups = 4;    // plane geometries per side and launch

struct RowSide {
  int64_t rows_per_block;
  int64_t block_stride;  // bytes
  int64_t row_stride;    // bytes
  int64_t num_rows;      // valid rows are [0, num_rows)
  int32_t lg_rows;       // log2(rows_per_block) when it is a power of two, else -1
  int32_t pad;
};

static int log2_or_neg(int64_t x) {
  if (x <= 0 || (x & (x - 1)) != 0) return -1;
  int l = 0;
  while ((int64_t{1} << l) < x) ++l;
  return l;
}

struct RowLaunch {
  uint64_t src[kRowPlanes];
  uint64_t dst[kRowPlanes];
  int32_t row_bytes[kRowPlanes];
  uint8_t sg[kRowPlanes];  // geometry of each plane on the source side
  uint8_t dg[kRowPlanes];  // ... and on the destination side
  RowSide s[kRowGroups], d[kRowGroups];
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
  uint8_t lgchunk[kRowPlanes];  // log2 of each plane's chunk length (items per warp chunk, <= 32)
  // Owner-table mode (dst_idx set): item i writes only while owner[dst] == tag_hi | i.
  const unsigned long long* owner;
  int64_t owner_rows;
  uint64_t tag_hi;
};
static_assert(sizeof(RowLaunch) <= 4096, "row launch parameters must fit the classic 4 KB parameter block");

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
  if (s.lg_rows >= 0) return (r >> s.lg_rows) * s.block_stride + (r & (s.rows_per_block - 1)) * s.row_stride;
  int64_t b, o;
  split_slot(r, s.rows_per_block, &b, &o);
  return b * s.block_stride + o * s.row_stride;
}

constexpr int kRowChunk = 32;       // largest chunk: one item per lane
constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;

// Raw destination / source row of item i (range checks come later); -1 = none.
__device__ __forceinline__ void fetch_item(const RowLaunch& p, int64_t i, bool live, int64_t* dr, int64_t* sr) {
  *dr = -1;
  *sr = -1;
  if (!live) return;
  const bool indexed = i < p.n_items;
  if (p.dst_idx != nullptr) {
    if (indexed) {
      *dr = load_index(p.dst_idx, p.dst_idx64, i);
      if (p.owner != nullptr) {
        const int64_t r = *dr;
        const bool own = r >= 0 && r < p.owner_rows && __ldcg(p.owner + r) == (p.tag_hi | static_cast<uint64_t>(i));
        *dr = own ? r : -1;
      }
    }
  } else {
    *dr = i + p.dst_base;
  }
  if (indexed) *sr = (p.src_idx != nullptr) ? load_index(p.src_idx, p.src_idx64, i) : i + p.src_base;
}

// grid = (x, planes of this launch): block (bx, plane) walks the plane's chunks
// bx*8 + warp, stepping by gridDim.x*8, so no division maps work to rows.
template <int VEC>
__global__ void __launch_bounds__(kRowThreads) rows_kernel(const __grid_constant__ RowLaunch p) {
  using V = typename VecT<VEC>::T;
  constexpr int U = (VEC >= 8) ? 4 : 8;  // independent vectors in flight per lane
  __shared__ int64_t s_src[kRowWarps][kRowChunk];  // source byte offset, -1 = zero row
  __shared__ int64_t s_dst[kRowWarps][kRowChunk];  // destination byte offset, -1 = skip
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int plane = blockIdx.y;
  const int nv = p.row_bytes[plane] / VEC;  // vectors per row
  if (nv <= 0) return;
  const int lgc = p.lgchunk[plane];
  const int chunk = 1 << lgc;
  const int64_t nch = (p.n_total + chunk - 1) >> lgc;
  const RowSide& S = p.s[p.sg[plane]];
  const RowSide& D = p.d[p.dg[plane]];
  const unsigned char* srcb = reinterpret_cast<const unsigned char*>(p.src[plane]);
  unsigned char* dstb = reinterpret_cast<unsigned char*>(p.dst[plane]);
  // Streaming shape: L = 2^lg lanes per row, 32/L rows per warp pass, kv vectors per lane and row.
  const int lg = nv >= 32 ? 5 : 32 - __clz(nv - 1);
  const int sub = lane >> lg;
  const int lv = lane & ((1 << lg) - 1);
  const int kv = (nv + (1 << lg) - 1) >> lg;
  const bool whole_batches = lg == 5 && (kv % U) == 0;  // each batch stays inside one row
  const int64_t step = static_cast<int64_t>(gridDim.x) * kRowWarps;
  int64_t cx = static_cast<int64_t>(blockIdx.x) * kRowWarps + wib;
  // The next chunk's index loads are issued before the current chunk's rows
  // stream, so the index latency hides behind the row traffic.
  int64_t next_dr, next_sr;
  {
    const int64_t i = (cx << lgc) + lane;
    fetch_item(p, i, cx < nch && lane < chunk && i < p.n_total, &next_dr, &next_sr);
  }
  for (; cx < nch; cx += step) {
    const int64_t i0 = cx << lgc;
    const int64_t dr = next_dr, sr = next_sr;
    {
      const int64_t i = ((cx + step) << lgc) + lane;
      fetch_item(p, i, cx + step < nch && lane < chunk && i < p.n_total, &next_dr, &next_sr);
    }
    // ---- resolve this lane's item --------------------------------------------------
    int64_t so = -1, dof = -1;
    if (dr >= 0 && dr < D.num_rows) {
      if (sr >= 0 && sr < S.num_rows) {
        so = row_offset(S, sr);
        dof = row_offset(D, dr);
      } else if (p.zero_fill) {
        dof = row_offset(D, dr);
      }
    }
    __syncwarp();  // the previous chunk's readers are done with the slots
    s_src[wib][lane] = so;
    s_dst[wib][lane] = dof;
    __syncwarp();
    // ---- stream the chunk's rows -----------------------------------------------------
    const int64_t left = p.n_total - i0;
    const int nitems = left < chunk ? static_cast<int>(left) : chunk;
    if (whole_batches) {
      for (int j = 0; j < nitems; ++j) {
        const int64_t d = s_dst[wib][j];
        if (d < 0) continue;
        const int64_t sb = s_src[wib][j];
        const V* src = reinterpret_cast<const V*>(srcb + sb);
        V* dst = reinterpret_cast<V*>(dstb + d);
        for (int v0 = lv; v0 < 32 * kv; v0 += 32 * U) {
          V r[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int v = v0 + 32 * u;
            if (v < nv) {
              if (sb >= 0) {
                r[u] = src[v];
              } else {
                memset(&r[u], 0, sizeof(V));
              }
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int v = v0 + 32 * u;
            if (v < nv) dst[v] = r[u];
          }
        }
      }
      continue;
    }
    // General shape: lane (sub, lv) walks rows j = sub, sub + 32/L, ... and in each
    // row the vectors lv, lv + L, ...; a row's two offsets are read from shared
    // memory once, and U vectors (possibly from consecutive rows) stay in flight.
    const int rows_step = 32 >> lg;
    int j = sub, k = 0;
    bool live = false, zero = false;
    const V* sp = nullptr;
    V* dp = nullptr;
    if (j < nitems) {
      const int64_t d = s_dst[wib][j];
      const int64_t sb = s_src[wib][j];
      live = d >= 0;
      zero = sb < 0;
      dp = reinterpret_cast<V*>(dstb + d);
      sp = reinterpret_cast<const V*>(srcb + sb);
    }
    while (j < nitems) {
      V r[U];
      V* at[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        at[u] = nullptr;
        if (j < nitems) {
          const int v = lv + (k << lg);
          if (live && v < nv) {
            at[u] = dp + v;
            if (zero) {
              memset(&r[u], 0, sizeof(V));
            } else {
              r[u] = sp[v];
            }
          }
          if (++k == kv) {
            k = 0;
            j += rows_step;
            live = false;
            if (j < nitems) {
              const int64_t d = s_dst[wib][j];
              const int64_t sb = s_src[wib][j];
              live = d >= 0;
              zero = sb < 0;
              dp = reinterpret_cast<V*>(dstb + d);
              sp = reinterpret_cast<const V*>(srcb + sb);
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (at[u] != nullptr) *at[u] = r[u];
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
  // x extent: enough warps for the plane with the most chunks, capped at 4 to 16
  // resident waves of blocks across all planes of the launch: about one block per
  // 64 KiB of the launch's rows (read side).  Blocks of a large call then stay
  // short, so the last wave drains quickly (cfg2 6326 -> 6553 GB/s against a fixed
  // four waves, SGLang MP per request 6262 -> 6409, 61-layer MLA per request 5946
  // -> 6299); small calls keep four waves, where more blocks of little work each
  // measured slower (8-layer MLA per request 4990 -> 4430 at sixteen).
  int64_t max_chunks = 0;
  for (int q = 0; q < p.num_planes; ++q) {
    const int64_t ch = (p.n_total + (int64_t{1} << p.lgchunk[q]) - 1) >> p.lgchunk[q];
    max_chunks = std::max(max_chunks, ch);
  }
  if (max_chunks == 0 || p.num_planes == 0) return MAK_OK;
  const int64_t resident_blocks =
      static_cast<int64_t>(blocks_per_sm(reinterpret_cast<const void*>(rows_kernel<VEC>), kRowThreads, 0)) * sm_count();
  const int64_t want = (max_chunks + kRowWarps - 1) / kRowWarps;
  int64_t call_bytes = 0;
  for (int q = 0; q < p.num_planes; ++q) call_bytes += static_cast<int64_t>(p.row_bytes[q]) * p.n_total;
  const int64_t waves = std::min<int64_t>(16, std::max<int64_t>(4, call_bytes / (resident_blocks * (int64_t{64} << 10))));
  const int64_t cap = std::max<int64_t>(1, (waves * resident_blocks + p.num_planes - 1) / p.num_planes);
  const dim3 grid(static_cast<unsigned>(std::min(want, cap)), static_cast<unsigned>(p.num_planes));
  return launch_pdl("rows_kernel", rows_kernel<VEC>, grid, dim3(kRowThreads), 0, st, p);
}

struct RowCall {
  const mak_rows_desc* src;  // n_groups descriptors per side; group g's planes follow group g-1's
  const mak_rows_desc* dst;
  int32_t n_groups;
  const int64_t* row_bytes;  // per plane (NULL -> group_row_bytes / row_bytes0)
  const int64_t* group_row_bytes;  // per group (NULL -> row_bytes0)
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
  const unsigned long long* owner;  // owner-table last-writer mode (see mak_rows_scatterv_owned)
  int64_t owner_rows;
  uint64_t tag_hi;
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
  if (c.n_groups < 1 || c.n_groups > kRowGroups)
    return fail(MAK_E_INVALID, "%s: %d plane groups (1..%d supported)", name, c.n_groups, kRowGroups);
  if (c.src == nullptr || c.dst == nullptr) return fail(MAK_E_INVALID, "%s: row descriptor is NULL", name);
  int64_t planes = 0;
  for (int g = 0; g < c.n_groups; ++g) {
    int rc = check_side(c.src + g, name);
    if (rc) return rc;
    rc = check_side(c.dst + g, name);
    if (rc) return rc;
    if (c.src[g].num_planes != c.dst[g].num_planes)
      return fail(MAK_E_INVALID, "%s: group %d: source has %lld planes, destination %lld", name, g,
                  (long long)c.src[g].num_planes, (long long)c.dst[g].num_planes);
    planes += c.src[g].num_planes;
  }
  if (planes > MAK_MAX_PLANES) return fail(MAK_E_INVALID, "%s: %lld planes exceed %d", name, (long long)planes, MAK_MAX_PLANES);
  if ((c.src_idx && !valid_index_dtype(c.src_idx_dtype)) || (c.dst_idx && !valid_index_dtype(c.dst_idx_dtype)))
    return fail(MAK_E_INVALID, "%s: index dtype must be int32 or int64", name);
  if (c.n_items < 0 || c.n_total < c.n_items) return fail(MAK_E_INVALID, "%s: bad item counts", name);
  if (planes == 0 || c.n_total == 0) return MAK_OK;
  // Flatten (group, plane) -> global plane list.
  struct PlaneRef {
    uint64_t src, dst;
    int64_t rb;
    uint8_t g;
  };
  std::vector<PlaneRef> all;
  all.reserve(static_cast<size_t>(planes));
  // Vector width: the largest power of two (<= 16) dividing every address, stride and row width.
  uint64_t bits = 0;
  for (int g = 0; g < c.n_groups; ++g) {
    const mak_rows_desc& S = c.src[g];
    const mak_rows_desc& D = c.dst[g];
    bits |= static_cast<uint64_t>(S.block_stride) | static_cast<uint64_t>(D.block_stride);
    if (S.rows_per_block > 1) bits |= static_cast<uint64_t>(S.row_stride);
    if (D.rows_per_block > 1) bits |= static_cast<uint64_t>(D.row_stride);
    for (int64_t q = 0; q < S.num_planes; ++q) {
      const int64_t idx = static_cast<int64_t>(all.size());
      const int64_t rb = c.row_bytes ? c.row_bytes[idx] : (c.group_row_bytes ? c.group_row_bytes[g] : c.row_bytes0);
      if (rb < 0 || rb > (int64_t)0x7fffffff) return fail(MAK_E_INVALID, "%s: bad row width %lld", name, (long long)rb);
      bits |= static_cast<uint64_t>(rb) | S.plane_ptrs[q] | D.plane_ptrs[q];
      all.push_back(PlaneRef{S.plane_ptrs[q], D.plane_ptrs[q], rb, static_cast<uint8_t>(g)});
    }
  }
  const int vec = vec_width(bits);
  // Chunk length per group: target ~1/8 of a resident warp's share of the call's
  // bytes (clamped to [2 KB, 64 KB]: at least one full batch of U 16-byte
  // vectors per lane), as whole rows of the group's widest plane.
  int64_t max_rb[kRowGroups] = {1, 1, 1, 1};
  int64_t bytes = 0;
  for (const PlaneRef& r : all) {
    max_rb[r.g] = std::max<int64_t>(max_rb[r.g], r.rb);
    bytes += r.rb * c.n_total;
  }
  const int64_t resident_warps =
      static_cast<int64_t>(blocks_per_sm(reinterpret_cast<const void*>(rows_kernel<16>), kRowThreads, 0)) * sm_count() *
      kRowWarps;
  const int64_t target = std::min<int64_t>(64 * 1024, std::max<int64_t>(2048, bytes / (8 * resident_warps)));
  int glg[kRowGroups];
  for (int g = 0; g < kRowGroups; ++g) {
    int lgc = 5;
    while (lgc > 0 && (int64_t{1} << lgc) * max_rb[g] > target) --lgc;
    glg[g] = lgc;
  }
  int rc = MAK_OK;
  for (int64_t p0 = 0; p0 < planes; p0 += kRowPlanes) {
    RowLaunch L;
    memset(&L, 0, sizeof(L));
    const int64_t np = std::min<int64_t>(kRowPlanes, planes - p0);
    for (int64_t q = 0; q < np; ++q) {
      const PlaneRef& r = all[static_cast<size_t>(p0 + q)];
      L.src[q] = r.src;
      L.dst[q] = r.dst;
      L.row_bytes[q] = static_cast<int32_t>(r.rb);
      L.sg[q] = r.g;
      L.dg[q] = r.g;
    }
    for (int g = 0; g < c.n_groups; ++g) {
      L.s[g] = RowSide{c.src[g].rows_per_block, c.src[g].block_stride, c.src[g].row_stride, c.src[g].num_rows,
                       log2_or_neg(c.src[g].rows_per_block), 0};
      L.d[g] = RowSide{c.dst[g].rows_per_block, c.dst[g].block_stride, c.dst[g].row_stride, c.dst[g].num_rows,
                       log2_or_neg(c.dst[g].rows_per_block), 0};
    }
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
    L.owner = c.owner;
    L.owner_rows = c.owner_rows;
    L.tag_hi = c.tag_hi;
    for (int64_t q = 0; q < np; ++q) L.lgchunk[q] = static_cast<uint8_t>(glg[L.sg[q]]);
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
  return mak_rows_gatherv(paged, linear, 1, row_bytes, row_bytes0, slots, slot_dtype, n_slots, fill_zero, stream);
}

int mak_rows_gatherv(const mak_rows_desc* paged, const mak_rows_desc* linear, int32_t n_groups, const int64_t* row_bytes,
                     int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots, int32_t fill_zero,
                     void* stream) {
  if (n_slots < 0 || (n_slots > 0 && slots == nullptr)) return fail(MAK_E_INVALID, "mak_rows_gather: bad slot vector");
  if (n_slots > 0 && !valid_index_dtype(slot_dtype)) return fail(MAK_E_INVALID, "mak_rows_gather: slot dtype must be int32 or int64");
  if (linear == nullptr || n_groups < 1) return fail(MAK_E_INVALID, "mak_rows_gather: linear descriptor is NULL");
  int64_t rows = 0;
  for (int g = 0; g < n_groups && g < kRowGroups; ++g) rows = std::max<int64_t>(rows, linear[g].num_rows);
  RowCall c{};
  c.src = paged;
  c.dst = linear;
  c.n_groups = n_groups;
  c.group_row_bytes = n_groups > 1 ? row_bytes : nullptr;
  c.row_bytes = n_groups > 1 ? nullptr : row_bytes;
  c.row_bytes0 = row_bytes0;
  c.src_idx = slots;
  c.src_idx_dtype = slot_dtype;
  c.n_items = std::min<int64_t>(n_slots, rows);
  c.n_total = fill_zero ? rows : c.n_items;
  c.zero_fill = fill_zero ? 1 : 0;
  return run_rows(c, as_stream(stream), "mak_rows_gather");
}

int mak_rows_scatter(const mak_rows_desc* linear, const mak_rows_desc* paged, const int64_t* row_bytes,
                     int64_t row_bytes0, const void* slots, int32_t slot_dtype, int64_t n_slots, int64_t skip_prefix,
                     void* workspace, size_t workspace_bytes, void* stream) {
  return mak_rows_scatterv(linear, paged, 1, row_bytes, row_bytes0, slots, slot_dtype, n_slots, skip_prefix, workspace,
                           workspace_bytes, stream);
}

int mak_rows_scatterv(const mak_rows_desc* linear, const mak_rows_desc* paged, int32_t n_groups, const int64_t* row_bytes,
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
  c.n_groups = n_groups;
  c.group_row_bytes = n_groups > 1 ? row_bytes : nullptr;
  c.row_bytes = n_groups > 1 ? nullptr : row_bytes;
  c.row_bytes0 = row_bytes0;
  c.dst_idx = ws.eff;
  c.dst_idx_dtype = MAK_DT_I64;
  c.n_items = n_slots;
  c.n_total = n_slots;
  c.src_base = skip_prefix;
  return run_rows(c, st, "mak_rows_scatter");
}

int mak_rows_scatterv_owned(const mak_rows_desc* linear, const mak_rows_desc* paged, int32_t n_groups,
                            const int64_t* row_bytes, int64_t row_bytes0, const void* slots, int32_t slot_dtype,
                            int64_t n_slots, int64_t skip_prefix, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                            void* stream) {
  const char* name = "mak_rows_scatterv_owned";
  if (n_slots < 0 || (n_slots > 0 && slots == nullptr)) return fail(MAK_E_INVALID, "%s: bad slot vector", name);
  if (n_slots == 0) return MAK_OK;
  if (!valid_index_dtype(slot_dtype)) return fail(MAK_E_INVALID, "%s: slot dtype must be int32 or int64", name);
  if (skip_prefix < 0) return fail(MAK_E_INVALID, "%s: skip_prefix must be non-negative", name);
  if (paged == nullptr || n_groups < 1 || n_groups > kRowGroups) return fail(MAK_E_INVALID, "%s: bad descriptors", name);
  for (int g = 0; g < n_groups; ++g)
    if (paged[g].num_rows > owner_rows)
      return fail(MAK_E_INVALID, "%s: owner table has %lld rows, group %d has %lld", name, (long long)owner_rows, g,
                  (long long)paged[g].num_rows);
  cudaStream_t st = as_stream(stream);
  int rc = mark_owners(slots, slot_dtype, n_slots, owner, owner_rows, epoch, st, name);
  if (rc) return rc;
  RowCall c{};
  c.src = linear;
  c.dst = paged;
  c.n_groups = n_groups;
  c.group_row_bytes = n_groups > 1 ? row_bytes : nullptr;
  c.row_bytes = n_groups > 1 ? nullptr : row_bytes;
  c.row_bytes0 = row_bytes0;
  c.dst_idx = slots;
  c.dst_idx_dtype = slot_dtype;
  c.n_items = n_slots;
  c.n_total = n_slots;
  c.src_base = skip_prefix;
  c.owner = reinterpret_cast<const unsigned long long*>(owner);
  c.owner_rows = owner_rows;
  c.tag_hi = static_cast<uint64_t>(epoch) << 32;
  return run_rows(c, st, name);
}

int mak_rows_copy_owned(const mak_rows_desc* src, const mak_rows_desc* dst, const int64_t* row_bytes,
                        int64_t row_bytes0, const void* src_idx, int32_t src_idx_dtype, const void* dst_idx,
                        int32_t dst_idx_dtype, int64_t n, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                        void* stream) {
  const char* name = "mak_rows_copy_owned";
  if (n < 0) return fail(MAK_E_INVALID, "%s: negative item count", name);
  if (n == 0) return MAK_OK;
  if (dst == nullptr) return fail(MAK_E_INVALID, "%s: row descriptor is NULL", name);
  if (dst_idx == nullptr || !valid_index_dtype(dst_idx_dtype))
    return fail(MAK_E_INVALID, "%s: needs an int32 or int64 destination index", name);
  if (dst->num_rows > owner_rows)
    return fail(MAK_E_INVALID, "%s: owner table has %lld rows, the destination %lld", name, (long long)owner_rows,
                (long long)dst->num_rows);
  cudaStream_t st = as_stream(stream);
  int rc = mark_owners(dst_idx, dst_idx_dtype, n, owner, owner_rows, epoch, st, name);
  if (rc) return rc;
  RowCall c{};
  c.src = src;
  c.dst = dst;
  c.n_groups = 1;
  c.row_bytes = row_bytes;
  c.row_bytes0 = row_bytes0;
  c.src_idx = src_idx;
  c.src_idx_dtype = src_idx_dtype;
  c.dst_idx = dst_idx;
  c.dst_idx_dtype = dst_idx_dtype;
  c.n_items = n;
  c.n_total = n;
  c.owner = reinterpret_cast<const unsigned long long*>(owner);
  c.owner_rows = owner_rows;
  c.tag_hi = static_cast<uint64_t>(epoch) << 32;
  return run_rows(c, st, name);
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
  c.n_groups = 1;
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
