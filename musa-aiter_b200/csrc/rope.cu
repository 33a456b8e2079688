// Rotary position embedding with the reference's per-operation rounding
// (musa_aiter/ops/cache.py:9-42): out1 = x1 * cos - x2 * sin,
// out2 = x1 * sin + x2 * cos.  Each product is formed in the promoted type of
// its two operands (operands are first cast to that type), the sum / difference
// in the promoted type of the two products, and the result is cast to x's
// dtype; f16 / bf16 steps are computed in fp32 and rounded to nearest-even
// after every operation, fp32 steps are single IEEE operations (no FMA
// contraction).  Dtype codes travel as runtime arguments.
//
// rope_dense_kernel: any x (up to 6 leading dims, strided) with cos / sin
// broadcast to x[..., :half]; writes a new contiguous output.
// rope_cache_kernel: in place on selected slots of a [NB][NH][HD][BS] key cache
// (musa_aiter/ops/cache.py:45-102), one warp per (32 tokens, 8 pairs, head group)
// with lane = token.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace mak {

__device__ __forceinline__ float ld_as_f32(const void* p, int64_t i, int dt) {
  if (dt == MAK_DT_F32) return static_cast<const float*>(p)[i];
  if (dt == MAK_DT_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ float round_to(float v, int dt) {
  if (dt == MAK_DT_F16) return __half2float(__float2half_rn(v));
  if (dt == MAK_DT_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

__device__ __forceinline__ void st_from_f32(void* p, int64_t i, int dt, float v) {
  if (dt == MAK_DT_F32) {
    static_cast<float*>(p)[i] = v;
  } else if (dt == MAK_DT_F16) {
    static_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
}

struct RopeTypes {
  int32_t x_dt, c_dt, s_dt;  // operand dtypes
  int32_t r1, r2, r3;        // x*cos / x*sin products, and their sum / difference
  int32_t out_dt;
  int32_t interleaved;
};

// (a1, a2) = rotated pair of (x1, x2) under (c, s), in the reference's rounding.
__device__ __forceinline__ void rotate(float x1, float x2, float c, float s, const RopeTypes& t, float* o1, float* o2) {
  const float p11 = round_to(__fmul_rn(round_to(x1, t.r1), round_to(c, t.r1)), t.r1);  // x1 * cos
  const float p22 = round_to(__fmul_rn(round_to(x2, t.r2), round_to(s, t.r2)), t.r2);  // x2 * sin
  const float p12 = round_to(__fmul_rn(round_to(x1, t.r2), round_to(s, t.r2)), t.r2);  // x1 * sin
  const float p21 = round_to(__fmul_rn(round_to(x2, t.r1), round_to(c, t.r1)), t.r1);  // x2 * cos
  *o1 = round_to(__fsub_rn(round_to(p11, t.r3), round_to(p22, t.r3)), t.r3);
  *o2 = round_to(__fadd_rn(round_to(p12, t.r3), round_to(p21, t.r3)), t.r3);
}

struct RopeDense {
  const void* x;
  const void* cos;
  const void* sin;
  void* out;
  int64_t rows;
  int64_t size[6];  // leading dims of the (broadcast) output
  int64_t xs[6], cs[6], ss[6];
  int64_t x_last, c_last, s_last;  // strides along the last dim (elements)
  int32_t nd;
  int32_t half;
  RopeTypes t;
};

__global__ void __launch_bounds__(256) rope_dense_kernel(const __grid_constant__ RopeDense p) {
  const int64_t total = p.rows * p.half;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t row = idx / p.half;
    const int j = static_cast<int>(idx - row * p.half);
    const int64_t out_row = row;
    int64_t xo = 0, co = 0, so = 0;
    for (int d = p.nd - 1; d >= 0; --d) {
      const int64_t q = row / p.size[d];
      const int64_t i = row - q * p.size[d];
      row = q;
      xo += i * p.xs[d];
      co += i * p.cs[d];
      so += i * p.ss[d];
    }
    const int64_t e1 = p.t.interleaved ? 2 * j : j;
    const int64_t e2 = p.t.interleaved ? 2 * j + 1 : j + p.half;
    const float x1 = ld_as_f32(p.x, xo + e1 * p.x_last, p.t.x_dt);
    const float x2 = ld_as_f32(p.x, xo + e2 * p.x_last, p.t.x_dt);
    const float c = ld_as_f32(p.cos, co + j * p.c_last, p.t.c_dt);
    const float s = ld_as_f32(p.sin, so + j * p.s_last, p.t.s_dt);
    float o1, o2;
    rotate(x1, x2, c, s, p.t, &o1, &o2);
    const int64_t ob = out_row * 2 * p.half;
    st_from_f32(p.out, ob + e1, p.t.out_dt, o1);
    st_from_f32(p.out, ob + e2, p.t.out_dt, o2);
  }
}

struct RopeCache {
  void* cache;
  const void* cos;
  const void* sin;
  const void* slots;
  const void* positions;
  int64_t n_tokens;
  int64_t num_blocks, num_heads, head_dim, block_size;
  int64_t sb, sh, sd;         // cache strides (elements); block offset stride 1
  int64_t c_row, c_last;      // cos strides (elements); c_row = 0 for a 1-D table
  int64_t s_row, s_last;
  int32_t slots64, pos64;
  int32_t heads_per_item;     // heads rotated by one warp item
  int32_t vec_tab;            // fp32 tables, unit last stride, rows and bases 16-byte aligned
  RopeTypes t;
};

constexpr int kRopeJ = 8;  // rotation pairs per warp item

// In the [NB][NH][HD][BS] cache one (block, head, dim) row holds the block's BS tokens
// side by side, so lanes = tokens makes the 16 tokens of a block-table block read and write
// one 32-byte sector per (head, dim) together (lanes = pairs touched a sector per element).
// A lane's cos / sin values for its item's pairs are loaded once and serve every head of the
// group; a head's 2 x 8 elements are loaded before any is stored.
template <typename X>
__device__ __forceinline__ float ld_x(const void* p, int64_t i) {
  if constexpr (sizeof(X) == 4) return static_cast<const float*>(p)[i];
  else if constexpr (std::is_same_v<X, __half>) return __half2float(static_cast<const __half*>(p)[i]);
  else return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

template <typename X>
__device__ __forceinline__ void st_x(void* p, int64_t i, float v) {
  if constexpr (sizeof(X) == 4) static_cast<float*>(p)[i] = v;
  else if constexpr (std::is_same_v<X, __half>) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// X = the cache dtype (also the output dtype); table dtypes stay runtime codes.  F32 = every
// product and sum is promoted to fp32 (a 16-bit cache with an fp32 table, or an fp32 cache), so
// the rotation is four single fp32 products and a sum / difference; otherwise the promotions are
// runtime codes.
template <typename X, bool F32>
__global__ void __launch_bounds__(256, F32 ? 3 : 2) rope_cache_kernel(const __grid_constant__ RopeCache p) {
  const int half = static_cast<int>(p.head_dim / 2);
  const int lane = threadIdx.x & 31;
  const int64_t groups = (p.n_tokens + 31) / 32;
  const int64_t chunks = (half + kRopeJ - 1) / kRopeJ;
  const int64_t hgroups = (p.num_heads + p.heads_per_item - 1) / p.heads_per_item;
  const int64_t items = groups * chunks * hgroups;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  pdl_wait();
  pdl_trigger();
  for (int64_t it = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; it < items; it += nwarps) {
    // head groups fastest: the warps sharing a (token group, pair chunk) share its cos / sin rows
    const int64_t hg = it % hgroups;
    const int64_t rest = it / hgroups;
    const int j0 = static_cast<int>(rest % chunks) * kRopeJ;
    const int64_t tok = (rest / chunks) * 32 + lane;
    if (tok >= p.n_tokens) continue;
    const int64_t slot = load_index(p.slots, p.slots64, tok);
    if (slot < 0) continue;
    int64_t b, o;
    split_slot(slot, p.block_size, &b, &o);
    if (b >= p.num_blocks) continue;  // rejected by the host check unless validation is off
    const int64_t pos = load_index(p.positions, p.pos64, tok);
    if (pos < 0) continue;  // rejected by the host check unless validation is off
    const int nj = min(kRopeJ, half - j0);
    float cs[kRopeJ], sn[kRopeJ];
    // element offsets of pair j0 + q: first at (e0 + q * es) * sd, second one stride further
    const int64_t es = p.t.interleaved ? 2 : 1;
    const int64_t e0 = p.t.interleaved ? 2 * j0 : j0;
    const int64_t gap = (p.t.interleaved ? 1 : half) * p.sd;
    if (p.vec_tab && nj == kRopeJ) {
      // the lane's 8 pairs are 32 contiguous bytes of its token's row: two 16-byte loads a table
      const float4* cr = reinterpret_cast<const float4*>(static_cast<const float*>(p.cos) + pos * p.c_row + j0);
      const float4* sr = reinterpret_cast<const float4*>(static_cast<const float*>(p.sin) + pos * p.s_row + j0);
#pragma unroll
      for (int v = 0; v < kRopeJ / 4; ++v) {
        const float4 c4 = __ldg(cr + v), s4 = __ldg(sr + v);
        cs[4 * v] = c4.x, cs[4 * v + 1] = c4.y, cs[4 * v + 2] = c4.z, cs[4 * v + 3] = c4.w;
        sn[4 * v] = s4.x, sn[4 * v + 1] = s4.y, sn[4 * v + 2] = s4.z, sn[4 * v + 3] = s4.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < kRopeJ; ++q) {
        const int j = j0 + q;
        cs[q] = sn[q] = 0.f;
        if (q < nj) {
          cs[q] = ld_as_f32(p.cos, pos * p.c_row + j * p.c_last, p.t.c_dt);
          sn[q] = ld_as_f32(p.sin, pos * p.s_row + j * p.s_last, p.t.s_dt);
        }
      }
    }
    const int64_t h0 = hg * p.heads_per_item;
    const int64_t h1 = min(h0 + p.heads_per_item, p.num_heads);
    for (int64_t h = h0; h < h1; ++h) {
      const int64_t ba = b * p.sb + h * p.sh + o + e0 * p.sd;
      const int64_t step = es * p.sd;
      float x1[kRopeJ], x2[kRopeJ];
#pragma unroll
      for (int q = 0; q < kRopeJ; ++q) {
        x1[q] = x2[q] = 0.f;
        if (q < nj) {
          x1[q] = ld_x<X>(p.cache, ba + q * step);
          x2[q] = ld_x<X>(p.cache, ba + q * step + gap);
        }
      }
#pragma unroll
      for (int q = 0; q < kRopeJ; ++q) {
        if (q < nj) {
          float o1, o2;
          if constexpr (F32) {
            o1 = __fsub_rn(__fmul_rn(x1[q], cs[q]), __fmul_rn(x2[q], sn[q]));
            o2 = __fadd_rn(__fmul_rn(x1[q], sn[q]), __fmul_rn(x2[q], cs[q]));
          } else {
            rotate(x1[q], x2[q], cs[q], sn[q], p.t, &o1, &o2);
          }
          st_x<X>(p.cache, ba + q * step, o1);
          st_x<X>(p.cache, ba + q * step + gap, o2);
        }
      }
    }
  }
}

template <typename X, bool F32>
static int launch_rope_cache(RopeCache& p, cudaStream_t st) {
  const int threads = 256;
  auto kern = rope_cache_kernel<X, F32>;
  // Heads per warp item: all of them (cos / sin loaded once per token and pair: lanes read 32
  // different table rows, so the table loads cost as much L1 time as 8 heads of cache loads),
  // halved only while the items would not fill the resident warps once.
  const int64_t groups = (p.n_tokens + 31) / 32;
  const int64_t chunks = (p.head_dim / 2 + kRopeJ - 1) / kRopeJ;
  const int64_t resident_warps =
      static_cast<int64_t>(blocks_per_sm(reinterpret_cast<const void*>(kern), threads, 0)) * sm_count() * (threads / 32);
  int64_t hpi = p.num_heads;
  while (hpi > 1 && groups * chunks * ((p.num_heads + hpi - 1) / hpi) < resident_warps) hpi = (hpi + 1) / 2;
  p.heads_per_item = static_cast<int32_t>(std::min<int64_t>(hpi, 0x7fffffff));
  const auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  p.vec_tab = p.t.c_dt == MAK_DT_F32 && p.t.s_dt == MAK_DT_F32 && p.c_last == 1 && p.s_last == 1 &&
              p.c_row % 4 == 0 && p.s_row % 4 == 0 && al16(p.cos) && al16(p.sin);
  const int64_t items = groups * chunks * ((p.num_heads + hpi - 1) / hpi);
  const int grid = grid_for(reinterpret_cast<const void*>(kern), threads, 0, (items + 7) / 8);
  return launch_pdl("rope_cache_kernel", kern, dim3(grid), dim3(threads), 0, st, p);
}

static bool float_dt(int32_t dt) { return dt == MAK_DT_F16 || dt == MAK_DT_BF16 || dt == MAK_DT_F32; }

static int check_types(const RopeTypes& t, const char* name) {
  if (!float_dt(t.x_dt) || !float_dt(t.c_dt) || !float_dt(t.s_dt) || !float_dt(t.r1) || !float_dt(t.r2) ||
      !float_dt(t.r3) || !float_dt(t.out_dt))
    return fail(MAK_E_INVALID, "%s: dtypes must be float16, bfloat16 or float32", name);
  return MAK_OK;
}

}  // namespace mak

using namespace mak;

extern "C" {

int mak_rope_dense(const mak_rope_dense_desc* d, void* stream) {
  if (d == nullptr || d->x == nullptr || d->cos == nullptr || d->sin == nullptr || d->out == nullptr)
    return fail(MAK_E_INVALID, "mak_rope_dense: NULL argument");
  if (d->ndim < 0 || d->ndim > 6 || d->half <= 0 || d->rows < 0)
    return fail(MAK_E_INVALID, "mak_rope_dense: bad shape (ndim %d, half %lld)", d->ndim, (long long)d->half);
  RopeDense p;
  memset(&p, 0, sizeof(p));
  p.t = RopeTypes{d->x_dtype, d->cos_dtype, d->sin_dtype, d->prod1_dtype, d->prod2_dtype, d->sum_dtype,
                  d->out_dtype, d->interleaved ? 1 : 0};
  int rc = check_types(p.t, "mak_rope_dense");
  if (rc) return rc;
  p.x = d->x;
  p.cos = d->cos;
  p.sin = d->sin;
  p.out = d->out;
  p.rows = d->rows;
  p.nd = d->ndim;
  p.half = static_cast<int32_t>(d->half);
  for (int i = 0; i < d->ndim; ++i) {
    if (d->sizes[i] <= 0) return fail(MAK_E_INVALID, "mak_rope_dense: leading sizes must be positive");
    p.size[i] = d->sizes[i];
    p.xs[i] = d->x_strides[i];
    p.cs[i] = d->cos_strides[i];
    p.ss[i] = d->sin_strides[i];
  }
  p.x_last = d->x_strides[6];
  p.c_last = d->cos_strides[6];
  p.s_last = d->sin_strides[6];
  if (p.rows == 0) return MAK_OK;
  const int threads = 256;
  const int grid = grid_for(reinterpret_cast<const void*>(rope_dense_kernel), threads, 0,
                            (p.rows * p.half + threads - 1) / threads);
  rope_dense_kernel<<<grid, threads, 0, as_stream(stream)>>>(p);
  return launch_status("rope_dense_kernel");
}

int mak_rope_key_cache(const mak_rope_cache_desc* d, void* stream) {
  if (d == nullptr || d->cache == nullptr || d->cos == nullptr || d->sin == nullptr)
    return fail(MAK_E_INVALID, "mak_rope_key_cache: NULL argument");
  if (d->n_tokens < 0 || d->num_blocks <= 0 || d->num_heads <= 0 || d->head_dim <= 0 || d->head_dim % 2 ||
      d->block_size <= 0)
    return fail(MAK_E_INVALID, "mak_rope_key_cache: bad cache geometry");
  if (d->n_tokens > 0 && (d->slots == nullptr || d->positions == nullptr || !valid_index_dtype(d->slot_dtype) ||
                          !valid_index_dtype(d->pos_dtype)))
    return fail(MAK_E_INVALID, "mak_rope_key_cache: slots and positions must be int32 or int64 vectors");
  RopeCache p;
  memset(&p, 0, sizeof(p));
  p.t = RopeTypes{d->cache_dtype, d->cos_dtype, d->sin_dtype, d->prod1_dtype, d->prod2_dtype, d->sum_dtype,
                  d->cache_dtype, d->interleaved ? 1 : 0};
  int rc = check_types(p.t, "mak_rope_key_cache");
  if (rc) return rc;
  p.cache = d->cache;
  p.cos = d->cos;
  p.sin = d->sin;
  p.slots = d->slots;
  p.positions = d->positions;
  p.n_tokens = d->n_tokens;
  p.num_blocks = d->num_blocks;
  p.num_heads = d->num_heads;
  p.head_dim = d->head_dim;
  p.block_size = d->block_size;
  p.sb = d->stride_block;
  p.sh = d->stride_head;
  p.sd = d->stride_dim;
  p.c_row = d->cos_stride_row;
  p.c_last = d->cos_stride_last;
  p.s_row = d->sin_stride_row;
  p.s_last = d->sin_stride_last;
  p.slots64 = d->slot_dtype == MAK_DT_I64;
  p.pos64 = d->pos_dtype == MAK_DT_I64;
  if (p.n_tokens == 0) return MAK_OK;
  const bool f32 = p.t.r1 == MAK_DT_F32 && p.t.r2 == MAK_DT_F32 && p.t.r3 == MAK_DT_F32;
  cudaStream_t st = as_stream(stream);
  if (p.t.x_dt == MAK_DT_F32)
    return f32 ? launch_rope_cache<float, true>(p, st) : launch_rope_cache<float, false>(p, st);
  if (p.t.x_dt == MAK_DT_F16)
    return f32 ? launch_rope_cache<__half, true>(p, st) : launch_rope_cache<__half, false>(p, st);
  return f32 ? launch_rope_cache<__nv_bfloat16, true>(p, st) : launch_rope_cache<__nv_bfloat16, false>(p, st);
}

}  // extern "C"
