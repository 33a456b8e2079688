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
// (musa_aiter/ops/cache.py:45-102), one thread per (token, head, pair).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

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
  RopeTypes t;
};

__global__ void __launch_bounds__(256) rope_cache_kernel(const __grid_constant__ RopeCache p) {
  const int half = static_cast<int>(p.head_dim / 2);
  const int64_t per_token = p.num_heads * half;
  const int64_t total = p.n_tokens * per_token;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = idx / per_token;
    const int64_t r = idx - tok * per_token;
    const int64_t h = r / half;
    const int j = static_cast<int>(r - h * half);
    const int64_t slot = load_index(p.slots, p.slots64, tok);
    if (slot < 0) continue;
    int64_t b, o;
    split_slot(slot, p.block_size, &b, &o);
    if (b >= p.num_blocks) continue;  // rejected by the host check unless validation is off
    const int64_t pos = load_index(p.positions, p.pos64, tok);
    const int64_t base = b * p.sb + h * p.sh + o;
    const int64_t e1 = p.t.interleaved ? 2 * j : j;
    const int64_t e2 = p.t.interleaved ? 2 * j + 1 : j + half;
    const float x1 = ld_as_f32(p.cache, base + e1 * p.sd, p.t.x_dt);
    const float x2 = ld_as_f32(p.cache, base + e2 * p.sd, p.t.x_dt);
    const float c = ld_as_f32(p.cos, pos * p.c_row + j * p.c_last, p.t.c_dt);
    const float s = ld_as_f32(p.sin, pos * p.s_row + j * p.s_last, p.t.s_dt);
    float o1, o2;
    rotate(x1, x2, c, s, p.t, &o1, &o2);
    st_from_f32(p.cache, base + e1 * p.sd, p.t.out_dt, o1);
    st_from_f32(p.cache, base + e2 * p.sd, p.t.out_dt, o2);
  }
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
  const int threads = 256;
  const int64_t work = p.n_tokens * p.num_heads * (p.head_dim / 2);
  const int grid = grid_for(reinterpret_cast<const void*>(rope_cache_kernel), threads, 0, (work + threads - 1) / threads);
  rope_cache_kernel<<<grid, threads, 0, as_stream(stream)>>>(p);
  return launch_status("rope_cache_kernel");
}

}  // extern "C"
