// MLA FP8 rows with per-group scales: the latent part of a token (kv_dim
// values) is quantised in groups of 128 with scale = amax / fp8_max (amax over
// the group's finite values) and stored
// next to its scales and the unquantised rope part, one row per token and
// layer:  [kv_dim codes][kv_dim/128 fp32 scales][pe_dim rope elements].
//
// kv_dim 512 (the DeepSeek shape) with rope rows of at most 128 bytes takes the
// pair kernels: a warp moves two tokens at once, a half-warp per token and 32
// values per lane, so the per-token work that does not depend on the values
// (slot and owner lookups, address arithmetic, the group scale, the loop) is
// shared by two tokens; slots and offsets are 32-bit after one range check.
// The store keeps the next pair's inputs in registers; the load streams rows
// through a per-warp ring of shared-memory stages filled by cp.async, with the
// slots of 16 pairs fetched by one warp load.
//
// Other shapes: one warp per (token, layer): lane l owns E = kv_dim / 32
// consecutive values (16-byte loads), the group amax is a shuffle reduction
// over the 128 / E lanes of a group, the codes leave as one E-byte store per
// lane.  The element codec is the musa-aiter reference rule (fp8.cuh).
// grid = (token warps or pairs, layers).
#include <algorithm>

#include "common.cuh"
#include "fp8.cuh"

namespace mak {

constexpr int kMlaPlanes = 256;  // layers per launch
constexpr int kMlaThreads = 256;

struct MlaLaunch {
  uint64_t cache[kMlaPlanes];
  const unsigned char* kv;
  const unsigned char* pe;
  int64_t kv_sl, kv_st, pe_sl, pe_st;  // byte strides
  int64_t rows_per_block, block_stride, row_stride, num_rows;
  const void* idx;
  int64_t num_tokens;
  int32_t idx64;
  int32_t lg_rows;    // log2(rows_per_block) or -1
  int32_t kv_dim;
  int32_t pe_bytes;   // rope bytes per row (multiple of 8)
  // store, owner-table mode: token t writes only while owner[row] == tag_hi | t
  const unsigned long long* owner;
  uint64_t tag_hi;
};

__device__ __forceinline__ int64_t mla_row_offset(const MlaLaunch& p, int64_t r) {
  if (p.rows_per_block == 1) return r * p.block_stride;
  if (p.lg_rows >= 0) return (r >> p.lg_rows) * p.block_stride + (r & (p.rows_per_block - 1)) * p.row_stride;
  int64_t b, o;
  split_slot(r, p.rows_per_block, &b, &o);
  return b * p.block_stride + o * p.row_stride;
}

// 16-bit element <-> fp32 through raw bits (keeps values in registers).
template <typename T>
__device__ __forceinline__ float bits_to_f32(uint32_t u);
template <>
__device__ __forceinline__ float bits_to_f32<__nv_bfloat16>(uint32_t u) { return __uint_as_float(u << 16); }
template <>
__device__ __forceinline__ float bits_to_f32<__half>(uint32_t u) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(u)));
}
template <typename T>
__device__ __forceinline__ uint32_t f32_to_bits(float x) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x)));
}
template <>
__device__ __forceinline__ uint32_t f32_to_bits<__half>(float x) {
  return static_cast<uint32_t>(__half_as_ushort(__float2half_rn(x)));
}

// Two fp32 values -> two RNE 16-bit elements in one conversion (lo = a, hi = b).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int F>
__device__ __forceinline__ float fp8_max_of() {
  return F == MAK_FP8_E4M3 ? 448.f : 57344.f;
}

// E bytes (8, 16 or 32) from/to a row, 8- or 16-byte accesses.
template <int E>
struct Bytes {
  uint32_t w[E / 4];
};

template <int E>
__device__ __forceinline__ void store_bytes(unsigned char* dst, const Bytes<E>& b) {
  if (E == 8) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(b.w[0], b.w[1]);
  } else {
#pragma unroll
    for (int k = 0; k < E / 16; ++k)
      reinterpret_cast<uint4*>(dst)[k] = make_uint4(b.w[4 * k], b.w[4 * k + 1], b.w[4 * k + 2], b.w[4 * k + 3]);
  }
}

template <int E>
__device__ __forceinline__ Bytes<E> load_bytes(const unsigned char* src) {
  Bytes<E> b;
  if (E == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(src);
    b.w[0] = v.x;
    b.w[1] = v.y;
  } else {
#pragma unroll
    for (int k = 0; k < E / 16; ++k) {
      const uint4 v = reinterpret_cast<const uint4*>(src)[k];
      b.w[4 * k] = v.x;
      b.w[4 * k + 1] = v.y;
      b.w[4 * k + 2] = v.z;
      b.w[4 * k + 3] = v.w;
    }
  }
  return b;
}

// 16-bit pattern of +infinity: |raw| at or above it is inf or nan.
template <typename T>
constexpr uint32_t kInfBits = 0x7F80u;  // bfloat16
template <>
constexpr uint32_t kInfBits<__half> = 0x7C00u;

// Per-token inputs of the store, fetched one token ahead so the next token's
// loads are in flight while this one is encoded.
template <int E>
struct StoreIn {
  uint4 v[E / 8];   // this lane's latent values (raw 16-bit elements)
  uint2 pe[2];      // this lane's rope bytes (b = 8 * lane and 8 * lane + 256)
  int64_t dr;       // destination row
  unsigned long long own;  // owner-table entry of dr (owner mode)
};

template <int E>
__device__ __forceinline__ void store_fetch(const MlaLaunch& p, const unsigned char* kv_layer,
                                            const unsigned char* pe_layer, int64_t t, int lane, StoreIn<E>& s) {
  const uint4* src = reinterpret_cast<const uint4*>(kv_layer + t * p.kv_st + lane * E * 2);
#pragma unroll
  for (int k = 0; k < E / 8; ++k) s.v[k] = src[k];
  const unsigned char* pe_src = pe_layer + t * p.pe_st;
  const int b0 = lane * 8;
  s.pe[0] = b0 < p.pe_bytes ? *reinterpret_cast<const uint2*>(pe_src + b0) : make_uint2(0u, 0u);
  s.pe[1] = b0 + 256 < p.pe_bytes ? *reinterpret_cast<const uint2*>(pe_src + b0 + 256) : make_uint2(0u, 0u);
  s.dr = load_index(p.idx, p.idx64, t);
  s.own = 0;
}

template <int E>
__device__ __forceinline__ void store_fetch_owner(const MlaLaunch& p, StoreIn<E>& s) {
  if (p.owner != nullptr && s.dr >= 0 && s.dr < p.num_rows) s.own = __ldcg(p.owner + s.dr);
}

// Quantise and write one token of the store (inputs fetched by store_fetch).
template <typename T, int F, int E>
__device__ __forceinline__ void store_token(const MlaLaunch& p, unsigned char* plane, const StoreIn<E>& cur, int64_t t,
                                            int lane) {
  constexpr int kLanesPerGroup = 128 / E;
  float x[E];
#pragma unroll
  for (int k = 0; k < E / 8; ++k) {
    const uint32_t w[4] = {cur.v[k].x, cur.v[k].y, cur.v[k].z, cur.v[k].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[8 * k + 2 * j] = bits_to_f32<T>(w[j] & 0xFFFFu);
      x[8 * k + 2 * j + 1] = bits_to_f32<T>(w[j] >> 16);
    }
  }
  // amax over the finite values only (every stored scale is finite): the
  // magnitudes' 16-bit patterns order like the values, so a packed unsigned
  // max of |raw| finds the lane's largest; a non-finite one (pattern at or
  // above the format's infinity, rare) sends the lane to the exact loop.
  uint32_t m2 = 0;
#pragma unroll
  for (int k = 0; k < E / 8; ++k) {
    m2 = __vmaxu2(m2, cur.v[k].x & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, cur.v[k].y & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, cur.v[k].z & 0x7FFF7FFFu);
    m2 = __vmaxu2(m2, cur.v[k].w & 0x7FFF7FFFu);
  }
  const uint32_t mraw = max(m2 & 0xFFFFu, m2 >> 16);
  float amax = bits_to_f32<T>(mraw);
  const bool all_finite = mraw < kInfBits<T>;
  if (!all_finite) {
    amax = 0.f;
#pragma unroll
    for (int j = 0; j < E; ++j) {
      const float a = fabsf(x[j]);
      if (a <= 3.40282346638528859812e+38f) amax = fmaxf(amax, a);
    }
  }
#pragma unroll
  for (int o = 1; o < kLanesPerGroup; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(amax, fp8_max_of<F>());
  Bytes<E> codes;
  if (fast_quot_ok(scale) && all_finite) {
    // one reciprocal per group; per value three fp32 operations for the
    // quotient and two multiplies for the flush (fp8.cuh), no compares
    const QuotPair qc = quot_pair(scale, __frcp_rn(scale));
#pragma unroll
    for (int j = 0; j < E / 4; ++j)
      codes.w[j] = fp8_encode2_quot_finite<F>(x[4 * j], x[4 * j + 1], qc) |
                   (fp8_encode2_quot_finite<F>(x[4 * j + 2], x[4 * j + 3], qc) << 16);
  } else if (fast_quot_ok(scale)) {
    const float y = __frcp_rn(scale);
#pragma unroll
    for (int j = 0; j < E / 4; ++j) {
      const FastQuot a = fast_quot(x[4 * j], scale, y), b = fast_quot(x[4 * j + 1], scale, y);
      const FastQuot c = fast_quot(x[4 * j + 2], scale, y), d = fast_quot(x[4 * j + 3], scale, y);
      codes.w[j] = fp8_encode2s_bounded<F>(a.q0, a.q1, b.q0, b.q1) |
                   (fp8_encode2s_bounded<F>(c.q0, c.q1, d.q0, d.q1) << 16);
    }
  } else {
#pragma unroll
    for (int j = 0; j < E / 4; ++j) {
      const uint32_t lo = fp8_encode2<F>(__fdiv_rn(x[4 * j], scale), __fdiv_rn(x[4 * j + 1], scale));
      const uint32_t hi = fp8_encode2<F>(__fdiv_rn(x[4 * j + 2], scale), __fdiv_rn(x[4 * j + 3], scale));
      codes.w[j] = lo | (hi << 16);
    }
  }
  const bool write = cur.dr >= 0 && cur.dr < p.num_rows &&
                     (p.owner == nullptr || cur.own == (p.tag_hi | static_cast<uint64_t>(t)));
  if (write) {
    unsigned char* row = plane + mla_row_offset(p, cur.dr);
    store_bytes<E>(row + lane * E, codes);
    if ((lane % kLanesPerGroup) == 0) reinterpret_cast<float*>(row + p.kv_dim)[lane / kLanesPerGroup] = scale;
    unsigned char* rope = row + p.kv_dim + (p.kv_dim / 128) * 4;
    const int b0 = lane * 8;
    if (b0 < p.pe_bytes) *reinterpret_cast<uint2*>(rope + b0) = cur.pe[0];
    if (b0 + 256 < p.pe_bytes) *reinterpret_cast<uint2*>(rope + b0 + 256) = cur.pe[1];
  }
}

template <typename T, int F, int E>
__global__ void __launch_bounds__(kMlaThreads) mla_fp8_store_kernel(const __grid_constant__ MlaLaunch p) {
  const int lane = threadIdx.x & 31;
  const int layer = blockIdx.y;
  const int64_t step = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  unsigned char* plane = reinterpret_cast<unsigned char*>(p.cache[layer]);
  const unsigned char* kv_layer = p.kv + layer * p.kv_sl;
  const unsigned char* pe_layer = p.pe + layer * p.pe_sl;
  pdl_wait();
  pdl_trigger();
  int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= p.num_tokens) return;
  // Two input buffers used in turn (no register copies between tokens): the
  // next token's loads are in flight while this one is encoded.
  StoreIn<E> a, b;
  store_fetch<E>(p, kv_layer, pe_layer, t, lane, a);
  store_fetch_owner<E>(p, a);
  while (true) {
    int64_t tn = t + step;
    bool more = tn < p.num_tokens;  // warp-uniform: a warp works on one token
    if (more) store_fetch<E>(p, kv_layer, pe_layer, tn, lane, b);
    store_token<T, F, E>(p, plane, a, t, lane);
    if (!more) break;
    store_fetch_owner<E>(p, b);
    t = tn;
    tn = t + step;
    more = tn < p.num_tokens;
    if (more) store_fetch<E>(p, kv_layer, pe_layer, tn, lane, a);
    store_token<T, F, E>(p, plane, b, t, lane);
    if (!more) break;
    store_fetch_owner<E>(p, a);
    t = tn;
  }
}

// Per-token inputs of the load: the cache row's codes, group scale and rope
// bytes, fetched one token ahead (and the row index two tokens ahead).
template <int E>
struct LoadIn {
  Bytes<E> codes;
  float scale;
  uint2 pe[2];
  bool have;
};

template <int E>
__device__ __forceinline__ void load_fetch(const MlaLaunch& p, const unsigned char* plane, int64_t sr, int lane,
                                           LoadIn<E>& r) {
  constexpr int kLanesPerGroup = 128 / E;
  r.have = sr >= 0 && sr < p.num_rows;
  if (!r.have) return;
  const unsigned char* row = plane + mla_row_offset(p, sr);
  r.codes = load_bytes<E>(row + lane * E);
  r.scale = reinterpret_cast<const float*>(row + p.kv_dim)[lane / kLanesPerGroup];
  const unsigned char* rope = row + p.kv_dim + (p.kv_dim / 128) * 4;
  const int b0 = lane * 8;
  r.pe[0] = b0 < p.pe_bytes ? *reinterpret_cast<const uint2*>(rope + b0) : make_uint2(0u, 0u);
  r.pe[1] = b0 + 256 < p.pe_bytes ? *reinterpret_cast<const uint2*>(rope + b0 + 256) : make_uint2(0u, 0u);
}

template <typename T, int F, int E>
__global__ void __launch_bounds__(kMlaThreads) mla_fp8_load_kernel(const __grid_constant__ MlaLaunch p,
                                                                   unsigned char* kv_out, unsigned char* pe_out) {
  const int lane = threadIdx.x & 31;
  const int layer = blockIdx.y;
  const int64_t step = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const unsigned char* plane = reinterpret_cast<const unsigned char*>(p.cache[layer]);
  unsigned char* kv_layer = kv_out + layer * p.kv_sl;
  unsigned char* pe_layer = pe_out + layer * p.pe_sl;
  pdl_wait();
  pdl_trigger();
  int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (t >= p.num_tokens) return;
  LoadIn<E> cur;
  load_fetch<E>(p, plane, load_index(p.idx, p.idx64, t), lane, cur);
  int64_t sr_next = t + step < p.num_tokens ? load_index(p.idx, p.idx64, t + step) : -1;
  while (true) {
    const int64_t tn = t + step;
    const bool more = tn < p.num_tokens;
    LoadIn<E> nxt;
    if (more) load_fetch<E>(p, plane, sr_next, lane, nxt);
    if (tn + step < p.num_tokens) sr_next = load_index(p.idx, p.idx64, tn + step);
    uint4* dst = reinterpret_cast<uint4*>(kv_layer + t * p.kv_st + lane * E * 2);
    unsigned char* pe_dst = pe_layer + t * p.pe_st;
    const int b0 = lane * 8;
    if (cur.have && fp8_ftz_scale_ok<F>(cur.scale)) {
      // flush-to-zero decode (fp8.cuh): three integer operations and one multiply per code
      const float sf = __fmul_rn(cur.scale, fp8_ftz_bias<F>());  // exact: a power of two
      const uint64_t sf2 = f2_pack(sf, sf);
#pragma unroll
      for (int k = 0; k < E / 8; ++k) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // codes 2j, 2j+1 of word 2k + j/2 (bytes b, b + 1), each shifted to the top byte
          const uint32_t cw = cur.codes.w[2 * k + (j >> 1)];
          const uint32_t x0 = (j & 1) ? (cw << 8) : (cw << 24);
          const uint32_t x1 = (j & 1) ? cw : (cw << 16);
          float v0, v1;
          f2_unpack(f2_mul_ftz(f2_pack(fp8_raw_top<F>(x0), fp8_raw_top<F>(x1)), sf2), v0, v1);
          w[j] = pack2<T>(v0, v1);
        }
        dst[k] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (b0 < p.pe_bytes) *reinterpret_cast<uint2*>(pe_dst + b0) = cur.pe[0];
      if (b0 + 256 < p.pe_bytes) *reinterpret_cast<uint2*>(pe_dst + b0 + 256) = cur.pe[1];
    } else if (cur.have) {
#pragma unroll
      for (int k = 0; k < E / 8; ++k) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // codes 2j, 2j+1 of word 2k + j/2, each moved to the top byte
          const uint32_t cw = cur.codes.w[2 * k + (j >> 1)];
          const int b = 2 * (j & 1);
          const uint32_t x0 = __byte_perm(cw, 0u, 0x0444u | (b << 12));
          const uint32_t x1 = __byte_perm(cw, 0u, 0x0444u | ((b + 1) << 12));
          w[j] = pack2<T>(__fmul_rn(fp8_decode_top<F>(x0), cur.scale), __fmul_rn(fp8_decode_top<F>(x1), cur.scale));
        }
        dst[k] = make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (b0 < p.pe_bytes) *reinterpret_cast<uint2*>(pe_dst + b0) = cur.pe[0];
      if (b0 + 256 < p.pe_bytes) *reinterpret_cast<uint2*>(pe_dst + b0 + 256) = cur.pe[1];
    } else {
#pragma unroll
      for (int k = 0; k < E / 8; ++k) dst[k] = make_uint4(0u, 0u, 0u, 0u);
      if (b0 < p.pe_bytes) *reinterpret_cast<uint2*>(pe_dst + b0) = make_uint2(0u, 0u);
      if (b0 + 256 < p.pe_bytes) *reinterpret_cast<uint2*>(pe_dst + b0 + 256) = make_uint2(0u, 0u);
    }
    if (!more) break;
    cur = nxt;
    t = tn;
  }
}

// ---- pair kernels (kv_dim 512, rope rows of at most 128 bytes) --------------

// max(|a|, |b|) per 16-bit half with NaN propagation (the result's sign bits
// are not meaningful); a non-finite input leaves a magnitude at or above the
// format's infinity pattern.
template <typename T>
__device__ __forceinline__ uint32_t amax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <>
__device__ __forceinline__ uint32_t amax2<__half>(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// amax / fp8_max rounded to nearest in fp32 without a division: Markstein's
// correction step with the constant reciprocal (see fast_quot in fp8.cuh),
// exact for every finite 16-bit amax >= 2^-100 (mak_fp8_quotient_selfcheck
// compares it with the IEEE division for all of them); smaller ones divide.
template <int F>
__device__ __forceinline__ float group_scale(float amax) {
  constexpr float M = F == MAK_FP8_E4M3 ? 448.f : 57344.f;
  constexpr float Y = F == MAK_FP8_E4M3 ? (1.f / 448.f) : (1.f / 57344.f);
  if (amax >= 0x1p-100f) {
    const float q0 = __fmul_rn(amax, Y);
    return __fmaf_rn(__fmaf_rn(-q0, M, amax), Y, q0);
  }
  return __fdiv_rn(amax, M);
}

// Slot i as a row index below num_rows, or -1 (negative or out of range).
template <bool I64>
__device__ __forceinline__ int slot_row(const MlaLaunch& p, int64_t i) {
  const int64_t v = I64 ? static_cast<int64_t>(__ldg(reinterpret_cast<const long long*>(p.idx) + i))
                        : static_cast<int64_t>(__ldg(reinterpret_cast<const int*>(p.idx) + i));
  return (v >= 0 && v < p.num_rows) ? static_cast<int>(v) : -1;
}

// Row address from a row index (rows_per_block a power of two; block and row
// strides below 2^32 and rows below 2^31, checked on the host).
__device__ __forceinline__ unsigned char* row_at(const MlaLaunch& p, unsigned char* plane, int r) {
  const uint32_t b = static_cast<uint32_t>(r) >> p.lg_rows;
  const uint32_t o = static_cast<uint32_t>(r) & ((1u << p.lg_rows) - 1u);
  return plane + (static_cast<uint64_t>(b) * static_cast<uint32_t>(p.block_stride) +
                  static_cast<uint64_t>(o) * static_cast<uint32_t>(p.row_stride));
}

// Inputs of one token of a store pair, per lane: 32 values, 8 rope bytes.
struct PairIn {
  uint4 v[4];
  uint2 pe;
};

// Quantise one token (the calling half-warp's) and write its row.  Lane j of
// the half owns values [32j, 32j + 32): a 128-value group is 4 lanes.
template <typename T, int F, bool OWN>
__device__ __forceinline__ void pair_store_token(const MlaLaunch& p, unsigned char* plane, const PairIn& in, int row,
                                                 unsigned long long own, uint32_t epoch, int tt, int j) {
  const uint32_t wd[16] = {in.v[0].x, in.v[0].y, in.v[0].z, in.v[0].w, in.v[1].x, in.v[1].y, in.v[1].z, in.v[1].w,
                           in.v[2].x, in.v[2].y, in.v[2].z, in.v[2].w, in.v[3].x, in.v[3].y, in.v[3].z, in.v[3].w};
  uint32_t m8[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m8[i] = amax2<T>(wd[2 * i], wd[2 * i + 1]);
  uint32_t m = amax2<T>(amax2<T>(amax2<T>(m8[0], m8[1]), amax2<T>(m8[2], m8[3])),
                        amax2<T>(amax2<T>(m8[4], m8[5]), amax2<T>(m8[6], m8[7])));
  m &= 0x7FFF7FFFu;
  const uint32_t mraw = max(m & 0xFFFFu, m >> 16);
  const bool all_finite = mraw < kInfBits<T>;
  float amax = bits_to_f32<T>(mraw);
  if (!all_finite) {  // rare: the amax over this lane's finite values only
    amax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = fabsf(bits_to_f32<T>(wd[i] & 0xFFFFu)), b = fabsf(bits_to_f32<T>(wd[i] >> 16));
      if (a <= 3.40282346638528859812e+38f) amax = fmaxf(amax, a);
      if (b <= 3.40282346638528859812e+38f) amax = fmaxf(amax, b);
    }
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float scale = group_scale<F>(amax);
  uint32_t codes[8];
  if (fast_quot_ok(scale) && all_finite) {
    const QuotPair qc = quot_pair(scale, __frcp_rn(scale));
#pragma unroll
    for (int i = 0; i < 8; ++i)
      codes[i] = fp8_encode2_quot_finite<F>(bits_to_f32<T>(wd[2 * i] & 0xFFFFu), bits_to_f32<T>(wd[2 * i] >> 16), qc) |
                 (fp8_encode2_quot_finite<F>(bits_to_f32<T>(wd[2 * i + 1] & 0xFFFFu), bits_to_f32<T>(wd[2 * i + 1] >> 16),
                                             qc) << 16);
  } else if (fast_quot_ok(scale)) {
    const float y = __frcp_rn(scale);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const FastQuot a = fast_quot(bits_to_f32<T>(wd[2 * i] & 0xFFFFu), scale, y);
      const FastQuot b = fast_quot(bits_to_f32<T>(wd[2 * i] >> 16), scale, y);
      const FastQuot c = fast_quot(bits_to_f32<T>(wd[2 * i + 1] & 0xFFFFu), scale, y);
      const FastQuot d = fast_quot(bits_to_f32<T>(wd[2 * i + 1] >> 16), scale, y);
      codes[i] = fp8_encode2s_bounded<F>(a.q0, a.q1, b.q0, b.q1) | (fp8_encode2s_bounded<F>(c.q0, c.q1, d.q0, d.q1) << 16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = fp8_encode2<F>(__fdiv_rn(bits_to_f32<T>(wd[2 * i] & 0xFFFFu), scale),
                                         __fdiv_rn(bits_to_f32<T>(wd[2 * i] >> 16), scale));
      const uint32_t hi = fp8_encode2<F>(__fdiv_rn(bits_to_f32<T>(wd[2 * i + 1] & 0xFFFFu), scale),
                                         __fdiv_rn(bits_to_f32<T>(wd[2 * i + 1] >> 16), scale));
      codes[i] = lo | (hi << 16);
    }
  }
  const bool write = row >= 0 && (!OWN || (static_cast<uint32_t>(own >> 32) == epoch &&
                                            static_cast<uint32_t>(own) == static_cast<uint32_t>(tt)));
  if (write) {
    unsigned char* dst = row_at(p, plane, row);
    reinterpret_cast<uint4*>(dst + j * 32)[0] = make_uint4(codes[0], codes[1], codes[2], codes[3]);
    reinterpret_cast<uint4*>(dst + j * 32)[1] = make_uint4(codes[4], codes[5], codes[6], codes[7]);
    if ((j & 3) == 0) reinterpret_cast<float*>(dst + 512)[j >> 2] = scale;
    if (j * 8 < p.pe_bytes) *reinterpret_cast<uint2*>(dst + 528 + j * 8) = in.pe;
  }
}

// Store, two tokens per warp: tokens 2q and 2q + 1 of pair q (q = warp, warp +
// warps, ...); the next pair's inputs and slots load while this pair is
// encoded, its owner entries one pair ahead, slots two pairs ahead.
template <typename T, int F, bool OWN, bool I64>
__global__ void __launch_bounds__(256, 3) mla_fp8_store2_kernel(const __grid_constant__ MlaLaunch p) {
  const int lane = threadIdx.x & 31, hl = lane >> 4, j = lane & 15;
  const int layer = blockIdx.y;
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int n = static_cast<int>(p.num_tokens);
  const int npairs = (n + 1) >> 1;
  unsigned char* plane = reinterpret_cast<unsigned char*>(p.cache[layer]);
  pdl_wait();
  pdl_trigger();
  if (w >= npairs) return;
  const int tstep = 2 * nw;
  int t = 2 * w + hl;  // this half's token
  const unsigned char* kvp = p.kv + layer * p.kv_sl + j * 64 + static_cast<int64_t>(t) * p.kv_st;
  const unsigned char* pep = p.pe + layer * p.pe_sl + j * 8 + static_cast<int64_t>(t) * p.pe_st;
  const int64_t kv_inc = static_cast<int64_t>(tstep) * p.kv_st, pe_inc = static_cast<int64_t>(tstep) * p.pe_st;
  const bool pe_lane = j * 8 < p.pe_bytes;
  const uint32_t epoch = static_cast<uint32_t>(p.tag_hi >> 32);
  int64_t st = t;  // token whose slot loads next
  auto fetch = [&](int tt, PairIn& in) {
    if (tt < n) {
      const uint4* src = reinterpret_cast<const uint4*>(kvp);
      in.v[0] = src[0];
      in.v[1] = src[1];
      in.v[2] = src[2];
      in.v[3] = src[3];
      in.pe = pe_lane ? *reinterpret_cast<const uint2*>(pep) : make_uint2(0u, 0u);
    }
    kvp += kv_inc;
    pep += pe_inc;
  };
  auto next_slot = [&]() -> int {
    const int r = st < n ? slot_row<I64>(p, st) : -1;
    st += tstep;
    return r;
  };
  auto owner_of = [&](int r) -> unsigned long long { return (OWN && r >= 0) ? __ldcg(p.owner + r) : 0ull; };
  PairIn a, b;
  fetch(t, a);
  int r0 = next_slot(), r1 = next_slot();
  unsigned long long o0 = owner_of(r0);
  // Two input buffers used in turn (no register copies between pairs).
  while (true) {
    int tn = t + tstep;
    bool more = tn - hl < n;  // the next pair exists (warp-uniform)
    if (more) fetch(tn, b);
    unsigned long long o1 = owner_of(r1);
    int r2 = next_slot();
    pair_store_token<T, F, OWN>(p, plane, a, r0, o0, epoch, t, j);
    if (!more) break;
    t = tn;
    r0 = r1;
    r1 = r2;
    o0 = o1;
    tn = t + tstep;
    more = tn - hl < n;
    if (more) fetch(tn, a);
    o1 = owner_of(r1);
    r2 = next_slot();
    pair_store_token<T, F, OWN>(p, plane, b, r0, o0, epoch, t, j);
    if (!more) break;
    t = tn;
    r0 = r1;
    r1 = r2;
    o0 = o1;
  }
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 16 codes (one 16-byte chunk) of one group -> 16 elements (32 bytes) at dst.
template <typename T, int F>
__device__ __forceinline__ void decode_chunk16(uint4 c, float sc, bool have, uint4* dst) {
  const uint32_t cw4[4] = {c.x, c.y, c.z, c.w};
  if (have && fp8_ftz_scale_ok<F>(sc)) {
    const float sf = __fmul_rn(sc, fp8_ftz_bias<F>());  // exact: a power of two
    const uint64_t sf2 = f2_pack(sf, sf);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t cw = cw4[2 * h + (i >> 1)];
        const uint32_t x0 = (i & 1) ? (cw << 8) : (cw << 24);
        const uint32_t x1 = (i & 1) ? cw : (cw << 16);
        float v0, v1;
        f2_unpack(f2_mul_ftz(f2_pack(fp8_raw_top<F>(x0), fp8_raw_top<F>(x1)), sf2), v0, v1);
        o[i] = pack2<T>(v0, v1);
      }
      dst[h] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else if (have) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t cw = cw4[2 * h + (i >> 1)];
        const int b = 2 * (i & 1);
        const uint32_t x0 = __byte_perm(cw, 0u, 0x0444u | (b << 12));
        const uint32_t x1 = __byte_perm(cw, 0u, 0x0444u | ((b + 1) << 12));
        o[i] = pack2<T>(__fmul_rn(fp8_decode_top<F>(x0), sc), __fmul_rn(fp8_decode_top<F>(x1), sc));
      }
      dst[h] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  } else {
    dst[0] = make_uint4(0u, 0u, 0u, 0u);
    dst[1] = make_uint4(0u, 0u, 0u, 0u);
  }
}

constexpr int kMlaLoadStages = 4;  // ring stages per warp (a power of two)

// Load, two tokens per warp: each warp streams its pairs' cache rows through a
// ring of kMlaLoadStages shared-memory stages (cp.async, three stages in flight
// while one is decoded); a half-warp takes one row: lane j decodes codes
// [16j, 16j + 16) and [256 + 16j, 256 + 16j + 16) (conflict-free 16-byte shared
// reads), the group scales come from one broadcast read.  Slots of 16 pairs
// are loaded by one warp instruction, lane l holding pair l / 2, half l % 2.
// Dynamic shared memory: warps x stages x 2 x row_bytes.
template <typename T, int F, bool I64>
__global__ void __launch_bounds__(256) mla_fp8_load2_kernel(const __grid_constant__ MlaLaunch p, unsigned char* kv_out,
                                                            unsigned char* pe_out) {
  constexpr int D = kMlaLoadStages;
  extern __shared__ __align__(16) unsigned char mla_ring[];
  const int lane = threadIdx.x & 31, hl = lane >> 4, j = lane & 15, wid = threadIdx.x >> 5;
  const int rb = 528 + p.pe_bytes;  // row bytes, a multiple of 16
  const int stage = 2 * rb;
  unsigned char* my = mla_ring + wid * (D * stage) + hl * rb;
  const int layer = blockIdx.y;
  const int nw = gridDim.x * (blockDim.x >> 5);
  const int w = blockIdx.x * (blockDim.x >> 5) + wid;
  const int n = static_cast<int>(p.num_tokens);
  const int npairs = (n + 1) >> 1;
  unsigned char* plane = reinterpret_cast<unsigned char*>(p.cache[layer]);
  pdl_wait();
  pdl_trigger();
  if (w >= npairs) return;
  const int n_my = (npairs - 1 - w) / nw + 1;  // pairs of this warp
  const int tail_chunks = rb / 16 - 32;         // chunks of a row beyond the first 512 bytes
  auto slot_batch = [&](int kb) -> int {
    const int k = kb + (lane >> 1);
    const int tt = 2 * (w + k * nw) + (lane & 1);
    return (k < n_my && tt < n) ? slot_row<I64>(p, tt) : -1;
  };
  int cur = slot_batch(0), nxt = slot_batch(16);
  uint32_t have = 0;  // bit i: the row of pair k + i (this half) was fetched
  auto issue = [&](int ki, int bit) {
    const int r = __shfl_sync(0xffffffffu, cur, 2 * (ki & 15) + hl);
    if (ki < n_my && r >= 0) {
      const unsigned char* src = row_at(p, plane, r) + j * 16;
      unsigned char* dst = my + (ki & (D - 1)) * stage + j * 16;
      cp_async16(dst, src);
      cp_async16(dst + 256, src + 256);
      if (j < tail_chunks) cp_async16(dst + 512, src + 512);
      have |= 1u << bit;
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < D - 1; ++i) issue(i, i);
  int t = 2 * w + hl;
  unsigned char* kvo = kv_out + layer * p.kv_sl + j * 32 + static_cast<int64_t>(t) * p.kv_st;
  unsigned char* peo = pe_out + layer * p.pe_sl + j * 8 + static_cast<int64_t>(t) * p.pe_st;
  const int64_t kvo_inc = static_cast<int64_t>(2 * nw) * p.kv_st, peo_inc = static_cast<int64_t>(2 * nw) * p.pe_st;
  const bool pe_lane = j * 8 < p.pe_bytes;
  for (int k = 0; k < n_my; ++k) {
    const int ki = k + D - 1;
    if ((ki & 15) == 0) {
      cur = nxt;
      nxt = slot_batch(ki + 16);
    }
    issue(ki, D - 1);
    cp_async_wait<D - 1>();
    __syncwarp();
    const unsigned char* rs = my + (k & (D - 1)) * stage;
    const bool ok = have & 1u;
    have >>= 1;
    uint4 c0 = make_uint4(0u, 0u, 0u, 0u), c1 = c0;
    float4 sc = make_float4(0.f, 0.f, 0.f, 0.f);
    uint2 pev = make_uint2(0u, 0u);
    if (ok) {
      c0 = *reinterpret_cast<const uint4*>(rs + j * 16);
      c1 = *reinterpret_cast<const uint4*>(rs + 256 + j * 16);
      sc = *reinterpret_cast<const float4*>(rs + 512);
      if (pe_lane) pev = *reinterpret_cast<const uint2*>(rs + 528 + j * 8);
    }
    __syncwarp();  // the stage is refilled by the next iteration's issue
    if (t < n) {
      const bool g1 = j >= 8;  // chunk j lies in group j / 8, chunk j + 16 in group 2 + j / 8
      decode_chunk16<T, F>(c0, g1 ? sc.y : sc.x, ok, reinterpret_cast<uint4*>(kvo));
      decode_chunk16<T, F>(c1, g1 ? sc.w : sc.z, ok, reinterpret_cast<uint4*>(kvo + 512));
      if (pe_lane) *reinterpret_cast<uint2*>(peo) = pev;
    }
    t += 2 * nw;
    kvo += kvo_inc;
    peo += peo_inc;
  }
}

static int64_t mla_row_bytes(int64_t kv_dim, int64_t pe_dim, int elem_bytes) {
  return kv_dim + (kv_dim / 128) * 4 + pe_dim * elem_bytes;
}

// Shared argument checks; fills everything in `L` except cache pointers and idx.
static int mla_prepare(const mak_mla_linear_desc* lin, const mak_rows_desc* cache, int32_t fp8_format, const char* name,
                       MlaLaunch* L) {
  if (lin == nullptr || cache == nullptr) return fail(MAK_E_INVALID, "%s: NULL descriptor", name);
  if (lin->dtype != MAK_DT_BF16 && lin->dtype != MAK_DT_F16)
    return fail(MAK_E_UNSUPPORTED, "%s: linear dtype must be float16 or bfloat16", name);
  if (fp8_format != MAK_FP8_E4M3 && fp8_format != MAK_FP8_E5M2) return fail(MAK_E_INVALID, "%s: bad fp8 format", name);
  if (lin->kv_dim != 256 && lin->kv_dim != 512 && lin->kv_dim != 1024)
    return fail(MAK_E_UNSUPPORTED, "%s: kv_dim must be 256, 512 or 1024 (got %lld)", name, (long long)lin->kv_dim);
  if (lin->pe_dim < 0 || lin->pe_dim % 8 != 0 || lin->pe_dim > 256)
    return fail(MAK_E_UNSUPPORTED, "%s: pe_dim must be a multiple of 8 in [0, 256]", name);
  if (lin->num_layers < 0 || lin->num_tokens < 0) return fail(MAK_E_INVALID, "%s: negative extents", name);
  if (cache->num_planes != lin->num_layers)
    return fail(MAK_E_INVALID, "%s: cache has %lld planes for %lld layers", name, (long long)cache->num_planes,
                (long long)lin->num_layers);
  if (cache->num_planes > 0 && cache->plane_ptrs == nullptr) return fail(MAK_E_INVALID, "%s: plane_ptrs is NULL", name);
  if (cache->rows_per_block <= 0 || cache->num_rows < 0 || cache->block_stride < 0 || cache->row_stride < 0)
    return fail(MAK_E_INVALID, "%s: bad cache row geometry", name);
  const int e = 2;
  const int64_t need = mla_row_bytes(lin->kv_dim, lin->pe_dim, e);
  if ((cache->rows_per_block == 1 ? cache->block_stride : cache->row_stride) < need && cache->num_rows > 1)
    return fail(MAK_E_INVALID, "%s: cache rows are narrower than the %lld-byte FP8 row", name, (long long)need);
  const uint64_t kv_bits = reinterpret_cast<uintptr_t>(lin->kv) | static_cast<uint64_t>(lin->kv_stride_layer * e) |
                           static_cast<uint64_t>(lin->kv_stride_token * e);
  const uint64_t pe_bits = reinterpret_cast<uintptr_t>(lin->pe) | static_cast<uint64_t>(lin->pe_stride_layer * e) |
                           static_cast<uint64_t>(lin->pe_stride_token * e);
  if ((kv_bits & 15u) != 0) return fail(MAK_E_UNSUPPORTED, "%s: latent rows must be 16-byte aligned", name);
  if (lin->pe_dim > 0 && (pe_bits & 7u) != 0) return fail(MAK_E_UNSUPPORTED, "%s: rope rows must be 8-byte aligned", name);
  uint64_t c_bits = static_cast<uint64_t>(cache->block_stride) |
                    (cache->rows_per_block > 1 ? static_cast<uint64_t>(cache->row_stride) : 0u);
  for (int64_t q = 0; q < cache->num_planes; ++q) c_bits |= cache->plane_ptrs[q];
  const uint64_t c_align = lin->kv_dim >= 512 ? 15u : 7u;
  if ((c_bits & c_align) != 0)
    return fail(MAK_E_UNSUPPORTED, "%s: cache rows must be %d-byte aligned", name, static_cast<int>(c_align + 1));
  memset(L, 0, sizeof(*L));
  L->kv = static_cast<const unsigned char*>(lin->kv);
  L->pe = static_cast<const unsigned char*>(lin->pe);
  L->kv_sl = lin->kv_stride_layer * e;
  L->kv_st = lin->kv_stride_token * e;
  L->pe_sl = lin->pe_stride_layer * e;
  L->pe_st = lin->pe_stride_token * e;
  L->rows_per_block = cache->rows_per_block;
  L->block_stride = cache->block_stride;
  L->row_stride = cache->row_stride;
  L->num_rows = cache->num_rows;
  int lg = -1;
  if ((cache->rows_per_block & (cache->rows_per_block - 1)) == 0) {
    lg = 0;
    while ((int64_t{1} << lg) < cache->rows_per_block) ++lg;
  }
  L->lg_rows = lg;
  L->num_tokens = lin->num_tokens;
  L->kv_dim = static_cast<int32_t>(lin->kv_dim);
  L->pe_bytes = static_cast<int32_t>(lin->pe_dim * e);
  return MAK_OK;
}

// Can this call take the pair kernels?  kv_dim 512, rope rows of at most 128
// bytes (the load: a multiple of 16, so rows stay 16-byte aligned for
// cp.async), rows_per_block a power of two, 32-bit row indices and strides,
// fewer than 2^30 tokens.
static bool mla_pair_ok(const MlaLaunch& L, bool store) {
  return L.kv_dim == 512 && L.pe_bytes <= 128 && (store || L.pe_bytes % 16 == 0) && L.lg_rows >= 0 &&
         L.num_rows < (int64_t{1} << 31) && L.block_stride < (int64_t{1} << 32) && L.row_stride < (int64_t{1} << 32) &&
         L.num_tokens < (int64_t{1} << 30);
}

// Resident waves of blocks for a launch of nl layers: about one block per 64 KiB of the launch's
// bf16 side, clamped to 4..16 (the row engine's rule: a large call's last wave then drains fast,
// a small one keeps four waves).
static int64_t mla_waves(const MlaLaunch& L, int64_t nl, int64_t resident) {
  const int64_t bytes = nl * L.num_tokens * (static_cast<int64_t>(L.kv_dim) * 2 + L.pe_bytes);
  return std::min<int64_t>(16, std::max<int64_t>(4, bytes / (std::max<int64_t>(resident, 1) * (int64_t{64} << 10))));
}

template <bool STORE, typename T, int F, bool OWN, bool I64>
static int launch_mla_pairs(MlaLaunch& L, int64_t layers, unsigned char* kv_out, unsigned char* pe_out, cudaStream_t st,
                            const mak_rows_desc* cache) {
  const void* kern = STORE ? reinterpret_cast<const void*>(mla_fp8_store2_kernel<T, F, OWN, I64>)
                           : reinterpret_cast<const void*>(mla_fp8_load2_kernel<T, F, I64>);
  const size_t smem = STORE ? 0 : static_cast<size_t>(kMlaThreads / 32) * kMlaLoadStages * 2 * (528 + L.pe_bytes);
  const int64_t resident = static_cast<int64_t>(blocks_per_sm(kern, kMlaThreads, smem)) * sm_count();
  const int64_t pairs = (L.num_tokens + 1) / 2;
  for (int64_t l0 = 0; l0 < layers; l0 += kMlaPlanes) {
    const int64_t nl = std::min<int64_t>(kMlaPlanes, layers - l0);
    for (int64_t q = 0; q < nl; ++q) L.cache[q] = cache->plane_ptrs[l0 + q];
    const int64_t want = (pairs + (kMlaThreads / 32) - 1) / (kMlaThreads / 32);
    const int64_t cap = std::max<int64_t>(1, (mla_waves(L, nl, resident) * resident + nl - 1) / nl);
    const dim3 grid(static_cast<unsigned>(std::min(want, cap)), static_cast<unsigned>(nl));
    MlaLaunch P = L;
    P.kv = L.kv + l0 * L.kv_sl;
    P.pe = L.pe + l0 * L.pe_sl;
    const int rc = STORE ? launch_pdl("mla_fp8_store2_kernel", mla_fp8_store2_kernel<T, F, OWN, I64>, grid,
                                      dim3(kMlaThreads), 0, st, P)
                         : launch_pdl("mla_fp8_load2_kernel", mla_fp8_load2_kernel<T, F, I64>, grid, dim3(kMlaThreads),
                                      smem, st, P, kv_out + l0 * L.kv_sl, pe_out + l0 * L.pe_sl);
    if (rc) return rc;
  }
  return MAK_OK;
}

template <bool STORE, typename T, int F>
static int launch_mla_pairs(MlaLaunch& L, int64_t layers, unsigned char* kv_out, unsigned char* pe_out, cudaStream_t st,
                            const mak_rows_desc* cache) {
  const bool own = STORE && L.owner != nullptr;
  if (L.idx64) {
    return own ? launch_mla_pairs<STORE, T, F, true, true>(L, layers, kv_out, pe_out, st, cache)
               : launch_mla_pairs<STORE, T, F, false, true>(L, layers, kv_out, pe_out, st, cache);
  }
  return own ? launch_mla_pairs<STORE, T, F, true, false>(L, layers, kv_out, pe_out, st, cache)
             : launch_mla_pairs<STORE, T, F, false, false>(L, layers, kv_out, pe_out, st, cache);
}

template <bool STORE, typename T, int F, int E>
static int launch_mla(MlaLaunch& L, int64_t layers, unsigned char* kv_out, unsigned char* pe_out, cudaStream_t st,
                      const mak_rows_desc* cache) {
  if (E == 16 && mla_pair_ok(L, STORE)) return launch_mla_pairs<STORE, T, F>(L, layers, kv_out, pe_out, st, cache);
  const void* kern = STORE ? reinterpret_cast<const void*>(mla_fp8_store_kernel<T, F, E>)
                           : reinterpret_cast<const void*>(mla_fp8_load_kernel<T, F, E>);
  const int64_t resident = static_cast<int64_t>(blocks_per_sm(kern, kMlaThreads, 0)) * sm_count();
  for (int64_t l0 = 0; l0 < layers; l0 += kMlaPlanes) {
    const int64_t nl = std::min<int64_t>(kMlaPlanes, layers - l0);
    for (int64_t q = 0; q < nl; ++q) L.cache[q] = cache->plane_ptrs[l0 + q];
    const int64_t want = (L.num_tokens + (kMlaThreads / 32) - 1) / (kMlaThreads / 32);
    const int64_t cap = std::max<int64_t>(1, (mla_waves(L, nl, resident) * resident + nl - 1) / nl);
    const dim3 grid(static_cast<unsigned>(std::min(want, cap)), static_cast<unsigned>(nl));
    MlaLaunch P = L;
    P.kv = L.kv + l0 * L.kv_sl;
    P.pe = L.pe + l0 * L.pe_sl;
    const int rc = STORE ? launch_pdl("mla_fp8_store_kernel", mla_fp8_store_kernel<T, F, E>, grid, dim3(kMlaThreads), 0,
                                      st, P)
                         : launch_pdl("mla_fp8_load_kernel", mla_fp8_load_kernel<T, F, E>, grid, dim3(kMlaThreads), 0,
                                      st, P, kv_out + l0 * L.kv_sl, pe_out + l0 * L.pe_sl);
    if (rc) return rc;
  }
  return MAK_OK;
}

template <bool STORE, typename T, int F>
static int dispatch_e(MlaLaunch& L, const mak_mla_linear_desc* lin, const mak_rows_desc* cache, cudaStream_t st) {
  unsigned char* kv_out = static_cast<unsigned char*>(lin->kv);
  unsigned char* pe_out = static_cast<unsigned char*>(lin->pe);
  switch (lin->kv_dim) {
    case 256: return launch_mla<STORE, T, F, 8>(L, lin->num_layers, kv_out, pe_out, st, cache);
    case 512: return launch_mla<STORE, T, F, 16>(L, lin->num_layers, kv_out, pe_out, st, cache);
    default: return launch_mla<STORE, T, F, 32>(L, lin->num_layers, kv_out, pe_out, st, cache);
  }
}

template <bool STORE>
static int dispatch(MlaLaunch& L, const mak_mla_linear_desc* lin, const mak_rows_desc* cache, int32_t fmt,
                    cudaStream_t st) {
  if (lin->dtype == MAK_DT_BF16) {
    return fmt == MAK_FP8_E4M3 ? dispatch_e<STORE, __nv_bfloat16, MAK_FP8_E4M3>(L, lin, cache, st)
                               : dispatch_e<STORE, __nv_bfloat16, MAK_FP8_E5M2>(L, lin, cache, st);
  }
  return fmt == MAK_FP8_E4M3 ? dispatch_e<STORE, __half, MAK_FP8_E4M3>(L, lin, cache, st)
                             : dispatch_e<STORE, __half, MAK_FP8_E5M2>(L, lin, cache, st);
}

// Self-check of the store's fast path (fp8_encode2_quot_finite for finite
// values, fast_quot + fp8_encode2s_bounded next to non-finite ones) against the
// IEEE fp32 division and the full encoder: thread k takes the scale
// s = 2^scale_exp * (1 + k / 2^23) and every 16-bit input x of type T that a
// group with that scale can hold (|x / s| <= fp8_max up to rounding, and the
// non-finite inputs), and counts (a) FP8 codes that differ from
// fp8_encode(x / s) and (b) quotients with |x / s| >= 2^-14 that differ in any
// bit.  Only scales the store kernel sends down the fast path are tested.
// Threads k < 2^15 also check group_scale(amax) for the 16-bit amax of bits k.
template <typename T, int F>
__global__ void fp8_quotient_check_kernel(int scale_exp, unsigned long long* counts) {
  const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= (1u << 23)) return;
  if (k < 0x8000u) {
    // the pair store's group scale: group_scale(amax) against the IEEE division for every
    // finite non-negative 16-bit amax (counted as a differing quotient)
    const float amax = bits_to_f32<T>(k);
    if (amax <= 3.40282346638528859812e+38f &&
        __float_as_uint(group_scale<F>(amax)) != __float_as_uint(__fdiv_rn(amax, fp8_max_of<F>())))
      atomicAdd(counts + 1, 1ull);
  }
  const float s = __uint_as_float((static_cast<uint32_t>(scale_exp + 127) << 23) | k);
  unsigned long long bad_code = 0, bad_quot = 0;
  if (fast_quot_ok(s)) {
    const float y = __frcp_rn(s);
    const QuotPair qc = quot_pair(s, y);
    const float lim = fp8_max_of<F>() * (1.f + 0x1p-20f);
    for (uint32_t u = 0; u < 65536u; u += 2) {
      const float x0 = bits_to_f32<T>(u), x1 = bits_to_f32<T>(u + 1);
      const FastQuot a = fast_quot(x0, s, y), b = fast_quot(x1, s, y);
      const float w0 = __fdiv_rn(x0, s), w1 = __fdiv_rn(x1, s);
      // the store's choice: finite values through fp8_encode2_finite, a non-finite one
      // sends its lane to fp8_encode2s_bounded
      const uint32_t got = (isfinite(x0) && isfinite(x1)) ? fp8_encode2_quot_finite<F>(x0, x1, qc)
                                                          : fp8_encode2s_bounded<F>(a.q0, a.q1, b.q0, b.q1);
      // the inputs a group with scale s holds: |x / s| <= fp8_max up to rounding; inf / nan stay in
      const bool in0 = !(fabsf(w0) > lim) || !isfinite(x0), in1 = !(fabsf(w1) > lim) || !isfinite(x1);
      bad_code += (in0 && (got & 0xFFu) != fp8_encode<F>(w0)) + (in1 && (got >> 8) != fp8_encode<F>(w1));
      bad_quot += (in0 && isfinite(x0) && fabsf(w0) >= 0x1p-14f && __float_as_uint(w0) != __float_as_uint(a.q1)) +
                  (in1 && isfinite(x1) && fabsf(w1) >= 0x1p-14f && __float_as_uint(w1) != __float_as_uint(b.q1));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    bad_code += __shfl_xor_sync(0xffffffffu, bad_code, o);
    bad_quot += __shfl_xor_sync(0xffffffffu, bad_quot, o);
  }
  if ((threadIdx.x & 31) == 0 && (bad_code | bad_quot)) {
    atomicAdd(counts, bad_code);
    atomicAdd(counts + 1, bad_quot);
  }
}

}  // namespace mak

using namespace mak;

extern "C" {

int64_t mak_mla_fp8_row_bytes(int64_t kv_dim, int64_t pe_dim) { return mla_row_bytes(kv_dim, pe_dim, 2); }

int mak_mla_fp8_rows_store(const mak_mla_linear_desc* lin, const mak_rows_desc* cache, const void* slots,
                           int32_t slot_dtype, int32_t fp8_format, void* workspace, size_t workspace_bytes,
                           void* stream) {
  MlaLaunch L;
  int rc = mla_prepare(lin, cache, fp8_format, "mak_mla_fp8_rows_store", &L);
  if (rc) return rc;
  if (lin->num_tokens == 0 || lin->num_layers == 0) return MAK_OK;
  if (slots == nullptr || !valid_index_dtype(slot_dtype))
    return fail(MAK_E_INVALID, "mak_mla_fp8_rows_store: slot vector must be int32 or int64");
  cudaStream_t st = as_stream(stream);
  ScatterWs ws{};
  rc = carve_scatter_ws(workspace, workspace_bytes, lin->num_tokens, &ws);
  if (rc) return rc;
  rc = resolve_last_writer(slots, slot_dtype, lin->num_tokens, ws, st);
  if (rc) return rc;
  L.idx = ws.eff;
  L.idx64 = 1;
  return dispatch<true>(L, lin, cache, fp8_format, st);
}

int mak_mla_fp8_rows_store_owned(const mak_mla_linear_desc* lin, const mak_rows_desc* cache, const void* slots,
                                 int32_t slot_dtype, int32_t fp8_format, uint64_t* owner, int64_t owner_rows,
                                 uint32_t epoch, void* stream) {
  const char* name = "mak_mla_fp8_rows_store_owned";
  MlaLaunch L;
  int rc = mla_prepare(lin, cache, fp8_format, name, &L);
  if (rc) return rc;
  if (lin->num_tokens == 0 || lin->num_layers == 0) return MAK_OK;
  if (slots == nullptr || !valid_index_dtype(slot_dtype))
    return fail(MAK_E_INVALID, "%s: slot vector must be int32 or int64", name);
  if (owner_rows < cache->num_rows)
    return fail(MAK_E_INVALID, "%s: owner table has %lld rows, the cache %lld", name, (long long)owner_rows,
                (long long)cache->num_rows);
  cudaStream_t st = as_stream(stream);
  rc = mark_owners(slots, slot_dtype, lin->num_tokens, owner, owner_rows, epoch, st, name);
  if (rc) return rc;
  L.idx = slots;
  L.idx64 = slot_dtype == MAK_DT_I64;
  L.owner = reinterpret_cast<const unsigned long long*>(owner);
  L.tag_hi = static_cast<uint64_t>(epoch) << 32;
  return dispatch<true>(L, lin, cache, fp8_format, st);
}

int mak_mla_fp8_rows_load(const mak_rows_desc* cache, const mak_mla_linear_desc* lin, const void* slots,
                          int32_t slot_dtype, int32_t fp8_format, void* stream) {
  MlaLaunch L;
  int rc = mla_prepare(lin, cache, fp8_format, "mak_mla_fp8_rows_load", &L);
  if (rc) return rc;
  if (lin->num_tokens == 0 || lin->num_layers == 0) return MAK_OK;
  if (slots == nullptr || !valid_index_dtype(slot_dtype))
    return fail(MAK_E_INVALID, "mak_mla_fp8_rows_load: slot vector must be int32 or int64");
  L.idx = slots;
  L.idx64 = slot_dtype == MAK_DT_I64;
  return dispatch<false>(L, lin, cache, fp8_format, as_stream(stream));
}

int mak_fp8_quotient_selfcheck(int32_t elem_dtype, int32_t fp8_format, int32_t scale_exp, uint64_t* counts,
                               void* stream) {
  if (counts == nullptr) return fail(MAK_E_INVALID, "mak_fp8_quotient_selfcheck: counts is NULL");
  if (elem_dtype != MAK_DT_BF16 && elem_dtype != MAK_DT_F16)
    return fail(MAK_E_UNSUPPORTED, "mak_fp8_quotient_selfcheck: element dtype must be float16 or bfloat16");
  if (fp8_format != MAK_FP8_E4M3 && fp8_format != MAK_FP8_E5M2)
    return fail(MAK_E_INVALID, "mak_fp8_quotient_selfcheck: bad fp8 format");
  if (scale_exp < -126 || scale_exp > 127) return fail(MAK_E_INVALID, "mak_fp8_quotient_selfcheck: scale_exp out of range");
  cudaStream_t st = as_stream(stream);
  auto* c = reinterpret_cast<unsigned long long*>(counts);
  const dim3 grid((1u << 23) / 256);
  if (elem_dtype == MAK_DT_BF16) {
    if (fp8_format == MAK_FP8_E4M3) fp8_quotient_check_kernel<__nv_bfloat16, MAK_FP8_E4M3><<<grid, 256, 0, st>>>(scale_exp, c);
    else fp8_quotient_check_kernel<__nv_bfloat16, MAK_FP8_E5M2><<<grid, 256, 0, st>>>(scale_exp, c);
  } else {
    if (fp8_format == MAK_FP8_E4M3) fp8_quotient_check_kernel<__half, MAK_FP8_E4M3><<<grid, 256, 0, st>>>(scale_exp, c);
    else fp8_quotient_check_kernel<__half, MAK_FP8_E5M2><<<grid, 256, 0, st>>>(scale_exp, c);
  }
  return launch_status("fp8_quotient_check_kernel");
}

}  // extern "C"
