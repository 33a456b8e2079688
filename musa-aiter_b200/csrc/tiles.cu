// Tile engine: gather/scatter between "tile" caches that keep block_size
// innermost ([L][NB][NH][HD][BS], the musa-aiter paged layout of
// musa_aiter/ops/kv_transfer.py:2987-3000) and token-major rows ([L][T][NH][HD]).
//
// Main path: warps take windows of tokens of one (kv, layer) plane, split the
// window's slot mapping into segments (runs of consecutive slots inside one
// block) with ballots, and move each segment through 16-byte chunks of the
// cache rows ([d][o0 .. o0 + G)), transposing in registers.  Runs of two or
// more tokens (block-table traffic and its ragged ends) go through
// tile_run_kernel, single tokens (random slots) through a second launch
// (tile_single_kernel, or tile_single_fp8_kernel for FP8 caches with
// head_dim a multiple of 128), so the single-token, latency-bound path runs
// at high occupancy while the run path keeps the registers its transposes
// need.
//
// Fallback (tile_kernel): any head_dim / block_size / alignment, through a
// shared-memory transpose of 32-token chunks.
//
// FP8 caches (raw uint8) fuse the musa-aiter reference codec into the moves:
// decode(byte) * scale on gather, encode(x / scale) on scatter
// (musa_aiter/ops/kv_transfer.py:2161-2200).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "fp8.cuh"

namespace mak {

constexpr int kTT = 32;  // tokens per chunk (multiple of every G: 4, 8, 16)

struct TileLaunch {
  uint64_t cache[2];
  uint64_t lin[2];
  const float* scale[2];
  const void* slots;
  int64_t c_sl, c_sb, c_sh, c_sd;  // cache strides (elements); block offset stride is 1
  int64_t l_sl, l_st, l_sh;        // linear strides (elements); head_dim stride is 1
  int64_t num_layers, num_heads, head_dim, block_size, num_slots, n_tokens, n_chunks;
  int32_t slots64, n_kv, fill_zero, cache_vec, lin_vec, scale_mode, heads_per_step;
  int32_t window;       // tokens per warp window of the segment kernel (8, 16 or 32)
  int32_t run_heads;    // heads per item of the run kernel's walk (fills a warp's 32 lanes)
  int32_t single_all;   // tile_single_fp8_kernel takes every token (runs, zero rows) with no run launch
  int32_t plane_group;  // (kv, layer) planes a segment-kernel block walks per window
  // Single-token launch (tile_single_kernel): a window's heads are split into 2^head_split_shift groups,
  // each a separate warp item, when the call has too few windows to fill the device (decode
  // batches); 0 elsewhere.
  int32_t head_split_shift;
  // Segment map (optional): the run launch (tile_run_kernel) stores, per window of map_window
  // tokens, (epoch << 2) | (single tokens of the window are left to the single-token launch);
  // that launch skips the tokens whose window entry has this epoch and the bit clear.  Entries of
  // another epoch are never trusted.
  uint32_t* seg_map;
  uint32_t seg_epoch;
  int32_t map_window;       // tokens per map entry (the run launch's window: 8, 16 or 32)
  int32_t map_shift;        // log2(map_window)
  int64_t seg_map_entries;  // host side: capacity of seg_map
  int64_t windows;          // ceil(n_tokens / window), set per launch
  // Owned scatter (optional): owner[slot] holds (epoch << 32) | last token writing the slot,
  // marked by owner_mark_kernel just before; a token whose entry names another token is skipped.
  const unsigned long long* owner;
  unsigned long long tag_hi;
};

// Slot of token t; -1 when it lies past the cache or, in an owned scatter, when a later token
// writes the same slot (negative slots are returned as they are: skipped by the callers).
template <bool SCATTER>
__device__ __forceinline__ int64_t token_slot(const TileLaunch& p, int64_t t) {
  const int64_t s = load_index(p.slots, p.slots64, t);
  if (s >= p.num_slots) return -1;
  if (SCATTER && s >= 0 && p.owner != nullptr &&
      __ldcg(p.owner + s) != (p.tag_hi | static_cast<unsigned long long>(t)))
    return -1;
  return s;
}

// Four consecutive linear elements as one aligned vector.
template <typename LT>
struct Vec4Of {
  using T = uint2;
};
template <>
struct Vec4Of<float> {
  using T = uint4;
};

template <typename CT, typename LT, int CODEC>
struct Codec {
  // raw copy: CT and LT are same-width integer carriers
  __device__ static __forceinline__ LT load(CT c, float) { return c; }
  __device__ static __forceinline__ CT store(LT x, float) { return x; }
};
template <typename LT>
struct Codec<uint8_t, LT, MAK_FP8_E4M3> {
  __device__ static __forceinline__ LT load(uint8_t c, float sc) {
    return from_f32<LT>(__fmul_rn(fp8_decode_top<MAK_FP8_E4M3>(static_cast<uint32_t>(c) << 24), sc));
  }
  __device__ static __forceinline__ uint8_t store(LT x, float sc) {
    return fp8_encode<MAK_FP8_E4M3>(__fdiv_rn(to_f32<LT>(x), sc));
  }
};
template <typename LT>
struct Codec<uint8_t, LT, MAK_FP8_E5M2> {
  __device__ static __forceinline__ LT load(uint8_t c, float sc) {
    return from_f32<LT>(__fmul_rn(fp8_decode_top<MAK_FP8_E5M2>(static_cast<uint32_t>(c) << 24), sc));
  }
  __device__ static __forceinline__ uint8_t store(LT x, float sc) {
    return fp8_encode<MAK_FP8_E5M2>(__fdiv_rn(to_f32<LT>(x), sc));
  }
};

// FP8 store of one full (R dims x G tokens) chunk from 16-bit token vectors (TV:
// R = 8 dims in a uint4 or R = 4 in a uint2 per token) when
// every value is finite and |x| / scale stays below the FP8 maximum (the usual
// case: scales from an amax): one reciprocal per chunk and, per value pair, the
// packed division-free quotient + flush-to-zero encoder of the MLA FP8 rows
// (fp8_encode2_quot_finite), which mak_fp8_quotient_selfcheck checks against the
// IEEE division for every 16-bit input in that range.  Returns false (nothing
// written) when the chunk needs the per-element reference encoder.
template <typename CT, typename LT, int CODEC, int G, int R, typename TV>
__device__ __forceinline__ bool encode_chunk_bounded(const TV (&toks)[G], float sc, CT* dst, int64_t row_pitch) {
  if constexpr (CODEC == 0 || sizeof(LT) != 2 || sizeof(CT) != 1 || G != 16 || R * 2 != sizeof(TV)) {
    return false;
  } else {
    constexpr int W = sizeof(TV) / 4;  // 32-bit words per token vector
    constexpr uint32_t kInf = std::is_same<LT, __half>::value ? 0x7C00u : 0x7F80u;
    constexpr float kBound = CODEC == MAK_FP8_E4M3 ? 447.99f : 57343.f;
    if (!fast_quot_ok(sc)) return false;
    uint32_t m2 = 0;
#pragma unroll
    for (int i = 0; i < G; ++i) {
#pragma unroll
      for (int k = 0; k < W; ++k) m2 = __vmaxu2(m2, reinterpret_cast<const uint32_t*>(&toks[i])[k] & 0x7FFF7FFFu);
    }
    const uint32_t mraw = max(m2 & 0xFFFFu, m2 >> 16);
    if (mraw >= kInf) return false;
    const float y = __frcp_rn(sc);
    const unsigned short mbits = static_cast<unsigned short>(mraw);
    if (!(__fmul_rn(to_f32<LT>(*reinterpret_cast<const LT*>(&mbits)), y) <= kBound)) return false;
    const QuotPair qc = quot_pair(sc, y);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float a = to_f32<LT>(reinterpret_cast<const LT*>(&toks[4 * q])[r]);
        const float b = to_f32<LT>(reinterpret_cast<const LT*>(&toks[4 * q + 1])[r]);
        const float c = to_f32<LT>(reinterpret_cast<const LT*>(&toks[4 * q + 2])[r]);
        const float d = to_f32<LT>(reinterpret_cast<const LT*>(&toks[4 * q + 3])[r]);
        w[q] = fp8_encode2_quot_finite<CODEC>(a, b, qc) | (fp8_encode2_quot_finite<CODEC>(c, d, qc) << 16);
      }
      *reinterpret_cast<uint4*>(dst + r * row_pitch) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return true;
  }
}

// Four 16-bit values -> four FP8 codes (byte i = code of x[i]) through the packed
// division-free encoder when they are finite and |x| / scale stays below the FP8
// maximum, as encode_chunk_bounded; false (nothing computed) otherwise or for
// fp32 inputs.
template <typename LT, int CODEC>
__device__ __forceinline__ bool encode4_bounded(const LT (&x)[4], float sc, uint32_t* out) {
  if constexpr (CODEC == 0 || sizeof(LT) != 2) {
    return false;
  } else {
    constexpr uint32_t kInf = std::is_same<LT, __half>::value ? 0x7C00u : 0x7F80u;
    constexpr float kBound = CODEC == MAK_FP8_E4M3 ? 447.99f : 57343.f;
    if (!fast_quot_ok(sc)) return false;
    uint32_t mraw = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) mraw = max(mraw, static_cast<uint32_t>(*reinterpret_cast<const unsigned short*>(&x[i])) & 0x7FFFu);
    if (mraw >= kInf) return false;
    const float y = __frcp_rn(sc);
    const unsigned short mbits = static_cast<unsigned short>(mraw);
    if (!(__fmul_rn(to_f32<LT>(*reinterpret_cast<const LT*>(&mbits)), y) <= kBound)) return false;
    const QuotPair qc = quot_pair(sc, y);
    *out = fp8_encode2_quot_finite<CODEC>(to_f32<LT>(x[0]), to_f32<LT>(x[1]), qc) |
           (fp8_encode2_quot_finite<CODEC>(to_f32<LT>(x[2]), to_f32<LT>(x[3]), qc) << 16);
    return true;
  }
}

// FP8 load of one full (R dims x G tokens) chunk through the flush-to-zero
// decode of the MLA FP8 rows (fp8_raw_top + one flush-to-zero multiply by
// scale * 2^(127 - bias), exact for scales in fp8_ftz_scale_ok's range): three
// integer operations and one multiply per code instead of the field-by-field
// decoder.  Returns false (nothing written) for other scales.
template <typename CT, typename LT, int CODEC, int G, int R>
__device__ __forceinline__ bool decode_chunk_ftz(const uint4 (&rows)[R], float sc, LT* out, int64_t token_pitch) {
  if constexpr (CODEC == 0 || sizeof(CT) != 1) {
    return false;
  } else {
    if (!fp8_ftz_scale_ok<CODEC>(sc)) return false;
    const float sf = __fmul_rn(sc, fp8_ftz_bias<CODEC>());  // exact: a power of two
#pragma unroll
    for (int i = 0; i < G; ++i) {
      uint4 outv;
      LT* o = reinterpret_cast<LT*>(&outv);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t w = reinterpret_cast<const uint32_t*>(&rows[r])[i >> 2];
        const uint32_t x = w << (8 * (3 - (i & 3)));  // code i in the top byte
        o[r] = from_f32<LT>(fmul_ftz(fp8_raw_top<CODEC>(x), sf));
      }
      *reinterpret_cast<uint4*>(out + i * token_pitch) = outv;
    }
    return true;
  }
}

template <typename CT, typename LT, int CODEC, bool SCATTER>
__global__ void __launch_bounds__(256) tile_kernel(const __grid_constant__ TileLaunch p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  constexpr int G = 16 / sizeof(CT);  // tokens per 16-byte cache vector
  constexpr int NG = kTT / G;
  constexpr int VL = 16 / sizeof(LT);  // elements per 16-byte linear vector
  using C = Codec<CT, LT, CODEC>;
  __shared__ int64_t s_off[kTT];
  __shared__ int s_packed[NG];
  LT* tile = reinterpret_cast<LT*>(smem_raw);
  const int HD = static_cast<int>(p.head_dim);
  const int NH = static_cast<int>(p.num_heads);
  const int HPS = p.heads_per_step;
  const int pitch = HD + VL;            // smem row pitch (elements), keeps 16-byte alignment
  const int head_tile = kTT * pitch;    // elements per head in the tile
  const int tid = threadIdx.x, nthr = blockDim.x;
  const int64_t work = p.n_chunks * p.num_layers * p.n_kv;

  for (int64_t w = blockIdx.x; w < work; w += gridDim.x) {
    const int64_t chunk = w % p.n_chunks;
    const int64_t rest = w / p.n_chunks;
    const int64_t l = rest % p.num_layers;
    const int kv = static_cast<int>(rest / p.num_layers);
    const int64_t t0 = chunk * kTT;
    const int cnt = static_cast<int>(min(static_cast<int64_t>(kTT), p.n_tokens - t0));
    __syncthreads();  // the previous work item is done with s_off / tile
    if (tid < kTT) {
      int64_t off = -1;
      if (tid < cnt) {
        const int64_t s = token_slot<SCATTER>(p, t0 + tid);
        if (s >= 0) {
          int64_t b, o;
          split_slot(s, p.block_size, &b, &o);
          off = b * p.c_sb + o;
        }
      }
      s_off[tid] = off;
    }
    __syncthreads();
    if (tid < NG) {
      const int64_t o0 = s_off[tid * G];
      bool ok = p.cache_vec && o0 >= 0 && (o0 % G) == 0;
      for (int i = 1; ok && i < G; ++i) ok = (s_off[tid * G + i] == o0 + i);
      s_packed[tid] = ok ? 1 : 0;
    }
    __syncthreads();

    const CT* cache_l = reinterpret_cast<const CT*>(p.cache[kv]) + l * p.c_sl;
    CT* cache_lw = reinterpret_cast<CT*>(p.cache[kv]) + l * p.c_sl;
    LT* lin_l = reinterpret_cast<LT*>(p.lin[kv]) + l * p.l_sl + t0 * p.l_st;
    const float* scl = CODEC ? p.scale[kv] : nullptr;

    for (int h0 = 0; h0 < NH; h0 += HPS) {
      const int nh = min(HPS, NH - h0);
      if (!SCATTER) {
        // (1) cache -> tile, group-fastest so a warp's packed loads cover whole cache rows
        const int items = nh * NG * HD;
        for (int it = tid; it < items; it += nthr) {
          const int g = it % NG;
          const int rem = it / NG;
          const int d = rem % HD;
          const int hh = rem / HD;
          const int h = h0 + hh;
          float sc = 1.f;
          if (CODEC) sc = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? h : l * NH + h)];
          const CT* ch = cache_l + h * p.c_sh + d * p.c_sd;
          LT* trow = tile + hh * head_tile + (g * G) * pitch + d;
          if (s_packed[g]) {
            const uint4 raw = __ldg(reinterpret_cast<const uint4*>(ch + s_off[g * G]));
            const CT* e = reinterpret_cast<const CT*>(&raw);
#pragma unroll
            for (int i = 0; i < G; ++i) trow[i * pitch] = C::load(e[i], sc);
          } else {
#pragma unroll
            for (int i = 0; i < G; ++i) {
              const int64_t off = s_off[g * G + i];
              trow[i * pitch] = off >= 0 ? C::load(ch[off], sc) : zero_of<LT>();
            }
          }
        }
        __syncthreads();
        // (2) tile -> linear rows
        if (p.lin_vec) {
          const int vpr = HD / VL;
          const int items2 = nh * cnt * vpr;
          for (int it = tid; it < items2; it += nthr) {
            const int c = it % vpr;
            const int rem = it / vpr;
            const int t = rem % cnt;
            const int hh = rem / cnt;
            uint4* dst = reinterpret_cast<uint4*>(lin_l + t * p.l_st + (h0 + hh) * p.l_sh + c * VL);
            if (s_off[t] >= 0) {
              *dst = *reinterpret_cast<const uint4*>(tile + hh * head_tile + t * pitch + c * VL);
            } else if (p.fill_zero) {
              *dst = make_uint4(0u, 0u, 0u, 0u);
            }
          }
        } else {
          const int items2 = nh * cnt * HD;
          for (int it = tid; it < items2; it += nthr) {
            const int d = it % HD;
            const int rem = it / HD;
            const int t = rem % cnt;
            const int hh = rem / cnt;
            LT* dst = lin_l + t * p.l_st + (h0 + hh) * p.l_sh + d;
            if (s_off[t] >= 0) {
              *dst = tile[hh * head_tile + t * pitch + d];
            } else if (p.fill_zero) {
              *dst = zero_of<LT>();
            }
          }
        }
        __syncthreads();
      } else {
        // (1) linear rows -> tile (only tokens that will be stored)
        if (p.lin_vec) {
          const int vpr = HD / VL;
          const int items = nh * cnt * vpr;
          for (int it = tid; it < items; it += nthr) {
            const int c = it % vpr;
            const int rem = it / vpr;
            const int t = rem % cnt;
            const int hh = rem / cnt;
            if (s_off[t] < 0) continue;
            *reinterpret_cast<uint4*>(tile + hh * head_tile + t * pitch + c * VL) =
                __ldg(reinterpret_cast<const uint4*>(lin_l + t * p.l_st + (h0 + hh) * p.l_sh + c * VL));
          }
        } else {
          const int items = nh * cnt * HD;
          for (int it = tid; it < items; it += nthr) {
            const int d = it % HD;
            const int rem = it / HD;
            const int t = rem % cnt;
            const int hh = rem / cnt;
            if (s_off[t] < 0) continue;
            tile[hh * head_tile + t * pitch + d] = lin_l[t * p.l_st + (h0 + hh) * p.l_sh + d];
          }
        }
        __syncthreads();
        // (2) tile -> cache (+ FP8 encode)
        const int items = nh * NG * HD;
        for (int it = tid; it < items; it += nthr) {
          const int g = it % NG;
          const int rem = it / NG;
          const int d = rem % HD;
          const int hh = rem / HD;
          const int h = h0 + hh;
          float sc = 1.f;
          if (CODEC) sc = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? h : l * NH + h)];
          CT* ch = cache_lw + h * p.c_sh + d * p.c_sd;
          const LT* trow = tile + hh * head_tile + (g * G) * pitch + d;
          if (s_packed[g]) {
            uint4 raw;
            CT* e = reinterpret_cast<CT*>(&raw);
#pragma unroll
            for (int i = 0; i < G; ++i) e[i] = C::store(trow[i * pitch], sc);
            *reinterpret_cast<uint4*>(ch + s_off[g * G]) = raw;
          } else {
#pragma unroll
            for (int i = 0; i < G; ++i) {
              const int64_t off = s_off[g * G + i];
              if (off >= 0) ch[off] = C::store(trow[i * pitch], sc);
            }
          }
        }
        __syncthreads();
      }
    }
  }
}

// Runs of two or more tokens take the 16-byte chunk path of tile_run_kernel: a gather reads
// whole chunks, so even a ragged end of 2..G-1 tokens costs one round trip per item where the
// element path would walk its tokens one after another; a scatter stores the covered part of a
// partly covered chunk element by element.  Single tokens (random slots) take the element path
// of the single-token launch, unless their window holds at most kRunSingles of them (the ragged
// ends of block-table calls) and a segment map tells that launch to skip them.
constexpr int kRunSingles = 4;

// ---------------------------------------------------------------------------
// One segment (a run of consecutive slots inside one cache block, at most 32
// tokens, chunk-aligned in slot space) of one (kv, layer) plane, heads
// [h_lo, h_hi), through the 16-byte cache chunks it touches.  The lanes split
// the (head, head_dim-group) units x chunks; neighbouring lanes take neighbouring chunks of one unit, so
// one warp instruction covers whole 32-byte sectors of a cache row.  A unit
// moves R head_dim rows (R = 16 / sizeof(linear element)) of G token columns
// (G = 16 / sizeof(cache element)):
//   gather : R chunk loads, then one 16-byte token row per covered column (a
//            partly covered chunk is read whole, only its tokens are written);
//   scatter: a fully covered chunk takes G token-row loads then R chunk
//            stores; a partly covered one element stores on the cache side (the
//            chunk's other slots belong to other tokens: no read-modify-write,
//            so concurrent segments of one block never race), its token rows
//            loaded KTOK at a time.  FP8 stores from 16-bit rows take R = 4
//            (8-byte token loads): the 16 token rows of a chunk then fit half
//            the registers, and every cache store still writes a whole 16-byte
//            row.
// cbase = element offset of the block in the plane, o_s = first in-block
// offset, ts = first token.
// ---------------------------------------------------------------------------
template <typename CT, typename LT, int CODEC, bool SCATTER, int KTOK>
__device__ __forceinline__ void move_run(const TileLaunch& p, const CT* cache_r, CT* cache_w, LT* lin_l, const float* scl,
                                         int64_t l, int64_t cbase, int o_s, int len, int64_t ts, int h_lo, int h_hi,
                                         int lane) {
  constexpr int G = 16 / sizeof(CT);
  constexpr bool kHalfRows = SCATTER && CODEC != 0 && sizeof(CT) == 1 && sizeof(LT) == 2;
  constexpr int R = kHalfRows ? 4 : 16 / sizeof(LT);
  using TV = typename std::conditional<kHalfRows, uint2, uint4>::type;  // R dims of one token
  using C = Codec<CT, LT, CODEC>;
  const int upr = static_cast<int>(p.head_dim) / R;
  const int NH = static_cast<int>(p.num_heads);
  const int units = (h_hi - h_lo) * upr;
  const int c_first = o_s / G, nch = (o_s + len - 1) / G - c_first + 1;
  for (int it = lane; it < units * nch; it += 32) {
    const int u = it / nch;
    const int c = c_first + (it - u * nch);
    const int hr = u / upr, dg = u - hr * upr;
    const int h = h_lo + hr;
    float sc = 1.f;
    if (CODEC) sc = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? h : l * NH + h)];
    const int64_t row0 = cbase + h * p.c_sh + static_cast<int64_t>(dg) * R * p.c_sd;
    LT* lrow = lin_l + ts * p.l_st + h * p.l_sh + dg * R;  // token ts, head h, head_dim dg*R
    const int col0 = c * G;
    const int lo = max(col0, o_s), hi = min(col0 + G, o_s + len);  // covered columns [lo, hi)
    if (lo == col0 && hi == col0 + G) {
      if (!SCATTER) {
        uint4 rows[R];
#pragma unroll
        for (int r = 0; r < R; ++r) rows[r] = __ldg(reinterpret_cast<const uint4*>(cache_r + row0 + r * p.c_sd + col0));
        if (!decode_chunk_ftz<CT, LT, CODEC, G, R>(rows, sc, lrow + (col0 - o_s) * p.l_st, p.l_st)) {
#pragma unroll
          for (int i = 0; i < G; ++i) {
            uint4 outv;
            LT* o = reinterpret_cast<LT*>(&outv);
#pragma unroll
            for (int r = 0; r < R; ++r) o[r] = C::load(reinterpret_cast<const CT*>(&rows[r])[i], sc);
            *reinterpret_cast<uint4*>(lrow + (col0 + i - o_s) * p.l_st) = outv;
          }
        }
      } else {
        TV toks[G];
#pragma unroll
        for (int i = 0; i < G; ++i) toks[i] = __ldg(reinterpret_cast<const TV*>(lrow + (col0 + i - o_s) * p.l_st));
        if (!encode_chunk_bounded<CT, LT, CODEC, G, R>(toks, sc, cache_w + row0 + col0, p.c_sd)) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            uint4 v;
            CT* e = reinterpret_cast<CT*>(&v);
#pragma unroll
            for (int i = 0; i < G; ++i) e[i] = C::store(reinterpret_cast<const LT*>(&toks[i])[r], sc);
            *reinterpret_cast<uint4*>(cache_w + row0 + r * p.c_sd + col0) = v;
          }
        }
      }
    } else if (!SCATTER) {
      uint4 rows[R];
#pragma unroll
      for (int r = 0; r < R; ++r) rows[r] = __ldg(reinterpret_cast<const uint4*>(cache_r + row0 + r * p.c_sd + col0));
#pragma unroll
      for (int i = 0; i < G; ++i) {
        if (col0 + i < lo || col0 + i >= hi) continue;
        uint4 outv;
        LT* o = reinterpret_cast<LT*>(&outv);
#pragma unroll
        for (int r = 0; r < R; ++r) o[r] = C::load(reinterpret_cast<const CT*>(&rows[r])[i], sc);
        *reinterpret_cast<uint4*>(lrow + (col0 + i - o_s) * p.l_st) = outv;
      }
    } else {
#pragma unroll 1
      for (int c0 = lo; c0 < hi; c0 += KTOK) {
        TV tv[KTOK];
#pragma unroll
        for (int i = 0; i < KTOK; ++i)
          if (c0 + i < hi) tv[i] = __ldg(reinterpret_cast<const TV*>(lrow + (c0 + i - o_s) * p.l_st));
#pragma unroll
        for (int i = 0; i < KTOK; ++i) {
          if (c0 + i >= hi) continue;
          const LT* x = reinterpret_cast<const LT*>(&tv[i]);
#pragma unroll
          for (int r = 0; r < R; ++r) cache_w[row0 + r * p.c_sd + c0 + i] = C::store(x[r], sc);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Segment tile kernel: the single tokens and the scatter run ends.
//
// A warp owns a window of 32 tokens of one (kv, layer) plane.  It loads the
// window's slots (plus the next 32, since runs may cross the window end), and
// finds "segments": runs of tokens whose slots are consecutive inside one
// cache block, capped at 32 tokens and cut at offsets that are multiples of
// min(block_size, 32) so every segment stays chunk-aligned in slot space.  The
// warp handles every segment that STARTS in its window, whole.
// It moves the single tokens (element items); the runs of two or more tokens
// go through tile_run_kernel, launched first, which also writes the segment
// map this launch uses to skip windows.  In calls of at most kSingleAllTokens
// tokens (single_all) it is the only tile launch: every token with a slot is
// moved element by element, and a filling gather writes the zero rows.  Each launch keeps the register budget
// its path needs.  No shared memory, no block barriers; FP8 codecs run in
// registers.
// ---------------------------------------------------------------------------
template <typename CT, typename LT, int CODEC, bool SCATTER, bool GROUPED>
__global__ void __launch_bounds__(256, 4) tile_single_kernel(const __grid_constant__ TileLaunch p) {
  using C = Codec<CT, LT, CODEC>;
  const int lane = threadIdx.x & 31;
  const int NH = static_cast<int>(p.num_heads);
  const int64_t cap = p.block_size < 32 ? p.block_size : 32;
  const int planes = static_cast<int>(p.num_layers) * p.n_kv;
  const int plane_lo = GROUPED ? static_cast<int>(blockIdx.y) * p.plane_group : static_cast<int>(blockIdx.y);
  const int plane_hi = GROUPED ? min(plane_lo + p.plane_group, planes) : plane_lo + 1;
  // plane variables (set here for the first plane; a grouped block resets them per plane);
  // planes <= 65535, so 32-bit division
  const int nl = static_cast<int>(p.num_layers);
  int64_t l = plane_lo % nl;
  int kv = plane_lo / nl;
  const CT* cache_r = reinterpret_cast<const CT*>(p.cache[kv]) + l * p.c_sl;
  CT* cache_w = reinterpret_cast<CT*>(p.cache[kv]) + l * p.c_sl;
  LT* lin_l = reinterpret_cast<LT*>(p.lin[kv]) + l * p.l_sl;
  const float* scl = CODEC ? p.scale[kv] : nullptr;
  const int W = p.window;
  const uint32_t wmask = W >= 32 ? 0xffffffffu : ((1u << W) - 1u);
  const int64_t windows = p.windows;
  const int64_t wstride = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  // head groups of an item: heads [h_lo, h_lo + NHp)
  const int hs_shift = p.head_split_shift;
  const int NHp = NH >> hs_shift;
  pdl_wait();
  pdl_trigger();

  for (int64_t wi = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); wi < (windows << hs_shift);
       wi += wstride) {
    const int64_t w = wi >> hs_shift;
    const int h_lo = static_cast<int>(wi & ((1 << hs_shift) - 1)) * NHp;
    const int h_hi = h_lo + NHp;
    const int64_t t0 = w * W;
    // Segment map entries of the map windows that cover [t0, t0 + W) (at most 32 / 8 = 4), one
    // per lane: the window is skipped when the run launch of this call left no single token in
    // any of them, and a single token is moved only if its own map window left it here.
    const uint32_t tag = p.seg_epoch << 2;
    const int64_t m0 = p.seg_map != nullptr ? t0 >> p.map_shift : 0;
    uint32_t v = 1u;  // no map: every single token is this launch's
    if (p.seg_map != nullptr) {
      const int64_t m1 = (min(t0 + W, p.n_tokens) - 1) >> p.map_shift;
      v = tag;
      if (lane <= m1 - m0) v = p.seg_map[m0 + lane];
      if (__all_sync(0xffffffffu, (v & ~3u) == tag && (v & 1u) == 0u)) continue;
    }
    // Slots of tokens t0 + lane (A) and t0 + 32 + lane (B), as (block element offset, in-block offset).
    int64_t offA = -1, sA = -1, sB = -1, oA = 0, oB = 0;
    {
      const int64_t ta = t0 + lane, tb = t0 + 32 + lane;
      if (ta < p.n_tokens) sA = token_slot<SCATTER>(p, ta);
      if (tb < p.n_tokens) sB = token_slot<SCATTER>(p, tb);
      int64_t b;
      if (sA >= 0) { split_slot(sA, p.block_size, &b, &oA); offA = b * p.c_sb + oA; }
      if (sB >= 0) split_slot(sB, p.block_size, &b, &oB);
    }
    int64_t sPrev = -1;  // slot of token t0 - 1 (for lane 0)
    if (lane == 0 && t0 > 0) {
      sPrev = token_slot<SCATTER>(p, t0 - 1);
    }
    const int64_t upA = __shfl_up_sync(0xffffffffu, sA, 1);
    const int64_t lastA = __shfl_sync(0xffffffffu, sA, 31);
    int64_t upB = __shfl_up_sync(0xffffffffu, sB, 1);
    const int64_t prevA = lane == 0 ? sPrev : upA;
    const int64_t prevB = lane == 0 ? lastA : upB;
    const bool startA = sA >= 0 && (prevA < 0 || sA != prevA + 1 || (oA % cap) == 0);
    const bool startB = sB >= 0 && (prevB < 0 || sB != prevB + 1 || (oB % cap) == 0);
    const uint32_t validA = __ballot_sync(0xffffffffu, sA >= 0);
    uint32_t mStartA = __ballot_sync(0xffffffffu, startA);  // segments starting at t0 + lane
    uint64_t bound = static_cast<uint64_t>(mStartA) |
                     (static_cast<uint64_t>(__ballot_sync(0xffffffffu, startB)) << 32) |
                     ~(static_cast<uint64_t>(validA) | (static_cast<uint64_t>(__ballot_sync(0xffffffffu, sB >= 0)) << 32));
    // Small calls (single_all, no run launch): every token with a slot is moved as a single
    // token, and a filling gather writes the zero rows of the tokens without one.
    uint32_t zmask = 0;
    if (p.single_all) {
      mStartA = validA;
      bound = ~0ull;
      if (!SCATTER && p.fill_zero) {
        const int64_t left = p.n_tokens - t0;
        zmask = ~validA & wmask & (left < 32 ? (1u << left) - 1u : 0xffffffffu);
      }
    }
    // The window's segments are the same for every plane: skip the planes when
    // none is this launch's kind.
    if (GROUPED) {
      bool work = zmask != 0u;
      for (uint32_t m = mStartA & wmask; m && !work; m &= m - 1) {
        const int q = __ffs(m) - 1;
        const uint64_t rest = bound >> (q + 1);
        work = (rest & 1u) != 0u;  // a single token: the next token is a boundary
      }
      if (!work) continue;
    }
    for (int plane = plane_lo; plane < plane_hi; ++plane) {
    if (GROUPED) {
      l = plane % nl;
      kv = plane / nl;
      cache_r = reinterpret_cast<const CT*>(p.cache[kv]) + l * p.c_sl;
      cache_w = reinterpret_cast<CT*>(p.cache[kv]) + l * p.c_sl;
      lin_l = reinterpret_cast<LT*>(p.lin[kv]) + l * p.l_sl;
      scl = CODEC ? p.scale[kv] : nullptr;
    }
    uint32_t mSeg = mStartA & wmask;  // the warp owns the segments that start inside its window
    while (mSeg) {
      const int q = __ffs(mSeg) - 1;
      mSeg &= mSeg - 1;
      const uint64_t rest = bound >> (q + 1);
      const int len = rest ? (__ffsll(static_cast<long long>(rest))) : (64 - q);
      const int64_t soff = __shfl_sync(0xffffffffu, offA, q);  // element offset of the segment's first slot
      const int o_s = static_cast<int>(__shfl_sync(0xffffffffu, oA, q));
      const int64_t ts = t0 + q;
      const int64_t cbase = soff - o_s;  // block start (element offset)
      if (len != 1) continue;
      {
        // left to this launch by the run launch? (the map entry of the token's own window)
        const uint32_t vq = __shfl_sync(0xffffffffu, v, p.seg_map != nullptr ? static_cast<int>((ts >> p.map_shift) - m0) : 0);
        if ((vq & ~3u) == tag && (vq & 1u) == 0u) continue;
      }
      {
        // Single-token segment (random slots): one element per item, head_dim fastest
        // across lanes, so a warp instruction touches consecutive cache rows (whole
        // sectors per instruction) and a contiguous piece of the token row; four items
        // per lane in flight.
        const int hd = static_cast<int>(p.head_dim);
        if (CODEC && (hd & 127) == 0) {
          // FP8 caches, head_dim a multiple of 128: a lane takes dims lane + 32e (e < 4) of a
          // 128-dim group, so each of its four cache loads (stores) is one warp access to 32
          // consecutive cache rows and each token-row access 64 contiguous bytes; items
          // (token, head, group) are walked with carried counters, two in flight per lane.
          const int gpr = hd >> 7;
          const int items = len * NHp * gpr;
          const int64_t sd = p.c_sd;
          int j = 0, h = h_lo, g = 0;
          for (int i0 = 0; i0 < items; i0 += 2) {
            CT code[2][4];
            LT vals[2][4];
            int pk[2];  // (token << 16) | (head << 8) | group of each item in flight, -1 = none
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              pk[k] = -1;
              if (i0 + k < items) {
                pk[k] = (j << 16) | (h << 8) | g;
                const int d0 = (g << 7) + lane;
                if (!SCATTER) {
                  const CT* c = cache_r + cbase + h * p.c_sh + static_cast<int64_t>(d0) * sd + o_s + j;
#pragma unroll
                  for (int e = 0; e < 4; ++e) code[k][e] = c[32 * e * sd];
                } else {
                  const LT* x = lin_l + (ts + j) * p.l_st + h * p.l_sh + d0;
#pragma unroll
                  for (int e = 0; e < 4; ++e) vals[k][e] = x[32 * e];
                }
                if (++g == gpr) {
                  g = 0;
                  if (++h == h_hi) {
                    h = h_lo;
                    ++j;
                  }
                }
              }
            }
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              if (pk[k] < 0) continue;
              const int jj = pk[k] >> 16, hh = (pk[k] >> 8) & 0xFF, d0 = ((pk[k] & 0xFF) << 7) + lane;
              const float sc = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? hh : l * NH + hh)];
              if (!SCATTER) {
                LT* o = lin_l + (ts + jj) * p.l_st + hh * p.l_sh + d0;
#pragma unroll
                for (int e = 0; e < 4; ++e) o[32 * e] = C::load(code[k][e], sc);
              } else {
                CT* c = cache_w + cbase + hh * p.c_sh + static_cast<int64_t>(d0) * sd + o_s + jj;
#pragma unroll
                for (int e = 0; e < 4; ++e) c[32 * e * sd] = C::store(vals[k][e], sc);
              }
            }
          }
          continue;
        }
        if ((hd & 31) == 0) {
          // head_dim a multiple of 32: lane = dim within a 32-dim group; every lane walks the
          // same (token, head, group) sequence with carried counters (no divisions), eight
          // elements in flight per lane.
          const int mpr = hd >> 5;
          const int steps = len * NHp * mpr;
          int j = 0, h = h_lo, m = 0;
          for (int s0 = 0; s0 < steps; s0 += 8) {
            CT cv[8];
            LT lv[8];
            int pk[8];  // (token << 16) | (head << 8) | group of each element in flight, -1 = none
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              pk[k] = -1;
              if (s0 + k < steps) {
                const int d = (m << 5) + lane;
                pk[k] = (j << 16) | (h << 8) | m;
                if (!SCATTER) cv[k] = cache_r[cbase + h * p.c_sh + static_cast<int64_t>(d) * p.c_sd + o_s + j];
                else lv[k] = lin_l[(ts + j) * p.l_st + h * p.l_sh + d];
                if (++m == mpr) {
                  m = 0;
                  if (++h == h_hi) {
                    h = h_lo;
                    ++j;
                  }
                }
              }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              if (pk[k] < 0) continue;
              const int jj = pk[k] >> 16, hh = (pk[k] >> 8) & 0xFF, d = ((pk[k] & 0xFF) << 5) + lane;
              float sc = 1.f;
              if (CODEC) sc = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? hh : l * NH + hh)];
              if (!SCATTER) lin_l[(ts + jj) * p.l_st + hh * p.l_sh + d] = C::load(cv[k], sc);
              else cache_w[cbase + hh * p.c_sh + static_cast<int64_t>(d) * p.c_sd + o_s + jj] = C::store(lv[k], sc);
            }
          }
          continue;
        }
        const int per_col = NH * hd;
        const int items = per_col * len;
        for (int base = 0; base < items; base += 128) {
          CT cv[4];
          LT lv[4];
          int64_t ck[4];
          LT* lk[4];
          float sck[4];
          bool ok[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int it = base + k * 32 + lane;
            ok[k] = it < items;
            const int j = ok[k] ? it / per_col : 0;
            const int hdid = ok[k] ? it - j * per_col : 0;
            const int h = hdid / hd, d = hdid - h * hd;
            sck[k] = 1.f;
            if (CODEC) sck[k] = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? h : l * NH + h)];
            ck[k] = cbase + h * p.c_sh + static_cast<int64_t>(d) * p.c_sd + o_s + j;
            lk[k] = lin_l + (ts + j) * p.l_st + h * p.l_sh + d;
            if (ok[k]) {
              if (!SCATTER) cv[k] = cache_r[ck[k]];
              else lv[k] = lk[k][0];
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (!ok[k]) continue;
            if (!SCATTER) lk[k][0] = C::load(cv[k], sck[k]);
            else cache_w[ck[k]] = C::store(lv[k], sck[k]);
          }
        }
      }
    }
    if (zmask) {
      // zero rows of this item's heads [h_lo, h_hi), 16-byte stores
      constexpr int R = 16 / sizeof(LT);
      const int upr = static_cast<int>(p.head_dim) / R;
      for (uint32_t mz = zmask; mz; mz &= mz - 1) {
        const int q = __ffs(mz) - 1;
        for (int u = lane; u < NHp * upr; u += 32) {
          const int h = h_lo + u / upr, dg = u - (u / upr) * upr;
          *reinterpret_cast<uint4*>(lin_l + (t0 + q) * p.l_st + h * p.l_sh + dg * R) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
    }  // planes of the group
  }
}

// ---------------------------------------------------------------------------
// Run launch (the main path): segments of two or more tokens, i.e. the
// block-table traffic and its ragged ends, in two phases per block.
//   1. Each of the block's 8 warps scans a window of W tokens of the slot
//      mapping (the same segment rule as the single-token kernel), appends the
//      runs that start in it to a shared-memory list (first token, slot offset,
//      length) -- and its single tokens too when there are at most kRunSingles
//      of them and a segment map records that -- marks the zero rows (gather,
//      fill mode) and, in the blocks of the first plane, writes the segment map
//      entry of its window for the single-token launch that follows.
//   2. The warps take (segment, head group) items of the list in turn and move
//      each through move_run; a group holds as many heads as fill the 32 lanes
//      with the (unit, chunk) pairs of a run as long as a block's chunk span
//      (bf16, head_dim 128, block_size 16: one head; FP8: two).
// One plane per block (grid = token ranges of 8W tokens x planes): nothing of
// the scan stays live in the walk, blocks are small enough that the last wave
// stays balanced, and the run path keeps 80 registers for its transposes
// (3 blocks per SM; 2 for FP8 stores from fp32 rows, whose 16 token rows of a chunk
// take 64 registers).
// ---------------------------------------------------------------------------
constexpr int kRunWarps = 8;
// segments listed per window: s single tokens and r runs (two or more tokens, the last one may
// end past the window) fit W >= s + 2(r - 1) + 1 tokens, so r + s <= (W + 1 + s) / 2
constexpr int kRunMaxSeg = kRunWarps * ((32 + 1 + kRunSingles) / 2);

template <typename CT, typename LT, int CODEC, bool SCATTER>
__global__ void __launch_bounds__(256, (CODEC != 0 && SCATTER && sizeof(LT) == 4) ? 2 : 3) tile_run_kernel(const __grid_constant__ TileLaunch p) {
  constexpr int R = 16 / sizeof(LT);
  __shared__ int64_t s_soff[kRunMaxSeg];  // element offset of the run's first slot in the plane
  __shared__ int s_ts[kRunMaxSeg];        // first token, relative to the block's first token
  __shared__ int s_os[kRunMaxSeg];        // in-block offset of the first slot
  __shared__ int s_len[kRunMaxSeg];
  __shared__ uint32_t s_zero[kRunWarps];
  __shared__ int s_cnt;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = p.window;  // 8, 16 or 32
  const uint32_t wmask = W >= 32 ? 0xffffffffu : ((1u << W) - 1u);
  const int64_t tb = static_cast<int64_t>(blockIdx.x) * (kRunWarps * W);
  const int64_t t0 = tb + warp * W;
  const int64_t cap = p.block_size < 32 ? p.block_size : 32;
  if (threadIdx.x == 0) s_cnt = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  uint32_t zmask = 0;
  if (t0 < p.n_tokens) {
    // slots of tokens t0 + lane (A) and t0 + 32 + lane (B): a run that starts in the window may
    // end past it
    int64_t offA = -1, sA = -1, sB = -1, oA = 0, oB = 0;
    {
      const int64_t ta = t0 + lane, tbb = t0 + 32 + lane;
      if (ta < p.n_tokens) sA = token_slot<SCATTER>(p, ta);
      if (tbb < p.n_tokens) sB = token_slot<SCATTER>(p, tbb);
      int64_t b;
      if (sA >= 0) { split_slot(sA, p.block_size, &b, &oA); offA = b * p.c_sb + oA; }
      if (sB >= 0) split_slot(sB, p.block_size, &b, &oB);
    }
    int64_t sPrev = -1;  // slot of token t0 - 1 (for lane 0)
    if (lane == 0 && t0 > 0) sPrev = token_slot<SCATTER>(p, t0 - 1);
    const int64_t upA = __shfl_up_sync(0xffffffffu, sA, 1);
    const int64_t lastA = __shfl_sync(0xffffffffu, sA, 31);
    const int64_t upB = __shfl_up_sync(0xffffffffu, sB, 1);
    const int64_t prevA = lane == 0 ? sPrev : upA;
    const int64_t prevB = lane == 0 ? lastA : upB;
    const bool startA = sA >= 0 && (prevA < 0 || sA != prevA + 1 || (oA % cap) == 0);
    const bool startB = sB >= 0 && (prevB < 0 || sB != prevB + 1 || (oB % cap) == 0);
    const uint32_t validA = __ballot_sync(0xffffffffu, sA >= 0);
    const uint32_t mStartA = __ballot_sync(0xffffffffu, startA);
    const uint64_t bound = static_cast<uint64_t>(mStartA) |
                           (static_cast<uint64_t>(__ballot_sync(0xffffffffu, startB)) << 32) |
                           ~(static_cast<uint64_t>(validA) |
                             (static_cast<uint64_t>(__ballot_sync(0xffffffffu, sB >= 0)) << 32));
    // the segment starting at this lane's token (len 0 = none): its length is bounded by the
    // next boundary in the 64 loaded slots; 64 - lane > 32, so a run that reaches past them is
    // long whatever follows, and the single-token launch classifies alike
    int len = 0;
    if (lane < W && ((mStartA >> lane) & 1u)) {
      const uint64_t rest = bound >> (lane + 1);
      len = rest ? __ffsll(static_cast<long long>(rest)) : (64 - lane);
    }
    // a window with few single tokens moves them here, when the map can tell the single-token
    // launch to leave them (the choice depends on the slots only: every plane makes it alike)
    const uint32_t singles = __ballot_sync(0xffffffffu, len == 1);
    const bool take_singles = p.seg_map != nullptr && __popc(singles) <= kRunSingles;
    if (p.seg_map != nullptr && blockIdx.y == 0 && lane == 0)
      p.seg_map[t0 / W] = (p.seg_epoch << 2) | (singles != 0u && !take_singles ? 1u : 0u);
    const int mode = len >= 2 || (len == 1 && take_singles) ? 1 : 0;
    if (!SCATTER && p.fill_zero) {
      zmask = ~validA & wmask;
      const int64_t left = p.n_tokens - t0;
      if (left < 32) zmask &= (1u << left) - 1u;
    }
    const uint32_t m = __ballot_sync(0xffffffffu, mode == 1);
    int base = 0;
    if (lane == 0 && m) base = atomicAdd(&s_cnt, __popc(m));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (mode == 1) {
      const int k = base + __popc(m & ((1u << lane) - 1u));
      s_soff[k] = offA;
      s_ts[k] = static_cast<int>(t0 - tb) + lane;
      s_os[k] = static_cast<int>(oA);
      s_len[k] = len;
    }
  }
  if (lane == 0) s_zero[warp] = zmask;
  __syncthreads();
  const int nl = static_cast<int>(p.num_layers);  // planes <= 65535: 32-bit division
  const int64_t l = static_cast<int>(blockIdx.y) % nl;
  const int kv = static_cast<int>(blockIdx.y) / nl;
  const CT* cache_r = reinterpret_cast<const CT*>(p.cache[kv]) + l * p.c_sl;
  CT* cache_w = reinterpret_cast<CT*>(p.cache[kv]) + l * p.c_sl;
  LT* lin_l = reinterpret_cast<LT*>(p.lin[kv]) + l * p.l_sl;
  const float* scl = CODEC ? p.scale[kv] : nullptr;
  const int NH = static_cast<int>(p.num_heads);
  const int hpi = p.run_heads;
  const int groups = (NH + hpi - 1) / hpi;
  const int items = s_cnt * groups;
  for (int it = warp; it < items; it += kRunWarps) {
    const int e = it / groups, h = (it - e * groups) * hpi;
    const int o_s = s_os[e];
    // (two token rows loaded at a time in a partly covered scatter chunk: more spill the run path)
    move_run<CT, LT, CODEC, SCATTER, 2>(p, cache_r, cache_w, lin_l, scl, l, s_soff[e] - o_s, o_s, s_len[e], tb + s_ts[e], h,
                                        min(h + hpi, NH), lane);
  }
  // zero rows for the skipped tokens of this warp's window (gather, fill mode)
  if (!SCATTER) {
    const int upr = static_cast<int>(p.head_dim) / R;
    const int units = static_cast<int>(p.num_heads) * upr;
    for (uint32_t mz = s_zero[warp]; mz; mz &= mz - 1) {
      const int q = __ffs(mz) - 1;
      for (int u = lane; u < units; u += 32) {
        const int h = u / upr, dg = u - h * upr;
        *reinterpret_cast<uint4*>(lin_l + (t0 + q) * p.l_st + h * p.l_sh + dg * R) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// FP8 single tokens (head_dim a multiple of 128): the single-token launch of
// FP8 calls, in two phases per block.
//   1. The block's warps find the single-token segments among its token range
//      (one slot per lane plus the neighbours by shuffles: a token is a segment
//      of its own when it starts one and the next token does not continue it,
//      the same rule the window scans apply) and append (token, slot offset)
//      to a shared-memory list.
//   2. All warps walk list entry x plane x head x 128-dim group items: a lane
//      takes dims lane + 32e (e < 4) of a group, so every cache access is one
//      warp access to 32 consecutive cache rows; four items per warp in flight.
// Nothing of phase 1 stays live in phase 2, so the kernel runs with few
// registers and a full SM of warps: the single tokens are bound by DRAM sector
// traffic (a token touches every sector of its head tile), and the number of
// sector requests in flight decides the rate.
// For calls of at most kSingleAllTokens tokens (single_all) it is the only tile
// launch: phase 1 lists every token with a slot, and in a filling gather every
// token without one as a zero row, and the runs are moved element by element.
// grid = (token ranges of tpc tokens, planes, head groups of hpc heads).
// ---------------------------------------------------------------------------
constexpr int kSingleMaxTok = 256;  // tokens per block, at most (8 scanning warps)
constexpr int kSingleInFlight = 4;  // items per warp in flight
// Calls of at most this many tokens skip the run launch: the single-token kernel (or, for FP8
// caches with head_dim a multiple of 128, tile_single_fp8_kernel) takes every token (a decode
// batch's random slots are single tokens; the run launch would only scan them).
constexpr int64_t kSingleAllTokens = 512;

template <typename LT, int CODEC, bool SCATTER>
__global__ void __launch_bounds__(256, 4) tile_single_fp8_kernel(const __grid_constant__ TileLaunch p, int tpc, int hpc) {
  using C = Codec<uint8_t, LT, CODEC>;
  __shared__ int64_t s_off[kSingleMaxTok];  // slot's element offset in the plane: block * c_sb + in-block offset
  __shared__ int s_tok[kSingleMaxTok];
  __shared__ int s_cnt;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n = p.n_tokens;
  if (threadIdx.x == 0) s_cnt = 0;
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const int64_t cap = p.block_size < 32 ? p.block_size : 32;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * tpc + warp * 32;
  if (warp * 32 < tpc && t0 < n) {
    // the run launch of this call marked, per map window, whether it left single tokens there
    bool scan = true, mine = true;
    if (p.seg_map != nullptr) {
      const int64_t m0 = t0 >> p.map_shift, m1 = (min(t0 + 32, n) - 1) >> p.map_shift;
      const uint32_t tag = p.seg_epoch << 2;
      uint32_t v = tag;
      if (lane <= m1 - m0) v = p.seg_map[m0 + lane];
      scan = !__all_sync(0xffffffffu, (v & ~3u) == tag && (v & 1u) == 0u);
      const uint32_t vt = __shfl_sync(0xffffffffu, v, static_cast<int>(((t0 + lane) >> p.map_shift) - m0));
      mine = !((vt & ~3u) == tag && (vt & 1u) == 0u);
    }
    if (scan) {
      const int64_t t = t0 + lane;
      const int64_t s = t < n ? token_slot<SCATTER>(p, t) : -1;
      int64_t sp = __shfl_up_sync(0xffffffffu, s, 1);
      int64_t sn = __shfl_down_sync(0xffffffffu, s, 1);
      if (lane == 0) sp = t0 > 0 ? token_slot<SCATTER>(p, t0 - 1) : -1;
      if (lane == 31) sn = t0 + 32 < n ? token_slot<SCATTER>(p, t0 + 32) : -1;
      int64_t b = 0, o = 0;
      if (s >= 0) split_slot(s, p.block_size, &b, &o);
      const bool start = s >= 0 && (sp < 0 || s != sp + 1 || (o % cap) == 0);
      const bool cont = sn >= 0 && sn == s + 1 && ((o + 1) % cap) != 0;
      // small calls (single_all): every token is listed, element by element for the tokens of
      // runs too, and in a filling gather the tokens without a slot as zero rows (offset -1)
      const bool zero_row = !SCATTER && p.single_all && p.fill_zero && t < n && s < 0;
      const bool single = p.single_all ? (s >= 0 || zero_row) : (start && !cont && mine);
      const uint32_t m = __ballot_sync(0xffffffffu, single);
      int base = 0;
      if (lane == 0 && m) base = atomicAdd(&s_cnt, __popc(m));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (single) {
        const int k = base + __popc(m & ((1u << lane) - 1u));
        s_tok[k] = static_cast<int>(t);
        s_off[k] = s >= 0 ? b * p.c_sb + o : -1;
      }
    }
  }
  __syncthreads();
  const int cnt = s_cnt;
  if (cnt == 0) return;
  const int plane = blockIdx.y;
  const int nl = static_cast<int>(p.num_layers);
  const int64_t l = plane % nl;
  const int kv = plane / nl;
  const uint8_t* cache_r = reinterpret_cast<const uint8_t*>(p.cache[kv]) + l * p.c_sl;
  uint8_t* cache_w = reinterpret_cast<uint8_t*>(p.cache[kv]) + l * p.c_sl;
  LT* lin_l = reinterpret_cast<LT*>(p.lin[kv]) + l * p.l_sl;
  const float* scl = p.scale[kv];
  const int NH = static_cast<int>(p.num_heads);
  const int h_lo = blockIdx.z * hpc;
  const int gpr = static_cast<int>(p.head_dim) >> 7;
  const int per_entry = hpc * gpr;
  const int64_t sd = p.c_sd;
  // this warp's contiguous share of the cnt x per_entry items, walked with carried counters
  const int total = cnt * per_entry;
  const int share = (total + 7) >> 3;
  int q = warp * share;
  const int q_end = min(q + share, total);
  if (q >= q_end) return;
  int e = q / per_entry;
  int j = q - e * per_entry;
  int hh = j / gpr;
  int g = j - hh * gpr;
  for (; q < q_end; q += kSingleInFlight) {
    uint8_t code[kSingleInFlight][4];
    LT vals[kSingleInFlight][4];
    int it_e[kSingleInFlight], it_h[kSingleInFlight], it_d[kSingleInFlight];
#pragma unroll
    for (int k = 0; k < kSingleInFlight; ++k) {
      it_e[k] = -1;
      if (q + k < q_end) {
        it_e[k] = e;
        it_h[k] = h_lo + hh;
        it_d[k] = (g << 7) + lane;
        if (!SCATTER) {
          const int64_t off = s_off[e];
#pragma unroll
          for (int i = 0; i < 4; ++i) code[k][i] = 0;
          if (off >= 0) {
            const uint8_t* c = cache_r + off + it_h[k] * p.c_sh + static_cast<int64_t>(it_d[k]) * sd;
#pragma unroll
            for (int i = 0; i < 4; ++i) code[k][i] = c[32 * i * sd];
          }
        } else {
          const LT* x = lin_l + static_cast<int64_t>(s_tok[e]) * p.l_st + it_h[k] * p.l_sh + it_d[k];
#pragma unroll
          for (int i = 0; i < 4; ++i) vals[k][i] = x[32 * i];
        }
        if (++g == gpr) {
          g = 0;
          if (++hh == hpc) {
            hh = 0;
            ++e;
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kSingleInFlight; ++k) {
      if (it_e[k] < 0) continue;
      const int h = it_h[k];
      const float sc = scl[p.scale_mode == MAK_SCALE_SCALAR ? 0 : (p.scale_mode == MAK_SCALE_PER_HEAD ? h : l * NH + h)];
      if (!SCATTER) {
        LT* o = lin_l + static_cast<int64_t>(s_tok[it_e[k]]) * p.l_st + h * p.l_sh + it_d[k];
        if (s_off[it_e[k]] < 0) {  // zero row of a filling gather (single_all)
#pragma unroll
          for (int i = 0; i < 4; ++i) o[32 * i] = zero_of<LT>();
        } else if (fp8_ftz_scale_ok<CODEC>(sc)) {
          const float sf = __fmul_rn(sc, fp8_ftz_bias<CODEC>());  // exact: a power of two
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o[32 * i] = from_f32<LT>(fmul_ftz(fp8_raw_top<CODEC>(static_cast<uint32_t>(code[k][i]) << 24), sf));
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) o[32 * i] = C::load(code[k][i], sc);
        }
      } else {
        uint8_t* c = cache_w + s_off[it_e[k]] + h * p.c_sh + static_cast<int64_t>(it_d[k]) * sd;
        uint32_t w = 0;
        if (!encode4_bounded<LT, CODEC>(vals[k], sc, &w)) {
#pragma unroll
          for (int i = 0; i < 4; ++i) w |= static_cast<uint32_t>(C::store(vals[k][i], sc)) << (8 * i);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) c[32 * i * sd] = static_cast<uint8_t>(w >> (8 * i));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// The single-token launch (tile_single_kernel).
template <typename CT, typename LT, int CODEC, bool SCATTER>
static int launch_tile_single(TileLaunch& p, cudaStream_t st) {
  const int threads = 256;
  const int64_t planes = p.num_layers * p.n_kv;
  auto kern = tile_single_kernel<CT, LT, CODEC, SCATTER, false>;
  const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(kern), threads, 0);
  // Narrower windows when 32-token windows would not give every resident warp a few windows
  // (short batches; runs of random slots are one token each, so parallelism comes from windows).
  const int64_t resident_warps = static_cast<int64_t>(per_sm) * sm_count() * (threads / 32);
  p.window = 32;
  while (p.window > 8 && (p.n_tokens + p.window - 1) / p.window * planes < 4 * resident_warps) p.window /= 2;
  const int64_t windows = (p.n_tokens + p.window - 1) / p.window;
  p.windows = windows;
  // Planes per block: a window's slot scan serves all planes of its group, so
  // group as many planes (up to 8) as still leave every resident warp a few
  // (window, group) items.
  p.plane_group = 8;
  while (p.plane_group > 1 && windows * ((planes + p.plane_group - 1) / p.plane_group) < 4 * resident_warps)
    p.plane_group /= 2;
  const int64_t groups = (planes + p.plane_group - 1) / p.plane_group;
  // Single tokens with few windows (decode batches): split each window's heads over up to
  // num_heads warp items (head_dim a multiple of 32, power-of-two splits dividing num_heads).
  p.head_split_shift = 0;
  if (p.head_dim % 32 == 0) {
    while ((windows << p.head_split_shift) * groups < 4 * resident_warps &&
           p.num_heads % (int64_t{2} << p.head_split_shift) == 0)
      ++p.head_split_shift;
  }
  const int64_t items = windows << p.head_split_shift;
  // About 4 device-fulls of CTAs, spread over the groups; each CTA walks windows grid-stride.
  const int64_t target = static_cast<int64_t>(per_sm) * sm_count() * 4;
  int64_t gx = std::max<int64_t>(1, target / groups);
  gx = std::min<int64_t>(gx, (items + (threads / 32) - 1) / (threads / 32));
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(groups));
  if (p.plane_group > 1)
    return launch_pdl("tile_single_kernel", tile_single_kernel<CT, LT, CODEC, SCATTER, true>, grid, dim3(threads), 0, st,
                      p);
  return launch_pdl("tile_single_kernel", kern, grid, dim3(threads), 0, st, p);
}

// The single-token launch of FP8 calls with head_dim a multiple of 128 (cfg3's random slots,
// ragged ends of block-table calls): tile_single_fp8_kernel.  Token ranges of up to 256 tokens
// per block, narrowed (and the heads split) until there are about four blocks per resident one.
template <typename LT, int CODEC, bool SCATTER>
static int launch_tile_single_fp8(TileLaunch& p, cudaStream_t st) {
  const int threads = 256;
  auto kern = tile_single_fp8_kernel<LT, CODEC, SCATTER>;
  const int64_t resident = static_cast<int64_t>(blocks_per_sm(reinterpret_cast<const void*>(kern), threads, 0)) * sm_count();
  const int64_t planes = p.num_layers * p.n_kv;
  int tpc = kSingleMaxTok, hpc = static_cast<int>(p.num_heads);
  auto blocks = [&]() { return (p.n_tokens + tpc - 1) / tpc * planes * (p.num_heads / hpc); };
  while (blocks() < 4 * resident && tpc > 32) tpc >>= 1;
  while (blocks() < 4 * resident && hpc % 2 == 0) hpc >>= 1;
  const dim3 grid(static_cast<unsigned>((p.n_tokens + tpc - 1) / tpc), static_cast<unsigned>(planes),
                  static_cast<unsigned>(p.num_heads / hpc));
  return launch_pdl("tile_single_fp8_kernel", kern, grid, dim3(threads), 0, st, p, tpc, hpc);
}

// The run launch: blocks of 8 windows of one plane; windows of 32 tokens (gathers: 16 or 8 when
// that leaves resident warps without a few windows; a scatter's scan also reads the owner table,
// which the smaller blocks pay for more often than they gain).  It sets the segment map fields
// the launches after it read.
template <typename CT, typename LT, int CODEC, bool SCATTER>
static int launch_tile_run(TileLaunch& p, cudaStream_t st) {
  const int threads = kRunWarps * 32;
  const int64_t planes = p.num_layers * p.n_kv;
  auto kern = tile_run_kernel<CT, LT, CODEC, SCATTER>;
  const int per_sm = blocks_per_sm(reinterpret_cast<const void*>(kern), threads, 0);
  const int64_t resident_warps = static_cast<int64_t>(per_sm) * sm_count() * kRunWarps;
  p.window = 32;
  // Gathers shrink the window to 8 tokens while the call has fewer than 4 waves of warps;
  // scatters keep 32-token windows (measured faster, Flash cache-back 3701 -> 4506 GB/s) unless
  // the call would fill under half of the resident warps (one-layer copy_to_kv_cache of 16384
  // tokens: 2395 -> 3110 GB/s at 16-token windows).
  while (p.window > 8 && (p.n_tokens + p.window - 1) / p.window * planes <
                             (SCATTER ? resident_warps / 2 : 4 * resident_warps))
    p.window /= 2;
  const int64_t windows = (p.n_tokens + p.window - 1) / p.window;
  p.windows = windows;
  // heads per walk item: (unit, chunk) pairs of one head for a run spanning a block's chunks
  const int64_t cap = std::min<int64_t>(p.block_size, 32);
  const int64_t g = 16 / static_cast<int64_t>(sizeof(CT));
  const int64_t r = (SCATTER && CODEC != 0 && sizeof(CT) == 1 && sizeof(LT) == 2) ? 4 : 16 / static_cast<int64_t>(sizeof(LT));
  const int64_t per_head = (p.head_dim / r) * ((cap + g - 1) / g);  // move_run's units x chunks of one head
  p.run_heads = static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(p.num_heads, 32 / std::max<int64_t>(per_head, 1))));
  // A scatter with enough whole runs to give every resident warp several moves them whole: on
  // large calls that measured faster than head groups (FP8 merged store 4683 -> 4896 GB/s), on
  // small ones slower (Flash cache-back 4509 -> 3812).
  if (SCATTER && (p.n_tokens + cap - 1) / cap * planes >= 8 * resident_warps) p.run_heads = static_cast<int32_t>(p.num_heads);
  if (p.seg_map != nullptr) {
    if (windows > p.seg_map_entries) p.seg_map = nullptr;  // too small: the later launches scan every window
    else {
      p.map_window = p.window;
      p.map_shift = p.window == 32 ? 5 : (p.window == 16 ? 4 : 3);
    }
  }
  const int64_t tblocks = (p.n_tokens + kRunWarps * p.window - 1) / (kRunWarps * p.window);
  if (tblocks > 0x7fffffff) return fail(MAK_E_UNSUPPORTED, "tile run launch: %lld token blocks", (long long)tblocks);
  const dim3 grid(static_cast<unsigned>(tblocks), static_cast<unsigned>(planes));
  return launch_pdl("tile_run_kernel", kern, grid, dim3(threads), 0, st, p);
}

template <typename CT, typename LT, int CODEC, bool SCATTER>
static int launch_tile_segments(TileLaunch& p, cudaStream_t st) {
  if constexpr (CODEC != 0 && sizeof(CT) == 1) {
    if (p.head_dim % 128 == 0 && p.n_tokens < (int64_t{1} << 31) && p.num_heads <= 65535) {
      if (p.n_tokens <= kSingleAllTokens) {
        // small calls (decode batches): the single-token kernel takes every token, runs
        // element by element and zero rows included, and the run launch is skipped
        p.seg_map = nullptr;
        p.single_all = 1;
        return launch_tile_single_fp8<LT, CODEC, SCATTER>(p, st);
      }
      const int rc = launch_tile_run<CT, LT, CODEC, SCATTER>(p, st);
      if (rc) return rc;
      return launch_tile_single_fp8<LT, CODEC, SCATTER>(p, st);
    }
  }
  if (p.n_tokens <= kSingleAllTokens) {
    // small calls: the single-token kernel takes every token, with no run launch
    p.seg_map = nullptr;
    p.single_all = 1;
    return launch_tile_single<CT, LT, CODEC, SCATTER>(p, st);
  }
  const int rc = launch_tile_run<CT, LT, CODEC, SCATTER>(p, st);
  if (rc) return rc;
  return launch_tile_single<CT, LT, CODEC, SCATTER>(p, st);
}

template <typename CT, typename LT, int CODEC, bool SCATTER>
static int launch_tile(TileLaunch& p, cudaStream_t st) {
  constexpr int VL = 16 / sizeof(LT);
  // Segment path: 16-byte chunks on both sides; needs aligned chunks and whole linear vectors
  // (and fewer than 256 heads: the single-token walk packs a head index into 8 bits).
  if (p.lin_vec && p.cache_vec && p.head_dim % VL == 0 && p.num_layers * p.n_kv <= 65535 && p.num_heads < 256)
    return launch_tile_segments<CT, LT, CODEC, SCATTER>(p, st);
  const int threads = 256;
  const size_t per_head = static_cast<size_t>(kTT) * (p.head_dim + VL) * sizeof(LT);
  // Heads per step: keep ~24 KB of tile per CTA so each thread has several 16-byte accesses in flight.
  int hps = static_cast<int>(std::max<size_t>(1, (24u << 10) / per_head));
  hps = static_cast<int>(std::min<int64_t>(hps, p.num_heads));
  p.heads_per_step = hps;
  const size_t smem = per_head * hps;
  auto kern = tile_kernel<CT, LT, CODEC, SCATTER>;
  if (smem > (48u << 10)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_fail(e, "tile_kernel smem attribute");
  }
  const int64_t work = p.n_chunks * p.num_layers * p.n_kv;
  const int grid = grid_for(reinterpret_cast<const void*>(kern), threads, smem, work);
  if (grid <= 0) return MAK_OK;
  kern<<<grid, threads, smem, st>>>(p);
  return launch_status("tile_kernel");
}

struct TileCall {
  const mak_paged_desc* cache;
  const mak_linear_desc* lin;
  const void* slots;
  int32_t slot_dtype;
  int32_t fill_zero;
  const float* k_scale;
  const float* v_scale;
  int32_t scale_mode;
  int32_t fp8_format;  // 0 = plain copy
  bool scatter;
  uint32_t* seg_map;  // optional segment map (see TileLaunch)
  int64_t seg_map_entries;
  uint32_t seg_epoch;
  const uint64_t* owner;  // owned scatter: marked owner table (see TileLaunch)
  uint32_t owner_epoch;
};

static int run_tile(const TileCall& c, cudaStream_t st, const char* name) {
  const mak_paged_desc* pc = c.cache;
  const mak_linear_desc* pl = c.lin;
  if (!pc || !pl) return fail(MAK_E_INVALID, "%s: NULL descriptor", name);
  if (pc->num_layers <= 0 || pc->num_blocks <= 0 || pc->num_heads <= 0 || pc->head_dim <= 0 || pc->block_size <= 0)
    return fail(MAK_E_INVALID, "%s: all cache extents must be positive", name);
  if (pl->num_tokens < 0) return fail(MAK_E_INVALID, "%s: negative token count", name);
  if (pl->num_tokens == 0) return MAK_OK;
  if (!c.slots || !valid_index_dtype(c.slot_dtype)) return fail(MAK_E_INVALID, "%s: slots must be int32/int64", name);
  if (pc->head_dim > 4096) return fail(MAK_E_UNSUPPORTED, "%s: head_dim %lld > 4096", name, (long long)pc->head_dim);
  const int n_kv = pc->v ? 2 : 1;
  if (!pc->k || !pl->k || (n_kv == 2 && !pl->v)) return fail(MAK_E_INVALID, "%s: NULL data pointer", name);

  const int ce = dtype_bytes(pc->dtype), le = dtype_bytes(pl->dtype);
  if (c.fp8_format) {
    if (pc->dtype != MAK_DT_U8) return fail(MAK_E_INVALID, "%s: FP8 cache must be stored as uint8", name);
    if (pl->dtype != MAK_DT_F16 && pl->dtype != MAK_DT_BF16 && pl->dtype != MAK_DT_F32)
      return fail(MAK_E_INVALID, "%s: FP8 linear dtype must be f16/bf16/f32", name);
    if (!c.k_scale || (n_kv == 2 && !c.v_scale)) return fail(MAK_E_INVALID, "%s: NULL scale pointer", name);
    if (c.scale_mode < MAK_SCALE_SCALAR || c.scale_mode > MAK_SCALE_PER_LAYER_HEAD)
      return fail(MAK_E_INVALID, "%s: bad scale mode %d", name, c.scale_mode);
  } else {
    if (pc->dtype != pl->dtype || (ce != 2 && ce != 4))
      return fail(MAK_E_INVALID, "%s: cache and linear dtypes must match (f16/bf16/f32)", name);
  }
  TileLaunch p;
  memset(&p, 0, sizeof(p));
  p.cache[0] = reinterpret_cast<uint64_t>(pc->k);
  p.cache[1] = reinterpret_cast<uint64_t>(pc->v);
  p.lin[0] = reinterpret_cast<uint64_t>(pl->k);
  p.lin[1] = reinterpret_cast<uint64_t>(pl->v);
  p.scale[0] = c.k_scale;
  p.scale[1] = c.v_scale;
  p.slots = c.slots;
  p.c_sl = pc->stride_layer;
  p.c_sb = pc->stride_block;
  p.c_sh = pc->stride_head;
  p.c_sd = pc->stride_dim;
  p.l_sl = pl->stride_layer;
  p.l_st = pl->stride_token;
  p.l_sh = pl->stride_head;
  p.num_layers = pc->num_layers;
  p.num_heads = pc->num_heads;
  p.head_dim = pc->head_dim;
  p.block_size = pc->block_size;
  p.num_slots = pc->num_blocks * pc->block_size;
  p.n_tokens = pl->num_tokens;
  p.n_chunks = (pl->num_tokens + kTT - 1) / kTT;
  p.slots64 = c.slot_dtype == MAK_DT_I64;
  p.n_kv = n_kv;
  p.fill_zero = c.fill_zero ? 1 : 0;
  p.scale_mode = c.scale_mode;
  if (c.seg_map != nullptr) {
    if (c.seg_epoch == 0 || c.seg_epoch >= (1u << 30) || c.seg_map_entries < 0)
      return fail(MAK_E_INVALID, "%s: segment map epoch must be in [1, 2^30) and its size non-negative", name);
    if ((reinterpret_cast<uintptr_t>(c.seg_map) & 3u) != 0) return fail(MAK_E_INVALID, "%s: misaligned segment map", name);
    p.seg_map = c.seg_map;
    p.seg_map_entries = c.seg_map_entries;
    p.seg_epoch = c.seg_epoch;
  }
  if (c.owner != nullptr) {
    p.owner = reinterpret_cast<const unsigned long long*>(c.owner);
    p.tag_hi = static_cast<unsigned long long>(c.owner_epoch) << 32;
  }
  // 16-byte cache vectors need every cache address of a packed group aligned.
  const int G = 16 / ce;
  const uint64_t cbits = static_cast<uint64_t>(p.c_sl | p.c_sb | p.c_sh | p.c_sd) * ce;
  p.cache_vec = aligned16(pc->k) && (n_kv == 1 || aligned16(pc->v)) && (cbits & 15u) == 0 && (pc->block_size % G) == 0;
  const uint64_t lbits = static_cast<uint64_t>(p.l_sl | p.l_st | p.l_sh | pc->head_dim) * le;
  p.lin_vec = aligned16(pl->k) && (n_kv == 1 || aligned16(pl->v)) && (lbits & 15u) == 0;

  if (c.fp8_format == 0) {
    if (ce == 2) return c.scatter ? launch_tile<uint16_t, uint16_t, 0, true>(p, st) : launch_tile<uint16_t, uint16_t, 0, false>(p, st);
    return c.scatter ? launch_tile<uint32_t, uint32_t, 0, true>(p, st) : launch_tile<uint32_t, uint32_t, 0, false>(p, st);
  }
#define MAK_TILE_FP8(FMT)                                                                                              \
  switch (pl->dtype) {                                                                                                 \
    case MAK_DT_F16:                                                                                                   \
      return c.scatter ? launch_tile<uint8_t, __half, FMT, true>(p, st) : launch_tile<uint8_t, __half, FMT, false>(p, st); \
    case MAK_DT_BF16:                                                                                                  \
      return c.scatter ? launch_tile<uint8_t, __nv_bfloat16, FMT, true>(p, st)                                         \
                       : launch_tile<uint8_t, __nv_bfloat16, FMT, false>(p, st);                                       \
    default:                                                                                                           \
      return c.scatter ? launch_tile<uint8_t, float, FMT, true>(p, st) : launch_tile<uint8_t, float, FMT, false>(p, st); \
  }
  if (c.fp8_format == MAK_FP8_E4M3) {
    MAK_TILE_FP8(MAK_FP8_E4M3)
  } else if (c.fp8_format == MAK_FP8_E5M2) {
    MAK_TILE_FP8(MAK_FP8_E5M2)
  }
#undef MAK_TILE_FP8
  return fail(MAK_E_INVALID, "%s: unknown FP8 format %d", name, c.fp8_format);
}

static int tile_scatter(TileCall c, void* workspace, size_t ws_bytes, cudaStream_t st, const char* name) {
  if (!c.lin || c.lin->num_tokens <= 0) return MAK_OK;
  if (!c.slots || !valid_index_dtype(c.slot_dtype)) return fail(MAK_E_INVALID, "%s: slots must be int32/int64", name);
  ScatterWs ws{};
  int rc = carve_scatter_ws(workspace, ws_bytes, c.lin->num_tokens, &ws);
  if (rc) return rc;
  rc = resolve_last_writer(c.slots, c.slot_dtype, c.lin->num_tokens, ws, st);
  if (rc) return rc;
  c.slots = ws.eff;
  c.slot_dtype = MAK_DT_I64;
  c.scatter = true;
  return run_tile(c, st, name);
}

// Owned scatter: one marking launch (atomicMax of (epoch << 32) | token per slot) replaces the
// workspace's clear / insert / resolve launches; the tile kernels skip tokens that lost.
static int tile_scatter_owned(TileCall c, uint64_t* owner, int64_t owner_rows, uint32_t epoch, cudaStream_t st,
                              const char* name) {
  if (!c.lin || c.lin->num_tokens <= 0) return MAK_OK;
  if (!c.cache) return fail(MAK_E_INVALID, "%s: NULL descriptor", name);
  if (!c.slots || !valid_index_dtype(c.slot_dtype)) return fail(MAK_E_INVALID, "%s: slots must be int32/int64", name);
  if (c.cache->num_blocks <= 0 || c.cache->block_size <= 0) return fail(MAK_E_INVALID, "%s: all cache extents must be positive", name);
  if (owner_rows < c.cache->num_blocks * c.cache->block_size)
    return fail(MAK_E_INVALID, "%s: owner table has %lld rows, the cache %lld slots", name, (long long)owner_rows,
                (long long)(c.cache->num_blocks * c.cache->block_size));
  int rc = mark_owners(c.slots, c.slot_dtype, c.lin->num_tokens, owner, owner_rows, epoch, st, name);
  if (rc) return rc;
  c.owner = owner;
  c.owner_epoch = epoch;
  c.scatter = true;
  return run_tile(c, st, name);
}

}  // namespace mak

using namespace mak;

extern "C" {

int mak_kv_paged_to_linear(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                           int32_t slot_dtype, int32_t fill_zero, void* stream) {
  return mak_kv_paged_to_linear_mapped(cache, out, slots, slot_dtype, fill_zero, nullptr, 0, 0, stream);
}

int mak_kv_paged_to_linear_mapped(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                                  int32_t slot_dtype, int32_t fill_zero, uint32_t* seg_map, int64_t seg_map_entries,
                                  uint32_t epoch, void* stream) {
  TileCall c{};
  c.cache = cache;
  c.lin = out;
  c.slots = slots;
  c.slot_dtype = slot_dtype;
  c.fill_zero = fill_zero;
  c.seg_map = seg_map;
  c.seg_map_entries = seg_map_entries;
  c.seg_epoch = epoch;
  return run_tile(c, as_stream(stream), "mak_kv_paged_to_linear");
}

int mak_kv_linear_to_paged(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                           int32_t slot_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return mak_kv_linear_to_paged_mapped(in, cache, slots, slot_dtype, workspace, workspace_bytes, nullptr, 0, 0, stream);
}

int mak_kv_linear_to_paged_mapped(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                                  int32_t slot_dtype, void* workspace, size_t workspace_bytes, uint32_t* seg_map,
                                  int64_t seg_map_entries, uint32_t epoch, void* stream) {
  TileCall c{};
  c.cache = cache;
  c.lin = in;
  c.slots = slots;
  c.slot_dtype = slot_dtype;
  c.seg_map = seg_map;
  c.seg_map_entries = seg_map_entries;
  c.seg_epoch = epoch;
  return tile_scatter(c, workspace, workspace_bytes, as_stream(stream), "mak_kv_linear_to_paged");
}

int mak_kv_linear_to_paged_owned(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                                 int32_t slot_dtype, uint64_t* owner, int64_t owner_rows, uint32_t epoch,
                                 uint32_t* seg_map, int64_t seg_map_entries, uint32_t seg_epoch, void* stream) {
  TileCall c{};
  c.cache = cache;
  c.lin = in;
  c.slots = slots;
  c.slot_dtype = slot_dtype;
  c.seg_map = seg_map;
  c.seg_map_entries = seg_map_entries;
  c.seg_epoch = seg_epoch;
  return tile_scatter_owned(c, owner, owner_rows, epoch, as_stream(stream), "mak_kv_linear_to_paged_owned");
}

int mak_kv_paged_fp8_to_linear(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                               int32_t slot_dtype, const float* k_scale, const float* v_scale, int32_t scale_mode,
                               int32_t fp8_format, void* stream) {
  return mak_kv_paged_fp8_to_linear_mapped(cache, out, slots, slot_dtype, k_scale, v_scale, scale_mode, fp8_format,
                                           nullptr, 0, 0, stream);
}

int mak_kv_paged_fp8_to_linear_mapped(const mak_paged_desc* cache, const mak_linear_desc* out, const void* slots,
                                      int32_t slot_dtype, const float* k_scale, const float* v_scale,
                                      int32_t scale_mode, int32_t fp8_format, uint32_t* seg_map,
                                      int64_t seg_map_entries, uint32_t epoch, void* stream) {
  if (fp8_format != MAK_FP8_E4M3 && fp8_format != MAK_FP8_E5M2)
    return fail(MAK_E_INVALID, "mak_kv_paged_fp8_to_linear: unknown FP8 format %d", fp8_format);
  TileCall c{};
  c.cache = cache;
  c.lin = out;
  c.slots = slots;
  c.slot_dtype = slot_dtype;
  c.fill_zero = 1;
  c.k_scale = k_scale;
  c.v_scale = v_scale;
  c.scale_mode = scale_mode;
  c.fp8_format = fp8_format;
  c.seg_map = seg_map;
  c.seg_map_entries = seg_map_entries;
  c.seg_epoch = epoch;
  return run_tile(c, as_stream(stream), "mak_kv_paged_fp8_to_linear");
}

int mak_kv_linear_to_paged_fp8(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                               int32_t slot_dtype, const float* k_scale, const float* v_scale, int32_t scale_mode,
                               int32_t fp8_format, void* workspace, size_t workspace_bytes, void* stream) {
  return mak_kv_linear_to_paged_fp8_mapped(in, cache, slots, slot_dtype, k_scale, v_scale, scale_mode, fp8_format,
                                           workspace, workspace_bytes, nullptr, 0, 0, stream);
}

int mak_kv_linear_to_paged_fp8_mapped(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                                      int32_t slot_dtype, const float* k_scale, const float* v_scale,
                                      int32_t scale_mode, int32_t fp8_format, void* workspace,
                                      size_t workspace_bytes, uint32_t* seg_map, int64_t seg_map_entries,
                                      uint32_t epoch, void* stream) {
  if (fp8_format != MAK_FP8_E4M3 && fp8_format != MAK_FP8_E5M2)
    return fail(MAK_E_INVALID, "mak_kv_linear_to_paged_fp8: unknown FP8 format %d", fp8_format);
  TileCall c{};
  c.cache = cache;
  c.lin = in;
  c.slots = slots;
  c.slot_dtype = slot_dtype;
  c.k_scale = k_scale;
  c.v_scale = v_scale;
  c.scale_mode = scale_mode;
  c.fp8_format = fp8_format;
  c.seg_map = seg_map;
  c.seg_map_entries = seg_map_entries;
  c.seg_epoch = epoch;
  return tile_scatter(c, workspace, workspace_bytes, as_stream(stream), "mak_kv_linear_to_paged_fp8");
}

int mak_kv_linear_to_paged_fp8_owned(const mak_linear_desc* in, const mak_paged_desc* cache, const void* slots,
                                     int32_t slot_dtype, const float* k_scale, const float* v_scale,
                                     int32_t scale_mode, int32_t fp8_format, uint64_t* owner, int64_t owner_rows,
                                     uint32_t epoch, uint32_t* seg_map, int64_t seg_map_entries, uint32_t seg_epoch,
                                     void* stream) {
  if (fp8_format != MAK_FP8_E4M3 && fp8_format != MAK_FP8_E5M2)
    return fail(MAK_E_INVALID, "mak_kv_linear_to_paged_fp8_owned: unknown FP8 format %d", fp8_format);
  TileCall c{};
  c.cache = cache;
  c.lin = in;
  c.slots = slots;
  c.slot_dtype = slot_dtype;
  c.k_scale = k_scale;
  c.v_scale = v_scale;
  c.scale_mode = scale_mode;
  c.fp8_format = fp8_format;
  c.seg_map = seg_map;
  c.seg_map_entries = seg_map_entries;
  c.seg_epoch = seg_epoch;
  return tile_scatter_owned(c, owner, owner_rows, epoch, as_stream(stream), "mak_kv_linear_to_paged_fp8_owned");
}

}  // extern "C"
