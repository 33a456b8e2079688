// CacheGen-style uniform-bin codec (musa_aiter/ops/kv_transfer.py:1111-1217).
//
// Encode, fully on the device:
//   1. min/max reduction (order-preserving uint32 keys + atomics, no workspace);
//   2. per element: scale = reciprocal(max - min) * (bins - 1) (PyTorch evaluates
//      `int / tensor` as `tensor.reciprocal() * int`), code = clamp(round_half_even(
//      (x - min) * scale), 0, bins - 1); a shared-memory histogram of the codes;
//   3. CDF: sequential float32 prefix sum of the counts divided by numel (the
//      reference's host bincount + cumsum).
// Decode: out = codebook[code] converted to the output dtype.
// All three passes read 16-byte vectors of the input (scalar tails), the
// histogram is kept per warp in shared memory and the decode codebook sits in
// shared memory as output-type bit patterns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace mak {

__device__ __forceinline__ float load_f32(const void* p, int dt, int64_t i) {
  switch (dt) {
    case MAK_DT_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    case MAK_DT_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

__device__ __forceinline__ void store_from_f32(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case MAK_DT_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case MAK_DT_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    default: reinterpret_cast<float*>(p)[i] = v; break;
  }
}

// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t f2key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Element types as 16-byte vectors: VE elements per vector, each widened to fp32.
template <int DT>
struct Elem;
template <>
struct Elem<MAK_DT_F16> {
  static constexpr int VE = 8;
  __device__ static float at(const uint4& v, int i) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(&v)[i >> 1];
    return __half2float(__ushort_as_half(static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xFFFFu))));
  }
};
template <>
struct Elem<MAK_DT_BF16> {
  static constexpr int VE = 8;
  __device__ static float at(const uint4& v, int i) {
    const uint32_t w = reinterpret_cast<const uint32_t*>(&v)[i >> 1];
    return __uint_as_float((i & 1) ? (w & 0xFFFF0000u) : (w << 16));
  }
};
template <>
struct Elem<MAK_DT_F32> {
  static constexpr int VE = 4;
  __device__ static float at(const uint4& v, int i) { return reinterpret_cast<const float*>(&v)[i]; }
};

// Grid-stride over 16-byte vectors (when x is 16-byte aligned) with a scalar tail.
constexpr int kMinmaxU = 8;
template <int DT>
__global__ void __launch_bounds__(256, 4) minmax_kernel(const void* x, int64_t n, int vec_ok, uint32_t* keys) {
  constexpr int VE = Elem<DT>::VE;
  float lo = 3.402823466e38f, hi = -3.402823466e38f;
  const int64_t nv = vec_ok ? n / VE : 0;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, nt = (int64_t)gridDim.x * blockDim.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  pdl_wait();
  // eight independent 16-byte loads per thread in flight (four left the pass at 0.66 of DRAM
  // peak, stalled on each iteration's round trip)
  for (int64_t i0 = tid; i0 < nv; i0 += kMinmaxU * nt) {
    uint4 v[kMinmaxU];
#pragma unroll
    for (int u = 0; u < kMinmaxU; ++u)
      if (i0 + u * nt < nv) v[u] = __ldg(xv + i0 + u * nt);
#pragma unroll
    for (int u = 0; u < kMinmaxU; ++u) {
      if (i0 + u * nt >= nv) continue;
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        const float f = Elem<DT>::at(v[u], e);
        lo = fminf(lo, f);
        hi = fmaxf(hi, f);
      }
    }
  }
  for (int64_t i = nv * VE + tid; i < n; i += nt) {
    const float f = load_f32(x, DT, i);
    lo = fminf(lo, f);
    hi = fmaxf(hi, f);
  }
  pdl_trigger();
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  // one pair of atomics per block, not per warp: thousands of warps updating the same two
  // words serialise in L2 (the pass took 30 us for 128 MiB with per-warp atomics)
  __shared__ float s_lo[32], s_hi[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) {
    s_lo[wid] = lo;
    s_hi[wid] = hi;
  }
  __syncthreads();
  if (wid == 0) {
    lo = lane < nw ? s_lo[lane] : 3.402823466e38f;
    hi = lane < nw ? s_hi[lane] : -3.402823466e38f;
    for (int o = 16; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lane == 0) {
      atomicMin(keys + 0, f2key(lo));
      atomicMax(keys + 1, f2key(hi));
    }
  }
}

// The CacheGen chain (key init, min/max, finish, count clear, encode, CDF, codebook) is launched
// with programmatic dependent launch: each small kernel's launch overlaps the previous one's drain.
__global__ void minmax_init_kernel(uint32_t* keys) {
  pdl_wait();
  keys[0] = 0xFFFFFFFFu;  // the min key starts at the largest key, the max key at the smallest
  keys[1] = 0u;
  pdl_trigger();
}

__global__ void clear_counts_kernel(unsigned long long* counts, int bins) {
  pdl_wait();
  for (int b = threadIdx.x; b < bins; b += blockDim.x) counts[b] = 0;
  pdl_trigger();
}

__global__ void minmax_finish_kernel(uint32_t* keys) {
  pdl_wait();
  pdl_trigger();
  float* out = reinterpret_cast<float*>(keys);
  const float lo = key2f(keys[0]), hi = key2f(keys[1]);
  out[0] = lo;
  out[1] = hi;
}

// The code of v as the bits of an fp32 number 1.5 * 2^23 + code: q is clamped to [0, top] first
// (fmaxf drops a NaN, the max == min case, to 0), then adding 1.5 * 2^23 rounds it to the nearest
// integer, ties to even (the sum's unit in the last place is 1), which lands in the low mantissa
// bits.  Clamping before rounding equals rounding before clamping for integer bounds.  This is
// the classic magic-number rounding: no conversion-pipe instruction (rint, float-to-int), which
// run at a quarter of the fp32 rate and bounded the encode pass at two per element.
constexpr uint32_t kCodeBias = 0x4B400000u;  // bits of 1.5 * 2^23
__device__ __forceinline__ uint32_t cachegen_code_bits(float v, float lo, float scale, float top) {
  const float q = fminf(fmaxf(__fmul_rn(__fsub_rn(v, lo), scale), 0.f), top);
  return __float_as_uint(__fadd_rn(q, 12582912.0f));
}

// Codes of VE elements per 16-byte vector (one VE-byte store), counted in
// shared-memory histograms that are folded into `counts` at the end.  Each warp
// keeps kHistCopies copies (lane % kHistCopies picks one), padded to 257 words so
// that one bin of different copies falls in different banks: lanes whose codes
// collide (the middle bins of a bell-shaped slab) serialise kHistCopies times less.
template <int DT>
__global__ void __launch_bounds__(256) cachegen_encode_kernel(const void* x, int64_t n, int vec_ok, const float* minmax,
                                                              int bins, uint8_t* codes, unsigned long long* counts) {
  constexpr int VE = Elem<DT>::VE;
  constexpr int kHistCopies = 4;
  constexpr int kHistPitch = 257;
  __shared__ unsigned int hist[8 * kHistCopies][kHistPitch];
  const int wib = threadIdx.x >> 5;
  for (int b = threadIdx.x; b < 8 * kHistCopies * kHistPitch; b += blockDim.x) (&hist[0][0])[b] = 0;
  __syncthreads();
  pdl_wait();
  const float lo = minmax[0], hi = minmax[1];
  const float scale = __fmul_rn(__frcp_rn(__fsub_rn(hi, lo)), static_cast<float>(bins - 1));
  const float top = static_cast<float>(bins - 1);
  const int64_t nv = vec_ok ? n / VE : 0;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, nt = (int64_t)gridDim.x * blockDim.x;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  unsigned int* h = hist[wib * kHistCopies + (threadIdx.x & (kHistCopies - 1))];
  // two independent 16-byte loads per thread in flight; the slab is walked from its end, so the
  // first vectors read are the ones the min/max pass read last and are likely still in L2
  for (int64_t i0 = tid; i0 < nv; i0 += 2 * nt) {
    uint4 vv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u)
      if (i0 + u * nt < nv) vv[u] = __ldg(xv + (nv - 1 - (i0 + u * nt)));
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (i0 + u * nt >= nv) continue;
      const int64_t i = nv - 1 - (i0 + u * nt);
      uint32_t cb[VE], packed[VE / 4];
#pragma unroll
      for (int e = 0; e < VE; ++e) {
        cb[e] = cachegen_code_bits(Elem<DT>::at(vv[u], e), lo, scale, top);
        atomicAdd(h + (cb[e] - kCodeBias), 1u);
      }
      // the low byte of each code's bits is the code: three byte permutes pack four
#pragma unroll
      for (int w = 0; w < VE / 4; ++w)
        packed[w] = __byte_perm(__byte_perm(cb[4 * w], cb[4 * w + 1], 0x0040),
                                __byte_perm(cb[4 * w + 2], cb[4 * w + 3], 0x0040), 0x5410);
      if (VE == 8) {
        reinterpret_cast<uint2*>(codes)[i] = make_uint2(packed[0], packed[VE / 4 - 1]);
      } else {
        reinterpret_cast<uint32_t*>(codes)[i] = packed[0];
      }
    }
  }
  for (int64_t i = nv * VE + tid; i < n; i += nt) {
    const uint32_t c = cachegen_code_bits(load_f32(x, DT, i), lo, scale, top) - kCodeBias;
    codes[i] = static_cast<uint8_t>(c);
    atomicAdd(h + c, 1u);
  }
  pdl_trigger();
  __syncthreads();
  for (int b = threadIdx.x; b < bins; b += blockDim.x) {
    unsigned int t = 0;
#pragma unroll
    for (int w = 0; w < 8 * kHistCopies; ++w) t += hist[w][b];
    if (t) atomicAdd(counts + b, static_cast<unsigned long long>(t));
  }
}

// CDF = [0, cumsum(counts) / n], summed strictly in bin order in fp32 (sums past 2^24 round,
// so the order is part of the result).  Lane l holds bins 8l .. 8l + 7 in registers; the running
// sum passes from lane to lane by shuffles, each lane adding its eight counts in order, and every
// lane then divides its own bins.  (A single thread summing counts from shared memory took
// 12-13 us.)
__global__ void cachegen_cdf_kernel(const unsigned long long* counts, int bins, int64_t n, float* cdf) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x;
  float v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int b = lane * 8 + j;
    v[j] = b < bins ? static_cast<float>(counts[b]) : 0.f;
  }
  float run = 0.f;
  for (int k = 0; k < 32; ++k) {
    if (lane == k) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        run = __fadd_rn(run, v[j]);
        v[j] = run;
      }
    }
    run = __shfl_sync(0xffffffffu, run, k);
  }
  const float denom = static_cast<float>(n);
  if (lane == 0) cdf[0] = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int b = lane * 8 + j;
    if (b < bins) cdf[b + 1] = __fdiv_rn(v[j], denom);
  }
}

// torch.linspace(min, max, bins) in float32 as PyTorch's CUDA kernel evaluates it: a step
// divided once, the first half counted up from min and the second half down from max, each a
// fused multiply-add; a slab with max == min gets min in every bin (the reference's torch.full).
__global__ void cachegen_codebook_kernel(const float* minmax, int bins, float* codebook) {
  pdl_wait();
  pdl_trigger();
  const float lo = minmax[0], hi = minmax[1];
  const float step = __fdiv_rn(__fsub_rn(hi, lo), static_cast<float>(bins - 1));
  const int halfway = bins / 2;
  for (int i = threadIdx.x; i < bins; i += blockDim.x) {
    float v = lo;
    if (!(lo == hi)) {
      v = i < halfway ? __fmaf_rn(step, static_cast<float>(i), lo)
                      : __fmaf_rn(-step, static_cast<float>(bins - 1 - i), hi);
    }
    codebook[i] = v;
  }
}

// 16 codes per 16-byte load, the codebook (as the output type's bits) in shared
// memory, 16 outputs per thread iteration; a scalar tail for the rest.
template <int OUT>
__global__ void __launch_bounds__(256) cachegen_decode_kernel(const uint8_t* codes, int64_t n, int vec_ok,
                                                              const void* codebook, int cb_dt, int bins, void* out) {
  __shared__ uint32_t book[256];  // output-type bit pattern of each code (0 beyond the codebook)
  pdl_wait();
  pdl_trigger();
  for (int c = threadIdx.x; c < 256; c += blockDim.x) {
    const float v = c < bins ? load_f32(codebook, cb_dt, c) : 0.f;
    uint32_t b;
    if (OUT == MAK_DT_F16) b = __half_as_ushort(__float2half_rn(v));
    else if (OUT == MAK_DT_BF16) b = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else b = __float_as_uint(v);
    book[c] = b;
  }
  __syncthreads();
  const int64_t nv = vec_ok ? n / 16 : 0;
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x, nt = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < nv; i += nt) {
    const uint4 cv = __ldg(reinterpret_cast<const uint4*>(codes) + i);
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w};
    if (OUT == MAK_DT_F32) {
      uint4* o = reinterpret_cast<uint4*>(out) + 4 * i;
#pragma unroll
      for (int w = 0; w < 4; ++w)
        o[w] = make_uint4(book[cw[w] & 0xFF], book[(cw[w] >> 8) & 0xFF], book[(cw[w] >> 16) & 0xFF], book[cw[w] >> 24]);
    } else {
      uint4* o = reinterpret_cast<uint4*>(out) + 2 * i;
      uint32_t r[8];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        r[2 * w] = book[cw[w] & 0xFF] | (book[(cw[w] >> 8) & 0xFF] << 16);
        r[2 * w + 1] = book[(cw[w] >> 16) & 0xFF] | (book[cw[w] >> 24] << 16);
      }
      o[0] = make_uint4(r[0], r[1], r[2], r[3]);
      o[1] = make_uint4(r[4], r[5], r[6], r[7]);
    }
  }
  for (int64_t i = nv * 16 + tid; i < n; i += nt) {
    const uint32_t b = book[codes[i]];
    if (OUT == MAK_DT_F32) reinterpret_cast<uint32_t*>(out)[i] = b;
    else reinterpret_cast<unsigned short*>(out)[i] = static_cast<unsigned short>(b);
  }
}

static bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool float_dtype(int32_t dt) { return dt == MAK_DT_F16 || dt == MAK_DT_BF16 || dt == MAK_DT_F32; }

}  // namespace mak

using namespace mak;

extern "C" {

int mak_minmax(const void* x, int32_t dtype, int64_t n, float* out_minmax, void* stream) {
  if (!float_dtype(dtype)) return fail(MAK_E_INVALID, "mak_minmax: dtype must be f16/bf16/f32");
  if (n <= 0 || !x || !out_minmax) return fail(MAK_E_INVALID, "mak_minmax: empty input or NULL pointer");
  cudaStream_t st = as_stream(stream);
  uint32_t* keys = reinterpret_cast<uint32_t*>(out_minmax);
  int rc = launch_pdl("minmax_init_kernel", minmax_init_kernel, dim3(1), dim3(32), 0, st, keys);
  if (rc) return rc;
  const int threads = 256;
  const int vec_ok = aligned16p(x);
  const void* kern = dtype == MAK_DT_F16 ? reinterpret_cast<const void*>(minmax_kernel<MAK_DT_F16>)
                     : dtype == MAK_DT_BF16 ? reinterpret_cast<const void*>(minmax_kernel<MAK_DT_BF16>)
                                            : reinterpret_cast<const void*>(minmax_kernel<MAK_DT_F32>);
  const int grid = grid_for(kern, threads, 0, (n / 4 + threads - 1) / threads + 1);
  auto mm = dtype == MAK_DT_F16 ? minmax_kernel<MAK_DT_F16> : dtype == MAK_DT_BF16 ? minmax_kernel<MAK_DT_BF16>
                                                                                     : minmax_kernel<MAK_DT_F32>;
  rc = launch_pdl("minmax_kernel", mm, dim3(grid), dim3(threads), 0, st, x, n, vec_ok, keys);
  if (rc) return rc;
  return launch_pdl("minmax_finish_kernel", minmax_finish_kernel, dim3(1), dim3(1), 0, st, keys);
}

int mak_cachegen_encode(const void* x, int32_t dtype, int64_t n, const float* minmax, int32_t num_bins, uint8_t* codes,
                        uint64_t* counts, float* cdf, void* stream) {
  if (!float_dtype(dtype)) return fail(MAK_E_INVALID, "mak_cachegen_encode: dtype must be f16/bf16/f32");
  if (num_bins < 2 || num_bins > 256) return fail(MAK_E_INVALID, "mak_cachegen_encode: num_bins must be in [2, 256]");
  if (n <= 0) return MAK_OK;
  if (!x || !minmax || !codes || !counts || !cdf) return fail(MAK_E_INVALID, "mak_cachegen_encode: NULL pointer");
  cudaStream_t st = as_stream(stream);
  auto* cnt0 = reinterpret_cast<unsigned long long*>(counts);
  int rc = launch_pdl("clear_counts_kernel", clear_counts_kernel, dim3(1), dim3(256), 0, st, cnt0, num_bins);
  if (rc) return rc;
  const int threads = 256;
  // vector path: 16-byte input vectors and VE-byte code stores (codes aligned to VE bytes)
  const int ve = dtype == MAK_DT_F32 ? 4 : 8;
  const int vec_ok = aligned16p(x) && (reinterpret_cast<uintptr_t>(codes) % ve) == 0;
  auto* cnt = reinterpret_cast<unsigned long long*>(counts);
  const void* kern = dtype == MAK_DT_F16 ? reinterpret_cast<const void*>(cachegen_encode_kernel<MAK_DT_F16>)
                     : dtype == MAK_DT_BF16 ? reinterpret_cast<const void*>(cachegen_encode_kernel<MAK_DT_BF16>)
                                            : reinterpret_cast<const void*>(cachegen_encode_kernel<MAK_DT_F32>);
  const int grid = grid_for(kern, threads, 0, (n / ve + threads - 1) / threads + 1);
  auto enc = dtype == MAK_DT_F16    ? cachegen_encode_kernel<MAK_DT_F16>
             : dtype == MAK_DT_BF16 ? cachegen_encode_kernel<MAK_DT_BF16>
                                    : cachegen_encode_kernel<MAK_DT_F32>;
  rc = launch_pdl("cachegen_encode_kernel", enc, dim3(grid), dim3(threads), 0, st, x, n, vec_ok, minmax, num_bins, codes,
                  cnt);
  if (rc) return rc;
  return launch_pdl("cachegen_cdf_kernel", cachegen_cdf_kernel, dim3(1), dim3(32), 0, st,
                    reinterpret_cast<const unsigned long long*>(counts), num_bins, n, cdf);
}

int mak_cachegen_codebook(const float* minmax, int32_t num_bins, float* codebook, void* stream) {
  if (num_bins < 2 || num_bins > 256) return fail(MAK_E_INVALID, "mak_cachegen_codebook: num_bins must be in [2, 256]");
  if (!minmax || !codebook) return fail(MAK_E_INVALID, "mak_cachegen_codebook: NULL pointer");
  return launch_pdl("cachegen_codebook_kernel", cachegen_codebook_kernel, dim3(1), dim3(256), 0, as_stream(stream),
                    minmax, num_bins, codebook);
}

int mak_cachegen_decode(const uint8_t* codes, int64_t n, const void* codebook, int32_t codebook_dtype, int32_t num_bins,
                        void* out, int32_t out_dtype, void* stream) {
  if (!float_dtype(codebook_dtype) || !float_dtype(out_dtype))
    return fail(MAK_E_INVALID, "mak_cachegen_decode: codebook/output dtype must be f16/bf16/f32");
  if (num_bins < 1 || num_bins > 256) return fail(MAK_E_INVALID, "mak_cachegen_decode: bad codebook size");
  if (n <= 0) return MAK_OK;
  if (!codes || !codebook || !out) return fail(MAK_E_INVALID, "mak_cachegen_decode: NULL pointer");
  const int threads = 256;
  const int vec_ok = aligned16p(codes) && aligned16p(out);
  cudaStream_t st = as_stream(stream);
  const void* kern = out_dtype == MAK_DT_F16 ? reinterpret_cast<const void*>(cachegen_decode_kernel<MAK_DT_F16>)
                     : out_dtype == MAK_DT_BF16 ? reinterpret_cast<const void*>(cachegen_decode_kernel<MAK_DT_BF16>)
                                                : reinterpret_cast<const void*>(cachegen_decode_kernel<MAK_DT_F32>);
  const int grid = grid_for(kern, threads, 0, (n / 16 + threads - 1) / threads + 1);
  auto dec = out_dtype == MAK_DT_F16    ? cachegen_decode_kernel<MAK_DT_F16>
             : out_dtype == MAK_DT_BF16 ? cachegen_decode_kernel<MAK_DT_BF16>
                                        : cachegen_decode_kernel<MAK_DT_F32>;
  return launch_pdl("cachegen_decode_kernel", dec, dim3(grid), dim3(threads), 0, st, codes, n, vec_ok, codebook,
                    codebook_dtype, num_bins, out);
}

}  // extern "C"
