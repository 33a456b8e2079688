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

__global__ void minmax_kernel(const void* x, int dt, int64_t n, uint32_t* keys) {
  float lo = 3.402823466e38f, hi = -3.402823466e38f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = load_f32(x, dt, i);
    lo = fminf(lo, v);
    hi = fmaxf(hi, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(keys + 0, f2key(lo));
    atomicMax(keys + 1, f2key(hi));
  }
}

__global__ void minmax_finish_kernel(uint32_t* keys) {
  float* out = reinterpret_cast<float*>(keys);
  const float lo = key2f(keys[0]), hi = key2f(keys[1]);
  out[0] = lo;
  out[1] = hi;
}

__global__ void cachegen_encode_kernel(const void* x, int dt, int64_t n, const float* minmax, int bins, uint8_t* codes,
                                       unsigned long long* counts) {
  __shared__ unsigned int hist[256];
  for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
  __syncthreads();
  const float lo = minmax[0], hi = minmax[1];
  const float scale = __fmul_rn(__frcp_rn(__fsub_rn(hi, lo)), static_cast<float>(bins - 1));
  const float top = static_cast<float>(bins - 1);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = load_f32(x, dt, i);
    float q = rintf(__fmul_rn(__fsub_rn(v, lo), scale));
    q = fminf(fmaxf(q, 0.f), top);  // fmaxf drops a NaN (max == min case) to 0
    const uint32_t c = static_cast<uint32_t>(q);
    codes[i] = static_cast<uint8_t>(c);
    atomicAdd(&hist[c], 1u);
  }
  __syncthreads();
  for (int b = threadIdx.x; b < bins; b += blockDim.x)
    if (hist[b]) atomicAdd(counts + b, static_cast<unsigned long long>(hist[b]));
}

__global__ void cachegen_cdf_kernel(const unsigned long long* counts, int bins, int64_t n, float* cdf) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float run = 0.f;
  const float denom = static_cast<float>(n);
  cdf[0] = 0.f;
  for (int b = 0; b < bins; ++b) {
    run = __fadd_rn(run, static_cast<float>(counts[b]));
    cdf[b + 1] = __fdiv_rn(run, denom);
  }
}

__global__ void cachegen_decode_kernel(const uint8_t* codes, int64_t n, const void* codebook, int cb_dt, int bins,
                                       void* out, int out_dt) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int c = codes[i];
    const float v = c < bins ? load_f32(codebook, cb_dt, c) : 0.f;
    store_from_f32(out, out_dt, i, v);
  }
}

static bool float_dtype(int32_t dt) { return dt == MAK_DT_F16 || dt == MAK_DT_BF16 || dt == MAK_DT_F32; }

}  // namespace mak

using namespace mak;

extern "C" {

int mak_minmax(const void* x, int32_t dtype, int64_t n, float* out_minmax, void* stream) {
  if (!float_dtype(dtype)) return fail(MAK_E_INVALID, "mak_minmax: dtype must be f16/bf16/f32");
  if (n <= 0 || !x || !out_minmax) return fail(MAK_E_INVALID, "mak_minmax: empty input or NULL pointer");
  cudaStream_t st = as_stream(stream);
  uint32_t* keys = reinterpret_cast<uint32_t*>(out_minmax);
  cudaError_t e = cudaMemsetAsync(keys, 0xFF, sizeof(uint32_t), st);  // min key starts at the largest key
  if (e == cudaSuccess) e = cudaMemsetAsync(keys + 1, 0x00, sizeof(uint32_t), st);
  if (e != cudaSuccess) return cuda_fail(e, "mak_minmax: init");
  const int threads = 256;
  const int grid = grid_for(reinterpret_cast<const void*>(minmax_kernel), threads, 0, (n + threads - 1) / threads);
  minmax_kernel<<<grid, threads, 0, st>>>(x, dtype, n, keys);
  int rc = launch_status("minmax_kernel");
  if (rc) return rc;
  minmax_finish_kernel<<<1, 1, 0, st>>>(keys);
  return launch_status("minmax_finish_kernel");
}

int mak_cachegen_encode(const void* x, int32_t dtype, int64_t n, const float* minmax, int32_t num_bins, uint8_t* codes,
                        uint64_t* counts, float* cdf, void* stream) {
  if (!float_dtype(dtype)) return fail(MAK_E_INVALID, "mak_cachegen_encode: dtype must be f16/bf16/f32");
  if (num_bins < 2 || num_bins > 256) return fail(MAK_E_INVALID, "mak_cachegen_encode: num_bins must be in [2, 256]");
  if (n <= 0) return MAK_OK;
  if (!x || !minmax || !codes || !counts || !cdf) return fail(MAK_E_INVALID, "mak_cachegen_encode: NULL pointer");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(uint64_t) * num_bins, st);
  if (e != cudaSuccess) return cuda_fail(e, "mak_cachegen_encode: clear counts");
  const int threads = 256;
  const int grid = grid_for(reinterpret_cast<const void*>(cachegen_encode_kernel), threads, 0, (n + threads - 1) / threads);
  cachegen_encode_kernel<<<grid, threads, 0, st>>>(x, dtype, n, minmax, num_bins, codes,
                                                   reinterpret_cast<unsigned long long*>(counts));
  int rc = launch_status("cachegen_encode_kernel");
  if (rc) return rc;
  cachegen_cdf_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const unsigned long long*>(counts), num_bins, n, cdf);
  return launch_status("cachegen_cdf_kernel");
}

int mak_cachegen_decode(const uint8_t* codes, int64_t n, const void* codebook, int32_t codebook_dtype, int32_t num_bins,
                        void* out, int32_t out_dtype, void* stream) {
  if (!float_dtype(codebook_dtype) || !float_dtype(out_dtype))
    return fail(MAK_E_INVALID, "mak_cachegen_decode: codebook/output dtype must be f16/bf16/f32");
  if (num_bins < 1 || num_bins > 256) return fail(MAK_E_INVALID, "mak_cachegen_decode: bad codebook size");
  if (n <= 0) return MAK_OK;
  if (!codes || !codebook || !out) return fail(MAK_E_INVALID, "mak_cachegen_decode: NULL pointer");
  const int threads = 256;
  const int grid = grid_for(reinterpret_cast<const void*>(cachegen_decode_kernel), threads, 0, (n + threads - 1) / threads);
  cachegen_decode_kernel<<<grid, threads, 0, as_stream(stream)>>>(codes, n, codebook, codebook_dtype, num_bins, out,
                                                                  out_dtype);
  return launch_status("cachegen_decode_kernel");
}

}  // extern "C"
