// Element conversions and the musa-aiter FP8 codec shared by the tile engine
// and the MLA FP8 row kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "mak_kvcache.h"

namespace mak {

// ---- element conversions (round-to-nearest-even everywhere) ---------------
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

template <typename T>
__device__ __forceinline__ T zero_of() {
  T z;
  memset(&z, 0, sizeof(T));
  return z;
}

// ---- musa-aiter FP8 codec ---------------------------------------------------
// Encoder semantics (musa_aiter/ops/kv_transfer.py:2161-2183): w = x / scale in
// fp32; non-finite -> zero carrying the sign of (w < 0); |w| below the smallest
// normal -> signed zero; |w| clamped to (2 - 2^-m) * 2^emax (480 for E4M3 with
// exponent field 15 / mantissa 7, 114688 for E5M2 with exponent field 31); the
// mantissa rounds half-to-even.  Inside the formats' standard finite range this
// is exactly cvt.rn.satfinite; the extra top codes are handled explicitly.
__device__ __forceinline__ uint32_t cvt_e4m3(float a) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(r) : "f"(a));
  return r & 0xFFu;
}
__device__ __forceinline__ uint32_t cvt_e5m2(float a) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %1;" : "=h"(r) : "f"(a));
  return r & 0xFFu;
}

template <int F>
__device__ __forceinline__ uint8_t fp8_encode(float w) {
  const uint32_t sign = (w < 0.f) ? 0x80u : 0u;
  const float a = fabsf(w);
  if (!(a <= 3.40282346638528859812e+38f)) return static_cast<uint8_t>(sign);  // inf / nan
  if (F == MAK_FP8_E4M3) {
    if (a < 0.015625f) return static_cast<uint8_t>(sign);  // below 2^-6
    // 464 is the midpoint of 448 (mantissa 6) and 480 (mantissa 7): ties go to 448.
    if (a > 464.f) return static_cast<uint8_t>(sign | 0x7Fu);
    return static_cast<uint8_t>(sign | cvt_e4m3(a));
  } else {
    if (a < 6.103515625e-05f) return static_cast<uint8_t>(sign);  // below 2^-14
    if (a >= 61440.f) {
      // Exponent field 31: scale by 2^-16 (exact) into field 15, add 16 back.
      const float y = fminf(a, 114688.f) * 1.52587890625e-05f;
      return static_cast<uint8_t>(sign | (cvt_e5m2(y) + 0x40u));
    }
    return static_cast<uint8_t>(sign | cvt_e5m2(a));
  }
}

// Two values at once, same rule as fp8_encode: one paired conversion, the
// special ranges chosen per value with selects.  Returns code(w0) | code(w1) << 8.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_e5m2x2(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// fp8_encode2 with the sign read from separate values (g0, g1): the sign of
// w is the sign of g wherever the two differ only by rounding (see fast_quot).
template <int F>
__device__ __forceinline__ uint32_t fp8_encode2s(float g0, float w0, float g1, float w1) {
  const uint32_t s0 = (g0 < 0.f) ? 0x80u : 0u;
  const uint32_t s1 = (g1 < 0.f) ? 0x80u : 0u;
  const float a0 = fabsf(w0), a1 = fabsf(w1);
  const bool fin0 = a0 <= 3.40282346638528859812e+38f, fin1 = a1 <= 3.40282346638528859812e+38f;
  uint32_t c0, c1;
  if (F == MAK_FP8_E4M3) {
    const uint32_t c = cvt_e4m3x2(a1, a0);
    c0 = (a0 > 464.f) ? 0x7Fu : (c & 0xFFu);
    c1 = (a1 > 464.f) ? 0x7Fu : (c >> 8);
    c0 = (fin0 && a0 >= 0.015625f) ? c0 : 0u;
    c1 = (fin1 && a1 >= 0.015625f) ? c1 : 0u;
  } else {
    const bool top0 = a0 >= 61440.f, top1 = a1 >= 61440.f;
    const float y0 = top0 ? fminf(a0, 114688.f) * 1.52587890625e-05f : a0;
    const float y1 = top1 ? fminf(a1, 114688.f) * 1.52587890625e-05f : a1;
    const uint32_t c = cvt_e5m2x2(y1, y0);
    c0 = (c & 0xFFu) + (top0 ? 0x40u : 0u);
    c1 = (c >> 8) + (top1 ? 0x40u : 0u);
    c0 = (fin0 && a0 >= 6.103515625e-05f) ? c0 : 0u;
    c1 = (fin1 && a1 >= 6.103515625e-05f) ? c1 : 0u;
  }
  return (s0 | c0) | ((s1 | c1) << 8);
}

template <int F>
__device__ __forceinline__ uint32_t fp8_encode2(float w0, float w1) {
  return fp8_encode2s<F>(w0, w0, w1, w1);
}

// fp8_encode2s for callers whose finite values never exceed the format's
// standard maximum by more than rounding (|w| <= 448.001 for E4M3, 57344.01
// for E5M2: a value divided by its own group's amax / fp8_max).  The extended
// top codes are then unreachable and cvt.rn.satfinite rounds every in-range
// magnitude exactly as the reference rule does; what remains is the flush
// below the smallest normal, non-finite values (both to magnitude 0, decided
// by one range test on |w|) and the sign from g < 0.
template <int F>
__device__ __forceinline__ uint32_t fp8_encode2s_bounded(float g0, float w0, float g1, float w1) {
  constexpr float kMin = (F == MAK_FP8_E4M3) ? 0.015625f : 6.103515625e-05f;
  const float a0 = fabsf(w0), a1 = fabsf(w1);
  const float v0 = (a0 >= kMin && a0 <= 3.40282346638528859812e+38f) ? a0 : 0.f;
  const float v1 = (a1 >= kMin && a1 <= 3.40282346638528859812e+38f) ? a1 : 0.f;
  const uint32_t c = (F == MAK_FP8_E4M3) ? cvt_e4m3x2(v1, v0) : cvt_e5m2x2(v1, v0);
  return c | ((g0 < 0.f) ? 0x80u : 0u) | ((g1 < 0.f) ? 0x8000u : 0u);
}

// fp8_encode2s_bounded for a pair of finite values (w0, w1: the correctly
// rounded quotients x / s, e.g. fast_quot's q1).  The reference's flush of
// |w| < 2^-6 (E4M3) / 2^-14 (E5M2) to a signed zero is one flush-to-zero
// multiply by 2^-K (K = 120 / 112 puts the threshold on fp32's smallest
// normal, so the product is exact above it and flushed below it), undone by a
// multiply by 2^K; the signed result then goes straight through
// cvt.rn.satfinite.  Its sign equals the reference's (w < 0) rule for every
// finite x: x = -0 gives q1 = +0 (the remainder step adds +0 to -0), and a
// flushed negative value keeps its sign.  Four multiplies, no compares.
template <int F>
__device__ __forceinline__ uint32_t fp8_encode2_finite(float w0, float w1);

// x / s rounded to nearest in fp32 without a division per value, by
// Markstein's correction step (P. Markstein, "IA-64 and Elementary Functions",
// 2000): with y = RN(1/s) and q0 = RN(x * y), q0 is within one ulp of x / s,
// the remainder r = x - s * q0 is exact in one fma, and RN(q0 + r * y) is the
// correctly rounded quotient, as long as r does not underflow.  For s in
// [2^-60, 2^16] (fast_quot_ok) and |x / s| at most a few times the FP8
// maximum, that holds wherever the FP8 code depends on the magnitude
// (|x / s| >= 2^-14); below that only the sign and non-zero-ness of the
// quotient reach the encoder, and q0 and q1 both keep them (|x / s| >= 2^-149
// for every non-zero 16-bit x).  Non-finite x: q0 = x * y carries the IEEE
// quotient's sign and class while q1 is nan, so callers read the sign from q0
// (fp8_encode2s).  mak_fp8_quotient_selfcheck compares the path with the IEEE
// division for every 16-bit input and every scale significand.
struct FastQuot {
  float q0, q1;
};
__device__ __forceinline__ bool fast_quot_ok(float s) { return s >= 0x1p-60f && s <= 0x1p16f; }
__device__ __forceinline__ FastQuot fast_quot(float x, float s, float y) {
  const float q0 = __fmul_rn(x, y);
  const float r = __fmaf_rn(-q0, s, x);
  return {q0, __fmaf_rn(r, y, q0)};
}

// Decoder (musa_aiter/ops/kv_transfer.py:2186-2200): exponent field 0 -> 0,
// otherwise (1 + m / 2^mb) * 2^(e - bias), all codes finite; built bit-exactly.
template <int F>
__device__ __forceinline__ float fp8_decode(uint32_t code) {
  constexpr int mb = (F == MAK_FP8_E4M3) ? 3 : 2;
  constexpr int bias = (F == MAK_FP8_E4M3) ? 7 : 15;
  const uint32_t e = (code >> mb) & ((1u << (7 - mb)) - 1u);
  const uint32_t m = code & ((1u << mb) - 1u);
  uint32_t bits = e ? (((e - bias + 127u) << 23) | (m << (23 - mb))) : 0u;
  bits |= (code & 0x80u) << 24;
  return __uint_as_float(bits);
}

// The same decoder for a code held in the top byte of x (the low 24 bits zero,
// as __byte_perm leaves it): the magnitude bits shift straight into the fp32
// exponent and mantissa fields, the exponent bias is one add, and exponent
// field 0 keeps only the sign.
template <int F>
__device__ __forceinline__ float fp8_decode_top(uint32_t x) {
  constexpr int mb = (F == MAK_FP8_E4M3) ? 3 : 2;
  constexpr int bias = (F == MAK_FP8_E4M3) ? 7 : 15;
  constexpr uint32_t kMag = 0x7Fu << (23 - mb);
  constexpr uint32_t kExp = ((1u << (7 - mb)) - 1u) << (24 + mb);
  const uint32_t sign = x & 0x80000000u;
  const uint32_t bits = (((x >> (1 + mb)) & kMag) + (static_cast<uint32_t>(127 - bias) << 23)) | sign;
  return __uint_as_float((x & kExp) ? bits : sign);
}

// Flush-to-zero decode (fast path of the MLA row loader).  The code's seven
// magnitude bits go straight into the fp32 exponent and mantissa fields with
// no bias added, so the code's exponent field e becomes the fp32 exponent
// field: e >= 1 gives 2^(e - 127) * (1 + m / 2^mb), a normal number, and e = 0
// gives an fp32 subnormal or zero.  One flush-to-zero multiply by
// s' = s * 2^(127 - bias) then yields RN(decode(code) * s) exactly: the power
// of two moves no rounding point, a subnormal input (e = 0) becomes the
// signed zero that the reference decoder gives, and no product is subnormal
// or overflows differently while s lies in [2^(bias - 127), 2^(bias + 1))
// (fp8_ftz_scale_ok).  The code sits in the top byte of x; the arithmetic
// shift copies its sign over the bits that the mask then clears.
template <int F>
__device__ __forceinline__ float fp8_raw_top(uint32_t x) {
  constexpr int sh = (F == MAK_FP8_E4M3) ? 4 : 3;
  constexpr uint32_t mask = (F == MAK_FP8_E4M3) ? 0x87F00000u : 0x8FE00000u;
  return __uint_as_float(static_cast<uint32_t>(static_cast<int32_t>(x) >> sh) & mask);
}
template <int F>
__device__ __forceinline__ float fp8_ftz_bias() {
  return F == MAK_FP8_E4M3 ? 0x1p120f : 0x1p112f;
}
template <int F>
__device__ __forceinline__ bool fp8_ftz_scale_ok(float s) {
  return F == MAK_FP8_E4M3 ? (s >= 0x1p-120f && s < 0x1p8f) : (s >= 0x1p-112f && s < 0x1p16f);
}
__device__ __forceinline__ float fmul_ftz(float a, float b) {
  float r;
  asm("mul.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Packed fp32 pairs (sm_100 .f32x2 arithmetic): each element is rounded
// exactly as the scalar operation would round it, two values per instruction.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul_ftz(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Per-group constants of the packed store path: the scale s, -s and y = RN(1/s)
// (fast_quot_ok(s) must hold), each in both halves.
struct QuotPair {
  uint64_t y, neg_s;
};
__device__ __forceinline__ QuotPair quot_pair(float s, float y) { return {f2_pack(y, y), f2_pack(-s, -s)}; }

// fast_quot + fp8_encode2_finite on a pair (x0, x1) of finite values in five
// packed operations: q0 = x * y, r = x - q0 * s (exact), q1 = q0 + r * y, then
// the flush-to-zero multiply pair.  Returns code(x0) | code(x1) << 8.
template <int F>
__device__ __forceinline__ uint32_t fp8_encode2_quot_finite(float x0, float x1, const QuotPair& c) {
  constexpr float kDown = (F == MAK_FP8_E4M3) ? 0x1p-120f : 0x1p-112f;
  constexpr float kUp = (F == MAK_FP8_E4M3) ? 0x1p120f : 0x1p112f;
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t q0 = f2_mul(x, c.y);
  const uint64_t r = f2_fma(q0, c.neg_s, x);
  const uint64_t q1 = f2_fma(r, c.y, q0);
  const uint64_t v = f2_mul(f2_mul_ftz(q1, f2_pack(kDown, kDown)), f2_pack(kUp, kUp));
  float v0, v1;
  f2_unpack(v, v0, v1);
  return (F == MAK_FP8_E4M3) ? cvt_e4m3x2(v1, v0) : cvt_e5m2x2(v1, v0);
}

template <int F>
__device__ __forceinline__ uint32_t fp8_encode2_finite(float w0, float w1) {
  constexpr float kDown = (F == MAK_FP8_E4M3) ? 0x1p-120f : 0x1p-112f;
  constexpr float kUp = (F == MAK_FP8_E4M3) ? 0x1p120f : 0x1p112f;
  const float v0 = __fmul_rn(fmul_ftz(w0, kDown), kUp);
  const float v1 = __fmul_rn(fmul_ftz(w1, kDown), kUp);
  return (F == MAK_FP8_E4M3) ? cvt_e4m3x2(v1, v0) : cvt_e5m2x2(v1, v0);
}

}  // namespace mak
