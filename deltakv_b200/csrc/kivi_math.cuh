// KIVI int4 group arithmetic shared by the KIVI kernels and the fused KIVI subspace route.
// Groups of 32: scale = fp16(max(hi - lo, 1e-8) / 15), zero = fp16(lo), both rounded before the
// codes are formed; q = clamp(rint((x - zero) / scale), 0, 15) (0 when the fp16 scale is 0);
// x = q * scale + zero.  Each step is one IEEE fp32 operation (_rn intrinsics, no contraction),
// so results match the numpy restatement bit for bit.
#pragma once

#include "dkv_common.cuh"

namespace dkv {
namespace kivi {

constexpr int kG = 32;

// group parameters from the group's min and max
__device__ __forceinline__ void group_params(float lo, float hi, __half &s16, __half &z16) {
  const float rng = fmaxf(__fsub_rn(hi, lo), 1e-8f);
  s16 = __float2half_rn(__fdiv_rn(rng, 15.f));
  z16 = __float2half_rn(lo);
}

__device__ __forceinline__ uint32_t quant_one(float x, float s, float z) {
  float v = 0.f;
  if (s > 0.f) v = fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(x, z), s)), 0.f), 15.f);
  return static_cast<uint32_t>(v);
}

// the exact quotient, kept out of line so the common path does not carry the division
static __device__ __noinline__ float exact_quotient(float a, float s) { return __fdiv_rn(a, s); }

// Same result as quant_one, with the group's reciprocal: y = (x - z) * (1/s) is within 2 ulp
// of the IEEE quotient (|y| < 16, so 2 ulp < 4e-6), hence rint(y) equals rint(quotient) unless
// y lies within that distance of a rounding tie; there (|frac(y) - 1/2| < 1e-5) the quotient
// is formed exactly.  `inv` = 1/s rounded to nearest.
__device__ __forceinline__ uint32_t quant_one_fast(float x, float s, float z, float inv) {
  if (!(s > 0.f)) return 0u;
  const float a = __fsub_rn(x, z);
  float y = __fmul_rn(a, inv);
  if (__builtin_expect(fabsf(y - floorf(y) - 0.5f) < 1e-5f, 0)) y = exact_quotient(a, s);
  return static_cast<uint32_t>(fminf(fmaxf(rintf(y), 0.f), 15.f));
}

// a 4-bit code as a float (exact): 2^23 + q built in the mantissa, minus 2^23
__device__ __forceinline__ float code_to_f(uint32_t q) { return __int_as_float(0x4B000000u | q) - 8388608.f; }

// codes 2p, 2p+1 of a packed word as an fp32 pair (exact)
__device__ __forceinline__ uint64_t codes_to_f2(uint32_t w, int p) {
  const uint32_t lo = 0x4B000000u | ((w >> (8 * p)) & 0xFu), hi = 0x4B000000u | ((w >> (8 * p + 4)) & 0xFu);
  return sub2(f2pack(__uint_as_float(lo), __uint_as_float(hi)), f2pack(8388608.f, 8388608.f));
}

// The reciprocal form alone: rint(y) clamped to [0, 15] for y = (x - z) * RN(1/s) (y = 0 when
// s = 0).  Equal to the division form except where y lies within ~2 ulp of a rounding tie
// (a few in a million codes); for outputs that are not held to bit equality with the
// division form.
__device__ __forceinline__ uint32_t quant_recip(float y) {
  const uint32_t q = __float2uint_rn(y);
  return q < 15u ? q : 15u;
}

// quant_one's codes for a pair, through the reciprocal: y = (x - z) * RN(1/s) lies within 2 ulp
// (< 4e-6 for |y| < 16) of the IEEE quotient, so rint(y) equals rint(quotient) unless y is
// that close to a rounding tie; where either value of the pair is within 1e-5 of a tie
// (|y - rint(y)| > 1/2 - 1e-5) both quotients are formed exactly.  a2 = the (x - z) pair,
// s = the group's fp16 scale as a float, inv = RN(1/s) (0 when s = 0: every code is 0).
__device__ __forceinline__ void quant_pair(uint64_t a2, float s, float inv, uint32_t &q0, uint32_t &q1) {
  float y0, y1;
  f2unpack(mul2(a2, f2pack(inv, inv)), y0, y1);
  const float d0 = fabsf(__fsub_rn(y0, rintf(y0))), d1 = fabsf(__fsub_rn(y1, rintf(y1)));
  if (__builtin_expect(fmaxf(d0, d1) > 0.49999f, 0)) {
    float a0, a1;
    f2unpack(a2, a0, a1);
    y0 = exact_quotient(a0, s);
    y1 = exact_quotient(a1, s);
  }
  q0 = quant_recip(y0);
  q1 = quant_recip(y1);
}

__device__ __forceinline__ void quant_group(const float (&x)[kG], int cnt, uint8_t (&q)[kG], __half &s16,
                                            __half &z16) {
  float lo = x[0], hi = x[0];
#pragma unroll
  for (int i = 1; i < kG; ++i)
    if (i < cnt) {
      lo = fminf(lo, x[i]);
      hi = fmaxf(hi, x[i]);
    }
  group_params(lo, hi, s16, z16);
  const float s = __half2float(s16), z = __half2float(z16);
  const float inv = s > 0.f ? __frcp_rn(s) : 0.f;
#pragma unroll
  for (int i = 0; i < kG; ++i) q[i] = static_cast<uint8_t>(quant_one_fast(x[i], s, z, inv));
}

__device__ __forceinline__ float deq(uint32_t q, float s, float z) {
  return __fadd_rn(__fmul_rn(code_to_f(q), s), z);
}

}  // namespace kivi
}  // namespace dkv
