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

// ---- packed forms for the fused route (one word = 8 codes, element j in bits 4j..4j+3) ----
//
// Decode without per-code shifts: nibble j of w (j < 4) or of w >> 16 (j >= 4) is masked in
// place and ORed under the exponent of 2^23, giving the float 2^23 + n_j 16^e (e = j mod 4,
// n_j 16^e < 2^16, so the float is exact); subtracting 2^23 is exact.  The factor 16^e is
// folded into the scale, s 16^-e (an exact power-of-two rescaling of an fp16 value), so
// fma(n_j 16^e, s 16^-e, z) = RN(n_j s + z): n_j s is exact in fp32 (4 x 11 significant bits),
// which makes this single rounding the reference's q * s + z.
// Pairs p = 0..3 hold elements (2p, 2p + 1), rescaled by 16^-e = (1, 1/16) for even p and
// (1/256, 1/4096) for odd p (pair_rescale).
__device__ __forceinline__ void code_pairs(uint32_t w, uint64_t (&raw)[4]) {
  const uint32_t h = w >> 16, m = 0x4B000000u;
  const uint64_t bias = f2pack(8388608.f, 8388608.f);
  raw[0] = sub2(f2pack(__uint_as_float((w & 0xFu) | m), __uint_as_float((w & 0xF0u) | m)), bias);
  raw[1] = sub2(f2pack(__uint_as_float((w & 0xF00u) | m), __uint_as_float((w & 0xF000u) | m)), bias);
  raw[2] = sub2(f2pack(__uint_as_float((h & 0xFu) | m), __uint_as_float((h & 0xF0u) | m)), bias);
  raw[3] = sub2(f2pack(__uint_as_float((h & 0xF00u) | m), __uint_as_float((h & 0xF000u) | m)), bias);
}
__device__ __forceinline__ uint64_t pair_rescale(int p) {
  return (p & 1) ? f2pack(0.00390625f, 0.000244140625f) : f2pack(1.f, 0.0625f);
}

// round to nearest even (ties to even, as rintf) as a signed integer
__device__ __forceinline__ int rni(float y) {
  int r;
  asm("cvt.rni.s32.f32 %0, %1;" : "=r"(r) : "f"(y));
  return r;
}
// (c << 8) | (clamp(a, 0, 15) << 4) | clamp(b, 0, 15): two codes saturated to [0, 15] and
// shifted in below c (PTX cvt.pack.sat.u4.s32.b32)
__device__ __forceinline__ uint32_t pack_u4(int a, int b, uint32_t c) {
  uint32_t d;
  asm("cvt.pack.sat.u4.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// the word of 8 codes clamp(rint((x_j - z_j) * inv_j), 0, 15) for the value pairs v[p] =
// (x_2p, x_2p+1) with the pairs' (z, inv) in z2[p], i2[p]
__device__ __forceinline__ uint32_t quant_word(const uint64_t (&v)[4], const uint64_t (&z2)[4],
                                               const uint64_t (&i2)[4]) {
  uint32_t w = 0u;
#pragma unroll
  for (int p = 3; p >= 0; --p) {
    float y0, y1;
    f2unpack(mul2(sub2(v[p], z2[p]), i2[p]), y0, y1);
    w = pack_u4(rni(y1), rni(y0), w);
  }
  return w;
}

// three-input minimum / maximum (sm_100)
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmin8(const float (&x)[8]) {
  return fminf(fmin3(fmin3(x[0], x[1], x[2]), fmin3(x[3], x[4], x[5]), x[6]), x[7]);
}
__device__ __forceinline__ float fmax8(const float (&x)[8]) {
  return fmaxf(fmax3(fmax3(x[0], x[1], x[2]), fmax3(x[3], x[4], x[5]), x[6]), x[7]);
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
