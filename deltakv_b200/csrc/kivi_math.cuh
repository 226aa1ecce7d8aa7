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
#pragma unroll
  for (int i = 0; i < kG; ++i) q[i] = static_cast<uint8_t>(quant_one(x[i], s, z));
}

__device__ __forceinline__ float deq(uint32_t q, float s, float z) {
  return __fadd_rn(__fmul_rn(static_cast<float>(q), s), z);
}

}  // namespace kivi
}  // namespace dkv
