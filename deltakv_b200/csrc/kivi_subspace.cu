// Subspace correction of a KIVI int4 KV cache, batched over (layer, projection) problems.
//
// Reference: deltakv.patches.subspace.subspace_correct (src/deltakv/patches/subspace.py:45-106)
// applied to a cache whose reused KV is stored KIVI int4 and whose corrected KV is written back
// in the same format (the multi-adapter maintenance step: every adapter view patches the
// shared int4 prefix):
//   reused = dequant(base);  R = fresh - reused
//   rhs = R B;  codes = rhs (B^T B + 1e-6 I)^-1;  fitted = codes B^T
//   orth_mu = mean_P(R - fitted);  w = min(||R|| / mean ||R||, 1)
//   corr = reused + fitted + w orth_mu;  corr[P] = fresh[P];  out = quant(corr)
// All problems of a call share d; each has its own token count, probes, basis (rank <= 64)
// and caches.  Launches (all problems at once):
//   flags   probe flags and probe count (probe indices are deduplicated)
//   pack    basis -> bf16, transposed copy for the first product, row copy for the second
//   pass1   dequant, R, ||R||, rhs = R B (mma.sync bf16, fp32 accumulate), sums
//   solve   one CTA per problem: (B^T B + 1e-6 I)^-1 in fp64, orth_mu, subspace, mean ||R||
//   pass2   codes = rhs G^-1, fitted = codes B^T (mma.sync bf16), corr, requantise
// The products use the basis rounded to bf16 (B~) throughout — G is formed from B~ as well —
// so `fitted` is the least-squares projection onto col(B~); R and the codes are rounded to
// bf16 as MMA operands.  These roundings sit far below the int4 step of the output.
#include <cstring>
#include <vector>

#include "dkv_common.cuh"
#include "kivi_math.cuh"

namespace dkv {
namespace ksub {

constexpr int kTM = 64;  // tokens per tile (two K groups)
constexpr int kKC = 64;  // channels per chunk
constexpr int kThreads = 256;
constexpr int kMaxRank = 64;
constexpr int kBP = 8;  // bf16 row padding (16 bytes) against ldmatrix bank conflicts

struct Prob {
  const uint8_t *codes;
  const __half *scale, *zero;
  int64_t crs, szrs;
  uint8_t *o_codes;
  __half *o_scale, *o_zero;
  int64_t o_crs, o_szrs;
  const void *fresh;
  int64_t frs;
  int64_t n;
  const int32_t *probes;
  int64_t n_probes;
  float *sub_out, *mu_out;
  // workspace
  float *rhs, *dist, *sums, *ginv, *mu, *subv;
  uint32_t *flag;
  __nv_bfloat16 *bt, *bb;
  const float *basis;
  int64_t tile0;
  int r, mode;
};

constexpr int kMaxProblems = 128;

// The problem table travels in the kernel parameters (read through the constant cache).
struct Batch {
  int n_probs;
  int64_t d, n_tiles;
  int32_t *status;
  Prob probs[kMaxProblems];
};
static_assert(sizeof(Batch) <= 32000, "kernel parameter limit");

// sums layout: [0] sum ||R||, [1] probe count, [2, 2+RP) sum rhs (all tokens),
// [2+RP, 2+2RP) sum rhs (probes), [2+2RP, 2+2RP+d) sum_P R
__device__ __forceinline__ int find_prob(const Batch &b, int64_t tile) {
  int lo = 0, hi = b.n_probs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.probs[mid].tile0 <= tile) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int FDT>
__device__ __forceinline__ void load16(const void *base, int64_t off, float (&v)[16]) {
  if (FDT == DKV_F32) {
    const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + off);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 q = p[i];
      v[4 * i] = q.x, v[4 * i + 1] = q.y, v[4 * i + 2] = q.z, v[4 * i + 3] = q.w;
    }
  } else {
    const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + off);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 q = p[i];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * i + 2 * j] = FDT == DKV_BF16 ? bf16lo(w[j]) : f16lo(w[j]);
        v[8 * i + 2 * j + 1] = FDT == DKV_BF16 ? bf16hi(w[j]) : f16hi(w[j]);
      }
    }
  }
}

template <int FDT>
__device__ __forceinline__ float load1(const void *base, int64_t off) {
  if (FDT == DKV_F32) return static_cast<const float *>(base)[off];
  if (FDT == DKV_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(base)[off]);
  return __half2float(static_cast<const __half *>(base)[off]);
}

// 16 dequantised values of token t, channels [c, c+16) (c % 16 == 0)
__device__ __forceinline__ void deq16(const Prob &P, int64_t t, int64_t c, float (&v)[16]) {
  const uint2 q = *reinterpret_cast<const uint2 *>(P.codes + t * P.crs + c / 2);
  const uint32_t w[2] = {q.x, q.y};
  if (P.mode == DKV_KIVI_PER_TOKEN) {
    const float s = __half2float(P.scale[t * P.szrs + c / kivi::kG]);
    const float z = __half2float(P.zero[t * P.szrs + c / kivi::kG]);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = kivi::deq((w[i >> 3] >> (4 * (i & 7))) & 0xFu, s, z);
  } else {
    const int64_t so = (t / kivi::kG) * P.szrs + c;
    const uint4 *sp = reinterpret_cast<const uint4 *>(P.scale + so);
    const uint4 *zp = reinterpret_cast<const uint4 *>(P.zero + so);
    uint32_t sw[8], zw[8];
    {
      const uint4 a = sp[0], b = sp[1], e = zp[0], f = zp[1];
      sw[0] = a.x, sw[1] = a.y, sw[2] = a.z, sw[3] = a.w, sw[4] = b.x, sw[5] = b.y, sw[6] = b.z, sw[7] = b.w;
      zw[0] = e.x, zw[1] = e.y, zw[2] = e.z, zw[3] = e.w, zw[4] = f.x, zw[5] = f.y, zw[6] = f.z, zw[7] = f.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float s = (i & 1) ? f16hi(sw[i >> 1]) : f16lo(sw[i >> 1]);
      const float z = (i & 1) ? f16hi(zw[i >> 1]) : f16lo(zw[i >> 1]);
      v[i] = kivi::deq((w[i >> 3] >> (4 * (i & 7))) & 0xFu, s, z);
    }
  }
}

// ---------------------------------------------------------------------------------------
__global__ void flags_kernel(const __grid_constant__ Batch b) {
  const Prob &P = b.probs[blockIdx.y];
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < P.n_probes;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = P.probes[i];
    if (t < 0 || t >= P.n) {
      record_error(b.status, DKV_ERR_INVALID_ARGUMENT);
      continue;
    }
    if (atomicExch(&P.flag[t], 1u) == 0u) atomicAdd(&P.sums[1], 1.f);
  }
}

// basis fp32 [d, r] -> bt [RP, d] and bb [d, RP] bf16, zero beyond r
__global__ void pack_kernel(const __grid_constant__ Batch b, int rp) {
  const Prob &P = b.probs[blockIdx.y];
  const int64_t total = b.d * rp;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = e / rp;
    const int k = static_cast<int>(e - c * rp);
    const float v = (k < P.r && P.basis != nullptr) ? P.basis[c * P.r + k] : 0.f;
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    P.bb[c * rp + k] = h;
    P.bt[static_cast<int64_t>(k) * b.d + c] = h;
  }
}

// ---------------------------------------------------------------------------------------
// pass 1
// ---------------------------------------------------------------------------------------
template <int RP, int FDT>
__global__ void __launch_bounds__(kThreads) pass1_kernel(const __grid_constant__ Batch b) {
  __shared__ __align__(16) __nv_bfloat16 Rs[kTM][kKC + kBP];
  __shared__ __align__(16) __nv_bfloat16 Bts[RP][kKC + kBP];
  __shared__ float sPR[kKC];
  __shared__ float sRhs[2][RP];
  __shared__ float red[kThreads / 32];
  __shared__ uint32_t sflag[kTM];
  __shared__ int any_probe;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const Prob &P = b.probs[find_prob(b, blockIdx.x)];
  const int64_t t0 = (blockIdx.x - P.tile0) * kTM;
  const int64_t n = P.n;
  if (tid == 0) any_probe = 0;
  __syncthreads();
  if (tid < kTM) {
    const uint32_t f = (t0 + tid < n) ? P.flag[t0 + tid] : 0u;
    sflag[tid] = f;
    if (f) any_probe = 1;
  }
  if (tid < kKC) sPR[tid] = 0.f;
  for (int e = tid; e < 2 * RP; e += kThreads) sRhs[e / RP][e % RP] = 0.f;
  __syncthreads();

  const int lt = tid >> 2, lc = (tid & 3) * 16;
  const int64_t tok = t0 + lt;
  const bool tv = tok < n;
  const bool myflag = tv && sflag[lt] != 0u;
  float dist2 = 0.f;
  const int mb = warp & 3, nb = warp >> 2;
  constexpr int NT = RP / 16;  // 8-wide n-tiles per warp (half of RP each)
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  for (int64_t c0 = 0; c0 < b.d; c0 += kKC) {
    {
      float f[16], rv[16];
      if (tv) {
        load16<FDT>(P.fresh, tok * P.frs + c0 + lc, f);
        deq16(P, tok, c0 + lc, rv);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) f[i] = rv[i] = 0.f;
      }
      uint32_t pk[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float r0 = f[2 * i] - rv[2 * i], r1 = f[2 * i + 1] - rv[2 * i + 1];
        dist2 = fmaf(r0, r0, dist2);
        dist2 = fmaf(r1, r1, dist2);
        pk[i] = pack_bf16x2(r0, r1);
        if (myflag) {
          atomicAdd(&sPR[lc + 2 * i], r0);
          atomicAdd(&sPR[lc + 2 * i + 1], r1);
        }
      }
      uint4 *dst = reinterpret_cast<uint4 *>(&Rs[lt][lc]);
      dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    for (int e = tid; e < RP * (kKC / 8); e += kThreads) {
      const int k = e / (kKC / 8), j = e % (kKC / 8);
      *reinterpret_cast<uint4 *>(&Bts[k][8 * j]) =
          *reinterpret_cast<const uint4 *>(P.bt + static_cast<int64_t>(k) * b.d + c0 + 8 * j);
    }
    __syncthreads();
    if (any_probe && tid < kKC) {
      atomicAdd(&P.sums[2 + 2 * RP + c0 + tid], sPR[tid]);
      sPR[tid] = 0.f;
    }
#pragma unroll
    for (int ks = 0; ks < kKC / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, smem_u32(&Rs[16 * mb + (lane & 15)][16 * ks + ((lane >> 4) << 3)]));
      const int nbase = nb * (RP / 2);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3,
                    smem_u32(&Bts[nbase + 16 * np + ((lane >> 4) << 3) + (lane & 7)][16 * ks + (((lane >> 3) & 1) << 3)]));
        mma16816_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
      if (NT & 1) {
        uint32_t b0, b1;
        ldmatrix_x2(b0, b1, smem_u32(&Bts[nbase + 16 * (NT / 2) + (lane & 7)][16 * ks + (((lane >> 3) & 1) << 3)]));
        mma16816_bf16(acc[NT - 1], a0, a1, a2, a3, b0, b1);
      }
    }
    __syncthreads();
  }

  // ||R|| per token (4 loader threads per token)
  dist2 += __shfl_xor_sync(0xffffffffu, dist2, 1);
  dist2 += __shfl_xor_sync(0xffffffffu, dist2, 2);
  float dsum = 0.f;
  if ((tid & 3) == 0 && tv) {
    const float dd = sqrtf(dist2);
    P.dist[tok] = dd;
    dsum = dd;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  if (lane == 0) red[warp] = dsum;

  // rhs rows and column sums (all tokens, probes)
  const int g = lane >> 2, q = lane & 3;
  const int ra = 16 * mb + g, rb = ra + 8;
  const bool va = t0 + ra < n, vb = t0 + rb < n;
  const bool fa = va && sflag[ra] != 0u, fb = vb && sflag[rb] != 0u;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int col = nb * (RP / 2) + 8 * nt + 2 * q;
    if (va) *reinterpret_cast<float2 *>(P.rhs + (t0 + ra) * RP + col) = make_float2(acc[nt][0], acc[nt][1]);
    if (vb) *reinterpret_cast<float2 *>(P.rhs + (t0 + rb) * RP + col) = make_float2(acc[nt][2], acc[nt][3]);
    float s0 = (va ? acc[nt][0] : 0.f) + (vb ? acc[nt][2] : 0.f);
    float s1 = (va ? acc[nt][1] : 0.f) + (vb ? acc[nt][3] : 0.f);
    float p0 = (fa ? acc[nt][0] : 0.f) + (fb ? acc[nt][2] : 0.f);
    float p1 = (fa ? acc[nt][1] : 0.f) + (fb ? acc[nt][3] : 0.f);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      p0 += __shfl_xor_sync(0xffffffffu, p0, o);
      p1 += __shfl_xor_sync(0xffffffffu, p1, o);
    }
    if (g == 0) {
      atomicAdd(&sRhs[0][col], s0);
      atomicAdd(&sRhs[0][col + 1], s1);
      atomicAdd(&sRhs[1][col], p0);
      atomicAdd(&sRhs[1][col + 1], p1);
    }
  }
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) s += red[i];
    atomicAdd(&P.sums[0], s);
  }
  if (tid < RP) {
    atomicAdd(&P.sums[2 + tid], sRhs[0][tid]);
    if (any_probe) atomicAdd(&P.sums[2 + RP + tid], sRhs[1][tid]);
  }
}

// ---------------------------------------------------------------------------------------
// solve: one CTA per problem
// ---------------------------------------------------------------------------------------
template <int RP>
__global__ void __launch_bounds__(kThreads) solve_kernel(const __grid_constant__ Batch b) {
  extern __shared__ double Mdyn[];  // [r][2r + 1]: [G | I]
  __shared__ float cp[RP], ca[RP];
  __shared__ double fac[RP];
  __shared__ int piv_row;
  const Prob &P = b.probs[blockIdx.x];
  const int r = P.r;
  const int ldm = 2 * r + 1;
  const float np = P.sums[1];
  for (int e = threadIdx.x; e < RP * RP; e += blockDim.x) P.ginv[e] = 0.f;
  if (threadIdx.x < RP) cp[threadIdx.x] = ca[threadIdx.x] = 0.f;
  __syncthreads();
  if (r > 0) {
    for (int e = threadIdx.x; e < r * r; e += blockDim.x) {
      const int i = e / r, j = e % r;
      double s = 0.0;
      for (int64_t c = 0; c < b.d; ++c)
        s += static_cast<double>(__bfloat162float(P.bb[c * RP + i])) * __bfloat162float(P.bb[c * RP + j]);
      Mdyn[i * ldm + j] = s + (i == j ? 1e-6 : 0.0);
      Mdyn[i * ldm + r + j] = (i == j) ? 1.0 : 0.0;
    }
    __syncthreads();
    for (int col = 0; col < r; ++col) {
      if (threadIdx.x == 0) {
        int best = col;
        double bv = fabs(Mdyn[col * ldm + col]);
        for (int i = col + 1; i < r; ++i)
          if (fabs(Mdyn[i * ldm + col]) > bv) {
            bv = fabs(Mdyn[i * ldm + col]);
            best = i;
          }
        piv_row = best;
      }
      __syncthreads();
      const int pr = piv_row;
      if (pr != col)
        for (int j = threadIdx.x; j < 2 * r; j += blockDim.x) {
          const double t = Mdyn[col * ldm + j];
          Mdyn[col * ldm + j] = Mdyn[pr * ldm + j];
          Mdyn[pr * ldm + j] = t;
        }
      __syncthreads();
      const double inv = 1.0 / Mdyn[col * ldm + col];
      __syncthreads();
      for (int j = threadIdx.x; j < 2 * r; j += blockDim.x) Mdyn[col * ldm + j] *= inv;
      for (int i = threadIdx.x; i < r; i += blockDim.x) fac[i] = Mdyn[i * ldm + col];
      __syncthreads();
      for (int e = threadIdx.x; e < r * 2 * r; e += blockDim.x) {
        const int i = e / (2 * r), j = e % (2 * r);
        if (i != col) Mdyn[i * ldm + j] -= fac[i] * Mdyn[col * ldm + j];
      }
      __syncthreads();
    }
    for (int e = threadIdx.x; e < r * r; e += blockDim.x)
      P.ginv[(e / r) * RP + e % r] = static_cast<float>(Mdyn[(e / r) * ldm + r + e % r]);
    if (threadIdx.x < r) {
      const int j = threadIdx.x;
      double sp = 0.0, sa = 0.0;
      for (int i = 0; i < r; ++i) {
        sp += static_cast<double>(P.sums[2 + RP + i]) * Mdyn[i * ldm + r + j];
        sa += static_cast<double>(P.sums[2 + i]) * Mdyn[i * ldm + r + j];
      }
      cp[j] = np > 0 ? static_cast<float>(sp / np) : 0.f;
      ca[j] = P.n > 0 ? static_cast<float>(sa / static_cast<double>(P.n)) : 0.f;
    }
    __syncthreads();
  }
  for (int64_t c = threadIdx.x; c < b.d; c += blockDim.x) {
    float fp = 0.f, fa = 0.f;
    for (int i = 0; i < r; ++i) {
      const float bv = __bfloat162float(P.bb[c * RP + i]);
      fp = fmaf(cp[i], bv, fp);
      fa = fmaf(ca[i], bv, fa);
    }
    const float meanR = np > 0 ? P.sums[2 + 2 * RP + c] / np : 0.f;
    P.mu[c] = meanR - fp;
    P.subv[c] = fa;
    if (P.mu_out) P.mu_out[c] = meanR - fp;
    if (P.sub_out) P.sub_out[c] = fa;
  }
  if (threadIdx.x == 0) P.subv[b.d] = fmaxf(P.n > 0 ? P.sums[0] / static_cast<float>(P.n) : 0.f, 1e-8f);
}

// ---------------------------------------------------------------------------------------
// pass 2
// ---------------------------------------------------------------------------------------
template <int RP>
struct Pass2Smem {
  union {
    struct {
      float G[RP][RP + 1];   // G^-1
      float Rt[kTM][RP + 1];  // rhs rows of the tile
    } pro;
    struct {
      float Y[kTM][kKC + 1];                       // reused, then corrected values of a chunk
      __nv_bfloat16 Bb[kKC][RP + kBP];             // basis rows of the chunk
    } loop;
  } u;
  __nv_bfloat16 Cb[kTM][RP + kBP];  // codes of the tile (mma A operand)
  float w[kTM], mus[kKC];
  uint32_t fl[kTM];
};

template <int RP, int FDT>
__global__ void __launch_bounds__(kThreads) pass2_kernel(const __grid_constant__ Batch b) {
  __shared__ __align__(16) Pass2Smem<RP> S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const Prob &P = b.probs[find_prob(b, blockIdx.x)];
  const int64_t t0 = (blockIdx.x - P.tile0) * kTM;
  const int64_t n = P.n;
  const float mean_dist = P.subv[b.d];

  // ---- prologue: codes = rhs G^-1 (fp32), token weights, probe flags ----
  for (int e = tid; e < RP * RP; e += kThreads) S.u.pro.G[e / RP][e % RP] = P.ginv[e];
  for (int e = tid; e < kTM * RP; e += kThreads) {
    const int t = e / RP, k = e % RP;
    S.u.pro.Rt[t][k] = (t0 + t < n) ? P.rhs[(t0 + t) * RP + k] : 0.f;
  }
  if (tid < kTM) {
    const int64_t t = t0 + tid;
    const bool v = t < n;
    S.fl[tid] = v ? P.flag[t] : 0u;
    S.w[tid] = v ? fminf(P.dist[t] / mean_dist, 1.f) : 0.f;
  }
  __syncthreads();
  for (int e = tid; e < kTM * RP; e += kThreads) {
    const int t = e / RP, k = e % RP;
    float s = 0.f;
#pragma unroll 8
    for (int i = 0; i < RP; ++i) s = fmaf(S.u.pro.Rt[t][i], S.u.pro.G[i][k], s);
    S.Cb[t][k] = __float2bfloat16_rn(s);
  }
  __syncthreads();

  const int lt = tid >> 2, lc = (tid & 3) * 16;
  const int64_t tok = t0 + lt;
  const bool tv = tok < n;
  const int mb = warp & 3, nb = warp >> 2;
  const int g = lane >> 2, q = lane & 3;
  const bool per_token = P.mode == DKV_KIVI_PER_TOKEN;

  for (int64_t c0 = 0; c0 < b.d; c0 += kKC) {
    // ---- reused values of the chunk, basis rows, orth_mu ----
    {
      float rv[16];
      if (tv) deq16(P, tok, c0 + lc, rv);
      else
#pragma unroll
        for (int i = 0; i < 16; ++i) rv[i] = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) S.u.loop.Y[lt][lc + i] = rv[i];
    }
    for (int e = tid; e < kKC * (RP / 8); e += kThreads) {
      const int c = e / (RP / 8), j = e % (RP / 8);
      *reinterpret_cast<uint4 *>(&S.u.loop.Bb[c][8 * j]) =
          *reinterpret_cast<const uint4 *>(P.bb + (c0 + c) * RP + 8 * j);
    }
    if (tid < kKC) S.mus[tid] = P.mu[c0 + tid];
    __syncthreads();

    // ---- fitted = codes B^T for 16 tokens x 32 channels per warp ----
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < RP / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(a0, a1, a2, a3, smem_u32(&S.Cb[16 * mb + (lane & 15)][16 * ks + ((lane >> 4) << 3)]));
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3,
                    smem_u32(&S.u.loop.Bb[32 * nb + 16 * np + ((lane >> 4) << 3) + (lane & 7)]
                                         [16 * ks + (((lane >> 3) & 1) << 3)]));
        mma16816_bf16(acc[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816_bf16(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- corr = reused + fitted + w orth_mu; probes take fresh ----
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mb + g + 8 * h;
        const int col = 32 * nb + 8 * nt + 2 * q;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v;
          if (S.fl[row]) {
            v = load1<FDT>(P.fresh, (t0 + row) * P.frs + c0 + col + e);
          } else {
            v = __fadd_rn(__fadd_rn(S.u.loop.Y[row][col + e], acc[nt][2 * h + e]),
                          __fmul_rn(S.w[row], S.mus[col + e]));
          }
          S.u.loop.Y[row][col + e] = v;
        }
      }
    }
    __syncthreads();

    // ---- requantise the chunk ----
    if (per_token) {
      // (token, 32-channel group) per thread pair, 16 channels each
      const int item = tid >> 1, half = tid & 1;
      const int rt = item >> 1, gg = item & 1;
      const int cb = 32 * gg + 16 * half;
      float x[16];
      float lo = INFINITY, hi = -INFINITY;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        x[j] = S.u.loop.Y[rt][cb + j];
        lo = fminf(lo, x[j]);
        hi = fmaxf(hi, x[j]);
      }
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, 1));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, 1));
      __half s16, z16;
      kivi::group_params(lo, hi, s16, z16);
      const float s = __half2float(s16), z = __half2float(z16);
      uint32_t wq[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 16; ++j) wq[j >> 3] |= kivi::quant_one(x[j], s, z) << (4 * (j & 7));
      const int64_t t = t0 + rt;
      if (t < n) {
        *reinterpret_cast<uint2 *>(P.o_codes + t * P.o_crs + (c0 + cb) / 2) = make_uint2(wq[0], wq[1]);
        if (half == 0) {
          P.o_scale[t * P.o_szrs + (c0 + 32 * gg) / kivi::kG] = s16;
          P.o_zero[t * P.o_szrs + (c0 + 32 * gg) / kivi::kG] = z16;
        }
      }
    } else {
      // (channel pair, 32-token group) per 4 threads, 8 tokens each
      const int item = tid >> 2, quarter = tid & 3;
      const int cp2 = item & 31, tg = item >> 5;
      const int64_t gt0 = t0 + 32 * tg;
      const int cnt = static_cast<int>(n - gt0 < 32 ? (n - gt0 > 0 ? n - gt0 : 0) : 32);
      float x0[8], x1[8];
      float lo0 = INFINITY, hi0 = -INFINITY, lo1 = INFINITY, hi1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int rt = 32 * tg + 8 * quarter + j;
        x0[j] = S.u.loop.Y[rt][2 * cp2];
        x1[j] = S.u.loop.Y[rt][2 * cp2 + 1];
        if (8 * quarter + j < cnt) {
          lo0 = fminf(lo0, x0[j]);
          hi0 = fmaxf(hi0, x0[j]);
          lo1 = fminf(lo1, x1[j]);
          hi1 = fmaxf(hi1, x1[j]);
        }
      }
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        lo0 = fminf(lo0, __shfl_xor_sync(0xffffffffu, lo0, o));
        hi0 = fmaxf(hi0, __shfl_xor_sync(0xffffffffu, hi0, o));
        lo1 = fminf(lo1, __shfl_xor_sync(0xffffffffu, lo1, o));
        hi1 = fmaxf(hi1, __shfl_xor_sync(0xffffffffu, hi1, o));
      }
      if (cnt > 0) {
        __half s0h, z0h, s1h, z1h;
        kivi::group_params(lo0, hi0, s0h, z0h);
        kivi::group_params(lo1, hi1, s1h, z1h);
        const float s0 = __half2float(s0h), z0 = __half2float(z0h);
        const float s1 = __half2float(s1h), z1 = __half2float(z1h);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (8 * quarter + j < cnt) {
            const uint32_t byte = kivi::quant_one(x0[j], s0, z0) | (kivi::quant_one(x1[j], s1, z1) << 4);
            P.o_codes[(gt0 + 8 * quarter + j) * P.o_crs + c0 / 2 + cp2] = static_cast<uint8_t>(byte);
          }
        }
        if (quarter == 0) {
          const int64_t so = (gt0 / kivi::kG) * P.o_szrs + c0 + 2 * cp2;
          P.o_scale[so] = s0h;
          P.o_scale[so + 1] = s1h;
          P.o_zero[so] = z0h;
          P.o_zero[so + 1] = z1h;
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
inline int64_t al(int64_t x) { return (x + 255) / 256 * 256; }

struct Layout {
  int64_t zero_begin, zero_end, total;
  std::vector<int64_t> flag, sums, rhs, dist, ginv, mu, subv, bt, bb;
};

inline int padded_rank(const dkv_kivi_subspace_problem *p, int np) {
  int rmax = 0;
  for (int i = 0; i < np; ++i) rmax = p[i].rank > rmax ? p[i].rank : rmax;
  const int rp = (rmax + 15) / 16 * 16;
  return rp < 16 ? 16 : rp;
}

inline Layout layout(const dkv_kivi_subspace_problem *p, int np, int64_t d, int rp) {
  Layout L;
  int64_t o = 0;
  L.zero_begin = o;
  for (int i = 0; i < np; ++i) {
    const int64_t n = p[i].base.n_tokens;
    L.flag.push_back(o);
    o = al(o + n * 4);
    L.sums.push_back(o);
    o = al(o + (2 + 2 * rp + d) * 4);
  }
  L.zero_end = o;
  for (int i = 0; i < np; ++i) {
    const int64_t n = p[i].base.n_tokens;
    L.rhs.push_back(o);
    o = al(o + n * rp * 4);
    L.dist.push_back(o);
    o = al(o + n * 4);
    L.ginv.push_back(o);
    o = al(o + static_cast<int64_t>(rp) * rp * 4);
    L.mu.push_back(o);
    o = al(o + d * 4);
    L.subv.push_back(o);
    o = al(o + (d + 1) * 4);
    L.bt.push_back(o);
    o = al(o + rp * d * 2);
    L.bb.push_back(o);
    o = al(o + rp * d * 2);
  }
  L.total = o;
  return L;
}

bool a16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_cache(const dkv_kivi_cache &c, int64_t n, int64_t d) {
  if (c.codes == nullptr || c.scale == nullptr || c.zero == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (c.n_tokens != n || c.d != d) return DKV_ERR_INVALID_ARGUMENT;
  if (c.mode != DKV_KIVI_PER_TOKEN && c.mode != DKV_KIVI_PER_CHANNEL) return DKV_ERR_INVALID_ARGUMENT;
  if (!a16(c.codes) || !a16(c.scale) || !a16(c.zero) || c.code_row_stride % 16) return DKV_ERR_ALIGNMENT;
  if (c.mode == DKV_KIVI_PER_CHANNEL && c.sz_row_stride % 8) return DKV_ERR_ALIGNMENT;  // 16-B scale rows
  if (c.code_row_stride < d / 2) return DKV_ERR_LAYOUT;
  if (c.mode == DKV_KIVI_PER_TOKEN ? c.sz_row_stride < d / 32 : c.sz_row_stride < d) return DKV_ERR_LAYOUT;
  return DKV_OK;
}

int validate(const dkv_kivi_subspace_problem *p, int np, int64_t &d, int &fdt) {
  if (p == nullptr || np <= 0 || np > kMaxProblems) return DKV_ERR_INVALID_ARGUMENT;
  d = p[0].base.d;
  fdt = p[0].fresh_dtype;
  if (d <= 0 || d % kKC) return DKV_ERR_UNSUPPORTED;
  if (fdt != DKV_F32 && fdt != DKV_F16 && fdt != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  const int esz = fdt == DKV_F32 ? 4 : 2;
  for (int i = 0; i < np; ++i) {
    const dkv_kivi_subspace_problem &q = p[i];
    if (q.base.d != d || q.fresh_dtype != fdt) return DKV_ERR_INVALID_ARGUMENT;
    if (q.rank < 0 || q.rank > kMaxRank) return DKV_ERR_INVALID_ARGUMENT;
    if (q.rank > 0 && q.basis == nullptr) return DKV_ERR_INVALID_ARGUMENT;
    const int64_t n = q.base.n_tokens;
    if (n < 0 || n > 0x7fffffffLL) return DKV_ERR_INVALID_ARGUMENT;
    if (n == 0) continue;
    int rc = check_cache(q.base, n, d);
    if (rc) return rc;
    rc = check_cache(q.out, n, d);
    if (rc) return rc;
    if (q.out.mode != q.base.mode) return DKV_ERR_INVALID_ARGUMENT;
    if (q.fresh == nullptr || !a16(q.fresh) || (q.fresh_row_stride * esz) % 16 || q.fresh_row_stride < d)
      return DKV_ERR_ALIGNMENT;
    if (q.n_probes < 0 || (q.n_probes > 0 && q.probe_index == nullptr)) return DKV_ERR_INVALID_ARGUMENT;
  }
  return DKV_OK;
}

template <int RP, int FDT>
int launch(const Batch &b, int np, int64_t max_probes, cudaStream_t st) {
  if (max_probes > 0) {
    const int bx = static_cast<int>((max_probes + 255) / 256 < 64 ? (max_probes + 255) / 256 : 64);
    flags_kernel<<<dim3(bx, np), 256, 0, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  {
    const int64_t total = b.d * RP;
    const int bx = static_cast<int>((total + 255) / 256 < 256 ? (total + 255) / 256 : 256);
    pack_kernel<<<dim3(bx, np), 256, 0, st>>>(b, RP);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (b.n_tiles > 0) {
    pass1_kernel<RP, FDT><<<static_cast<unsigned>(b.n_tiles), kThreads, 0, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  const int solve_smem = kMaxRank * (2 * kMaxRank + 1) * 8;
  DKV_CUDA_CHECK(cudaFuncSetAttribute(solve_kernel<RP>, cudaFuncAttributeMaxDynamicSharedMemorySize, solve_smem));
  solve_kernel<RP><<<np, kThreads, solve_smem, st>>>(b);
  DKV_CUDA_CHECK(cudaGetLastError());
  if (b.n_tiles > 0) {
    pass2_kernel<RP, FDT><<<static_cast<unsigned>(b.n_tiles), kThreads, 0, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  return DKV_OK;
}

template <int FDT>
int launch_rp(int rp, const Batch &b, int np, int64_t max_probes, cudaStream_t st) {
  switch (rp) {
    case 16: return launch<16, FDT>(b, np, max_probes, st);
    case 32: return launch<32, FDT>(b, np, max_probes, st);
    case 48: return launch<48, FDT>(b, np, max_probes, st);
    case 64: return launch<64, FDT>(b, np, max_probes, st);
    default: return DKV_ERR_UNSUPPORTED;
  }
}

}  // namespace ksub
}  // namespace dkv

using namespace dkv;
using namespace dkv::ksub;

extern "C" int dkv_kivi_subspace_workspace_bytes(const dkv_kivi_subspace_problem *problems, int32_t n_problems,
                                                 int64_t *bytes) {
  if (bytes == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  int64_t d;
  int fdt;
  const int rc = validate(problems, n_problems, d, fdt);
  if (rc) return rc;
  *bytes = layout(problems, n_problems, d, padded_rank(problems, n_problems)).total;
  return DKV_OK;
}

extern "C" int dkv_kivi_subspace_correct(const dkv_kivi_subspace_problem *problems, int32_t n_problems,
                                         void *workspace, int64_t workspace_bytes, int32_t *status,
                                         dkv_stream_t stream) {
  int64_t d;
  int fdt;
  int rc = validate(problems, n_problems, d, fdt);
  if (rc) return rc;
  const int rp = padded_rank(problems, n_problems);
  const Layout L = layout(problems, n_problems, d, rp);
  if (workspace == nullptr || workspace_bytes < L.total || !a16(workspace)) return DKV_ERR_WORKSPACE;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  static thread_local Batch b;  // ~25 KB: not on the caller's stack
  memset(&b, 0, sizeof(b));
  int64_t tiles = 0, max_probes = 0;
  for (int i = 0; i < n_problems; ++i) {
    const dkv_kivi_subspace_problem &q = problems[i];
    Prob &P = b.probs[i];
    memset(&P, 0, sizeof(P));
    P.codes = static_cast<const uint8_t *>(q.base.codes);
    P.scale = static_cast<const __half *>(q.base.scale);
    P.zero = static_cast<const __half *>(q.base.zero);
    P.crs = q.base.code_row_stride;
    P.szrs = q.base.sz_row_stride;
    P.o_codes = static_cast<uint8_t *>(q.out.codes);
    P.o_scale = static_cast<__half *>(q.out.scale);
    P.o_zero = static_cast<__half *>(q.out.zero);
    P.o_crs = q.out.code_row_stride;
    P.o_szrs = q.out.sz_row_stride;
    P.fresh = q.fresh;
    P.frs = q.fresh_row_stride;
    P.n = q.base.n_tokens;
    P.probes = q.probe_index;
    P.n_probes = q.n_probes;
    P.sub_out = q.subspace_out;
    P.mu_out = q.orth_mu_out;
    P.mode = q.base.mode;
    // the reference applies the column-space fit only with a basis and at least one probe
    P.r = (q.n_probes > 0 && q.basis != nullptr) ? q.rank : 0;
    P.basis = q.basis;
    P.flag = reinterpret_cast<uint32_t *>(ws + L.flag[i]);
    P.sums = reinterpret_cast<float *>(ws + L.sums[i]);
    P.rhs = reinterpret_cast<float *>(ws + L.rhs[i]);
    P.dist = reinterpret_cast<float *>(ws + L.dist[i]);
    P.ginv = reinterpret_cast<float *>(ws + L.ginv[i]);
    P.mu = reinterpret_cast<float *>(ws + L.mu[i]);
    P.subv = reinterpret_cast<float *>(ws + L.subv[i]);
    P.bt = reinterpret_cast<__nv_bfloat16 *>(ws + L.bt[i]);
    P.bb = reinterpret_cast<__nv_bfloat16 *>(ws + L.bb[i]);
    P.tile0 = tiles;
    tiles += (P.n + kTM - 1) / kTM;
    if (P.n_probes > max_probes) max_probes = P.n_probes;
  }
  if (tiles > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DKV_CUDA_CHECK(cudaMemsetAsync(ws + L.zero_begin, 0, L.zero_end - L.zero_begin, st));
  b.n_probs = n_problems;
  b.d = d;
  b.n_tiles = tiles;
  b.status = status;
  switch (fdt) {
    case DKV_BF16: rc = launch_rp<DKV_BF16>(rp, b, n_problems, max_probes, st); break;
    case DKV_F16: rc = launch_rp<DKV_F16>(rp, b, n_problems, max_probes, st); break;
    default: rc = launch_rp<DKV_F32>(rp, b, n_problems, max_probes, st); break;
  }
  return rc;
}
