// Rank-r subspace least-squares correction with an orthogonal residual shift.
//
// Reference: deltakv.patches.subspace.subspace_correct (src/deltakv/patches/subspace.py:45-106)
// with _solve_codes (21-34):
//   R = fresh - reused                                  [n, d]
//   codes = solve(B^T B + 1e-6 I, (R B)^T)^T             [n, r]
//   fitted = codes B^T;  subspace = mean_n(codes) B^T;  orth_mu = mean_P(R - fitted)
//   w = min(||R_j|| / mean_j ||R_j||, 1)  (or caller weights)
//   corr = reused + fitted + w * orth_mu;  corr[P] = fresh[P]
// Without a basis: corr = reused + w * mean_P(R), subspace = 0.
//
// Where d is a multiple of 32 and the rows are 16-byte aligned the call runs on the batched
// tensor-core pipeline of kivi_subspace.cu (ksub::dense_correct: R B and rhs (B G^-1)^T on
// split-bf16 mma.sync, the probe sums one warp per probe row, the solve register-blocked);
// the kernels below take every other shape.
// Four launches on the caller's stream, all arithmetic fp32 (the r x r inverse in fp64):
//   sub_pass1    R, ||R||, rhs = R B per token (CTA-tiled small GEMM), CTA-reduced sums
//   sub_probes   probe flags, sum_P R, sum_P rhs
//   sub_solve    (B^T B + 1e-6 I)^-1, orth_mu, subspace, mean ||R||
//   sub_pass2    corr = reused + (rhs G^-1) B^T + w orth_mu, probes <- fresh
// Scratch lives in a caller-provided workspace (dkv_subspace_workspace_bytes).
#include <mutex>

#include "dkv_common.cuh"

namespace dkv {
namespace ksub {
int dense_correct(const dkv_subspace_args *a, uint8_t *ws, int64_t ws_bytes, cudaStream_t st);
int64_t dense_workspace_bytes(int64_t n, int64_t d, int rank);
}  // namespace ksub
namespace sub {

constexpr int kTM = 64;   // tokens per CTA tile
constexpr int kKC = 64;   // d-chunk per smem stage
constexpr int kThreads = 256;
constexpr int kMaxRank = 64;

struct Work {  // offsets into the workspace (bytes), all 256-aligned
  int64_t rhs, dist, flag, sums, ginv, mu, sub, total;
};

inline int64_t al(int64_t x) { return (x + 255) / 256 * 256; }

inline Work layout(int64_t n, int64_t d, int r) {
  Work w;
  int64_t o = 0;
  w.rhs = o;  o = al(o + n * r * 4);
  w.dist = o; o = al(o + n * 4);
  w.flag = o; o = al(o + n);
  // sums: [0] sum ||R||, [1] probe count, [2..2+r) sum rhs (all), [2+r..2+2r) sum rhs (probes),
  //       [2+2r..2+2r+d) sum_P R
  w.sums = o; o = al(o + (2 + 2 * r + d) * 4);
  w.ginv = o; o = al(o + r * r * 4);
  w.mu = o;   o = al(o + d * 4);
  w.sub = o;  o = al(o + d * 4 + 16);  // + mean ||R|| at sub[d]
  w.total = o;
  return w;
}

struct P {
  const void *reused, *fresh;
  int kv_dtype;
  int64_t n, d, rs_stride, fs_stride;
  const int32_t *probes;
  int64_t n_probes;
  const float *basis;  // [d, r] or null
  int r;
  const float *token_weights;
  void *out;
  int out_dtype;
  int64_t out_stride;
  float *subspace_out, *orth_mu_out;
  uint8_t *ws;
  Work w;
};

__device__ __forceinline__ float ld(const void *p, int dt, int64_t i) { return load_as_float(p, dt, i); }
__device__ __forceinline__ void st(void *p, int dt, int64_t i, float v) {
  switch (dt) {
    case DKV_F32: static_cast<float *>(p)[i] = v; break;
    case DKV_F16: static_cast<__half *>(p)[i] = __float2half_rn(v); break;
    case DKV_BF16: static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v); break;
    default: break;
  }
}

__global__ void zero_kernel(float *p, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0.f;
}
__global__ void zero_u8(uint8_t *p, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) p[i] = 0;
}

// ---------------------------------------------------------------------------------
// pass 1: thread (tg, cg) of a 16 x (R/4) grid owns a 4-token x 4-column block of rhs
// ---------------------------------------------------------------------------------
template <int R>
__global__ void __launch_bounds__(kThreads) pass1_kernel(const P p) {
  __shared__ float Rs[kKC][kTM + 4];   // residual chunk, k-major
  __shared__ float Bs[kKC][R + 4];     // basis chunk
  __shared__ float red[kThreads / 32];
  const int tid = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kTM;
  // loader mapping: token lt = tid / 4, 16 consecutive k per thread
  const int lt = tid >> 2, lk = (tid & 3) * 16;
  const int64_t tok = t0 + lt;
  const bool tvalid = tok < p.n;
  float dist2 = 0.f;
  // compute mapping
  const int tg = tid / (R / 4), cg = tid % (R / 4);
  const bool active = tid < 16 * (R / 4);
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const bool have_basis = p.basis != nullptr;
  for (int64_t k0 = 0; k0 < p.d; k0 += kKC) {
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int64_t k = k0 + lk + i;
      float v = 0.f;
      if (tvalid && k < p.d)
        v = ld(p.fresh, p.kv_dtype, tok * p.fs_stride + k) - ld(p.reused, p.kv_dtype, tok * p.rs_stride + k);
      dist2 = fmaf(v, v, dist2);
      Rs[lk + i][lt] = v;
    }
    if (have_basis) {
      for (int i = tid; i < kKC * R; i += kThreads) {
        const int kk = i / R, c = i % R;
        const int64_t k = k0 + kk;
        Bs[kk][c] = (k < p.d && c < p.r) ? p.basis[k * p.r + c] : 0.f;
      }
    }
    __syncthreads();
    if (have_basis && active) {
#pragma unroll 8
      for (int kk = 0; kk < kKC; ++kk) {
        const float4 a = *reinterpret_cast<const float4 *>(&Rs[kk][4 * tg]);
        const float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][4 * cg]);
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
    }
    __syncthreads();
  }
  // ||R||: 4 loader threads per token
  dist2 += __shfl_xor_sync(0xffffffffu, dist2, 1);
  dist2 += __shfl_xor_sync(0xffffffffu, dist2, 2);
  float *dist = reinterpret_cast<float *>(p.ws + p.w.dist);
  float *sums = reinterpret_cast<float *>(p.ws + p.w.sums);
  float dsum = 0.f;
  if ((tid & 3) == 0 && tvalid) {
    const float dd = sqrtf(dist2);
    dist[tok] = dd;
    dsum = dd;
  }
  for (int o = 16; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  if ((tid & 31) == 0) red[tid >> 5] = dsum;
  // rhs rows + per-CTA column sums (reuse Rs as scratch)
  float *rhs = reinterpret_cast<float *>(p.ws + p.w.rhs);
  if (have_basis && active) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t tt = t0 + 4 * tg + i;
      if (tt < p.n) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = 4 * cg + j;
          if (c < p.r) rhs[tt * p.r + c] = acc[i][j];
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    float s = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) s += red[i];
    atomicAdd(&sums[0], s);
  }
  if (have_basis) {
    // column sums over this CTA's valid tokens
    float *colsum = &Rs[0][0];
    if (active) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) s += (t0 + 4 * tg + i < p.n) ? acc[i][j] : 0.f;
        colsum[tg * R + 4 * cg + j] = s;
      }
    }
    __syncthreads();
    if (tid < p.r) {
      float s = 0.f;
      for (int g2 = 0; g2 < 16; ++g2) s += colsum[g2 * R + tid];
      atomicAdd(&sums[2 + tid], s);
    }
  }
}

// probe flags, sum_P R (per column), sum_P rhs, probe count
__global__ void __launch_bounds__(kThreads) probes_kernel(const P p) {
  float *sums = reinterpret_cast<float *>(p.ws + p.w.sums);
  uint8_t *flag = p.ws + p.w.flag;
  const float *rhs = reinterpret_cast<const float *>(p.ws + p.w.rhs);
  const int64_t per_cta = 64;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * per_cta;
  const int64_t p1 = min(p0 + per_cta, p.n_probes);
  for (int64_t c = threadIdx.x; c < p.d; c += blockDim.x) {
    float s = 0.f;
    for (int64_t i = p0; i < p1; ++i) {
      const int64_t t = p.probes[i];
      if (t < 0 || t >= p.n) continue;
      s += ld(p.fresh, p.kv_dtype, t * p.fs_stride + c) - ld(p.reused, p.kv_dtype, t * p.rs_stride + c);
    }
    atomicAdd(&sums[2 + 2 * p.r + c], s);
  }
  if (threadIdx.x < p.r) {
    float s = 0.f;
    for (int64_t i = p0; i < p1; ++i) {
      const int64_t t = p.probes[i];
      if (t >= 0 && t < p.n) s += rhs[t * p.r + threadIdx.x];
    }
    atomicAdd(&sums[2 + p.r + threadIdx.x], s);
  }
  if (threadIdx.x == blockDim.x - 1) {
    int cnt = 0;
    for (int64_t i = p0; i < p1; ++i) {
      const int64_t t = p.probes[i];
      if (t >= 0 && t < p.n) {
        flag[t] = 1;
        ++cnt;
      }
    }
    atomicAdd(&sums[1], static_cast<float>(cnt));
  }
}

// one CTA: G^-1, orth_mu, subspace, mean ||R||
__global__ void __launch_bounds__(kThreads) solve_kernel(const P p) {
  extern __shared__ double Mdyn[];  // [r][2r + 1], augmented [G | I]
  __shared__ float cp[kMaxRank], ca[kMaxRank];
  __shared__ double fac[kMaxRank];
  __shared__ int piv_row;
  const int r = p.r;
  const int ldm = 2 * r + 1;
  float *sums = reinterpret_cast<float *>(p.ws + p.w.sums);
  float *ginv = reinterpret_cast<float *>(p.ws + p.w.ginv);
  float *mu = reinterpret_cast<float *>(p.ws + p.w.mu);
  float *subv = reinterpret_cast<float *>(p.ws + p.w.sub);
  const float np = sums[1];
  if (r > 0) {
    // G = B^T B + 1e-6 I  (fp32 products accumulated in fp64), augmented with I
    for (int e = threadIdx.x; e < r * r; e += blockDim.x) {
      const int i = e / r, j = e % r;
      double s = 0.0;
      for (int64_t k = 0; k < p.d; ++k) s += static_cast<double>(p.basis[k * r + i]) * p.basis[k * r + j];
      Mdyn[(i) * ldm + (j)] = s + (i == j ? 1e-6 : 0.0);
      Mdyn[(i) * ldm + (r + j)] = (i == j) ? 1.0 : 0.0;
    }
    __syncthreads();
    // Gauss-Jordan with partial pivoting
    for (int col = 0; col < r; ++col) {
      if (threadIdx.x == 0) {
        int best = col;
        double bv = fabs(Mdyn[(col) * ldm + (col)]);
        for (int i = col + 1; i < r; ++i)
          if (fabs(Mdyn[(i) * ldm + (col)]) > bv) {
            bv = fabs(Mdyn[(i) * ldm + (col)]);
            best = i;
          }
        piv_row = best;
      }
      __syncthreads();
      const int pr = piv_row;
      if (pr != col)
        for (int j = threadIdx.x; j < 2 * r; j += blockDim.x) {
          const double t = Mdyn[(col) * ldm + (j)];
          Mdyn[(col) * ldm + (j)] = Mdyn[(pr) * ldm + (j)];
          Mdyn[(pr) * ldm + (j)] = t;
        }
      __syncthreads();
      const double inv = 1.0 / Mdyn[(col) * ldm + (col)];
      __syncthreads();
      for (int j = threadIdx.x; j < 2 * r; j += blockDim.x) Mdyn[(col) * ldm + (j)] *= inv;
      for (int i = threadIdx.x; i < r; i += blockDim.x) fac[i] = Mdyn[(i) * ldm + (col)];
      __syncthreads();
      for (int e = threadIdx.x; e < r * 2 * r; e += blockDim.x) {
        const int i = e / (2 * r), j = e % (2 * r);
        if (i != col) Mdyn[(i) * ldm + (j)] -= fac[i] * Mdyn[(col) * ldm + (j)];
      }
      __syncthreads();
    }
    for (int e = threadIdx.x; e < r * r; e += blockDim.x) ginv[e] = static_cast<float>(Mdyn[(e / r) * ldm + (r + e % r)]);
    __syncthreads();
    // mean codes over probes and over all tokens: (mean rhs) G^-1
    if (threadIdx.x < r) {
      const int j = threadIdx.x;
      double sp = 0.0, sa = 0.0;
      for (int i = 0; i < r; ++i) {
        sp += static_cast<double>(sums[2 + r + i]) * Mdyn[(i) * ldm + (r + j)];
        sa += static_cast<double>(sums[2 + i]) * Mdyn[(i) * ldm + (r + j)];
      }
      cp[j] = np > 0 ? static_cast<float>(sp / np) : 0.f;
      ca[j] = static_cast<float>(sa / static_cast<double>(p.n));
    }
    __syncthreads();
  }
  for (int64_t c = threadIdx.x; c < p.d; c += blockDim.x) {
    float fp = 0.f, fa = 0.f;
    for (int i = 0; i < r; ++i) {
      fp = fmaf(cp[i], p.basis[c * r + i], fp);
      fa = fmaf(ca[i], p.basis[c * r + i], fa);
    }
    const float meanR = np > 0 ? sums[2 + 2 * r + c] / np : 0.f;
    mu[c] = meanR - fp;
    subv[c] = fa;
    if (p.orth_mu_out) p.orth_mu_out[c] = meanR - fp;
    if (p.subspace_out) p.subspace_out[c] = fa;
  }
  if (threadIdx.x == 0) subv[p.d] = fmaxf(sums[0] / static_cast<float>(p.n), 1e-8f);
}

// pass 2: thread (tg, dg) owns 4 tokens x 4 consecutive columns of a 64-column chunk
template <int R>
__global__ void __launch_bounds__(kThreads) pass2_kernel(const P p) {
  __shared__ float Cs[kTM][R + 1];       // codes of the tile
  __shared__ float GB[kKC > R ? kKC : R][R + 1];  // G^-1, then the basis rows of a column chunk
  float (*Gs)[R + 1] = GB;
  float (*Bs)[R + 1] = GB;
  const int tid = threadIdx.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kTM;
  const float *rhs = reinterpret_cast<const float *>(p.ws + p.w.rhs);
  const float *ginv = reinterpret_cast<const float *>(p.ws + p.w.ginv);
  const float *mu = reinterpret_cast<const float *>(p.ws + p.w.mu);
  const float *subv = reinterpret_cast<const float *>(p.ws + p.w.sub);
  const float *dist = reinterpret_cast<const float *>(p.ws + p.w.dist);
  const uint8_t *flag = p.ws + p.w.flag;
  const int r = p.r;
  if (r > 0) {
    for (int e = tid; e < r * r; e += kThreads) Gs[e / r][e % r] = ginv[e];
    __syncthreads();
    // codes = rhs G^-1 for the tile's tokens
    for (int e = tid; e < kTM * R; e += kThreads) {
      const int lt = e / R, c = e % R;
      const int64_t tok = t0 + lt;
      float s = 0.f;
      if (tok < p.n && c < r)
        for (int i = 0; i < r; ++i) s = fmaf(rhs[tok * r + i], Gs[i][c], s);
      Cs[lt][c] = s;
    }
  }
  const float mean_dist = subv[p.d];
  const int tg = tid >> 4, dg = tid & 15;
  float w[4];
  bool pr[4];
  int64_t tk[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    tk[i] = t0 + 4 * tg + i;
    const bool v = tk[i] < p.n;
    pr[i] = v && flag[tk[i]];
    if (p.token_weights) w[i] = v ? p.token_weights[tk[i]] : 0.f;
    else w[i] = v ? fminf(dist[tk[i]] / mean_dist, 1.f) : 0.f;
  }
  for (int64_t c0 = 0; c0 < p.d; c0 += kKC) {
    __syncthreads();
    if (r > 0)
      for (int e = tid; e < kKC * R; e += kThreads) {
        const int cc = e / R, i = e % R;
        const int64_t c = c0 + cc;
        Bs[cc][i] = (c < p.d && i < r) ? p.basis[c * r + i] : 0.f;
      }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (tk[i] >= p.n) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int cc = 4 * dg + j;
        const int64_t c = c0 + cc;
        if (c >= p.d) continue;
        float v;
        if (pr[i]) {
          v = ld(p.fresh, p.kv_dtype, tk[i] * p.fs_stride + c);
        } else {
          float f = 0.f;
          for (int k = 0; k < r; ++k) f = fmaf(Cs[4 * tg + i][k], Bs[cc][k], f);
          v = ld(p.reused, p.kv_dtype, tk[i] * p.rs_stride + c) + f + w[i] * mu[c];
        }
        st(p.out, p.out_dtype, tk[i] * p.out_stride + c, v);
      }
    }
  }
}

template <int R>
int launch_all(const P &p, cudaStream_t st) {
  const int grid = static_cast<int>((p.n + kTM - 1) / kTM);
  pass1_kernel<R><<<grid, kThreads, 0, st>>>(p);
  DKV_CUDA_CHECK(cudaGetLastError());
  if (p.n_probes > 0) {
    probes_kernel<<<static_cast<int>((p.n_probes + 63) / 64), kThreads, 0, st>>>(p);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  const int solve_smem = p.r * (2 * p.r + 1) * 8;
  DKV_CUDA_CHECK(cudaFuncSetAttribute(solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kMaxRank * (2 * kMaxRank + 1) * 8));
  solve_kernel<<<1, kThreads, solve_smem, st>>>(p);
  DKV_CUDA_CHECK(cudaGetLastError());
  pass2_kernel<R><<<grid, kThreads, 0, st>>>(p);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

}  // namespace sub
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_subspace_workspace_bytes(int64_t n_tokens, int64_t d, int32_t rank,
                                            int64_t *bytes) {
  if (bytes == nullptr || n_tokens < 0 || d <= 0 || rank < 0 || rank > sub::kMaxRank)
    return DKV_ERR_INVALID_ARGUMENT;
  const int rp = rank == 0 ? 0 : (rank + 15) / 16 * 16;
  const int64_t general = sub::layout(n_tokens, d, rp).total, dense = ksub::dense_workspace_bytes(n_tokens, d, rank);
  *bytes = dense > general ? dense : general;
  return DKV_OK;
}

// Shared set-up of both entry points: validate, build the launch parameters.
static int subspace_params(const dkv_subspace_args *a, uint8_t *ws, int64_t ws_bytes, sub::P &p) {
  if (a == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (a->n_tokens < 0 || a->d <= 0 || a->rank < 0 || a->rank > sub::kMaxRank) return DKV_ERR_INVALID_ARGUMENT;
  if (a->kv_dtype != DKV_F32 && a->kv_dtype != DKV_F16 && a->kv_dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (a->out_dtype != DKV_F32 && a->out_dtype != DKV_F16 && a->out_dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (a->n_tokens > 0 && (a->reused == nullptr || a->fresh == nullptr || a->corrected == nullptr))
    return DKV_ERR_INVALID_ARGUMENT;
  if (a->rank > 0 && a->basis == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (a->n_probes > 0 && a->probe_index == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  const int rp = a->rank == 0 ? 0 : (a->rank + 15) / 16 * 16;
  p.w = sub::layout(a->n_tokens, a->d, rp);
  if (ws == nullptr || ws_bytes < p.w.total) return DKV_ERR_WORKSPACE;
  p.reused = a->reused;
  p.fresh = a->fresh;
  p.kv_dtype = a->kv_dtype;
  p.n = a->n_tokens;
  p.d = a->d;
  p.rs_stride = a->reused_row_stride;
  p.fs_stride = a->fresh_row_stride;
  p.probes = a->probe_index;
  p.n_probes = a->n_probes;
  p.basis = a->rank > 0 ? a->basis : nullptr;
  p.r = a->rank;
  p.token_weights = a->token_weights;
  p.out = a->corrected;
  p.out_dtype = a->out_dtype;
  p.out_stride = a->out_row_stride;
  p.subspace_out = a->subspace_out;
  p.orth_mu_out = a->orth_mu_out;
  p.ws = ws;
  return DKV_OK;
}

// Clear the accumulators the launches add into, then run the four launches.
static int subspace_run(const sub::P &p, cudaStream_t st) {
  sub::zero_kernel<<<8, 256, 0, st>>>(reinterpret_cast<float *>(p.ws + p.w.sums), 2 + 2 * p.r + p.d);
  DKV_CUDA_CHECK(cudaGetLastError());
  if (p.n > 0) {
    sub::zero_u8<<<64, 256, 0, st>>>(p.ws + p.w.flag, p.n);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (p.n == 0) return DKV_OK;
  const int rp = p.r == 0 ? 0 : (p.r + 15) / 16 * 16;
  switch (rp) {
    case 0: return sub::launch_all<16>(p, st);  // no basis: the rank-16 kernels skip the products
    case 16: return sub::launch_all<16>(p, st);
    case 32: return sub::launch_all<32>(p, st);
    case 48: return sub::launch_all<48>(p, st);
    case 64: return sub::launch_all<64>(p, st);
    default: return DKV_ERR_UNSUPPORTED;
  }
}

extern "C" int dkv_subspace_correct(const dkv_subspace_args *a, dkv_stream_t stream) {
  if (a != nullptr) {
    const int rc = ksub::dense_correct(a, static_cast<uint8_t *>(a->workspace), a->workspace_bytes,
                                       reinterpret_cast<cudaStream_t>(stream));
    if (rc != DKV_ERR_UNSUPPORTED) return rc;
  }
  sub::P p;
  int rc = subspace_params(a, static_cast<uint8_t *>(a ? a->workspace : nullptr),
                           a ? a->workspace_bytes : 0, p);
  if (rc != DKV_OK) return rc;
  return subspace_run(p, reinterpret_cast<cudaStream_t>(stream));
}

// R[P] = fresh[P] - reused[P] as fp32 [n_probes, d] (the matrix whose right singular
// vectors are the K-path basis, subspace.py:37-42,71-73).
__global__ void probe_residual_kernel(const void *reused, const void *fresh, int dt, int64_t rs,
                                      int64_t fs, int64_t n, int64_t d, const int32_t *probes,
                                      int64_t n_probes, float *out) {
  const int64_t i = blockIdx.x;
  const int64_t t = probes[i];
  for (int64_t c = threadIdx.x; c < d; c += blockDim.x) {
    float v = 0.f;
    if (t >= 0 && t < n) v = sub::ld(fresh, dt, t * fs + c) - sub::ld(reused, dt, t * rs + c);
    out[i * d + c] = v;
  }
}

extern "C" int dkv_subspace_probe_residual(const void *reused, const void *fresh, int32_t kv_dtype,
                                           int64_t reused_row_stride, int64_t fresh_row_stride,
                                           int64_t n_tokens, int64_t d, const int32_t *probe_index,
                                           int64_t n_probes, float *out, dkv_stream_t stream) {
  if (n_probes == 0) return DKV_OK;
  if (reused == nullptr || fresh == nullptr || probe_index == nullptr || out == nullptr || d <= 0)
    return DKV_ERR_INVALID_ARGUMENT;
  if (kv_dtype != DKV_F32 && kv_dtype != DKV_F16 && kv_dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (n_probes > 0x7fffffff) return DKV_ERR_UNSUPPORTED;
  probe_residual_kernel<<<static_cast<unsigned>(n_probes), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reused, fresh, kv_dtype, reused_row_stride, fresh_row_stride, n_tokens, d, probe_index, n_probes, out);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

// ---------------------------------------------------------------------------------
// Allocation-free variant
// ---------------------------------------------------------------------------------
// Some callers cannot allocate device memory at the point where they want a correction:
// code running inside a framework that owns every allocation through its own pool (and
// forbids cudaMalloc while it serves requests), plugins that are handed only the buffers
// they must read and write, and host threads that must never block on the allocator's
// device-wide synchronisation.  For them the scratch lives in one fixed device array
// defined in this file.  The CUDA runtime places it on every GPU that loads this library
// and keeps it there until the process exits; it is never allocated or freed per call.
//
// The array's host-side name is only a stand-in for the symbol: its device address is
// looked up once per device (cudaGetSymbolAddress, with that device current) on the first
// call made while that device is current, cached, and passed to the kernels.
constexpr int64_t kNoAllocScratchBytes = 16ll << 20;  // 16 MiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_subspace_scratch[kNoAllocScratchBytes];

static std::mutex g_scratch_mu;
static void *g_scratch_addr[kNoAllocMaxDevices] = {};

static int noalloc_scratch(void **out) {
  int dev = 0;
  DKV_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return DKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_subspace_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      note_cuda_error(err != cudaSuccess ? err : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(scratch)");
      return DKV_ERR_CUDA;
    }
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return DKV_OK;
}

extern "C" int dkv_subspace_correct_noalloc(const dkv_subspace_args *a, dkv_stream_t stream) {
  if (a == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  const int rp = a->rank <= 0 ? 0 : (a->rank + 15) / 16 * 16;
  if (a->n_tokens < 0 || a->d <= 0 || a->rank < 0 || a->rank > sub::kMaxRank) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t general = sub::layout(a->n_tokens, a->d, rp).total;
  const int64_t dense = ksub::dense_workspace_bytes(a->n_tokens, a->d, a->rank);
  if (general > kNoAllocScratchBytes && (dense == 0 || dense > kNoAllocScratchBytes)) return DKV_ERR_WORKSPACE;
  void *scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != DKV_OK) return rc;
  if (dense > 0 && dense <= kNoAllocScratchBytes) {
    rc = ksub::dense_correct(a, static_cast<uint8_t *>(scratch), kNoAllocScratchBytes,
                             reinterpret_cast<cudaStream_t>(stream));
    if (rc != DKV_ERR_UNSUPPORTED) return rc;
  }
  if (general > kNoAllocScratchBytes) return DKV_ERR_WORKSPACE;
  sub::P p;
  rc = subspace_params(a, static_cast<uint8_t *>(scratch), kNoAllocScratchBytes, p);
  if (rc != DKV_OK) return rc;
  return subspace_run(p, reinterpret_cast<cudaStream_t>(stream));
}
