// Batched symmetric eigendecomposition of small matrices (n <= 96) in fp64 — the Rayleigh-Ritz
// step of the K-basis subspace iteration that stands in for the reference's svd_basis
// (src/deltakv/patches/subspace.py:37-42): the k x k projected Gram matrix Q^T C Q is
// diagonalised on the device, so the basis never leaves HBM.
//
// Method: cyclic two-sided Jacobi with the parallel round-robin ordering (Brent & Luk, SIAM
// J. Sci. Stat. Comput. 1985; Golub & Van Loan, Matrix Computations 4th ed., Sec. 8.5.3 and
// Alg. 8.5.1 for the 2x2 symmetric Schur rotation).  One CTA per matrix keeps A and the
// accumulated rotations V in shared memory; each round rotates n/2 disjoint index pairs at
// once — both sides of every 2x2 block in one pass, two barriers per round — n-1 rounds per
// sweep, and sweeps stop when the off-diagonal Frobenius norm falls below 1e-11 of the matrix
// norm or after max_sweeps.  Odd n is padded with a decoupled zero row/column that never
// rotates.
#include "dkv_common.cuh"

namespace dkv {
namespace eig {

constexpr int kMaxN = 96;
constexpr int kThreads = 1024;  // more of each round's 2x2 blocks in flight (512: 7 % slower at k = 72)

__device__ __forceinline__ double block_sum(double v, double *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double s = 0.0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) s += red[w];
  return s;
}

// players at positions 0..n-1 of round `round`: position 0 holds player 0, position i >= 1
// holds player ((i - 1 + round) mod (n - 1)) + 1; pair i couples positions i and n-1-i.
__device__ __forceinline__ int player(int pos, int round, int n) {
  return pos == 0 ? 0 : ((pos - 1 + round) % (n - 1)) + 1;
}

// Jacobi rotation (c, s) that annihilates apq (Alg. 8.5.1): t = tan(theta) is formed in fp32
// (relative error ~1e-7 leaves a'_pq ~ 1e-7 a_pq, which the next sweep removes), then
// c = 1/sqrt(1 + t^2) to full fp64 accuracy by two Newton steps from the fp32 estimate, so the
// rotation is orthogonal to fp64 rounding whatever the error in t.
__device__ __forceinline__ void rotation(double app, double aqq, double apq, double &c, double &s) {
  c = 1.0;
  s = 0.0;
  const float apq_f = static_cast<float>(apq);
  if (fabsf(apq_f) < 1e-30f) return;  // below the matrix norm by far more than the tolerance
  const float tau = static_cast<float>(aqq - app) / (2.0f * apq_f);
  const float at = fabsf(tau);
  const float tf = (at > 1e18f ? 0.5f / at : 1.0f / (at + sqrtf(fmaf(at, at, 1.0f))));
  const double t = static_cast<double>(tau >= 0.0f ? tf : -tf);
  const double x = fma(t, t, 1.0);
  double y = static_cast<double>(rsqrtf(static_cast<float>(x)));
  y = y * fma(-0.5 * x * y, y, 1.5);
  y = y * fma(-0.5 * x * y, y, 1.5);
  c = y;
  s = t * y;
}

__global__ void __launch_bounds__(kThreads) jacobi_kernel(const double *a_in, int64_t a_stride, int k, int n,
                                                          int max_sweeps, double *evals, double *evecs,
                                                          int32_t *info) {
  extern __shared__ double sm[];
  const int ld = n + 1;
  const int half = n / 2;
  double *A = sm;                    // [n][ld]
  double *V = A + n * ld;            // [n][ld]
  double *cs = V + n * ld;           // [half] c, [half] s
  double *red = cs + n;              // [kThreads/32]
  int *pq = reinterpret_cast<int *>(red + kThreads / 32);  // [half] p, [half] q
  const int tid = threadIdx.x;
  const int64_t bi = blockIdx.x;
  const double *src = a_in + bi * a_stride;

  double frob = 0.0;
  bool finite = true;
  for (int e = tid; e < n * n; e += kThreads) {
    const int i = e / n, j = e % n;
    double v = 0.0;
    if (i < k && j < k) v = 0.5 * (src[static_cast<int64_t>(i) * k + j] + src[static_cast<int64_t>(j) * k + i]);
    if (!isfinite(v)) {
      finite = false;
      v = 0.0;
    }
    A[i * ld + j] = v;
    V[i * ld + j] = i == j ? 1.0 : 0.0;
    frob = fma(v, v, frob);
  }
  frob = block_sum(frob, red);
  const int all_finite = __syncthreads_and(finite ? 1 : 0) && isfinite(frob);
  if (!isfinite(frob)) frob = 0.0;
  // work on A / ||A||_F so that every entry that matters is far inside the fp32 range
  const double norm = sqrt(frob);
  const double inv = frob > 0.0 ? 1.0 / norm : 0.0;
  for (int e = tid; e < n * n; e += kThreads) A[(e / n) * ld + e % n] *= inv;
  __syncthreads();

  const int m_half = (1 << 20) / half + 1, m_n = (1 << 20) / n + 1;  // e / half, f / n
  int converged = frob == 0.0 ? 1 : 0;
  for (int sweep = 0; sweep < max_sweeps && !converged; ++sweep) {
    for (int round = 0; round < n - 1; ++round) {
      if (tid < half) {
        int p = player(tid, round, n), q = player(n - 1 - tid, round, n);
        if (p > q) {
          const int t = p;
          p = q;
          q = t;
        }
        double c, s;
        rotation(A[p * ld + p], A[q * ld + q], A[p * ld + q], c, s);
        cs[tid] = c;
        cs[half + tid] = s;
        pq[tid] = p;
        pq[half + tid] = q;
      }
      __syncthreads();
      // A <- J^T A J one 2x2 block at a time: block (t, u) spans rows {p_t, q_t} and columns
      // {p_u, q_u} and depends only on rotations t and u; V <- V J alongside.  The flat index
      // is split by multiply-shift (exact for these ranges: e < 2^13, divisors <= 96).
      for (int e = tid; e < half * half + n * half; e += kThreads) {
        if (e < half * half) {
          const int t = (e * m_half) >> 20, u = e - t * half;
          const double ct = cs[t], st = cs[half + t], cu = cs[u], su = cs[half + u];
          if (st == 0.0 && su == 0.0) continue;
          const int pt = pq[t], qt = pq[half + t], pu = pq[u], qu = pq[half + u];
          const double a = A[pt * ld + pu], b = A[pt * ld + qu], c = A[qt * ld + pu], d = A[qt * ld + qu];
          const double r0 = ct * a - st * c, r1 = ct * b - st * d;
          const double r2 = st * a + ct * c, r3 = st * b + ct * d;
          A[pt * ld + pu] = cu * r0 - su * r1;
          A[pt * ld + qu] = su * r0 + cu * r1;
          A[qt * ld + pu] = cu * r2 - su * r3;
          A[qt * ld + qu] = su * r2 + cu * r3;
        } else {
          const int f = e - half * half;
          const int t = (f * m_n) >> 20, i = f - t * n;
          const double c = cs[t], s = cs[half + t];
          if (s == 0.0) continue;
          const int p = pq[t], q = pq[half + t];
          const double vp = V[i * ld + p], vq = V[i * ld + q];
          V[i * ld + p] = c * vp - s * vq;
          V[i * ld + q] = s * vp + c * vq;
        }
      }
      __syncthreads();
    }
    double off = 0.0;
    for (int e = tid; e < n * n; e += kThreads) {
      const int i = e / n, j = e % n;
      if (i != j) off = fma(A[i * ld + j], A[i * ld + j], off);
    }
    off = block_sum(off, red);
    converged = off <= 1e-22 ? 1 : 0;  // ||offdiag|| <= 1e-11 ||A||_F
  }

  // descending order over the k real indices (padding excluded); NaN ranks last, ties by index
  double *ev_out = evals + bi * k;
  double *vec_out = evecs + bi * static_cast<int64_t>(k) * k;
  for (int i = tid; i < k; i += kThreads) {
    const double di = A[i * ld + i];
    const double key_i = isnan(di) ? -INFINITY : di;
    int rank = 0;
    for (int j = 0; j < k; ++j) {
      const double dj = A[j * ld + j];
      const double key_j = isnan(dj) ? -INFINITY : dj;
      rank += (key_j > key_i) || (key_j == key_i && j < i);
    }
    ev_out[rank] = di * norm;
    for (int r = 0; r < k; ++r) vec_out[static_cast<int64_t>(r) * k + rank] = V[r * ld + i];
  }
  if (tid == 0) info[bi] = all_finite ? (converged ? 0 : 1) : 2;
}

}  // namespace eig
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_sym_eig_batched(const double *a, int64_t batch, int32_t k, int64_t a_stride, int32_t max_sweeps,
                                   double *evals, double *evecs, int32_t *info, dkv_stream_t stream) {
  if (batch < 0 || k <= 0 || k > eig::kMaxN || max_sweeps <= 0) return DKV_ERR_INVALID_ARGUMENT;
  if (batch == 0) return DKV_OK;
  if (a == nullptr || evals == nullptr || evecs == nullptr || info == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (a_stride < static_cast<int64_t>(k) * k) return DKV_ERR_INVALID_ARGUMENT;
  if (batch > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  const int n = (k + 1) & ~1;
  const size_t smem = (2 * static_cast<size_t>(n) * (n + 1) + n + eig::kThreads / 32) * sizeof(double) +
                      static_cast<size_t>(n) * sizeof(int);
  const int smem_max = static_cast<int>((2 * eig::kMaxN * (eig::kMaxN + 1) + eig::kMaxN + eig::kThreads / 32) *
                                        sizeof(double) + eig::kMaxN * sizeof(int));
  // set once per device (no runtime-API call on later launches, so they can be graph-captured)
  static unsigned long long set_on = 0;
  int dev = 0;
  DKV_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev >= 64 || !((set_on >> dev) & 1ull)) {
    DKV_CUDA_CHECK(cudaFuncSetAttribute(eig::jacobi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
    if (dev < 64) set_on |= 1ull << dev;
  }
  eig::jacobi_kernel<<<static_cast<unsigned>(batch), eig::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      a, a_stride, k, n, max_sweeps, evals, evecs, info);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}
