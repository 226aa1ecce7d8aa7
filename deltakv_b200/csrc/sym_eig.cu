// Batched symmetric eigendecomposition of small matrices (n <= 96) in fp64 — the Rayleigh-Ritz
// step of the K-basis subspace iteration that stands in for the reference's svd_basis
// (src/deltakv/patches/subspace.py:37-42): the k x k projected Gram matrix Q^T C Q is
// diagonalised on the device, so the basis never leaves HBM.
//
// Method: cyclic two-sided Jacobi with the parallel round-robin ordering (Brent & Luk, SIAM
// J. Sci. Stat. Comput. 1985; Golub & Van Loan, Matrix Computations 4th ed., Sec. 8.5.3 and
// Alg. 8.5.1 for the 2x2 symmetric Schur rotation).  One CTA per matrix keeps A and the
// accumulated rotations V in shared memory; each round rotates n/2 disjoint index pairs at
// once (rows, then columns), n-1 rounds per sweep, and sweeps stop when the off-diagonal
// Frobenius norm falls below 1e-13 of the matrix norm or after max_sweeps.  Odd n is padded
// with a decoupled zero row/column that never rotates.
#include "dkv_common.cuh"

namespace dkv {
namespace eig {

constexpr int kMaxN = 96;
constexpr int kThreads = 256;

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

__global__ void __launch_bounds__(kThreads) jacobi_kernel(const double *a_in, int64_t a_stride, int k, int n,
                                                          int max_sweeps, double *evals, double *evecs,
                                                          int32_t *info) {
  extern __shared__ double sm[];
  const int ld = n + 1;
  double *A = sm;                    // [n][ld]
  double *V = A + n * ld;            // [n][ld]
  double *cs = V + n * ld;           // [n/2] c, [n/2] s
  double *red = cs + n;              // [kThreads/32]
  int *pq = reinterpret_cast<int *>(red + kThreads / 32);  // [n/2] p, [n/2] q
  const int tid = threadIdx.x;
  const int64_t bi = blockIdx.x;
  const double *src = a_in + bi * a_stride;
  const int half = n / 2;

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
  const int all_finite = __syncthreads_and(finite ? 1 : 0);
  const double tol2 = 1e-26 * frob;  // (1e-13 ||A||_F)^2

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
        const double apq = A[p * ld + q];
        double c = 1.0, s = 0.0;
        if (apq != 0.0) {
          const double tau = (A[q * ld + q] - A[p * ld + p]) / (2.0 * apq);
          const double t = tau >= 0.0 ? 1.0 / (tau + sqrt(1.0 + tau * tau)) : -1.0 / (-tau + sqrt(1.0 + tau * tau));
          c = 1.0 / sqrt(1.0 + t * t);
          s = t * c;
        }
        cs[tid] = c;
        cs[half + tid] = s;
        pq[tid] = p;
        pq[half + tid] = q;
      }
      __syncthreads();
      // rows: A <- J^T A
      for (int e = tid; e < half * n; e += kThreads) {
        const int t = e / n, j = e % n;
        const double c = cs[t], s = cs[half + t];
        if (s == 0.0) continue;
        const int p = pq[t], q = pq[half + t];
        const double ap = A[p * ld + j], aq = A[q * ld + j];
        A[p * ld + j] = c * ap - s * aq;
        A[q * ld + j] = s * ap + c * aq;
      }
      __syncthreads();
      // columns: A <- A J, V <- V J
      for (int e = tid; e < 2 * half * n; e += kThreads) {
        const int m = e >= half * n;
        const int f = e - m * half * n;
        const int t = f / n, i = f % n;
        const double c = cs[t], s = cs[half + t];
        if (s == 0.0) continue;
        const int p = pq[t], q = pq[half + t];
        double *M = m ? V : A;
        const double ap = M[i * ld + p], aq = M[i * ld + q];
        M[i * ld + p] = c * ap - s * aq;
        M[i * ld + q] = s * ap + c * aq;
      }
      __syncthreads();
    }
    double off = 0.0;
    for (int e = tid; e < n * n; e += kThreads) {
      const int i = e / n, j = e % n;
      if (i != j) off = fma(A[i * ld + j], A[i * ld + j], off);
    }
    off = block_sum(off, red);
    converged = off <= tol2 ? 1 : 0;
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
    ev_out[rank] = di;
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
  DKV_CUDA_CHECK(cudaFuncSetAttribute(eig::jacobi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max));
  eig::jacobi_kernel<<<static_cast<unsigned>(batch), eig::kThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      a, a_stride, k, n, max_sweeps, evals, evecs, info);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}
