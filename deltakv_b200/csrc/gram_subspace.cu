// Block subspace iteration on a small symmetric positive semi-definite fp64 matrix G (d x d),
// the Gram matrix dX^T dX of the analytic route's rank truncation (rank_truncate,
// src/deltakv/patches/analytic.py:14-22): Q <- orth(G Q) with Cholesky QR, two kernels per
// iteration, followed by the Rayleigh quotient T = Q^T G Q for a Rayleigh-Ritz step
// (Golub & Van Loan, Matrix Computations 4th ed., Sec. 8.2.4).
//
//   gq_kernel     Y[rows] = G[rows, :] Q for 16 rows per CTA: Q (each 32-row chunk one
//                 contiguous range) and the CTA's columns of G stream through a 3-deep cp.async
//                 ring (two CTAs fit an SM, so launches of concurrent callers share SMs); each
//                 warp takes 4 rows of a chunk into a 16 x 96 register tile (every Q value
//                 loaded from shared memory feeds 16 FMAs); the warps' tiles are summed, then
//                 the partial product A^T Y of those rows is added into W with fp64 atomics
//                 (A = Y: the upper triangle of Y^T Y; A = Q: all of Q^T G Q)
//   cholqr_kernel W = U^T D^-1 U (right-looking elimination, the trailing matrix in the
//                 registers of 16 warps, one barrier per pivot) and, in the same loop, the
//                 forward substitution of this CTA's 64 rows of Y: Q = Y R^-1 with
//                 R = D^-1/2 U, so Q^T Q = I; every CTA factors W redundantly (64 rows per CTA
//                 keep that redundant work, and the SMs a launch holds, small)
//
// G is read by columns (G[j][row], contiguous for a CTA's rows): G must be symmetric.
#include "dkv_common.cuh"

namespace dkv {
namespace gsi {

constexpr int kMaxK = 96;
constexpr int kCols = kMaxK / 32;  // columns per lane: lane, lane + 32, lane + 64

// ---- gq_kernel: 16 rows of Y per CTA, 8 warps splitting each chunk's rows j ----
constexpr int kGRows = 16;
constexpr int kGWarps = 8;
constexpr int kGThreads = kGWarps * 32;
constexpr int kGWRows = kMaxK / kGWarps;  // rows a of the partial product per warp
constexpr int kChunk = 32;                // rows j of Q (and of G's columns) per ring stage
constexpr int kStages = 3;                // ring depth (86 KB of shared memory: two CTAs per SM)
constexpr int kQStage = kChunk * kMaxK;   // doubles (a chunk is 32 * k contiguous doubles of Q)
constexpr int kGStage = kChunk * kGRows;  // doubles: G[j][row0 .. row0 + 15] for the chunk's j
constexpr size_t kGqSmem = static_cast<size_t>(kStages) * (kQStage + kGStage) * sizeof(double);
static_assert(kGqSmem >= sizeof(double) * (kGWarps / 2) * kGRows * kMaxK, "the reduction tiles reuse the ring");
static_assert(kChunk % kGWarps == 0, "each warp takes kChunk / kGWarps rows of a chunk");

// ---- cholqr_kernel: 16 warps, four rows of Y each; W rows a = warp + 16 ia ----
constexpr int kCWarps = 16;
constexpr int kCThreads = kCWarps * 32;
constexpr int kCYRows = 4;  // rows of Y per warp: few CTAs factor W redundantly (SM time)
constexpr int kCRows = kCWarps * kCYRows;
constexpr int kCWRows = kMaxK / kCWarps;

template <bool kRayleigh, bool kVec16>
__global__ void __launch_bounds__(kGThreads) gq_kernel(const double *__restrict__ g, int d,
                                                       const double *__restrict__ q, int k,
                                                       double *__restrict__ y, double *__restrict__ w) {
  extern __shared__ double smem_d[];
  double *qs = smem_d;                      // [kStages][kChunk * k]
  double *gs = smem_d + kStages * kQStage;  // [kStages][kChunk][kGRows]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kGRows;
  const int nrows = min(kGRows, d - row0);
  const int n_chunks = (d + kChunk - 1) / kChunk;

  // one chunk: Q rows jbase .. jbase + 31 (one contiguous range of 32 k doubles) and
  // G[j][row0 .. row0 + 15] (= G[row0 ..][j]); out-of-range elements are zero-filled
  auto issue = [&](int ch) {
    const int st = ch % kStages, jbase = ch * kChunk;
    double *qd = qs + st * kQStage, *gd = gs + st * kGStage;
    const int nvalid = min(kChunk, d - jbase) * k, ntot = kChunk * k;
    const double *src = q + static_cast<int64_t>(jbase) * k;
    if (kVec16) {
      for (int e = 2 * threadIdx.x; e < ntot; e += 2 * kGThreads) {
        const bool ok = e < nvalid;
        cp_async16(qd + e, ok ? src + e : q, ok ? 16u : 0u);
      }
    } else {
      for (int e = threadIdx.x; e < ntot; e += kGThreads) {
        const bool ok = e < nvalid;
        cp_async8(qd + e, ok ? src + e : q, ok ? 8u : 0u);
      }
    }
    for (int e = threadIdx.x; e < kGStage; e += kGThreads) {
      const int jj = e / kGRows, r = e - jj * kGRows, j = jbase + jj;
      const bool ok = j < d && r < nrows;
      cp_async8(gd + e, ok ? g + static_cast<int64_t>(j) * d + row0 + r : g, ok ? 8u : 0u);
    }
  };

  double acc[kGRows][kCols];
#pragma unroll
  for (int r = 0; r < kGRows; ++r)
#pragma unroll
    for (int i = 0; i < kCols; ++i) acc[r][i] = 0.0;
  bool colv[kCols];
#pragma unroll
  for (int i = 0; i < kCols; ++i) colv[i] = lane + 32 * i < k;

#pragma unroll 1
  for (int st = 0; st < kStages - 1; ++st) {
    if (st < n_chunks) issue(st);
    cp_async_commit();
  }
#pragma unroll 1
  for (int ch = 0; ch < n_chunks; ++ch) {
    // the slot refilled here was read in iteration ch - 1, which ended with a barrier
    if (ch + kStages - 1 < n_chunks) issue(ch + kStages - 1);
    cp_async_commit();
    cp_async_wait<kStages - 1>();
    __syncthreads();
    const double *qd = qs + (ch % kStages) * kQStage, *gd = gs + (ch % kStages) * kGStage;
#pragma unroll
    for (int u = 0; u < kChunk / kGWarps; ++u) {
      const int jj = warp * (kChunk / kGWarps) + u;
      double qv[kCols], gv[kGRows];
#pragma unroll
      for (int i = 0; i < kCols; ++i) qv[i] = colv[i] ? qd[jj * k + lane + 32 * i] : 0.0;
#pragma unroll
      for (int r = 0; r < kGRows; r += 2) {
        const double2 two = *reinterpret_cast<const double2 *>(gd + jj * kGRows + r);
        gv[r] = two.x;
        gv[r + 1] = two.y;
      }
#pragma unroll
      for (int r = 0; r < kGRows; ++r)
#pragma unroll
        for (int i = 0; i < kCols; ++i) acc[r][i] = fma(gv[r], qv[i], acc[r][i]);
    }
    __syncthreads();
  }
  cp_async_wait<0>();  // only empty groups remain; the ring is reused below

  // the warps' tiles, summed in two rounds through kGWarps / 2 tiles: warps 0-3 store, then
  // warps 4-7 add theirs to the same positions
  constexpr int kHalf = kGWarps / 2;
  double(*part)[kGRows][kMaxK] = reinterpret_cast<double(*)[kGRows][kMaxK]>(smem_d);  // [kHalf]
  if (warp < kHalf)
#pragma unroll
    for (int r = 0; r < kGRows; ++r)
#pragma unroll
      for (int i = 0; i < kCols; ++i) part[warp][r][lane + 32 * i] = acc[r][i];
  __syncthreads();
  if (warp >= kHalf)
#pragma unroll
    for (int r = 0; r < kGRows; ++r)
#pragma unroll
      for (int i = 0; i < kCols; ++i) part[warp - kHalf][r][lane + 32 * i] += acc[r][i];
  __syncthreads();

  // element (r, c) has one owner thread, which alone reads part[*][r][c] and then overwrites
  // part[0][r][c] (Y) and part[1][r][c] (A)
  for (int o = threadIdx.x; o < kGRows * kMaxK; o += kGThreads) {
    const int r = o / kMaxK, c = o - r * kMaxK;
    double s = 0.0;
#pragma unroll
    for (int v = 0; v < kHalf; ++v) s += part[v][r][c];
    const bool live = r < nrows && c < k;
    if (!live) s = 0.0;
    if (live) y[static_cast<int64_t>(row0 + r) * k + c] = s;
    part[0][r][c] = s;
    if (kRayleigh) part[1][r][c] = live ? q[static_cast<int64_t>(row0 + r) * k + c] : 0.0;
  }
  __syncthreads();

  const double(*ys)[kMaxK] = part[0];
  const double(*as)[kMaxK] = kRayleigh ? part[1] : part[0];
#pragma unroll
  for (int ia = 0; ia < kGWRows; ++ia) {
    const int a = warp + kGWarps * ia;
    double av[kGRows];
#pragma unroll
    for (int r = 0; r < kGRows; ++r) av[r] = as[r][a];
#pragma unroll
    for (int i = 0; i < kCols; ++i) {
      const int b = lane + 32 * i;
      if (a < k && b < k && (kRayleigh || b >= a)) {
        double s = 0.0;
#pragma unroll
        for (int r = 0; r < kGRows; ++r) s = fma(av[r], ys[r][b], s);
        atomicAdd(w + static_cast<int64_t>(a) * k + b, s);
      }
    }
  }
}

// 1/a and 1/sqrt(a) for a > 0 to ~1 ulp: a hardware approximation refined by two
// Newton-Raphson steps (x <- x (2 - a x); y <- y (3 - a y^2) / 2), each of which squares the
// relative error (Muller et al., Handbook of Floating-Point Arithmetic, 2nd ed., Sec. 4.7)
__device__ __forceinline__ double recip(double a) {
  double x;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(x) : "d"(a));
  x = fma(x, fma(-a, x, 1.0), x);
  return fma(x, fma(-a, x, 1.0), x);
}
__device__ __forceinline__ double rsqrt_nr(double a) {
  double y;
  asm("rsqrt.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(a));
  y = y * fma(-0.5 * a * y, y, 1.5);
  return y * fma(-0.5 * a * y, y, 1.5);
}

__global__ void __launch_bounds__(kCThreads) cholqr_kernel(const double *__restrict__ w, int k,
                                                           const double *__restrict__ y, int d,
                                                           double *__restrict__ q, double *__restrict__ w_clear,
                                                           int32_t *__restrict__ status) {
  __shared__ double prow[2][kMaxK];  // pivot row of the trailing matrix, double-buffered
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kCRows + warp * kCYRows;  // this warp's rows

  // element (a, b) = (warp + 16 ia, lane + 32 ib) of the symmetric W (stored: upper triangle)
  double wr[kCWRows][kCols];
#pragma unroll
  for (int ia = 0; ia < kCWRows; ++ia)
#pragma unroll
    for (int ib = 0; ib < kCols; ++ib) {
      const int a = warp + kCWarps * ia, b = lane + 32 * ib;
      wr[ia][ib] = (a < k && b < k) ? w[static_cast<int64_t>(min(a, b)) * k + max(a, b)] : 0.0;
    }
  double yv[kCYRows][kCols], qv[kCYRows][kCols];
#pragma unroll
  for (int u = 0; u < kCYRows; ++u)
#pragma unroll
    for (int ib = 0; ib < kCols; ++ib) {
      const int c = lane + 32 * ib;
      yv[u][ib] = (row0 + u < d && c < k) ? y[static_cast<int64_t>(row0 + u) * k + c] : 0.0;
      qv[u][ib] = 0.0;
    }
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e < k * k; e += kCThreads) w_clear[e] = 0.0;
  if (warp == 0)
#pragma unroll
    for (int ib = 0; ib < kCols; ++ib) prow[0][lane + 32 * ib] = wr[0][ib];
  __syncthreads();

  const double w00 = prow[0][0];
  bool ok = true;
  // pivot j = 16 jb + jw: the outer loop is unrolled so that the register rows a pivot touches
  // (ia >= jb), the row it publishes next (ia = jb or jb + 1) and the lane slot of y_j
  // (jb / 2) are compile-time indices; the updates are branch-free (rows and columns at or
  // before the pivot get a zero multiplier) so that every shared-memory load of a step is in
  // flight at once
#pragma unroll
  for (int jb = 0; jb < kCWRows; ++jb) {
#pragma unroll 1
    for (int jw = 0; jw < kCWarps; ++jw) {
      const int j = kCWarps * jb + jw;
      if (j >= k) break;
      const double *pr = prow[j & 1];
      double pa[kCWRows], pbr[kCols];
#pragma unroll
      for (int ia = jb; ia < kCWRows; ++ia) {
        const int a = warp + kCWarps * ia;
        pa[ia] = (a > j && a < k) ? pr[a] : 0.0;
      }
#pragma unroll
      for (int ib = 0; ib < kCols; ++ib) {
        const int b = lane + 32 * ib;
        pbr[ib] = (b > j && b < k) ? pr[b] : 0.0;
      }
      const double piv = pr[j];
      // uniform (every thread reads the same pivot); below 1e-12 of the first the block has
      // lost rank (kappa(Y) > 1e6) and Cholesky QR no longer keeps its span
      if (!(piv > 1e-12 * w00) || !isfinite(piv)) {
        ok = false;
        break;
      }
      const double inv = recip(piv), rs = rsqrt_nr(piv);
      double pb[kCols];
#pragma unroll
      for (int ib = 0; ib < kCols; ++ib) pb[ib] = pbr[ib] * inv;
#pragma unroll
      for (int ia = jb; ia < kCWRows; ++ia)
#pragma unroll
        for (int ib = 0; ib < kCols; ++ib) wr[ia][ib] = fma(-pa[ia], pb[ib], wr[ia][ib]);
      // forward substitution of this warp's rows: q_j = y_j / sqrt(piv), y_c -= (y_j / piv) U_jc
      const int kSlot = jb / 2;  // j / 32 (jb is a compile-time index after unrolling)
#pragma unroll
      for (int u = 0; u < kCYRows; ++u) {
        const double yj = __shfl_sync(0xffffffffu, yv[u][kSlot], j & 31);
        if (lane == (j & 31)) qv[u][kSlot] = yj * rs;
#pragma unroll
        for (int ib = 0; ib < kCols; ++ib) yv[u][ib] = fma(-yj, pb[ib], yv[u][ib]);
      }
      // the owner warp of row j + 1 publishes it (already updated by this pivot)
      const int nj = j + 1;
      if (nj < k && warp == (nj & (kCWarps - 1))) {
        if (jw == kCWarps - 1) {
          if (jb + 1 < kCWRows)
#pragma unroll
            for (int ib = 0; ib < kCols; ++ib)
              prow[nj & 1][lane + 32 * ib] = wr[jb + 1 < kCWRows ? jb + 1 : jb][ib];
        } else {
#pragma unroll
          for (int ib = 0; ib < kCols; ++ib) prow[nj & 1][lane + 32 * ib] = wr[jb][ib];
        }
      }
      __syncthreads();
    }
    if (!ok) break;
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicOr(status, 1);
    return;
  }
#pragma unroll
  for (int u = 0; u < kCYRows; ++u)
#pragma unroll
    for (int ib = 0; ib < kCols; ++ib) {
      const int c = lane + 32 * ib;
      if (row0 + u < d && c < k) q[static_cast<int64_t>(row0 + u) * k + c] = qv[u][ib];
    }
}

template <bool kRayleigh, bool kVec16>
int launch_gq(const double *g, int d, const double *q, int k, double *y, double *w, cudaStream_t s) {
  // the shared-memory attribute, set once per device for this instantiation (a repeated set
  // from racing threads is harmless)
  static unsigned long long set_on = 0;
  int dev = 0;
  DKV_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev >= 64 || !((set_on >> dev) & 1ull)) {
    DKV_CUDA_CHECK(cudaFuncSetAttribute(gq_kernel<kRayleigh, kVec16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(kGqSmem)));
    if (dev < 64) set_on |= 1ull << dev;
  }
  const unsigned grid = static_cast<unsigned>((d + kGRows - 1) / kGRows);
  gq_kernel<kRayleigh, kVec16><<<grid, kGThreads, kGqSmem, s>>>(g, d, q, k, y, w);
  return DKV_OK;
}

}  // namespace gsi
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_gram_subspace_iterate(const double *g, int32_t d, double *q, int32_t k, int32_t iters, double *y,
                                         double *w, double *t, int32_t *status, dkv_stream_t stream) {
  if (d <= 0 || k <= 0 || k > gsi::kMaxK || k > d || iters < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (!g || !q || !y || !w || !status) return DKV_ERR_INVALID_ARGUMENT;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 16-byte copies of Q's chunks need 16-byte aligned rows
  const bool vec16 = (k % 2 == 0) && (reinterpret_cast<uintptr_t>(q) % 16 == 0);
  auto gq = [&](bool rayleigh, double *acc) {
    if (rayleigh) return vec16 ? gsi::launch_gq<true, true>(g, d, q, k, y, acc, s)
                               : gsi::launch_gq<true, false>(g, d, q, k, y, acc, s);
    return vec16 ? gsi::launch_gq<false, true>(g, d, q, k, y, acc, s) : gsi::launch_gq<false, false>(g, d, q, k, y, acc, s);
  };
  const unsigned cgrid = static_cast<unsigned>((d + gsi::kCRows - 1) / gsi::kCRows);
  const size_t kk = static_cast<size_t>(k) * k;
  DKV_CUDA_CHECK(cudaMemsetAsync(status, 0, sizeof(int32_t), s));
  DKV_CUDA_CHECK(cudaMemsetAsync(w, 0, 2 * kk * sizeof(double), s));
  for (int it = 0; it < iters; ++it) {
    double *cur = w + (it & 1) * kk, *nxt = w + ((it + 1) & 1) * kk;
    const int rc = gq(false, cur);
    if (rc != DKV_OK) return rc;
    gsi::cholqr_kernel<<<cgrid, gsi::kCThreads, 0, s>>>(cur, k, y, d, q, nxt, status);
  }
  if (t) {
    DKV_CUDA_CHECK(cudaMemsetAsync(t, 0, kk * sizeof(double), s));
    const int rc = gq(true, t);
    if (rc != DKV_OK) return rc;
  }
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}
