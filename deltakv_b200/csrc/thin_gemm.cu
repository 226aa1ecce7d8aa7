// Thin batched products of the K basis' subspace iteration, C[b] = op(A[b]) B[b] in fp32, on
// the tensor cores with split-precision operands.
//
// The K path's basis (svd_basis, src/deltakv/patches/subspace.py:37-42) is computed by block
// subspace iteration on the probe residual X [m, d] (deltakv_b200.subspace.topr_basis): every
// step forms Y = X Q and Z = X^T Y with Q, Y only 16-96 columns wide, and the Rayleigh-Ritz step
// forms W = X Q.  Those products read X (m x d fp32, ~13 MB per layer) once each and do ~2 k
// flops per element read, so they belong near the HBM roofline — a library fp32 SIMT GEMM runs
// them at 40-60 % of it at these widths.  Here every operand is carried as two bf16 terms
// (x = hi + lo to 2^-16 |x|) and each product as lo*hi + hi*lo + hi*hi with fp32 accumulation on
// mma.sync m16n8k16 (the dropped lo*lo is below 2^-16 of a product), the precision the route's
// own split products use; in the iteration the result agrees with fp32 products to the level
// the converged basis is determined at (projector error against an exact fp64 basis ~1e-6).
//
// Layout: A[b] is [M, K] row-major (lda) or, with trans_a, stored [K, M] row-major (lda) and
// used transposed; B[b] is [K, N] row-major (ldb) with N a multiple of 16 (at most 96); C[b] is
// [M, N] row-major (ldc).  One CTA of 4 warps computes 64 rows of C (128 when N >= 48: two
// m-tiles per warp share each B fragment) x all N columns; K is walked in chunks of 32 staged
// by cp.async two deep.  Within a 16-wide k-step lane (g, q) holds
// physical k = 4q..4q+3 of its rows (a float4), and the B fragments are permuted the same way,
// which leaves the product unchanged; each chunk's B is split into bf16 fragment images once per
// CTA, the A fragments by each warp for its own rows.
#include <algorithm>

#include "dkv_common.cuh"

namespace dkv {
namespace tg {

constexpr int kThreads = 128;
constexpr int kKC = 32;         // k per staged chunk: two 16-wide MMA k-steps
constexpr int kStrideN = 36;    // floats per staged A row, A [M, K]: 32 k + 4 of padding
constexpr int kMaxN = 96;

// MT m-tiles of 16 rows per warp: a CTA computes 64 MT rows of C
template <int MT>
constexpr int tile_m() {
  return 64 * MT;
}
template <int MT>
constexpr int stride_t() {  // floats per staged A row, A stored [K, M]: 64 MT m + 4 of padding
  return tile_m<MT>() + 4;
}
template <int MT>
constexpr int a_stage() {  // floats
  return std::max(tile_m<MT>() * kStrideN, kKC * stride_t<MT>());
}
template <int MT, int NP>
constexpr int smem_bytes() {
  // two stages of A and B (fp32), then the B fragment image [2 terms][2 k-steps][NP/8][32] (uint2)
  return 2 * (a_stage<MT>() + kKC * NP) * 4 + 2 * 2 * (NP / 8) * 32 * 8;
}

template <bool TRANS, int MT, int NP>
__global__ void __launch_bounds__(kThreads) split_gemm_kernel(const float *__restrict__ A, int64_t a_bs,
                                                              int64_t lda, const float *__restrict__ B,
                                                              int64_t b_bs, int64_t ldb, float *__restrict__ Cm,
                                                              int64_t c_bs, int64_t ldc, int M, int K) {
  constexpr int NT = NP / 8;
  constexpr int kTM = tile_m<MT>(), kStrideT = stride_t<MT>(), kAStage = a_stage<MT>();
  extern __shared__ __align__(16) float tg_smem[];
  float *const a_st = tg_smem;                       // [2][kAStage]
  float *const b_st = tg_smem + 2 * kAStage;         // [2][kKC * NP]
  uint2 *const bimg = reinterpret_cast<uint2 *>(tg_smem + 2 * kAStage + 2 * kKC * NP);
  const int64_t bi = blockIdx.y;
  A += bi * a_bs;
  B += bi * b_bs;
  Cm += bi * c_bs;
  const int m0 = blockIdx.x * kTM;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  const int nchunks = (K + kKC - 1) / kKC;

  // one chunk of A and B into stage `buf`; out-of-range float4s are zero-filled from a valid
  // address (K % 4 == 0 for A [M, K], M % 4 == 0 for A stored [K, M]: a float4 is wholly in or out)
  auto stage = [&](int ch, int buf) {
    const int k0 = ch * kKC;
    float *const as = a_st + buf * kAStage;
#pragma unroll
    for (int i = 0; i < 4 * MT; ++i) {
      if constexpr (!TRANS) {
        const int r = (tid >> 3) + 16 * i, c4 = tid & 7;
        const int gm = m0 + r, gk = k0 + 4 * c4;
        const bool ok = gm < M && gk < K;
        cp_async16(as + r * kStrideN + 4 * c4, ok ? A + static_cast<int64_t>(gm) * lda + gk : A, ok ? 16u : 0u);
      } else {
        constexpr int kRow4 = kTM / 4;  // float4s per staged row
        const int e = tid + kThreads * i, r = e / kRow4, c4 = e - r * kRow4;
        const int gk = k0 + r, gm = m0 + 4 * c4;
        const bool ok = gk < K && gm < M;
        cp_async16(as + r * kStrideT + 4 * c4, ok ? A + static_cast<int64_t>(gk) * lda + gm : A, ok ? 16u : 0u);
      }
    }
    float *const bs = b_st + buf * kKC * NP;
    constexpr int kRow4 = NP / 4;
    for (int e = tid; e < kKC * kRow4; e += kThreads) {
      const int r = e / kRow4, c4 = e - r * kRow4;
      const int gk = k0 + r;
      const bool ok = gk < K;
      cp_async16(bs + r * NP + 4 * c4, ok ? B + static_cast<int64_t>(gk) * ldb + 4 * c4 : B, ok ? 16u : 0u);
    }
    cp_async_commit();
  };

  float acc[MT][NT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[t][j][0] = acc[t][j][1] = acc[t][j][2] = acc[t][j][3] = 0.f;

  if (nchunks > 0) stage(0, 0);
  for (int ch = 0; ch < nchunks; ++ch) {
    const int buf = ch & 1;
    if (ch + 1 < nchunks) {
      stage(ch + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // chunk ch is in shared memory for every thread
    const float *const as = a_st + buf * kAStage;
    const float *const bs = b_st + buf * kKC * NP;
    // B fragment image: entry (term, s, j, lane ln = (gg, gq)) holds B[16s + 4gq + {0,1}][8j + gg]
    // and B[16s + 4gq + {2,3}][8j + gg] as bf16 pairs
    for (int e = tid; e < 2 * NT * 32; e += kThreads) {
      const int s = e / (NT * 32), j = (e >> 5) % NT, ln = e & 31;
      const float *col = bs + (16 * s + 4 * (ln & 3)) * NP + 8 * j + (ln >> 2);
      uint32_t h01, l01, h23, l23;
      split_bf16x2(col[0], col[NP], h01, l01);
      split_bf16x2(col[2 * NP], col[3 * NP], h23, l23);
      bimg[(s * NT + j) * 32 + ln] = make_uint2(h01, h23);
      bimg[((2 + s) * NT + j) * 32 + ln] = make_uint2(l01, l23);
    }
    // this warp's A fragments: m-tile t covers rows 16 (MT warp + t) + g and + 8, physical
    // k = 16 s + 4 q .. + 3
    uint32_t ah[MT][2][4], al[MT][2][4];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int rw = 16 * (MT * warp + t) + g;
        float x0[4], x1[4];
        if constexpr (!TRANS) {
          const float4 u = *reinterpret_cast<const float4 *>(as + rw * kStrideN + 16 * s + 4 * q);
          const float4 w = *reinterpret_cast<const float4 *>(as + (rw + 8) * kStrideN + 16 * s + 4 * q);
          x0[0] = u.x, x0[1] = u.y, x0[2] = u.z, x0[3] = u.w;
          x1[0] = w.x, x1[1] = w.y, x1[2] = w.z, x1[3] = w.w;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            x0[i] = as[(16 * s + 4 * q + i) * kStrideT + rw];
            x1[i] = as[(16 * s + 4 * q + i) * kStrideT + rw + 8];
          }
        }
        split_bf16x2(x0[0], x0[1], ah[t][s][0], al[t][s][0]);
        split_bf16x2(x1[0], x1[1], ah[t][s][1], al[t][s][1]);
        split_bf16x2(x0[2], x0[3], ah[t][s][2], al[t][s][2]);
        split_bf16x2(x1[2], x1[3], ah[t][s][3], al[t][s][3]);
      }
    __syncthreads();  // the image is complete
#pragma unroll
    for (int s = 0; s < 2; ++s)
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint2 bh = bimg[(s * NT + j) * 32 + lane], bl = bimg[((2 + s) * NT + j) * 32 + lane];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          mma16816_bf16(acc[t][j], al[t][s][0], al[t][s][1], al[t][s][2], al[t][s][3], bh.x, bh.y);
          mma16816_bf16(acc[t][j], ah[t][s][0], ah[t][s][1], ah[t][s][2], ah[t][s][3], bl.x, bl.y);
          mma16816_bf16(acc[t][j], ah[t][s][0], ah[t][s][1], ah[t][s][2], ah[t][s][3], bh.x, bh.y);
        }
      }
    __syncthreads();  // every warp is done with this stage and the image before they are reused
  }

#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int r0 = m0 + 16 * (MT * warp + t) + g, r1 = r0 + 8;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int col = 8 * j + 2 * q;
      if (r0 < M)
        *reinterpret_cast<float2 *>(Cm + static_cast<int64_t>(r0) * ldc + col) = make_float2(acc[t][j][0], acc[t][j][1]);
      if (r1 < M)
        *reinterpret_cast<float2 *>(Cm + static_cast<int64_t>(r1) * ldc + col) = make_float2(acc[t][j][2], acc[t][j][3]);
    }
  }
}

template <bool TRANS, int NP>
int launch(const float *a, int64_t a_bs, int64_t lda, const float *b, int64_t b_bs, int64_t ldb, float *c,
           int64_t c_bs, int64_t ldc, int64_t batch, int m, int k, cudaStream_t st) {
  // 48 or more columns (the products at ranks 32 and 64, bound by the per-chunk fragment
  // work): 128 rows per CTA, so each chunk's B image serves twice the rows (measured for one
  // rank-64 view: three X Q products 0.81 -> 0.64 ms, two X^T Y 0.60 -> 0.48 ms); narrower
  // products, bound by memory, keep 64 rows and twice the CTAs (three X Q at 16 columns: 0.29
  // vs 0.34 ms)
  constexpr int MT = NP <= 32 ? 1 : 2;
  constexpr int smem = smem_bytes<MT, NP>();
  // set once per device (no runtime-API call on later launches)
  static unsigned long long set_on = 0;
  int dev = 0;
  DKV_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev >= 64 || !((set_on >> dev) & 1ull)) {
    DKV_CUDA_CHECK(cudaFuncSetAttribute(split_gemm_kernel<TRANS, MT, NP>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (dev < 64) set_on |= 1ull << dev;
  }
  const dim3 grid(static_cast<unsigned>((m + tile_m<MT>() - 1) / tile_m<MT>()), static_cast<unsigned>(batch));
  split_gemm_kernel<TRANS, MT, NP><<<grid, kThreads, smem, st>>>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, m, k);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

template <bool TRANS>
int dispatch(int n, const float *a, int64_t a_bs, int64_t lda, const float *b, int64_t b_bs, int64_t ldb, float *c,
             int64_t c_bs, int64_t ldc, int64_t batch, int m, int k, cudaStream_t st) {
  switch (n) {
    case 16: return launch<TRANS, 16>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, batch, m, k, st);
    case 32: return launch<TRANS, 32>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, batch, m, k, st);
    case 48: return launch<TRANS, 48>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, batch, m, k, st);
    case 64: return launch<TRANS, 64>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, batch, m, k, st);
    case 80: return launch<TRANS, 80>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, batch, m, k, st);
    case 96: return launch<TRANS, 96>(a, a_bs, lda, b, b_bs, ldb, c, c_bs, ldc, batch, m, k, st);
    default: return DKV_ERR_UNSUPPORTED;
  }
}

}  // namespace tg
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_split_gemm_batched(const float *a, int64_t a_batch_stride, int64_t lda, int32_t trans_a,
                                      const float *b, int64_t b_batch_stride, int64_t ldb, float *c,
                                      int64_t c_batch_stride, int64_t ldc, int64_t batch, int32_t m, int32_t n,
                                      int32_t k, dkv_stream_t stream) {
  if (batch < 0 || m < 0 || k < 0 || n <= 0) return DKV_ERR_INVALID_ARGUMENT;
  if (n % 16 != 0 || n > tg::kMaxN) return DKV_ERR_UNSUPPORTED;
  if (batch == 0 || m == 0) return DKV_OK;
  if (a == nullptr || b == nullptr || c == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (batch > 65535) return DKV_ERR_UNSUPPORTED;
  if (ldb < n || ldc < n || (trans_a ? lda < m : lda < k)) return DKV_ERR_INVALID_ARGUMENT;
  // 16-byte staging copies: aligned bases, strides in whole float4s, float4s wholly in or out
  auto al16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (!al16(a) || !al16(b) || (reinterpret_cast<uintptr_t>(c) & 7u) != 0) return DKV_ERR_ALIGNMENT;
  if (lda % 4 || ldb % 4 || ldc % 2 || a_batch_stride % 4 || b_batch_stride % 4 || c_batch_stride % 2)
    return DKV_ERR_ALIGNMENT;
  if (trans_a ? (m % 4 != 0) : (k % 4 != 0)) return DKV_ERR_ALIGNMENT;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k == 0) {  // an empty sum: C = 0
    for (int64_t i = 0; i < batch; ++i)
      DKV_CUDA_CHECK(cudaMemset2DAsync(c + i * c_batch_stride, static_cast<size_t>(ldc) * sizeof(float), 0,
                                       static_cast<size_t>(n) * sizeof(float), static_cast<size_t>(m), st));
    return DKV_OK;
  }
  return trans_a ? tg::dispatch<true>(n, a, a_batch_stride, lda, b, b_batch_stride, ldb, c, c_batch_stride, ldc,
                                      batch, m, k, st)
                 : tg::dispatch<false>(n, a, a_batch_stride, lda, b, b_batch_stride, ldb, c, c_batch_stride, ldc,
                                       batch, m, k, st);
}
