// Probe scoring and the CacheBlend residual gate of the subspace route.
//
//   dkv_lora_scores     out[t] (+)= || scale * x[t] @ A^T ||  — the reference's
//                       lora_activation_scores (src/deltakv/patches/exact.py:111-115), summed
//                       over the adapter's projections by weight_axis_scores
//                       (src/deltakv/patches/probe.py:30-47) to rank probe tokens.
//   dkv_row_diff_norms  out[i] = || a[r_i] - b[r_i] ||  — the per-token residual estimates of
//                       residual_gate (src/deltakv/patches/probe.py:85-109).
//
// Scores: 64 tokens per CTA, 256 threads (4 per token, each a quarter of the codes); x and A
// are staged in shared memory 128 channels at a time; fp32 accumulation.
#include "dkv_common.cuh"

namespace dkv {
namespace probe {

constexpr int kTok = 64;
constexpr int kKC = 128;
constexpr int kThreads = 256;
constexpr int kMaxRank = 64;

__global__ void __launch_bounds__(kThreads) lora_scores_kernel(const void *x, int xdt, int64_t rows, int64_t d,
                                                               int64_t xrs, const float *a, int r, float scale,
                                                               float *out, int accumulate) {
  extern __shared__ float sm[];
  float *xs = sm;                     // [kTok][kKC + 1]
  float *as = sm + kTok * (kKC + 1);  // [r][kKC + 1]
  const int tid = threadIdx.x;
  const int lt = tid >> 2, part = tid & 3;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kTok;
  const int per = (r + 3) / 4;  // codes per thread
  float acc[kMaxRank / 4];
#pragma unroll
  for (int j = 0; j < kMaxRank / 4; ++j) acc[j] = 0.f;
  for (int64_t c0 = 0; c0 < d; c0 += kKC) {
    for (int e = tid; e < kTok * kKC; e += kThreads) {
      const int tt = e / kKC, cc = e % kKC;
      const int64_t t = t0 + tt, c = c0 + cc;
      xs[tt * (kKC + 1) + cc] = (t < rows && c < d) ? load_as_float(x, xdt, t * xrs + c) : 0.f;
    }
    for (int e = tid; e < r * kKC; e += kThreads) {
      const int k = e / kKC, cc = e % kKC;
      const int64_t c = c0 + cc;
      as[k * (kKC + 1) + cc] = c < d ? a[k * d + c] : 0.f;
    }
    __syncthreads();
    const float *xr = xs + lt * (kKC + 1);
#pragma unroll 4
    for (int cc = 0; cc < kKC; ++cc) {
      const float xv = xr[cc];
#pragma unroll
      for (int j = 0; j < kMaxRank / 4; ++j) {
        const int k = part * per + j;
        if (j < per && k < r) acc[j] = fmaf(xv, as[k * (kKC + 1) + cc], acc[j]);
      }
    }
    __syncthreads();
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxRank / 4; ++j) {
    const float cv = scale * acc[j];
    if (j < per && part * per + j < r) ss = fmaf(cv, cv, ss);
  }
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  const int64_t t = t0 + lt;
  if (part == 0 && t < rows) {
    const float v = sqrtf(ss);
    out[t] = accumulate ? out[t] + v : v;
  }
}

// one warp per output row
__global__ void row_diff_norms_kernel(const void *a, const void *b, int dt, int64_t cols, int64_t as_,
                                      int64_t bs_, const int32_t *rows, int64_t n_out, int64_t n_rows, float *out,
                                      int32_t *status) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n_out) return;
  const int64_t r = rows ? rows[i] : i;
  if (r < 0 || r >= n_rows) {
    if (lane == 0) {
      record_error(status, DKV_ERR_INVALID_ARGUMENT);
      out[i] = 0.f;
    }
    return;
  }
  float s = 0.f;
  for (int64_t c = lane; c < cols; c += 32) {
    const float v = load_as_float(a, dt, r * as_ + c) - load_as_float(b, dt, r * bs_ + c);
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) out[i] = sqrtf(s);
}

}  // namespace probe
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_lora_scores(const void *x, int32_t x_dtype, int64_t rows, int64_t d, int64_t x_row_stride,
                               const float *a, int32_t rank, float scale, float *out, int32_t accumulate,
                               dkv_stream_t stream) {
  if (rows < 0 || d <= 0 || rank <= 0 || rank > probe::kMaxRank) return DKV_ERR_INVALID_ARGUMENT;
  if (x_dtype != DKV_F32 && x_dtype != DKV_F16 && x_dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (rows == 0) return DKV_OK;
  if (x == nullptr || a == nullptr || out == nullptr || x_row_stride < d) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t blocks = (rows + probe::kTok - 1) / probe::kTok;
  if (blocks > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  const size_t smem = static_cast<size_t>(probe::kTok + rank) * (probe::kKC + 1) * sizeof(float);
  DKV_CUDA_CHECK(cudaFuncSetAttribute(probe::lora_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>((probe::kTok + probe::kMaxRank) * (probe::kKC + 1) * 4)));
  probe::lora_scores_kernel<<<static_cast<unsigned>(blocks), probe::kThreads, smem,
                              static_cast<cudaStream_t>(stream)>>>(x, x_dtype, rows, d, x_row_stride, a, rank,
                                                                   scale, out, accumulate ? 1 : 0);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

extern "C" int dkv_row_diff_norms(const void *a, const void *b, int32_t dtype, int64_t n_rows, int64_t cols,
                                  int64_t a_row_stride, int64_t b_row_stride, const int32_t *rows, int64_t n_out,
                                  float *out, int32_t *status, dkv_stream_t stream) {
  if (n_rows < 0 || cols <= 0 || n_out < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (dtype != DKV_F32 && dtype != DKV_F16 && dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (n_out == 0) return DKV_OK;
  if (a == nullptr || b == nullptr || out == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (rows == nullptr && n_out > n_rows) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t threads = n_out * 32;
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  probe::row_diff_norms_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, b, dtype, cols, a_row_stride, b_row_stride, rows, n_out, n_rows, out, status);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}
