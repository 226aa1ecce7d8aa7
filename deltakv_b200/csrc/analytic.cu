// Elementwise and row-wise pieces of the analytic route (Route A,
// src/deltakv/patches/analytic.py), fp32, in the reference's operation order:
//
//   dkv_rmsnorm_first_order  y = x / rms * w, dy = (dx rms - x d_rms) / (rms rms) * w with
//                            rms = sqrt(mean(x^2) + eps), d_rms = 0.5 * 2 mean(x dx) / rms
//                            (rmsnorm_first_order, analytic.py:245-262); one warp per row
//   dkv_swiglu_first_order   h = silu(g) u, dh = silu'(g) dg u + silu(g) du
//                            (mlp_first_order, analytic.py:108-138; silu / silu_grad 98-105)
//   dkv_rope_rows            x * cos + rotate_half(x) * sin at positions 0..n-1 for a
//                            [n, heads, head_dim] tensor (rope.py:9-63), in place
#include "dkv_common.cuh"

namespace dkv {
namespace analytic {

__global__ void rmsnorm_fo_kernel(const float *x, const float *dx, const float *w, float eps, int64_t rows,
                                  int d, int64_t xs, int64_t dxs, float *y, float *dy, int64_t ys, int64_t dys) {
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float *xr = x + row * xs, *dxr = dx + row * dxs;
  float sxx = 0.f, sxd = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float a = xr[i], b = dxr[i];
    sxx = fmaf(a, a, sxx);
    sxd = fmaf(a, b, sxd);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sxx += __shfl_xor_sync(0xffffffffu, sxx, o);
    sxd += __shfl_xor_sync(0xffffffffu, sxd, o);
  }
  const float ms = __fdiv_rn(sxx, static_cast<float>(d));
  const float rms = __fsqrt_rn(__fadd_rn(ms, eps));
  const float d_ms = __fmul_rn(2.f, __fdiv_rn(sxd, static_cast<float>(d)));
  const float d_rms = __fdiv_rn(__fmul_rn(0.5f, d_ms), rms);
  const float rr = __fmul_rn(rms, rms);
  float *yr = y + row * ys, *dyr = dy + row * dys;
  for (int i = lane; i < d; i += 32) {
    const float a = xr[i], b = dxr[i], wi = w[i];
    yr[i] = __fmul_rn(__fdiv_rn(a, rms), wi);
    dyr[i] = __fmul_rn(__fdiv_rn(__fsub_rn(__fmul_rn(b, rms), __fmul_rn(a, d_rms)), rr), wi);
  }
}

__device__ __forceinline__ float sigmoid(float x) { return __fdiv_rn(1.f, __fadd_rn(1.f, expf(-x))); }

__global__ void swiglu_fo_kernel(const float *g, const float *u, const float *dg, const float *du, int64_t n,
                                 float *h, float *dh) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gi = g[i], ui = u[i];
    const float s = sigmoid(gi);
    const float silu = __fmul_rn(gi, s);
    const float grad = __fadd_rn(s, __fmul_rn(__fmul_rn(gi, s), __fsub_rn(1.f, s)));
    h[i] = __fmul_rn(silu, ui);
    dh[i] = __fadd_rn(__fmul_rn(__fmul_rn(grad, dg[i]), ui), __fmul_rn(silu, du[i]));
  }
}

// x[t, head, i] for i < hd/2 pairs with i + hd/2; cos/sin are the half-width tables
__global__ void rope_rows_kernel(float *x, int64_t rows, int heads, int hd, int64_t row_stride,
                                 const float *cos_t, const float *sin_t) {
  const int half = hd / 2;
  const int64_t total = rows * heads * half;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(e % half);
    const int64_t rh = e / half;
    const int hh = static_cast<int>(rh % heads);
    const int64_t t = rh / heads;
    float *p = x + t * row_stride + static_cast<int64_t>(hh) * hd;
    const float c = cos_t[t * half + i], s = sin_t[t * half + i];
    const float lo = p[i], hi = p[i + half];
    p[i] = __fadd_rn(__fmul_rn(lo, c), __fmul_rn(-hi, s));
    p[i + half] = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
  }
}

inline unsigned grid_for(int64_t n, int threads) {
  const int64_t b = (n + threads - 1) / threads;
  return static_cast<unsigned>(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

}  // namespace analytic
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_rmsnorm_first_order(const float *x, const float *dx, const float *w, float eps, int64_t rows,
                                       int32_t d, int64_t x_row_stride, int64_t dx_row_stride, float *y,
                                       float *dy, int64_t y_row_stride, int64_t dy_row_stride,
                                       dkv_stream_t stream) {
  if (rows < 0 || d <= 0) return DKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DKV_OK;
  if (!x || !dx || !w || !y || !dy) return DKV_ERR_INVALID_ARGUMENT;
  if (x_row_stride < d || dx_row_stride < d || y_row_stride < d || dy_row_stride < d) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t blocks = (rows * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  analytic::rmsnorm_fo_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, dx, w, eps, rows, d, x_row_stride, dx_row_stride, y, dy, y_row_stride, dy_row_stride);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

extern "C" int dkv_swiglu_first_order(const float *g, const float *u, const float *dg, const float *du, int64_t n,
                                      float *h, float *dh, dkv_stream_t stream) {
  if (n < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (n == 0) return DKV_OK;
  if (!g || !u || !dg || !du || !h || !dh) return DKV_ERR_INVALID_ARGUMENT;
  analytic::swiglu_fo_kernel<<<analytic::grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      g, u, dg, du, n, h, dh);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

extern "C" int dkv_rope_rows(float *x, int64_t rows, int32_t heads, int32_t head_dim, int64_t row_stride,
                             const float *cos_half, const float *sin_half, int64_t table_rows,
                             dkv_stream_t stream) {
  if (rows < 0 || heads <= 0 || head_dim <= 0 || head_dim % 2) return DKV_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DKV_OK;
  if (!x || !cos_half || !sin_half) return DKV_ERR_INVALID_ARGUMENT;
  if (rows > table_rows) return DKV_ERR_ROPE_RANGE;
  if (row_stride < static_cast<int64_t>(heads) * head_dim) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t total = rows * heads * (head_dim / 2);
  analytic::rope_rows_kernel<<<analytic::grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, rows, heads, head_dim, row_stride, cos_half, sin_half);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}
