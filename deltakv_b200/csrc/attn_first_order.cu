// First-order causal attention — the O(n^2) core of the analytic route (Route A,
// src/deltakv/patches/analytic.py:38-105 attention_first_order):
//
//   S = Q K^T / sqrt(hd) + causal,  A = softmax(S),  dS = (dQ K^T + Q dK^T) / sqrt(hd)
//   dA = A (.) (dS - rowsum(A (.) dS))          (softmax_jacobian_product, analytic.py:25-35)
//   ctx = A V,   dctx = dA V + A dV
//
// per query head h with its GQA key/value head h / (H / Hkv) (analytic.py:142-153), without
// materialising the [H, n, n] matrices.  Two passes over the causal keys of each query row:
// pass 1 forms the row statistics m = max S, l = sum exp(S - m), t = sum exp(S - m) dS
// online; pass 2 recomputes S and dS and accumulates
//   dctx = sum_k a_k (dS_k - t / l) v_k + a_k dv_k,   ctx = sum_k a_k v_k,   a_k = exp(S_k - m) / l.
// fp32 arithmetic throughout (the reference runs the route in the model dtype, fp32 for the
// toy).  Mapping: 64 query rows per CTA, a quad of 4 threads per row, each thread holding a
// quarter of head_dim of Q, dQ and of the outputs; key blocks of 32 rows of K, dK, V, dV are
// staged in shared memory; the quad reduces its partial dot products with two shuffles.
#include "dkv_common.cuh"

namespace dkv {
namespace afo {

constexpr int kRows = 64;   // query rows per CTA
constexpr int kKeys = 32;   // keys per staged block
constexpr int kThreads = 4 * kRows;
constexpr int kMaxHd = 128;
constexpr int kMaxSlice = kMaxHd / 4;

template <int DT>
__device__ __forceinline__ float ld(const void *p, int64_t i) {
  if (DT == DKV_F32) return static_cast<const float *>(p)[i];
  if (DT == DKV_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
  return __half2float(static_cast<const __half *>(p)[i]);
}

struct Args {
  const void *q, *dq, *k, *dk, *v, *dv;
  int64_t q_row, kv_row;  // element strides between tokens (heads x head_dim when packed)
  float *ctx, *dctx;      // [n, H, hd] fp32, row stride out_row; ctx may be null
  int64_t out_row;
  int n, n_heads, n_kv, hd;
  float scale;
};

template <int DT, int SL>  // SL: head_dim / 4 (values per thread)
__global__ void __launch_bounds__(kThreads) afo_kernel(const Args a) {
  extern __shared__ float sm[];
  // staged key block: [4 tensors][kKeys][hd]
  float *Ks = sm, *dKs = sm + kKeys * a.hd, *Vs = sm + 2 * kKeys * a.hd, *dVs = sm + 3 * kKeys * a.hd;
  const int h = blockIdx.y, hk = h / (a.n_heads / a.n_kv);
  const int q0 = blockIdx.x * kRows;
  const int r = threadIdx.x >> 2, part = threadIdx.x & 3;
  const int row = q0 + r;
  const bool valid = row < a.n;
  const int d0 = part * SL;
  float qv[SL], dqv[SL];
#pragma unroll
  for (int j = 0; j < SL; ++j) {
    const int64_t o = static_cast<int64_t>(valid ? row : 0) * a.q_row + static_cast<int64_t>(h) * a.hd + d0 + j;
    qv[j] = ld<DT>(a.q, o) * a.scale;  // the 1/sqrt(hd) of S and dS folded into Q and dQ
    dqv[j] = ld<DT>(a.dq, o) * a.scale;
  }
  const int last_key = min(q0 + kRows, a.n);  // keys [0, last_key) reach some row of this CTA
  const int n_blocks = (last_key + kKeys - 1) / kKeys;

  auto stage = [&](int kb) {
    const int k0 = kb * kKeys;
    for (int e = threadIdx.x; e < kKeys * a.hd; e += kThreads) {
      const int kk = e / a.hd, d = e - kk * a.hd;
      const int key = k0 + kk;
      const bool ok = key < a.n;
      const int64_t o = static_cast<int64_t>(ok ? key : 0) * a.kv_row + static_cast<int64_t>(hk) * a.hd + d;
      Ks[e] = ok ? ld<DT>(a.k, o) : 0.f;
      dKs[e] = ok ? ld<DT>(a.dk, o) : 0.f;
      Vs[e] = ok ? ld<DT>(a.v, o) : 0.f;
      dVs[e] = ok ? ld<DT>(a.dv, o) : 0.f;
    }
  };
  // s = q.k and ds = dq.k + q.dk for key kk of the staged block, summed over the quad
  auto scores = [&](int kk, float &s, float &ds) {
    const float *kr = Ks + kk * a.hd + d0, *dkr = dKs + kk * a.hd + d0;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < SL; ++j) {
      s0 = fmaf(qv[j], kr[j], s0);
      s1 = fmaf(dqv[j], kr[j], s1);
      s1 = fmaf(qv[j], dkr[j], s1);
    }
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    s = s0;
    ds = s1;
  };

  // pass 1: row statistics
  float m = -INFINITY, l = 0.f, t = 0.f;
  for (int kb = 0; kb < n_blocks; ++kb) {
    __syncthreads();
    stage(kb);
    __syncthreads();
    const int k0 = kb * kKeys;
    for (int kk = 0; kk < kKeys; ++kk) {
      const int key = k0 + kk;
      if (key >= last_key) break;  // uniform across the CTA
      float s, ds;
      scores(kk, s, ds);
      if (!valid || key > row) continue;  // causal (the shuffles above ran on all lanes)
      if (s > m) {
        const float c = expf(m - s);
        l *= c;
        t *= c;
        m = s;
      }
      const float p = expf(s - m);
      l += p;
      t = fmaf(p, ds, t);
    }
  }
  const float inv_l = valid && l > 0.f ? 1.f / l : 0.f;
  const float tbar = t * inv_l;  // rowsum(A (.) dS)

  // pass 2: outputs
  float oc[SL], od[SL];
#pragma unroll
  for (int j = 0; j < SL; ++j) oc[j] = od[j] = 0.f;
  for (int kb = 0; kb < n_blocks; ++kb) {
    __syncthreads();
    stage(kb);
    __syncthreads();
    const int k0 = kb * kKeys;
    for (int kk = 0; kk < kKeys; ++kk) {
      const int key = k0 + kk;
      if (key >= last_key) break;
      float s, ds;
      scores(kk, s, ds);
      if (!valid || key > row) continue;
      const float aa = expf(s - m) * inv_l;
      const float da = aa * (ds - tbar);
      const float *vr = Vs + kk * a.hd + d0, *dvr = dVs + kk * a.hd + d0;
#pragma unroll
      for (int j = 0; j < SL; ++j) {
        od[j] = fmaf(da, vr[j], fmaf(aa, dvr[j], od[j]));
        oc[j] = fmaf(aa, vr[j], oc[j]);
      }
    }
  }
  if (valid) {
    float *o = a.dctx + static_cast<int64_t>(row) * a.out_row + static_cast<int64_t>(h) * a.hd + d0;
#pragma unroll
    for (int j = 0; j < SL; ++j) o[j] = od[j];
    if (a.ctx) {
      float *c = a.ctx + static_cast<int64_t>(row) * a.out_row + static_cast<int64_t>(h) * a.hd + d0;
#pragma unroll
      for (int j = 0; j < SL; ++j) c[j] = oc[j];
    }
  }
}

template <int DT>
int launch(const Args &a, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(4) * kKeys * a.hd * sizeof(float);
  dim3 grid(static_cast<unsigned>((a.n + kRows - 1) / kRows), static_cast<unsigned>(a.n_heads));
#define DKV_AFO(SL)                                                                                   \
  if (a.hd == 4 * SL) {                                                                               \
    DKV_CUDA_CHECK(cudaFuncSetAttribute(afo_kernel<DT, SL>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                        static_cast<int>(smem)));                                     \
    afo_kernel<DT, SL><<<grid, kThreads, smem, st>>>(a);                                              \
    DKV_CUDA_CHECK(cudaGetLastError());                                                               \
    return DKV_OK;                                                                                    \
  }
  DKV_AFO(4)
  DKV_AFO(8)
  DKV_AFO(16)
  DKV_AFO(32)
#undef DKV_AFO
  return DKV_ERR_UNSUPPORTED;
}

}  // namespace afo
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_attn_first_order(const void *q, const void *dq, int64_t q_row_stride, const void *k,
                                    const void *dk, const void *v, const void *dv, int64_t kv_row_stride,
                                    int32_t dtype, int32_t n_tokens, int32_t n_heads, int32_t n_kv_heads,
                                    int32_t head_dim, float scale, float *ctx, float *dctx,
                                    int64_t out_row_stride, dkv_stream_t stream) {
  if (n_tokens < 0 || n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads) return DKV_ERR_INVALID_ARGUMENT;
  if (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128) return DKV_ERR_UNSUPPORTED;
  if (dtype != DKV_F32 && dtype != DKV_BF16 && dtype != DKV_F16) return DKV_ERR_UNSUPPORTED;
  if (n_tokens == 0) return DKV_OK;
  if (!q || !dq || !k || !dk || !v || !dv || !dctx) return DKV_ERR_INVALID_ARGUMENT;
  if (q_row_stride < static_cast<int64_t>(n_heads) * head_dim ||
      kv_row_stride < static_cast<int64_t>(n_kv_heads) * head_dim ||
      out_row_stride < static_cast<int64_t>(n_heads) * head_dim)
    return DKV_ERR_INVALID_ARGUMENT;
  if ((n_tokens + afo::kRows - 1) / afo::kRows > 0x7fffffff || n_heads > 65535) return DKV_ERR_UNSUPPORTED;
  afo::Args a{q, dq, k, dk, v, dv, q_row_stride, kv_row_stride, ctx, dctx, out_row_stride,
              n_tokens, n_heads, n_kv_heads, head_dim, scale};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DKV_F32) return afo::launch<DKV_F32>(a, st);
  if (dtype == DKV_BF16) return afo::launch<DKV_BF16>(a, st);
  return afo::launch<DKV_F16>(a, st);
}
