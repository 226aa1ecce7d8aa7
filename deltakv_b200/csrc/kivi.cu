// KIVI-style int4 KV cache: quantise, dequantise, and dequant -> add -> requant.
//
// The reference has no int4 cache; its int4 arithmetic is the fake-quant
// metrics._minmax_quantize (src/deltakv/metrics.py:115-132).  Stored format (this build's):
// asymmetric min-max over groups of 32 — V: 32 consecutive channels of a token, K: 32
// consecutive tokens of a channel — scale = max(hi - lo, 1e-8) / 15 and zero = lo stored as
// fp16 (rounded before q is formed), q = clamp(rint((x - zero) / scale), 0, 15), two codes
// per byte along channels with the even channel in the low nibble.  Every step is a single
// IEEE fp32 operation (explicit _rn intrinsics, no contraction), so results are bit-exact
// against the numpy restatement.
#include "dkv_common.cuh"
#include "kivi_math.cuh"

namespace dkv {
namespace kivi {

struct Cache {
  uint8_t *codes;
  __half *scale, *zero;
  int64_t crs, szrs, n, d;
};

// ---- per-token groups (V): one thread per (token, 32-channel group) ----
// SRC: 0 = dense x, 1 = dequantised base (+ dense delta when delta != null)
template <int SRC>
__global__ void v_kernel(const void *x, int xdt, int64_t xrs, Cache base, const void *delta, int ddt,
                         int64_t drs, Cache out) {
  const int64_t ng = base.d / kG;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= out.n * ng) return;
  const int64_t t = i / ng, gi = i % ng;
  float v[kG];
  if (SRC == 0) {
#pragma unroll
    for (int j = 0; j < kG; ++j) v[j] = load_as_float(x, xdt, t * xrs + gi * kG + j);
  } else {
    const uint4 c = *reinterpret_cast<const uint4 *>(base.codes + t * base.crs + gi * 16);
    const float s = __half2float(base.scale[t * base.szrs + gi]);
    const float z = __half2float(base.zero[t * base.szrs + gi]);
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < kG; ++j) v[j] = deq((w[j >> 3] >> (4 * (j & 7))) & 0xFu, s, z);
    if (delta != nullptr) {
#pragma unroll
      for (int j = 0; j < kG; ++j) v[j] = __fadd_rn(v[j], load_as_float(delta, ddt, t * drs + gi * kG + j));
    }
  }
  uint8_t q[kG];
  __half s16, z16;
  quant_group(v, kG, q, s16, z16);
  uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < kG; ++j) w[j >> 3] |= static_cast<uint32_t>(q[j]) << (4 * (j & 7));
  *reinterpret_cast<uint4 *>(out.codes + t * out.crs + gi * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  out.scale[t * out.szrs + gi] = s16;
  out.zero[t * out.szrs + gi] = z16;
}

// ---- per-channel groups (K): one thread per (32-token group, channel pair) ----
template <int SRC>
__global__ void k_kernel(const void *x, int xdt, int64_t xrs, Cache base, const void *delta, int ddt,
                         int64_t drs, Cache out) {
  const int64_t pairs = base.d / 2;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t ngroups = (out.n + kG - 1) / kG;
  if (i >= ngroups * pairs) return;
  const int64_t gi = i / pairs, cp = i % pairs;
  const int64_t t0 = gi * kG;
  const int64_t rem = out.n - t0;
  const int cnt = static_cast<int>(rem < kG ? rem : kG);
  float a[kG], b[kG];
  float sa = 0.f, za = 0.f, sb = 0.f, zb = 0.f;
  if (SRC == 1) {
    sa = __half2float(base.scale[gi * base.szrs + 2 * cp]);
    za = __half2float(base.zero[gi * base.szrs + 2 * cp]);
    sb = __half2float(base.scale[gi * base.szrs + 2 * cp + 1]);
    zb = __half2float(base.zero[gi * base.szrs + 2 * cp + 1]);
  }
#pragma unroll
  for (int j = 0; j < kG; ++j) {
    a[j] = b[j] = 0.f;
    if (j < cnt) {
      const int64_t t = t0 + j;
      if (SRC == 0) {
        a[j] = load_as_float(x, xdt, t * xrs + 2 * cp);
        b[j] = load_as_float(x, xdt, t * xrs + 2 * cp + 1);
      } else {
        const uint32_t c = base.codes[t * base.crs + cp];
        a[j] = deq(c & 0xFu, sa, za);
        b[j] = deq(c >> 4, sb, zb);
        if (delta != nullptr) {
          a[j] = __fadd_rn(a[j], load_as_float(delta, ddt, t * drs + 2 * cp));
          b[j] = __fadd_rn(b[j], load_as_float(delta, ddt, t * drs + 2 * cp + 1));
        }
      }
    }
  }
  uint8_t qa[kG], qb[kG];
  __half s16a, z16a, s16b, z16b;
  quant_group(a, cnt, qa, s16a, z16a);
  quant_group(b, cnt, qb, s16b, z16b);
#pragma unroll
  for (int j = 0; j < kG; ++j)
    if (j < cnt) out.codes[(t0 + j) * out.crs + cp] = static_cast<uint8_t>(qa[j] | (qb[j] << 4));
  out.scale[gi * out.szrs + 2 * cp] = s16a;
  out.zero[gi * out.szrs + 2 * cp] = z16a;
  out.scale[gi * out.szrs + 2 * cp + 1] = s16b;
  out.zero[gi * out.szrs + 2 * cp + 1] = z16b;
}

// dequantise to a dense tensor
__global__ void deq_kernel(Cache c, int mode, void *x, int xdt, int64_t xrs) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= c.n * (c.d / 2)) return;
  const int64_t t = i / (c.d / 2), cp = i % (c.d / 2);
  const uint32_t code = c.codes[t * c.crs + cp];
  float out[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t ch = 2 * cp + h;
    const int64_t si = mode == DKV_KIVI_PER_TOKEN ? t * c.szrs + ch / kG : (t / kG) * c.szrs + ch;
    out[h] = deq((code >> (4 * h)) & 0xFu, __half2float(c.scale[si]), __half2float(c.zero[si]));
  }
  switch (xdt) {
    case DKV_F32:
      static_cast<float *>(x)[t * xrs + 2 * cp] = out[0];
      static_cast<float *>(x)[t * xrs + 2 * cp + 1] = out[1];
      break;
    case DKV_BF16:
      static_cast<__nv_bfloat16 *>(x)[t * xrs + 2 * cp] = __float2bfloat16_rn(out[0]);
      static_cast<__nv_bfloat16 *>(x)[t * xrs + 2 * cp + 1] = __float2bfloat16_rn(out[1]);
      break;
    case DKV_F16:
      static_cast<__half *>(x)[t * xrs + 2 * cp] = __float2half_rn(out[0]);
      static_cast<__half *>(x)[t * xrs + 2 * cp + 1] = __float2half_rn(out[1]);
      break;
    default: break;
  }
}

// out[i, c] = fresh[rows[i], c] - dequant(base)[rows[i], c]: one thread per (row, 2 channels)
__global__ void probe_residual_kernel(Cache c, int mode, const void *fresh, int fdt, int64_t frs, const int32_t *rows,
                                      int64_t n_rows, float *out, int64_t ors, int32_t *status) {
  const int64_t half = c.d / 2;
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= n_rows * half) return;
  const int64_t k = i / half, cp = i % half;
  const int64_t t = rows[k];
  if (t < 0 || t >= c.n) {
    record_error(status, DKV_ERR_INVALID_ARGUMENT);
    return;
  }
  const uint32_t b = c.codes[t * c.crs + cp];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int64_t ch = 2 * cp + e;
    const int64_t si = mode == DKV_KIVI_PER_TOKEN ? t * c.szrs + ch / kG : (t / kG) * c.szrs + ch;
    const float v = deq((b >> (4 * e)) & 0xFu, __half2float(c.scale[si]), __half2float(c.zero[si]));
    out[k * ors + ch] = load_as_float(fresh, fdt, t * frs + ch) - v;
  }
}

// Batched probe residual: job j = (cache, fresh, probe rows); one warp per probe row, each
// lane 8 channels at a time (16-byte fresh loads, 4-byte codes, 16-byte K scale/zero).
constexpr int kMaxProbeJobs = 64;
struct ProbeJob {
  Cache c;
  int mode;
  const void *fresh;
  int64_t frs;
  const int32_t *rows;
};
struct ProbeJobs {
  int n_jobs, fdt;
  int64_t n_rows, ojs, ors;
  float *out;
  int32_t *status;
  ProbeJob jobs[kMaxProbeJobs];
};

__device__ __forceinline__ void fresh8(const void *base, int fdt, int64_t off, float (&f)[8]) {
  if (fdt == DKV_F32) {
    const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + off);
    const float4 a = p[0], b = p[1];
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  } else {
    const uint4 a = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + off);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = fdt == DKV_BF16 ? bf16lo(w[j]) : f16lo(w[j]);
      f[2 * j + 1] = fdt == DKV_BF16 ? bf16hi(w[j]) : f16hi(w[j]);
    }
  }
}

__global__ void __launch_bounds__(256) probe_residual_batched_kernel(const __grid_constant__ ProbeJobs J) {
  const ProbeJob &P = J.jobs[blockIdx.y];
  const int lane = threadIdx.x & 31;
  const int64_t wstep = static_cast<int64_t>(gridDim.x) * 8;
  for (int64_t k = blockIdx.x * 8 + (threadIdx.x >> 5); k < J.n_rows; k += wstep) {
    const int64_t t = P.rows[k];
    if (t < 0 || t >= P.c.n) {
      if (lane == 0) record_error(J.status, DKV_ERR_INVALID_ARGUMENT);
      continue;
    }
    float *o = J.out + blockIdx.y * J.ojs + k * J.ors;
    for (int64_t c0 = 8 * lane; c0 < P.c.d; c0 += 256) {
      float f[8], s[8], z[8];
      fresh8(P.fresh, J.fdt, t * P.frs + c0, f);
      const uint32_t w = *reinterpret_cast<const uint32_t *>(P.c.codes + t * P.c.crs + c0 / 2);
      if (P.mode == DKV_KIVI_PER_CHANNEL) {
        const uint4 sv = *reinterpret_cast<const uint4 *>(P.c.scale + (t / kG) * P.c.szrs + c0);
        const uint4 zv = *reinterpret_cast<const uint4 *>(P.c.zero + (t / kG) * P.c.szrs + c0);
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[2 * j] = f16lo(sw[j]), s[2 * j + 1] = f16hi(sw[j]);
          z[2 * j] = f16lo(zw[j]), z[2 * j + 1] = f16hi(zw[j]);
        }
      } else {
        const float vs = __half2float(P.c.scale[t * P.c.szrs + c0 / kG]);
        const float vz = __half2float(P.c.zero[t * P.c.szrs + c0 / kG]);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = vs, z[j] = vz;
      }
      float r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = f[j] - deq((w >> (4 * j)) & 0xFu, s[j], z[j]);
      float4 *op = reinterpret_cast<float4 *>(o + c0);
      op[0] = make_float4(r[0], r[1], r[2], r[3]);
      op[1] = make_float4(r[4], r[5], r[6], r[7]);
    }
  }
}

int check(const dkv_kivi_cache *c, Cache &o) {
  if (c == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (c->mode != DKV_KIVI_PER_CHANNEL && c->mode != DKV_KIVI_PER_TOKEN) return DKV_ERR_INVALID_ARGUMENT;
  if (c->d <= 0 || c->d % kG || c->n_tokens < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (c->n_tokens > 0 && (c->codes == nullptr || c->scale == nullptr || c->zero == nullptr))
    return DKV_ERR_INVALID_ARGUMENT;
  if (c->code_row_stride < c->d / 2) return DKV_ERR_LAYOUT;
  if (c->mode == DKV_KIVI_PER_TOKEN) {
    if (c->sz_row_stride < c->d / kG) return DKV_ERR_LAYOUT;
    if ((reinterpret_cast<uintptr_t>(c->codes) & 15) || (c->code_row_stride & 15)) return DKV_ERR_ALIGNMENT;
  } else if (c->sz_row_stride < c->d) {
    return DKV_ERR_LAYOUT;
  }
  o.codes = static_cast<uint8_t *>(c->codes);
  o.scale = static_cast<__half *>(c->scale);
  o.zero = static_cast<__half *>(c->zero);
  o.crs = c->code_row_stride;
  o.szrs = c->sz_row_stride;
  o.n = c->n_tokens;
  o.d = c->d;
  return DKV_OK;
}

bool float_dtype(int dt) { return dt == DKV_F32 || dt == DKV_F16 || dt == DKV_BF16; }

int launch(int mode, int src, const void *x, int xdt, int64_t xrs, const Cache &base, const void *delta,
           int ddt, int64_t drs, const Cache &out, cudaStream_t st) {
  const int threads = 128;
  int64_t work = mode == DKV_KIVI_PER_TOKEN ? out.n * (out.d / kG) : ((out.n + kG - 1) / kG) * (out.d / 2);
  if (work == 0) return DKV_OK;
  const unsigned blocks = static_cast<unsigned>((work + threads - 1) / threads);
  if (mode == DKV_KIVI_PER_TOKEN) {
    if (src == 0) v_kernel<0><<<blocks, threads, 0, st>>>(x, xdt, xrs, base, delta, ddt, drs, out);
    else v_kernel<1><<<blocks, threads, 0, st>>>(x, xdt, xrs, base, delta, ddt, drs, out);
  } else {
    if (src == 0) k_kernel<0><<<blocks, threads, 0, st>>>(x, xdt, xrs, base, delta, ddt, drs, out);
    else k_kernel<1><<<blocks, threads, 0, st>>>(x, xdt, xrs, base, delta, ddt, drs, out);
  }
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

}  // namespace kivi
}  // namespace dkv

using namespace dkv;
using namespace dkv::kivi;

extern "C" int dkv_kivi_quantize(const void *x, int32_t x_dtype, int64_t x_row_stride, const dkv_kivi_cache *out,
                                 dkv_stream_t stream) {
  kivi::Cache o;
  int rc = kivi::check(out, o);
  if (rc) return rc;
  if (!kivi::float_dtype(x_dtype)) return DKV_ERR_UNSUPPORTED;
  if (o.n > 0 && x == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  return kivi::launch(out->mode, 0, x, x_dtype, x_row_stride, o, nullptr, 0, 0, o,
                      reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dkv_kivi_dequantize(const dkv_kivi_cache *in, void *x, int32_t x_dtype, int64_t x_row_stride,
                                   dkv_stream_t stream) {
  kivi::Cache c;
  int rc = kivi::check(in, c);
  if (rc) return rc;
  if (!kivi::float_dtype(x_dtype)) return DKV_ERR_UNSUPPORTED;
  const int64_t work = c.n * (c.d / 2);
  if (work == 0) return DKV_OK;
  if (x == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  kivi::deq_kernel<<<static_cast<unsigned>((work + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      c, in->mode, x, x_dtype, x_row_stride);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

extern "C" int dkv_kivi_patch(const dkv_kivi_cache *base, const void *delta, int32_t delta_dtype,
                              int64_t delta_row_stride, const dkv_kivi_cache *out, dkv_stream_t stream) {
  kivi::Cache b, o;
  int rc = kivi::check(base, b);
  if (rc) return rc;
  rc = kivi::check(out, o);
  if (rc) return rc;
  if (base->mode != out->mode || b.n != o.n || b.d != o.d) return DKV_ERR_INVALID_ARGUMENT;
  if (delta != nullptr && !kivi::float_dtype(delta_dtype)) return DKV_ERR_UNSUPPORTED;
  return kivi::launch(out->mode, 1, nullptr, 0, 0, b, delta, delta_dtype, delta_row_stride, o,
                      reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dkv_kivi_probe_residual(const dkv_kivi_cache *base, const void *fresh, int32_t fresh_dtype,
                                       int64_t fresh_row_stride, const int32_t *rows, int64_t n_rows, float *out,
                                       int64_t out_row_stride, int32_t *status, dkv_stream_t stream) {
  Cache c;
  int rc = check(base, c);
  if (rc) return rc;
  if (fresh_dtype != DKV_F32 && fresh_dtype != DKV_F16 && fresh_dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (n_rows < 0 || out_row_stride < c.d) return DKV_ERR_INVALID_ARGUMENT;
  if (n_rows == 0) return DKV_OK;
  if (fresh == nullptr || rows == nullptr || out == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t work = n_rows * (c.d / 2);
  probe_residual_kernel<<<static_cast<unsigned>((work + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      c, base->mode, fresh, fresh_dtype, fresh_row_stride, rows, n_rows, out, out_row_stride, status);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

extern "C" int dkv_kivi_probe_residual_batched(const dkv_kivi_probe_job *jobs, int32_t n_jobs, int32_t fresh_dtype,
                                               int64_t n_rows, float *out, int64_t out_job_stride,
                                               int64_t out_row_stride, int32_t *status, dkv_stream_t stream) {
  if (n_jobs < 0 || n_rows < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (fresh_dtype != DKV_F32 && fresh_dtype != DKV_F16 && fresh_dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (n_jobs == 0 || n_rows == 0) return DKV_OK;
  if (jobs == nullptr || out == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  const int64_t d = jobs[0].base.d;
  const int esz = fresh_dtype == DKV_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (out_row_stride & 3) || (out_job_stride & 3)) return DKV_ERR_ALIGNMENT;
  if (out_row_stride < d || out_job_stride < (n_rows - 1) * out_row_stride + d) return DKV_ERR_INVALID_ARGUMENT;
  ProbeJobs J;
  J.fdt = fresh_dtype;
  J.n_rows = n_rows;
  J.ojs = out_job_stride;
  J.ors = out_row_stride;
  J.status = status;
  for (int32_t j0 = 0; j0 < n_jobs; j0 += kMaxProbeJobs) {
    const int nj = n_jobs - j0 < kMaxProbeJobs ? n_jobs - j0 : kMaxProbeJobs;
    for (int j = 0; j < nj; ++j) {
      const dkv_kivi_probe_job &q = jobs[j0 + j];
      Cache c;
      const int rc = check(&q.base, c);
      if (rc) return rc;
      if (c.d != d) return DKV_ERR_INVALID_ARGUMENT;
      if (q.fresh == nullptr || q.rows == nullptr || q.fresh_row_stride < d) return DKV_ERR_INVALID_ARGUMENT;
      if ((reinterpret_cast<uintptr_t>(q.fresh) & 15) || ((q.fresh_row_stride * esz) & 15)) return DKV_ERR_ALIGNMENT;
      if ((reinterpret_cast<uintptr_t>(c.codes) & 3) || (c.crs & 3)) return DKV_ERR_ALIGNMENT;
      if (q.base.mode == DKV_KIVI_PER_CHANNEL &&
          ((reinterpret_cast<uintptr_t>(c.scale) & 15) || (reinterpret_cast<uintptr_t>(c.zero) & 15) || (c.szrs & 7)))
        return DKV_ERR_ALIGNMENT;
      J.jobs[j] = ProbeJob{c, q.base.mode, q.fresh, q.fresh_row_stride, q.rows};
    }
    J.n_jobs = nj;
    J.out = out + static_cast<int64_t>(j0) * out_job_stride;
    const int64_t want = (n_rows + 7) / 8;  // one warp per row, 8 warps per CTA
    const unsigned gx = static_cast<unsigned>(want < 64 ? want : 64);
    probe_residual_batched_kernel<<<dim3(gx, nj), 256, 0, static_cast<cudaStream_t>(stream)>>>(J);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  return DKV_OK;
}
