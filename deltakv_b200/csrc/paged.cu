// Paged scatter-add / gather between token-major [rows, heads, dim] tensors and a
// paged KV cache, for a batch of sequences.
//
// Reference: deltakv.paged.scatter_into_paged / gather_from_paged
// (src/deltakv/paged.py:8-70).  The reference loops over blocks in Python and does
// `pages[bid, :span] = pages[bid, :span] + delta[start:end]`, i.e. fp32(page) +
// fp32(delta) rounded once to the page dtype; this kernel does the same per element,
// so results are bit-identical.
#include <stdio.h>

#include "dkv_common.cuh"

namespace dkv {
namespace {

constexpr int kTokPerCta = 4;
constexpr int kThreads = 256;

// Resolve token i of sequence b to an element offset of its page row, or -1.
__device__ __forceinline__ int64_t page_row_offset(const dkv_seq_batch &s, const dkv_paged_cache &c,
                                                   int b, int i, int32_t *status) {
  const int blk_i = i / c.block_size;
  const int64_t tlen = s.table_lens ? s.table_lens[b] : s.table_stride;
  if (blk_i >= tlen) {
    record_error(status, DKV_ERR_BLOCK_TABLE_SHORT);
    return -1;
  }
  const int32_t bid = s.block_tables[static_cast<int64_t>(b) * s.table_stride + blk_i];
  if (bid < 0 || bid >= c.num_blocks) {
    record_error(status, DKV_ERR_PAGE_RANGE);
    return -1;
  }
  return static_cast<int64_t>(bid) * c.stride_block +
         static_cast<int64_t>(i % c.block_size) * c.stride_slot;
}

template <int PDT, int DDT>
__global__ void __launch_bounds__(kThreads) scatter_kernel(const void *__restrict__ delta,
                                                           int64_t d_row, int64_t d_head,
                                                           dkv_paged_cache cache,
                                                           dkv_seq_batch seqs, int32_t *status) {
  using PT = typename Elem<PDT>::T;
  using DT = typename Elem<DDT>::T;
  const int b = blockIdx.y;
  const int row0 = seqs.cu_seqlens[b];
  const int len = seqs.cu_seqlens[b + 1] - row0;
  const int hd = cache.head_dim;
  const int row_elems = cache.n_heads * hd;
  PT *pages = static_cast<PT *>(cache.base);
  const DT *dl = static_cast<const DT *>(delta);
  for (int k = 0; k < kTokPerCta; ++k) {
    const int i = blockIdx.x * kTokPerCta + k;
    if (i >= len) break;
    const int64_t off = page_row_offset(seqs, cache, b, i, status);
    if (off < 0) continue;
    const int64_t drow = static_cast<int64_t>(row0 + i) * d_row;
    for (int e = threadIdx.x; e < row_elems; e += blockDim.x) {
      const int h = e / hd, j = e - h * hd;
      PT *pp = pages + off + h * cache.stride_head + j;
      const float v = Elem<PDT>::to_f(*pp) + Elem<DDT>::to_f(dl[drow + h * d_head + j]);
      *pp = Elem<PDT>::from_f(v);
    }
  }
}

template <int PDT, int ODT>
__global__ void __launch_bounds__(kThreads) gather_kernel(dkv_paged_cache cache, dkv_seq_batch seqs,
                                                          void *__restrict__ out, int64_t o_row,
                                                          int64_t o_head, int32_t *status) {
  using PT = typename Elem<PDT>::T;
  using OT = typename Elem<ODT>::T;
  const int b = blockIdx.y;
  const int row0 = seqs.cu_seqlens[b];
  const int len = seqs.cu_seqlens[b + 1] - row0;
  const int hd = cache.head_dim;
  const int row_elems = cache.n_heads * hd;
  const PT *pages = static_cast<const PT *>(cache.base);
  OT *o = static_cast<OT *>(out);
  for (int k = 0; k < kTokPerCta; ++k) {
    const int i = blockIdx.x * kTokPerCta + k;
    if (i >= len) break;
    const int64_t off = page_row_offset(seqs, cache, b, i, status);
    const int64_t orow = static_cast<int64_t>(row0 + i) * o_row;
    for (int e = threadIdx.x; e < row_elems; e += blockDim.x) {
      const int h = e / hd, j = e - h * hd;
      const float v = off < 0 ? 0.f : Elem<PDT>::to_f(pages[off + h * cache.stride_head + j]);
      o[orow + h * o_head + j] = Elem<ODT>::from_f(v);
    }
  }
}

// Per-layer sums for the measured error of patched pages against fresh KV (the reference's
// measured_error, src/deltakv/patches/compose.py:147-163): sums[2l] += sum (page - fresh)^2,
// sums[2l+1] += sum fresh^2 over every token of every sequence.  One CTA per 16 tokens of a
// (layer, sequence); fp32 partial sums per thread, one fp64 atomic pair per CTA.
struct ErrLayers {
  const void *base[DKV_MAX_LAYERS];
};

// NS = 2: sum (p - f)^2, sum f^2 (measured_error); NS = 4: + sum p f, sum p^2 (compare_kv)
template <int PDT, int FDT, int NS>
__global__ void __launch_bounds__(kThreads) error_sums_kernel(dkv_paged_cache cache, ErrLayers layers,
                                                              const void *__restrict__ fresh, int64_t f_layer,
                                                              int64_t f_row, int64_t f_head,
                                                              dkv_seq_batch seqs, double *sums,
                                                              int32_t *status) {
  using PT = typename Elem<PDT>::T;
  using FT = typename Elem<FDT>::T;
  __shared__ float red[NS][kThreads / 32];
  const int l = blockIdx.z, b = blockIdx.y;
  const int row0 = seqs.cu_seqlens[b];
  const int len = seqs.cu_seqlens[b + 1] - row0;
  const int hd = cache.head_dim;
  const int row_elems = cache.n_heads * hd;
  const PT *pages = static_cast<const PT *>(layers.base[l]);
  const FT *fr = static_cast<const FT *>(fresh) + static_cast<int64_t>(l) * f_layer;
  float s[NS];
#pragma unroll
  for (int k = 0; k < NS; ++k) s[k] = 0.f;
  for (int k = 0; k < 16; ++k) {
    const int i = blockIdx.x * 16 + k;
    if (i >= len) break;
    const int64_t off = page_row_offset(seqs, cache, b, i, status);
    if (off < 0) continue;
    const int64_t frow = static_cast<int64_t>(row0 + i) * f_row;
    for (int e = threadIdx.x; e < row_elems; e += blockDim.x) {
      const int h = e / hd, j = e - h * hd;
      const float pv = Elem<PDT>::to_f(pages[off + h * cache.stride_head + j]);
      const float fv = Elem<FDT>::to_f(fr[frow + h * f_head + j]);
      const float dv = pv - fv;
      s[0] = fmaf(dv, dv, s[0]);
      s[1] = fmaf(fv, fv, s[1]);
      if (NS == 4) {
        s[NS - 2] = fmaf(pv, fv, s[NS - 2]);
        s[NS - 1] = fmaf(pv, pv, s[NS - 1]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int k = 0; k < NS; ++k) s[k] += __shfl_xor_sync(0xffffffffu, s[k], o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0)
#pragma unroll
    for (int k = 0; k < NS; ++k) red[k][w] = s[k];
  __syncthreads();
  if (threadIdx.x < NS) {
    double a = 0.0;
    for (int i = 0; i < kThreads / 32; ++i) a += red[threadIdx.x][i];
    atomicAdd(sums + NS * l + threadIdx.x, a);
  }
}

bool valid_float_dtype(int dt) { return dt == DKV_F32 || dt == DKV_F16 || dt == DKV_BF16; }

int check_common(const dkv_paged_cache *cache, const dkv_seq_batch *seqs) {
  if (cache == nullptr || seqs == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (cache->base == nullptr && seqs->n_seqs > 0) return DKV_ERR_INVALID_ARGUMENT;
  if (!valid_float_dtype(cache->dtype)) return DKV_ERR_UNSUPPORTED;
  if (cache->block_size <= 0 || cache->head_dim <= 0 || cache->n_heads <= 0)
    return DKV_ERR_LAYOUT;
  if (seqs->n_seqs < 0 || seqs->max_seq_len < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (seqs->n_seqs > 0 && (seqs->cu_seqlens == nullptr || seqs->block_tables == nullptr))
    return DKV_ERR_INVALID_ARGUMENT;
  if (seqs->n_seqs > 65535) return DKV_ERR_UNSUPPORTED;
  return DKV_OK;
}

}  // namespace
}  // namespace dkv

using namespace dkv;

extern "C" int dkv_scatter_paged(const void *delta, int32_t delta_dtype, int64_t delta_stride_row,
                                 int64_t delta_stride_head, const dkv_paged_cache *cache,
                                 const dkv_seq_batch *seqs, int32_t *status,
                                 dkv_stream_t stream) {
  int rc = check_common(cache, seqs);
  if (rc != DKV_OK) return rc;
  if (!valid_float_dtype(delta_dtype)) return DKV_ERR_UNSUPPORTED;
  if (seqs->n_seqs == 0 || seqs->max_seq_len == 0) return DKV_OK;
  if (delta == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  dim3 grid((seqs->max_seq_len + kTokPerCta - 1) / kTokPerCta, seqs->n_seqs);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define DKV_SCATTER_CASE(P, D)                                                                 \
  if (cache->dtype == P && delta_dtype == D) {                                                 \
    scatter_kernel<P, D><<<grid, kThreads, 0, st>>>(delta, delta_stride_row, delta_stride_head, \
                                                    *cache, *seqs, status);                    \
    DKV_CUDA_CHECK(cudaGetLastError());                                                        \
    return DKV_OK;                                                                             \
  }
  DKV_SCATTER_CASE(DKV_BF16, DKV_F32)
  DKV_SCATTER_CASE(DKV_BF16, DKV_BF16)
  DKV_SCATTER_CASE(DKV_BF16, DKV_F16)
  DKV_SCATTER_CASE(DKV_F16, DKV_F32)
  DKV_SCATTER_CASE(DKV_F16, DKV_F16)
  DKV_SCATTER_CASE(DKV_F16, DKV_BF16)
  DKV_SCATTER_CASE(DKV_F32, DKV_F32)
  DKV_SCATTER_CASE(DKV_F32, DKV_F16)
  DKV_SCATTER_CASE(DKV_F32, DKV_BF16)
#undef DKV_SCATTER_CASE
  return DKV_ERR_UNSUPPORTED;
}

extern "C" int dkv_gather_paged(const dkv_paged_cache *cache, const dkv_seq_batch *seqs, void *out,
                                int32_t out_dtype, int64_t out_stride_row, int64_t out_stride_head,
                                int32_t *status, dkv_stream_t stream) {
  int rc = check_common(cache, seqs);
  if (rc != DKV_OK) return rc;
  if (!valid_float_dtype(out_dtype)) return DKV_ERR_UNSUPPORTED;
  if (seqs->n_seqs == 0 || seqs->max_seq_len == 0) return DKV_OK;
  if (out == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  dim3 grid((seqs->max_seq_len + kTokPerCta - 1) / kTokPerCta, seqs->n_seqs);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define DKV_GATHER_CASE(P, O)                                                             \
  if (cache->dtype == P && out_dtype == O) {                                              \
    gather_kernel<P, O><<<grid, kThreads, 0, st>>>(*cache, *seqs, out, out_stride_row,    \
                                                   out_stride_head, status);              \
    DKV_CUDA_CHECK(cudaGetLastError());                                                   \
    return DKV_OK;                                                                        \
  }
  DKV_GATHER_CASE(DKV_BF16, DKV_BF16)
  DKV_GATHER_CASE(DKV_BF16, DKV_F32)
  DKV_GATHER_CASE(DKV_F16, DKV_F16)
  DKV_GATHER_CASE(DKV_F16, DKV_F32)
  DKV_GATHER_CASE(DKV_F32, DKV_F32)
#undef DKV_GATHER_CASE
  return DKV_ERR_UNSUPPORTED;
}

namespace dkv {
template <int NS>
int error_sums(const dkv_paged_cache *pages, int32_t n_layers, const void *fresh, int32_t fresh_dtype,
               int64_t fresh_layer_stride, int64_t fresh_row_stride, int64_t fresh_head_stride,
               const dkv_seq_batch *seqs, double *sums, int32_t *status, dkv_stream_t stream) {
  if (pages == nullptr || n_layers <= 0 || n_layers > DKV_MAX_LAYERS) return DKV_ERR_INVALID_ARGUMENT;
  int rc = check_common(&pages[0], seqs);
  if (rc != DKV_OK) return rc;
  if (!valid_float_dtype(fresh_dtype)) return DKV_ERR_UNSUPPORTED;
  if (seqs->n_seqs == 0 || seqs->max_seq_len == 0) return DKV_OK;
  if (fresh == nullptr || sums == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  ErrLayers layers;
  for (int l = 0; l < n_layers; ++l) {
    if (pages[l].base == nullptr) return DKV_ERR_INVALID_ARGUMENT;
    layers.base[l] = pages[l].base;
  }
  dim3 grid((seqs->max_seq_len + 15) / 16, seqs->n_seqs, n_layers);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define DKV_ERR_CASE(P, F)                                                                             \
  if (pages[0].dtype == P && fresh_dtype == F) {                                                      \
    error_sums_kernel<P, F, NS><<<grid, kThreads, 0, st>>>(pages[0], layers, fresh, fresh_layer_stride, \
                                                           fresh_row_stride, fresh_head_stride, *seqs,  \
                                                           sums, status);                               \
    DKV_CUDA_CHECK(cudaGetLastError());                                                               \
    return DKV_OK;                                                                                    \
  }
  DKV_ERR_CASE(DKV_BF16, DKV_BF16)
  DKV_ERR_CASE(DKV_BF16, DKV_F32)
  DKV_ERR_CASE(DKV_F16, DKV_F16)
  DKV_ERR_CASE(DKV_F16, DKV_F32)
  DKV_ERR_CASE(DKV_F32, DKV_F32)
  DKV_ERR_CASE(DKV_F32, DKV_BF16)
#undef DKV_ERR_CASE
  return DKV_ERR_UNSUPPORTED;
}
}  // namespace dkv

extern "C" int dkv_paged_error_sums(const dkv_paged_cache *pages, int32_t n_layers, const void *fresh,
                                    int32_t fresh_dtype, int64_t fresh_layer_stride,
                                    int64_t fresh_row_stride, int64_t fresh_head_stride,
                                    const dkv_seq_batch *seqs, double *sums, int32_t *status,
                                    dkv_stream_t stream) {
  return dkv::error_sums<2>(pages, n_layers, fresh, fresh_dtype, fresh_layer_stride, fresh_row_stride,
                            fresh_head_stride, seqs, sums, status, stream);
}

extern "C" int dkv_paged_compare_sums(const dkv_paged_cache *pages, int32_t n_layers, const void *fresh,
                                      int32_t fresh_dtype, int64_t fresh_layer_stride,
                                      int64_t fresh_row_stride, int64_t fresh_head_stride,
                                      const dkv_seq_batch *seqs, double *sums, int32_t *status,
                                      dkv_stream_t stream) {
  return dkv::error_sums<4>(pages, n_layers, fresh, fresh_dtype, fresh_layer_stride, fresh_row_stride,
                            fresh_head_stride, seqs, sums, status, stream);
}

extern "C" const char *dkv_status_string(int status) {
  switch (status) {
    case DKV_OK: return "ok";
    case DKV_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DKV_ERR_BLOCK_TABLE_SHORT: return "block_table shorter than prefix";
    case DKV_ERR_LAYOUT: return "unsupported paged KV layout";
    case DKV_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case DKV_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case DKV_ERR_ROPE_RANGE: return "position exceeds RoPE cache";
    case DKV_ERR_BASIS_DIM: return "basis dimension does not match kv dimension";
    case DKV_ERR_CUDA: return "CUDA runtime error";
    case DKV_ERR_TIMEOUT: return "device-side wait timed out";
    case DKV_ERR_PAGE_RANGE: return "block id outside the paged cache";
    case DKV_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" int dkv_abi_version(void) { return 2; }

namespace dkv {
static thread_local char g_last_cuda_error[256] = "";
void note_cuda_error(cudaError_t err, const char *what) {
  snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s (%s)", cudaGetErrorName(err),
           cudaGetErrorString(err), what);
}
}  // namespace dkv

extern "C" const char *dkv_last_cuda_error(void) { return dkv::g_last_cuda_error; }
