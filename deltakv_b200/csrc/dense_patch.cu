// Dense-delta KV patch on 5th-generation tensor cores (sm_100a).
//
// For an RL step the weight delta of k_proj / v_proj is a full-rank matrix dW, so the patch
// is a real contraction:  dK = RoPE(X . dW_K^T),  dV = X . dW_V^T,  pages += (dK, dV).
// The reference computes it as exact_kv_patch with LowRankFactors(A = dW, B = I, scale = 1)
// (src/deltakv/patches/exact.py:14-63, factors.py:61-67) followed by scatter_into_paged
// (src/deltakv/paged.py:8-43).  Here it is one persistent warp-specialised GEMM per launch:
//
//   warp 0     TMA producer: X tile [128 tokens x 64] and W tile [256 outputs x 64] per
//              k-stage, both 128-B swizzled, into a 4-deep shared-memory ring;
//   warp 1     MMA issuer: tcgen05.mma kind::f16 (bf16 x bf16 -> fp32), M=128 N=256 K=16,
//              accumulating a 128x256 tile in tensor memory (two 256-column buffers, so the
//              epilogue of one tile overlaps the MMAs of the next);
//   warps 2-9  epilogue: each thread owns one token row and 128 output columns; it loads its
//              page rows before the tile's MMAs finish, reads the accumulator with
//              tcgen05.ld, applies the per-row scale and RoPE (pairs (i, i + hd/2), K only),
//              adds to the page values in fp32 and stores with one rounding.
//
// Output column c of the packed W (rows [0, d_kv) = dW_K, [d_kv, 2 d_kv) = dW_V) is head
// (c mod d_kv) / hd, dim (c mod d_kv) mod hd.  Tiles are (layer, sequence, 128-token chunk,
// 256-column block), the column block fastest, so the eight column blocks of one token chunk
// run at the same time and X is read from HBM once.  Every wait is bounded; a timeout is
// reported in the status word and the kernel drains its copies and frees tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "dkv_common.cuh"

namespace dkv {
namespace dense {

constexpr int kBM = 128;  // tokens per tile
constexpr int kBN = 256;  // output columns per tile
constexpr int kBK = 64;   // d_model elements per stage (128 bytes of bf16: one swizzle row)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kTmemCols = 512;
constexpr int kBarOff = kStages * kStageBytes;
constexpr int kSmemBytes = kBarOff + 256;

struct alignas(64) Params {
  CUtensorMap x_map;  // {d_model, x_rows, layers} bf16
  CUtensorMap w_map;  // {d_model, 2*d_kv, layers} bf16
  const float *x_scale;
  int64_t xs_stride;
  const float *rope_cos, *rope_sin;
  int rope_max_pos, has_rope;
  const int32_t *cu_seqlens, *block_tables, *table_lens, *positions;
  int64_t table_stride;
  int n_seqs, max_chunks, n_tiles_n, kc;
  int d_kv, hd, col_lo, col_hi;
  int block_size, accumulate;
  int64_t x_rows, n_tiles;
  int64_t k_sblock, k_sslot, k_shead, k_nblocks;
  int64_t v_sblock, v_sslot, v_shead, v_nblocks;
  int32_t *status;
  void *k_base[DKV_MAX_LAYERS];
  void *v_base[DKV_MAX_LAYERS];
};

struct Tile {
  int layer, seq, n, row0, c0, len;
};

__device__ __forceinline__ bool decode_tile(const Params &p, int64_t tile, Tile &t) {
  t.n = static_cast<int>(tile % p.n_tiles_n);
  int64_t rest = tile / p.n_tiles_n;
  const int chunk = static_cast<int>(rest % p.max_chunks);
  rest /= p.max_chunks;
  t.seq = static_cast<int>(rest % p.n_seqs);
  t.layer = static_cast<int>(rest / p.n_seqs);
  const int s0 = __ldg(p.cu_seqlens + t.seq);
  t.len = __ldg(p.cu_seqlens + t.seq + 1) - s0;
  t.c0 = chunk * kBM;
  t.row0 = s0 + t.c0;
  return t.c0 < t.len;
}

// 16 consecutive 16-bit page elements (32 bytes) as raw bits
struct Page16 {
  uint4 a, b;
};

template <int PDT>
__device__ __forceinline__ float page_get(const Page16 &v, int i) {
  const uint4 &q = i < 8 ? v.a : v.b;
  const int j = i & 7;
  const uint32_t w = j < 2 ? q.x : j < 4 ? q.y : j < 6 ? q.z : q.w;
  if (PDT == DKV_BF16) return (j & 1) ? bf16hi(w) : bf16lo(w);
  return (j & 1) ? f16hi(w) : f16lo(w);
}

template <int PDT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return PDT == DKV_BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <int PDT>
__device__ __forceinline__ void page_put(uint8_t *dst, const float (&v)[16]) {
  uint4 a, b;
  a.x = pack2<PDT>(v[0], v[1]);
  a.y = pack2<PDT>(v[2], v[3]);
  a.z = pack2<PDT>(v[4], v[5]);
  a.w = pack2<PDT>(v[6], v[7]);
  b.x = pack2<PDT>(v[8], v[9]);
  b.y = pack2<PDT>(v[10], v[11]);
  b.z = pack2<PDT>(v[12], v[13]);
  b.w = pack2<PDT>(v[14], v[15]);
  stg128_stream(dst, a);
  stg128_stream(dst + 16, b);
}

// One epilogue thread's view of a tile: row metadata and the 8 chunks of 16 columns it owns
// (4 head-halves pairs (lo, lo + hd/2)).  `col0` is the first global output column.
struct RowCtx {
  uint8_t *k_row, *v_row;  // page row of the token in this layer's K / V cache (or null)
  float xs;
  int pos;
  bool valid;
};

template <int PDT>
__device__ __forceinline__ RowCtx row_ctx(const Params &p, const Tile &t, int row) {
  RowCtx r;
  r.k_row = r.v_row = nullptr;
  r.xs = 1.f;
  r.pos = 0;
  const int tok = t.c0 + row;
  bool v = tok < t.len;
  const int64_t grow = static_cast<int64_t>(t.row0) + row;
  if (v && grow >= p.x_rows) {
    record_error(p.status, DKV_ERR_INVALID_ARGUMENT);
    v = false;
  }
  if (v) {
    int pos = tok;
    if (p.positions) pos = __ldg(p.positions + grow);
    if (p.has_rope && (pos < 0 || pos >= p.rope_max_pos)) {
      record_error(p.status, DKV_ERR_ROPE_RANGE);
      v = false;
    }
    r.pos = pos;
    const int bi = tok / p.block_size;
    const int64_t tlen = p.table_lens ? __ldg(p.table_lens + t.seq) : p.table_stride;
    if (v && bi >= tlen) {
      record_error(p.status, DKV_ERR_BLOCK_TABLE_SHORT);
      v = false;
    }
    if (v) {
      const int bid = __ldg(p.block_tables + static_cast<int64_t>(t.seq) * p.table_stride + bi);
      if (bid < 0 || bid >= p.k_nblocks || bid >= p.v_nblocks) {
        record_error(p.status, DKV_ERR_PAGE_RANGE);
        v = false;
      } else {
        const int slot = tok % p.block_size;
        constexpr int EB = 2;
        r.k_row = static_cast<uint8_t *>(p.k_base[t.layer]) +
                  (static_cast<int64_t>(bid) * p.k_sblock + static_cast<int64_t>(slot) * p.k_sslot) * EB;
        r.v_row = static_cast<uint8_t *>(p.v_base[t.layer]) +
                  (static_cast<int64_t>(bid) * p.v_sblock + static_cast<int64_t>(slot) * p.v_sslot) * EB;
      }
    }
    if (v && p.x_scale) r.xs = __ldg(p.x_scale + t.layer * p.xs_stride + grow);
  }
  r.valid = v;
  return r;
}

// address of chunk i (0..7) of this thread's 128 columns: i = 2*pair + half; pair walks the
// (head, 16-column block) pairs of the range in order.  Returns null when the chunk is not
// patched (outside [col_lo, col_hi) or an invalid row).
__device__ __forceinline__ uint8_t *chunk_ptr(const Params &p, const RowCtx &r, int col0, int i,
                                              bool &is_k, int &fi) {
  const int half_hd = p.hd >> 1;
  const int per_head = half_hd >> 4;  // 16-column blocks in half a head
  const int pr = i >> 1;
  const int hh = pr / per_head;       // head within the 128-column range
  const int jb = pr - hh * per_head;  // 16-column block within the half head
  const int c = col0 + hh * p.hd;     // first column of the head
  fi = jb * 16;                       // frequency index of the block's first column
  if (!r.valid || c < p.col_lo || c >= p.col_hi) return nullptr;
  is_k = c < p.d_kv;
  const int head = is_k ? c / p.hd : (c - p.d_kv) / p.hd;
  const int64_t off = static_cast<int64_t>(head) * (is_k ? p.k_shead : p.v_shead) + fi +
                      (i & 1) * half_hd;
  return (is_k ? r.k_row : r.v_row) + off * 2;
}

template <int PDT>
__global__ void __launch_bounds__(kThreads, 1) dense_patch_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *empty = full + kStages;
  uint64_t *tfull = empty + kStages;  // [2]
  uint64_t *tempty = tfull + 2;       // [2]
  uint64_t *done = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      prefetch_tensormap(&p.x_map);
      prefetch_tensormap(&p.w_map);
      int stage = 0;
      uint32_t phase = 0, issued = 0, parity = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        Tile t;
        if (!decode_tile(p, tile, t)) continue;
        const int wrow = p.col_lo + t.n * kBN;
        for (int kc = 0; kc < p.kc; ++kc) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t *sa = smem + stage * kStageBytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_3d(sa, &p.x_map, &full[stage], kc * kBK, t.row0, t.layer);
          tma_load_3d(sa + kABytes, &p.w_map, &full[stage], kc * kBK, wrow, t.layer);
          issued |= 1u << stage;
          parity = (parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // never leave with a copy still landing in shared memory
      for (int s = 0; s < kStages; ++s) {
        if (!(issued & (1u << s))) continue;
        const uint32_t par = (parity >> s) & 1u;
        const long long t0 = clock64();
        while (!mbar_try_wait(&full[s], par)) {
          if (clock64() - t0 > kWaitLimitCycles) {
            record_error(p.status, DKV_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(1 /* bf16 */, kBM, kBN);
      int stage = 0;
      uint32_t phase = 0;
      int64_t j = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        Tile t;
        if (!decode_tile(p, tile, t)) continue;
        const int b = static_cast<int>(j & 1);
        const int64_t use = j >> 1;
        if (use > 0 && !mbar_wait_bounded(&tempty[b], static_cast<uint32_t>((use - 1) & 1), abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + b * kBN;
        for (int kc = 0; kc < p.kc; ++kc) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint64_t da = umma_desc_k_sw128(sa), db = umma_desc_k_sw128(sa + kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)  // +32 bytes along K = +2 in the start-address field
            umma_f16(d, da + 2 * k, db + 2 * k, idesc, (kc | k) != 0);
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[b]);
        ++j;
      }
      if (!ok) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      umma_commit(done);
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int q = warp & 3;             // tensor-memory lane quarter this warp may read
    const int half = (warp - 2) >> 2;   // which 128 of the tile's 256 columns
    const int row = 32 * q + lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * q) << 16) + half * 128;
    int64_t j = 0;
    for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
      Tile t;
      if (!decode_tile(p, tile, t)) continue;
      const int b = static_cast<int>(j & 1);
      const int64_t use = j >> 1;
      const int col0 = p.col_lo + t.n * kBN + half * 128;
      const RowCtx rc = row_ctx<PDT>(p, t, row);

      // this row's page values, loaded while the tile's MMAs run
      Page16 pg[8];
      uint8_t *ptr[8];
      bool isk[8];
      int fi[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        isk[i] = false;
        ptr[i] = chunk_ptr(p, rc, col0, i, isk[i], fi[i]);
        if (ptr[i] != nullptr && p.accumulate) {
          pg[i].a = ldg128_stream(ptr[i]);
          pg[i].b = ldg128_stream(ptr[i] + 16);
        } else {
          pg[i].a = pg[i].b = make_uint4(0, 0, 0, 0);
        }
      }

      const bool ok = mbar_wait_bounded(&tfull[b], static_cast<uint32_t>(use & 1), abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t base = lane_addr + b * kBN;
      const int half_hd = p.hd >> 1;
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        // chunk pair (lo, hi = lo + hd/2) of one head
        const int per_head = half_hd >> 4;
        const int hh = pr / per_head, jb = pr - hh * per_head;
        const uint32_t clo = base + hh * p.hd + jb * 16;
        float lo[16], hi[16];
        __syncwarp();
        tmem_ld16(clo, lo);
        tmem_ld16(clo + half_hd, hi);
        tmem_ld_wait();
        uint8_t *plo = ptr[2 * pr], *phi = ptr[2 * pr + 1];
        if (plo != nullptr) {
          const float xs = rc.xs;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            lo[e] *= xs;
            hi[e] *= xs;
          }
          if (isk[2 * pr] && p.has_rope) {
            const int64_t tb = static_cast<int64_t>(rc.pos) * half_hd + fi[2 * pr];
            const float4 *cs = reinterpret_cast<const float4 *>(p.rope_cos + tb);
            const float4 *sn = reinterpret_cast<const float4 *>(p.rope_sin + tb);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              const float4 c4 = __ldg(cs + v4), s4 = __ldg(sn + v4);
              const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int e = 4 * v4 + u;
                const float a = lo[e], bb = hi[e];
                lo[e] = fmaf(a, cc[u], -bb * ss[u]);
                hi[e] = fmaf(bb, cc[u], a * ss[u]);
              }
            }
          }
          if (p.accumulate) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              lo[e] += page_get<PDT>(pg[2 * pr], e);
              hi[e] += page_get<PDT>(pg[2 * pr + 1], e);
            }
          }
          page_put<PDT>(plo, lo);
          page_put<PDT>(phi, hi);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      ++j;
    }
  }

  // ------------------------------- teardown -------------------------------
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      const long long t0 = clock64();
      while (!mbar_try_wait(done, 0)) {
        if (clock64() - t0 > kWaitLimitCycles) {
          record_error(p.status, DKV_ERR_TIMEOUT);
          break;
        }
      }
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ----------------------------------------------------------------------------
// packing: dW_K, dW_V (any float dtype) -> bf16 [layers][2 d_kv][d_model], with the RMSNorm
// weight folded in (dW . diag(w)) and the projection scales applied
// ----------------------------------------------------------------------------
__global__ void pack_kernel(const void *dw_k, const void *dw_v, int dt, int64_t k_ls, int64_t v_ls,
                            const void *norm_w, int ndt, int64_t n_ls, float sk, float sv,
                            int d_model, int d_kv, __nv_bfloat16 *out, int64_t out_ls) {
  const int layer = blockIdx.y;
  const int64_t per = static_cast<int64_t>(2) * d_kv * d_model;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / d_model;
    const int c = static_cast<int>(i - r * d_model);
    const bool is_v = r >= d_kv;
    const void *src = is_v ? dw_v : dw_k;
    float v = 0.f;
    if (src != nullptr) {
      const int64_t rr = is_v ? r - d_kv : r;
      v = load_as_float(src, dt, layer * (is_v ? v_ls : k_ls) + rr * d_model + c) * (is_v ? sv : sk);
      if (norm_w != nullptr) v *= load_as_float(norm_w, ndt, layer * n_ls + c);
    }
    out[layer * out_ls + i] = __float2bfloat16_rn(v);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

bool geometry_ok(const dkv_dense_geometry &g) {
  return g.d_model > 0 && g.d_model % kBK == 0 && g.n_kv_heads > 0 &&
         (g.head_dim == 32 || g.head_dim == 64 || g.head_dim == 128);
}

int check_pages(const dkv_paged_cache &c, const dkv_dense_geometry &g) {
  if (c.dtype != DKV_BF16 && c.dtype != DKV_F16) return DKV_ERR_UNSUPPORTED;
  if (c.n_heads != g.n_kv_heads || c.head_dim != g.head_dim) return DKV_ERR_LAYOUT;
  if (c.block_size <= 0 || c.num_blocks <= 0) return DKV_ERR_LAYOUT;
  if (c.stride_block % 8 || c.stride_slot % 8 || c.stride_head % 8) return DKV_ERR_ALIGNMENT;
  return DKV_OK;
}

}  // namespace dense
}  // namespace dkv

using namespace dkv;
using namespace dkv::dense;

extern "C" int dkv_pack_dense_delta(const dkv_dense_geometry *geom, const dkv_dense_delta *dw,
                                    void *packed, int64_t packed_layer_stride, dkv_stream_t stream) {
  if (geom == nullptr || dw == nullptr || packed == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (!geometry_ok(*geom)) return DKV_ERR_UNSUPPORTED;
  if (dw->n_layers <= 0 || dw->n_layers > DKV_MAX_LAYERS) return DKV_ERR_INVALID_ARGUMENT;
  if (dw->dtype != DKV_F32 && dw->dtype != DKV_F16 && dw->dtype != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (dw->dw_k == nullptr && dw->dw_v == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  const int d_kv = geom->n_kv_heads * geom->head_dim;
  const int64_t per = static_cast<int64_t>(2) * d_kv * geom->d_model;
  if (packed_layer_stride < per || packed_layer_stride % 8 || !aligned16(packed)) return DKV_ERR_ALIGNMENT;
  const int blocks_x = static_cast<int>((per + 255) / 256 < 1024 ? (per + 255) / 256 : 1024);
  pack_kernel<<<dim3(blocks_x, dw->n_layers), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      dw->dw_k, dw->dw_v, dw->dtype, dw->dw_k_layer_stride, dw->dw_v_layer_stride, dw->norm_weight,
      dw->norm_dtype, dw->norm_layer_stride, dw->scale_k, dw->scale_v, geom->d_model, d_kv,
      static_cast<__nv_bfloat16 *>(packed), packed_layer_stride);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

extern "C" int dkv_dense_patch_paged(const dkv_dense_patch_args *a, dkv_stream_t stream) {
  if (a == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  const dkv_dense_geometry &g = a->geom;
  if (!geometry_ok(g)) return DKV_ERR_UNSUPPORTED;
  const dkv_seq_batch &s = a->seqs;
  if (a->n_layers <= 0 || a->n_layers > DKV_MAX_LAYERS) return DKV_ERR_INVALID_ARGUMENT;
  if (s.n_seqs < 0 || s.max_seq_len < 0) return DKV_ERR_INVALID_ARGUMENT;
  if (!a->do_k && !a->do_v) return DKV_OK;
  if (s.n_seqs == 0 || s.max_seq_len == 0) return DKV_OK;
  if (s.cu_seqlens == nullptr || s.block_tables == nullptr || a->x == nullptr ||
      a->packed == nullptr || a->k_pages == nullptr || a->v_pages == nullptr)
    return DKV_ERR_INVALID_ARGUMENT;
  const dkv_paged_cache &kp = a->k_pages[0], &vp = a->v_pages[0];
  int rc = check_pages(kp, g);
  if (rc) return rc;
  rc = check_pages(vp, g);
  if (rc) return rc;
  if (kp.dtype != vp.dtype || kp.block_size != vp.block_size) return DKV_ERR_LAYOUT;
  if (!aligned16(a->x) || (a->x_row_stride * 2) % 16 || (a->x_layer_stride * 2) % 16) return DKV_ERR_ALIGNMENT;
  const int d_kv = g.n_kv_heads * g.head_dim;
  if (!aligned16(a->packed) || (a->packed_layer_stride * 2) % 16) return DKV_ERR_ALIGNMENT;
  if (a->n_layers > 1 && a->packed_layer_stride < static_cast<int64_t>(2) * d_kv * g.d_model)
    return DKV_ERR_INVALID_ARGUMENT;
  const bool rope = a->rope_cos != nullptr && a->rope_sin != nullptr;
  if (rope && (a->rope_max_pos <= 0 || !aligned16(a->rope_cos) || !aligned16(a->rope_sin)))
    return DKV_ERR_ALIGNMENT;
  if (a->x_rows <= 0 || a->x_rows > 0x7fffffffLL) return DKV_ERR_INVALID_ARGUMENT;

  Params p;
  memset(&p, 0, sizeof(p));
  auto enc = encoder();
  if (enc == nullptr) {
    note_cuda_error(cudaErrorNotSupported, "cuTensorMapEncodeTiled entry point");
    return DKV_ERR_CUDA;
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(g.d_model), static_cast<cuuint64_t>(a->x_rows),
                          static_cast<cuuint64_t>(a->n_layers)};
    const int64_t ls = a->n_layers > 1 ? a->x_layer_stride : a->x_rows * a->x_row_stride;
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(a->x_row_stride * 2), static_cast<cuuint64_t>(ls * 2)};
    cuuint32_t box[3] = {kBK, kBM, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&p.x_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(a->x), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DKV_ERR_ALIGNMENT;
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(g.d_model), static_cast<cuuint64_t>(2 * d_kv),
                          static_cast<cuuint64_t>(a->n_layers)};
    const int64_t ls = a->n_layers > 1 ? a->packed_layer_stride : static_cast<int64_t>(2) * d_kv * g.d_model;
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(g.d_model * 2), static_cast<cuuint64_t>(ls * 2)};
    cuuint32_t box[3] = {kBK, kBN, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    if (enc(&p.w_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(a->packed), dims, strides,
            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DKV_ERR_ALIGNMENT;
  }
  p.x_scale = a->x_scale;
  p.xs_stride = a->x_scale_layer_stride;
  p.rope_cos = rope ? a->rope_cos : nullptr;
  p.rope_sin = rope ? a->rope_sin : nullptr;
  p.rope_max_pos = rope ? a->rope_max_pos : 0;
  p.has_rope = rope ? 1 : 0;
  p.cu_seqlens = s.cu_seqlens;
  p.block_tables = s.block_tables;
  p.table_lens = s.table_lens;
  p.positions = s.positions;
  p.table_stride = s.table_stride;
  p.n_seqs = s.n_seqs;
  p.max_chunks = (s.max_seq_len + kBM - 1) / kBM;
  p.col_lo = a->do_k ? 0 : d_kv;
  p.col_hi = a->do_v ? 2 * d_kv : d_kv;
  p.n_tiles_n = (p.col_hi - p.col_lo + kBN - 1) / kBN;
  p.kc = g.d_model / kBK;
  p.d_kv = d_kv;
  p.hd = g.head_dim;
  p.block_size = kp.block_size;
  p.accumulate = a->accumulate ? 1 : 0;
  p.x_rows = a->x_rows;
  p.k_sblock = kp.stride_block;
  p.k_sslot = kp.stride_slot;
  p.k_shead = kp.stride_head;
  p.k_nblocks = kp.num_blocks;
  p.v_sblock = vp.stride_block;
  p.v_sslot = vp.stride_slot;
  p.v_shead = vp.stride_head;
  p.v_nblocks = vp.num_blocks;
  p.status = a->status;
  for (int l = 0; l < a->n_layers; ++l) {
    p.k_base[l] = a->k_pages[l].base;
    p.v_base[l] = a->v_pages[l].base;
    if (p.k_base[l] == nullptr || p.v_base[l] == nullptr) return DKV_ERR_INVALID_ARGUMENT;
    if (!aligned16(p.k_base[l]) || !aligned16(p.v_base[l])) return DKV_ERR_ALIGNMENT;
  }
  p.n_tiles = static_cast<int64_t>(a->n_layers) * s.n_seqs * p.max_chunks * p.n_tiles_n;

  int dev = 0, sms = 0;
  DKV_CUDA_CHECK(cudaGetDevice(&dev));
  DKV_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = static_cast<int>(p.n_tiles < sms ? p.n_tiles : sms);
  const size_t smem = 1024 + kSmemBytes;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (kp.dtype == DKV_BF16) {
    DKV_CUDA_CHECK(cudaFuncSetAttribute(dense_patch_kernel<DKV_BF16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    dense_patch_kernel<DKV_BF16><<<grid, kThreads, smem, st>>>(p);
  } else {
    DKV_CUDA_CHECK(cudaFuncSetAttribute(dense_patch_kernel<DKV_F16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    dense_patch_kernel<DKV_F16><<<grid, kThreads, smem, st>>>(p);
  }
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}
