// Fused exact / zeroth-order KV patch for B200 (sm_100a).
//
// Reference path replaced (adityaraj-09/DeltaKV):
//   DeltaKVEngine._patch exact branch           src/deltakv/engine.py:263-288
//   -> ToyTransformer.rmsnorm_tensors            src/deltakv/model.py:48-56,310-314
//   -> zeroth_order_patches / exact_kv_patch     src/deltakv/patches/exact.py:14-94
//      (LowRankFactors.codes/.apply              src/deltakv/deltas/factors.py:61-67,
//       RotaryEmbedding.forward                  src/deltakv/rope.py:9-63)
//   -> apply_layer_patches / materialize         src/deltakv/patches/compose.py:29-34,
//                                                src/deltakv/patches/tensors.py:105-123
//   -> scatter_into_paged (per block, additive)  src/deltakv/paged.py:8-43
//
// One persistent launch covers every (layer, sequence, 128-token chunk) tile:
//   * a producer warp streams the tile's stored activations X[128 x d] through a
//     4-stage shared-memory ring with TMA (cp.async.bulk.tensor, 128-B swizzle) and the
//     matching slice of the packed A factors with a bulk copy;
//   * 8 consumer warps (16 tokens each) compute codes = x.A^T for K and V together with
//     mma.sync (fp8 X converted to f16 on the fly, fp32 accumulate), plus sum(x^2) for
//     the RMSNorm via a diagonal X.X^T product on the same fragments (or, when the stored
//     activations carry it, the per-row sum of squared codes written with them: no extra
//     tensor work, which under the power cap raises the clock);
//   * the codes never leave registers: they are re-scaled per token, turned into the
//     A fragments of a second mma.sync (codes . B^T) that produces dK/dV directly in a
//     column order chosen so each thread holds 8 contiguous columns and both halves of
//     every RoPE pair; RoPE, the delta scaling and the bf16 page read-add-write follow
//     in registers, with the tile's page rows prefetched into L2 during the X stream.
#include <cudaTypedefs.h>

#include "dkv_common.cuh"

namespace dkv {
namespace exact {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = kConsumerWarps * 32;
constexpr int kMTile = 16 * kConsumerWarps;  // tokens per tile
constexpr int kXStageBytes = kMTile * 128;   // one 128-byte k-slab of the tile
constexpr int kHeaderBytes = 256;
constexpr int kStages = 4;

// ----------------------------------------------------------------------------
// geometry of the packed factor image
// ----------------------------------------------------------------------------
struct Geo {
  int d_model, n_kv, hd, d_kv, x_dtype, rank_k, rank_v;
  int rpad;      // padded rank shared by K and V (16..64)
  int r16;       // rpad / 16
  int n1;        // rows of the packed A (K rows then V rows) = 2 * rpad
  int srow;      // bytes of one packed-A row per stage (256 for fp8 X, 128 for f16 X)
  int stage_k;   // X elements per stage (128 fp8 / 64 f16)
  int kc;        // stages per token row
  int n_passes;  // expand passes per K (or V) row; each pass = 64 output columns
  bool tc;       // codes on tcgen05 (rank <= 32): A image in the tensor-core layout
  int terms;     // e4m3 terms per A entry in the tcgen05 image (3 for fp8 X, 1 for f16 X)
  int64_t a_off, a_stage_bytes, a_bytes, bk_off, b_bytes, bv_off, total;
};

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t align_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

inline bool make_geo(const dkv_exact_geometry &g, Geo &o) {
  o.d_model = g.d_model;
  o.n_kv = g.n_kv_heads;
  o.hd = g.head_dim;
  o.d_kv = g.n_kv_heads * g.head_dim;
  o.x_dtype = g.x_dtype;
  o.rank_k = g.rank_k;
  o.rank_v = g.rank_v;
  if (g.d_model <= 0 || g.n_kv_heads <= 0) return false;
  if (!(g.head_dim == 16 || g.head_dim == 32 || (g.head_dim % 64 == 0 && g.head_dim <= 256)))
    return false;
  if (g.rank_k < 0 || g.rank_v < 0 || g.rank_k > 64 || g.rank_v > 64) return false;
  if (g.x_dtype != DKV_E4M3 && g.x_dtype != DKV_F16) return false;
  const int esz = g.x_dtype == DKV_E4M3 ? 1 : 2;
  int rk = align_up(g.rank_k, 16), rv = align_up(g.rank_v, 16);
  o.rpad = rk > rv ? rk : rv;
  if (o.rpad < 16) o.rpad = 16;
  o.r16 = o.rpad / 16;
  o.tc = o.rpad <= 32;
  o.terms = (o.tc && g.x_dtype == DKV_E4M3) ? 3 : 1;
  o.n1 = 2 * o.rpad * o.terms;
  // mma.sync image: f16 rows of one stage's k-range; tcgen05 image: 128-byte rows
  o.srow = o.tc ? 128 : (g.x_dtype == DKV_E4M3 ? 256 : 128);
  o.stage_k = 128 / esz;
  o.kc = ceil_div(g.d_model, o.stage_k);
  if (o.hd >= 64) o.n_passes = o.n_kv * (o.hd / 64);
  else if (o.hd == 32) o.n_passes = ceil_div(o.n_kv, 2);
  else o.n_passes = ceil_div(o.n_kv, 4);
  o.a_off = kHeaderBytes;
  o.a_stage_bytes = static_cast<int64_t>(o.n1) * o.srow;
  o.a_bytes = o.a_stage_bytes * o.kc;
  o.bk_off = align_up(o.a_off + o.a_bytes, 256);
  o.b_bytes = static_cast<int64_t>(o.n_passes) * o.r16 * 4 * 32 * 16;
  o.bv_off = align_up(o.bk_off + o.b_bytes, 256);
  o.total = align_up(o.bv_off + o.b_bytes, 256);
  return true;
}

// Output-column order of the expand product.  A pass covers 64 columns; thread q of a
// quad owns two 8-column chunks (chunk_lo, chunk_lo + head_dim/16) holding both halves
// of its RoPE pairs (rotate-half pairs column i with i + head_dim/2, rope.py:9-13).
__host__ __device__ inline int chunk_lo(int pass, int q, int hd) {
  if (hd >= 64) {
    const int per = hd / 64;
    return (pass / per) * (hd / 8) + 4 * (pass % per) + q;
  }
  if (hd == 32) return (2 * pass + (q >> 1)) * 4 + (q & 1);
  return (4 * pass + q) * 2;  // hd == 16
}
__host__ __device__ inline int head_of(int pass, int q, int hd) {
  if (hd >= 64) return pass / (hd / 64);
  if (hd == 32) return 2 * pass + (q >> 1);
  return 4 * pass + q;
}
// Output column produced by expand n-tile jt (0..7) of `pass` at mma column n (0..7),
// or -1 when that head does not exist.
__host__ __device__ inline int expand_col(int pass, int jt, int n, int hd, int n_kv) {
  const int qo = n >> 1, b = n & 1;
  if (head_of(pass, qo, hd) >= n_kv) return -1;
  const int lo = chunk_lo(pass, qo, hd);
  const int ch = jt < 4 ? lo : lo + hd / 16;
  return 8 * ch + 2 * (jt & 3) + b;
}

// ----------------------------------------------------------------------------
// factor packing
// ----------------------------------------------------------------------------
struct PackParams {
  Geo g;
  dkv_lora_factors f;
  uint8_t *packed;
  int64_t pstride;
};

__device__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float w = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) w = fmaxf(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

// grid (n_layers, 4): part 0 = A_k, 1 = A_v, 2 = B_k, 3 = B_v
__global__ void __launch_bounds__(256) pack_kernel(const PackParams pp) {
  __shared__ float red[32];
  const Geo &g = pp.g;
  const dkv_lora_factors &f = pp.f;
  const int layer = blockIdx.x, part = blockIdx.y;
  uint8_t *img = pp.packed + layer * pp.pstride;
  const bool is_a = part < 2, is_k = (part & 1) == 0;
  const int rank = is_k ? f.rank_k : f.rank_v;
  const void *M = nullptr;
  if (part == 0) M = f.a_k;
  if (part == 1) M = f.a_v;
  if (part == 2) M = f.b_k;
  if (part == 3) M = f.b_v;
  const int64_t mstride = part == 0   ? f.a_k_layer_stride
                          : part == 1 ? f.a_v_layer_stride
                          : part == 2 ? f.b_k_layer_stride
                                      : f.b_v_layer_stride;
  const bool present = M != nullptr && rank > 0;
  const int64_t mbase = static_cast<int64_t>(layer) * mstride;
  const int64_t wbase = static_cast<int64_t>(layer) * f.norm_layer_stride;
  auto aval = [&](int r, int k) -> float {  // A[r][k] * w[k]
    float v = load_as_float(M, f.dtype, mbase + static_cast<int64_t>(r) * g.d_model + k);
    if (f.norm_weight != nullptr) v *= load_as_float(f.norm_weight, f.norm_dtype, wbase + k);
    return v;
  };
  auto bval = [&](int c, int r) -> float {  // B[c][r]
    return load_as_float(M, f.dtype, mbase + static_cast<int64_t>(c) * rank + r);
  };
  // 1. magnitude -> power-of-two scale that puts the largest entry in [2^14, 2^15)
  float mx = 0.f;
  if (present) {
    const int64_t n = is_a ? static_cast<int64_t>(rank) * g.d_model
                           : static_cast<int64_t>(g.d_kv) * rank;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const float v = is_a ? aval(static_cast<int>(i / g.d_model), static_cast<int>(i % g.d_model))
                           : bval(static_cast<int>(i / rank), static_cast<int>(i % rank));
      if (isfinite(v)) mx = fmaxf(mx, fabsf(v));
    }
  }
  mx = block_max(mx, red);
  int e = 0;
  const int top = (is_a && g.tc && g.x_dtype == DKV_E4M3) ? 7 : 14;  // e4m3 max 448, f16 max 65504
  if (mx > 0.f) e = top - ilogbf(mx);
  e = max(-120, min(120, e));
  const float sc = exp2i(e);
  if (threadIdx.x == 0) {
    float *hdr = reinterpret_cast<float *>(img);
    const float s = is_k ? f.scale_k : f.scale_v;
    // [0] codes mult K, [1] codes mult V, [2] out mult K, [3] out mult V
    if (is_a) hdr[is_k ? 0 : 1] = s * exp2i(-e);
    else hdr[is_k ? 2 : 3] = exp2i(-e);
    if (part == 0) {
      int32_t *ih = reinterpret_cast<int32_t *>(img);
      ih[4] = f.rank_k;
      ih[5] = f.rank_v;
      ih[6] = g.rpad;
    }
  }
  // 2. write the operand image
  if (is_a && g.tc) {
    // tcgen05 image: row ng = (K|V block) + term * rpad + n, 128 bytes per stage, the 16-byte
    // unit u of row ng stored at u ^ (ng & 7) (the SWIZZLE_128B K-major layout).  fp8 X:
    // three e4m3 terms with A*2^E ~= t0 + t1/16 + t2/256; f16 X: one f16 term.
    const int64_t units = static_cast<int64_t>(g.kc) * g.rpad * 8;
    const int vblk = is_k ? 0 : g.terms * g.rpad;
    for (int64_t i = threadIdx.x; i < units; i += blockDim.x) {
      const int kci = static_cast<int>(i / (g.rpad * 8));
      const int rem = static_cast<int>(i % (g.rpad * 8));
      const int n = rem >> 3, u = rem & 7;
      if (g.x_dtype == DKV_E4M3) {
        uint32_t w[3][4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          uint32_t b[3] = {0, 0, 0};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int k = kci * g.stage_k + 16 * u + 4 * jj + t;
            float v = (present && n < rank && k < g.d_model) ? aval(n, k) * sc : 0.f;
#pragma unroll
            for (int term = 0; term < 3; ++term) {
              const uint32_t q = f32_to_e4m3(v);
              b[term] |= q << (8 * t);
              v = (v - e4m3_to_f32(q)) * 16.f;
            }
          }
#pragma unroll
          for (int term = 0; term < 3; ++term) w[term][jj] = b[term];
        }
#pragma unroll
        for (int term = 0; term < 3; ++term) {
          const int ng = vblk + term * g.rpad + n;
          uint8_t *dst = img + g.a_off + kci * g.a_stage_bytes + static_cast<int64_t>(ng) * 128 +
                         ((u ^ (ng & 7)) << 4);
          *reinterpret_cast<uint4 *>(dst) = make_uint4(w[term][0], w[term][1], w[term][2], w[term][3]);
        }
      } else {
        uint32_t w[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float v2[2];
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int k = kci * g.stage_k + 8 * u + 2 * jj + t;
            v2[t] = (present && n < rank && k < g.d_model) ? aval(n, k) * sc : 0.f;
          }
          w[jj] = pack_f16x2(v2[0], v2[1]);
        }
        const int ng = vblk + n;
        uint8_t *dst = img + g.a_off + kci * g.a_stage_bytes + static_cast<int64_t>(ng) * 128 +
                       ((u ^ (ng & 7)) << 4);
        *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  } else if (is_a) {
    const int upr = g.srow / 16;  // 16-byte units per row per stage
    const int64_t units = static_cast<int64_t>(g.kc) * g.rpad * upr;
    const int row_base = is_k ? 0 : g.rpad;
    for (int64_t i = threadIdx.x; i < units; i += blockDim.x) {
      const int kci = static_cast<int>(i / (g.rpad * upr));
      const int rem = static_cast<int>(i % (g.rpad * upr));
      const int n = rem / upr, u = rem % upr;
      const int ng = row_base + n;
      const int grp = u >> 2, q = u & 3;
      uint32_t w[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        float v2[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int j = 2 * jj + t;
          int k;
          if (g.x_dtype == DKV_E4M3) k = 32 * grp + (j < 4 ? 4 * q + j : 16 + 4 * q + (j - 4));
          else k = 32 * grp + 8 * (j >> 1) + 2 * q + (j & 1);
          k += kci * g.stage_k;
          v2[t] = (present && n < rank && k < g.d_model) ? aval(n, k) * sc : 0.f;
        }
        w[jj] = pack_f16x2(v2[0], v2[1]);
      }
      uint8_t *dst = img + g.a_off + kci * g.a_stage_bytes + static_cast<int64_t>(ng) * g.srow +
                     ((u ^ ((ng & 1) << 2)) << 4);
      *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    const int64_t total = static_cast<int64_t>(g.n_passes) * g.r16 * 4 * 32;
    uint8_t *base = img + (is_k ? g.bk_off : g.bv_off);
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
      const int lane = static_cast<int>(i & 31);
      const int c = static_cast<int>((i >> 5) & 3);
      const int64_t pk = i >> 7;  // pass * r16 + ks
      const int ks = static_cast<int>(pk % g.r16);
      const int pass = static_cast<int>(pk / g.r16);
      const int gg = lane >> 2, q = lane & 3;
      uint32_t w[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int jt = 2 * c + h;
        const int col = expand_col(pass, jt, gg, g.hd, g.n_kv);
        float v[4];
        const int kk[4] = {16 * ks + 2 * q, 16 * ks + 2 * q + 1, 16 * ks + 2 * q + 8,
                           16 * ks + 2 * q + 9};
#pragma unroll
        for (int t = 0; t < 4; ++t)
          v[t] = (present && col >= 0 && kk[t] < rank) ? bval(col, kk[t]) * sc : 0.f;
        w[2 * h] = pack_f16x2(v[0], v[1]);
        w[2 * h + 1] = pack_f16x2(v[2], v[3]);
      }
      *reinterpret_cast<uint4 *>(base + i * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// ----------------------------------------------------------------------------
// fused patch kernel
// ----------------------------------------------------------------------------
struct alignas(64) Params {
  CUtensorMap x_map;
  const uint8_t *packed;
  int64_t packed_stride;
  const float *x_scale;
  int64_t xs_stride;
  const float *x_sumsq;  // optional per-row sum of squared codes (RMSNorm without the X.X^T product)
  int64_t xsq_stride;
  const float *rope_cos, *rope_sin;
  int32_t rope_max_pos, has_rope;
  float norm_eps, inv_d;
  int32_t d_model, n_kv, hd, d_kv, r16, n_passes, kc, stage_k;
  int64_t a_off, bk_off, bv_off;
  int32_t do_k, do_v, accumulate, n_layers;
  const int32_t *cu_seqlens, *block_tables, *table_lens, *positions;
  int64_t table_stride;
  int32_t n_seqs, max_chunks, block_size, prefetch_lead;
  int32_t nip, nh;  // expand passes = nip frequency blocks x nh heads (or head groups)
  int32_t k_shead_i, v_shead_i;  // head strides as 32-bit ints (row offsets stay below 2^31)
  int64_t k_sblock, k_sslot, k_shead, k_nblocks;
  int64_t v_sblock, v_sslot, v_shead, v_nblocks;
  int32_t *status;
  int64_t n_tiles, x_rows;
  void *k_base[DKV_MAX_LAYERS];
  void *v_base[DKV_MAX_LAYERS];
};

struct Tile {
  int layer, seq, row0, c0, len;
};

__device__ __forceinline__ bool decode_tile(const Params &p, int64_t tile, Tile &t) {
  const int64_t per_layer = static_cast<int64_t>(p.n_seqs) * p.max_chunks;
  t.layer = static_cast<int>(tile / per_layer);
  const int64_t rem = tile % per_layer;
  t.seq = static_cast<int>(rem / p.max_chunks);
  const int chunk = static_cast<int>(rem % p.max_chunks);
  const int s0 = __ldg(p.cu_seqlens + t.seq);
  t.len = __ldg(p.cu_seqlens + t.seq + 1) - s0;
  t.c0 = chunk * kMTile;
  t.row0 = s0 + t.c0;
  return t.c0 < t.len;
}

// 8 page elements (one chunk) held as raw bits
template <int PDT>
struct Chunk;
template <>
struct Chunk<DKV_BF16> {
  uint4 v;
  __device__ __forceinline__ void load(const void *p) { v = ldg128_stream(p); }
  __device__ __forceinline__ void lds(uint32_t a) { v = lds128(a); }
  __device__ __forceinline__ void store(void *p) const { stg128_stream(p, v); }
  __device__ __forceinline__ float get(int j) const {
    const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
    return (j & 1) ? bf16hi(w) : bf16lo(w);
  }
  // elements (2i, 2i+1) as an fp32 pair
  __device__ __forceinline__ uint64_t pair(int i) const {
    const uint32_t w = i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    return f2pack(bf16lo(w), bf16hi(w));
  }
  __device__ __forceinline__ void set_pairs(const uint64_t (&q)[4]) {
    float a, b;
    f2unpack(q[0], a, b); v.x = pack_bf16x2(a, b);
    f2unpack(q[1], a, b); v.y = pack_bf16x2(a, b);
    f2unpack(q[2], a, b); v.z = pack_bf16x2(a, b);
    f2unpack(q[3], a, b); v.w = pack_bf16x2(a, b);
  }
  __device__ __forceinline__ void set_all(const float (&f)[8]) {
    v.x = pack_bf16x2(f[0], f[1]);
    v.y = pack_bf16x2(f[2], f[3]);
    v.z = pack_bf16x2(f[4], f[5]);
    v.w = pack_bf16x2(f[6], f[7]);
  }
  static constexpr int kElemBytes = 2;
};
template <>
struct Chunk<DKV_F16> {
  uint4 v;
  __device__ __forceinline__ void load(const void *p) { v = ldg128_stream(p); }
  __device__ __forceinline__ void lds(uint32_t a) { v = lds128(a); }
  __device__ __forceinline__ void store(void *p) const { stg128_stream(p, v); }
  __device__ __forceinline__ float get(int j) const {
    const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
    return (j & 1) ? f16hi(w) : f16lo(w);
  }
  __device__ __forceinline__ uint64_t pair(int i) const {
    const uint32_t w = i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    return f2pack(f16lo(w), f16hi(w));
  }
  __device__ __forceinline__ void set_pairs(const uint64_t (&q)[4]) {
    float a, b;
    f2unpack(q[0], a, b); v.x = pack_f16x2(a, b);
    f2unpack(q[1], a, b); v.y = pack_f16x2(a, b);
    f2unpack(q[2], a, b); v.z = pack_f16x2(a, b);
    f2unpack(q[3], a, b); v.w = pack_f16x2(a, b);
  }
  __device__ __forceinline__ void set_all(const float (&f)[8]) {
    v.x = pack_f16x2(f[0], f[1]);
    v.y = pack_f16x2(f[2], f[3]);
    v.z = pack_f16x2(f[4], f[5]);
    v.w = pack_f16x2(f[6], f[7]);
  }
  static constexpr int kElemBytes = 2;
};
template <>
struct Chunk<DKV_F32> {
  uint4 a, b;
  __device__ __forceinline__ void load(const void *p) {
    a = ldg128_stream(p);
    b = ldg128_stream(static_cast<const uint8_t *>(p) + 16);
  }
  // the two 16-byte halves of a chunk sit 32 lanes apart in the page ring
  __device__ __forceinline__ void lds(uint32_t addr) {
    a = lds128(addr);
    b = lds128(addr + 32 * 16);
  }
  __device__ __forceinline__ void store(void *p) const {
    stg128_stream(p, a);
    stg128_stream(static_cast<uint8_t *>(p) + 16, b);
  }
  __device__ __forceinline__ float get(int j) const {
    const uint4 &s = j < 4 ? a : b;
    const int k = j & 3;
    return __uint_as_float(k == 0 ? s.x : k == 1 ? s.y : k == 2 ? s.z : s.w);
  }
  __device__ __forceinline__ uint64_t pair(int i) const {
    const uint4 &s = i < 2 ? a : b;
    return (i & 1) ? (static_cast<uint64_t>(s.w) << 32 | s.z) : (static_cast<uint64_t>(s.y) << 32 | s.x);
  }
  __device__ __forceinline__ void set_pairs(const uint64_t (&q)[4]) {
    a = make_uint4(static_cast<uint32_t>(q[0]), static_cast<uint32_t>(q[0] >> 32),
                   static_cast<uint32_t>(q[1]), static_cast<uint32_t>(q[1] >> 32));
    b = make_uint4(static_cast<uint32_t>(q[2]), static_cast<uint32_t>(q[2] >> 32),
                   static_cast<uint32_t>(q[3]), static_cast<uint32_t>(q[3] >> 32));
  }
  __device__ __forceinline__ void set_all(const float (&f)[8]) {
    a = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                   __float_as_uint(f[3]));
    b = make_uint4(__float_as_uint(f[4]), __float_as_uint(f[5]), __float_as_uint(f[6]),
                   __float_as_uint(f[7]));
  }
  static constexpr int kElemBytes = 4;
};

struct RowInfo {
  int64_t off_k[2], off_v[2];  // element offset of the row inside a layer's K / V pages
  float xs[2];                 // dequantisation scale
  float ss[2];                 // sum of squared codes from x_sumsq (when given)
  int pos[2];
  bool valid[2];
};

// ----------------------------------------------------------------------------
// phase 2: expand passes with the page rows streamed through a per-warp cp.async ring
// ----------------------------------------------------------------------------
// A tile's expand passes, in order: K then V; within a projection, frequency block ip
// (head_dim >= 64) outer and head h inner, so a tile loads each cos/sin block once.  The
// cursor advances without divisions; chunk offsets are closed forms of (ip, h, q).
struct Cursor {
  int kv, ip, h;  // kv: 0 = K, 1 = V, 2 = past the end
  __device__ __forceinline__ void begin(const Params &p) {
    kv = p.do_k ? 0 : (p.do_v ? 1 : 2);
    ip = h = 0;
  }
  __device__ __forceinline__ void next(const Params &p) {
    if (++h == p.nh) {
      h = 0;
      if (++ip == p.nip) {
        ip = 0;
        kv = (kv == 0 && p.do_v) ? 1 : 2;
      }
    }
  }
};

struct Chunks {
  int e_lo, e_hi;  // element offsets of this lane's two 8-column chunks inside a page row
  int pk;          // B-fragment block of the pass in the packed image
  bool hok;        // this lane's head exists
};

__device__ __forceinline__ Chunks chunks_of(const Params &p, const Cursor &c, int q, int shead) {
  Chunks o;
  if (p.hd >= 64) {
    o.e_lo = c.h * shead + 32 * c.ip + 8 * q;
    o.e_hi = o.e_lo + (p.hd >> 1);
    o.pk = c.h * p.nip + c.ip;
    o.hok = true;
  } else if (p.hd == 32) {
    const int head = 2 * c.h + (q >> 1);
    o.e_lo = head * shead + 8 * (q & 1);
    o.e_hi = o.e_lo + 16;
    o.pk = c.h;
    o.hok = head < p.n_kv;
  } else {  // 16
    const int head = 4 * c.h + q;
    o.e_lo = head * shead;
    o.e_hi = o.e_lo + 8;
    o.pk = c.h;
    o.hok = head < p.n_kv;
  }
  return o;
}

// Row pointers of this lane's two rows in the layer's K and V pages (or null when invalid).
struct RowPtrs {
  uint8_t *k[2], *v[2];
};

template <int PDT>
__device__ __forceinline__ RowPtrs row_ptrs(const Params &p, const Tile &t, const RowInfo &ri) {
  constexpr int EB = Chunk<PDT>::kElemBytes;
  RowPtrs rp;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    rp.k[r] = ri.valid[r] ? static_cast<uint8_t *>(p.k_base[t.layer]) + ri.off_k[r] * EB : nullptr;
    rp.v[r] = ri.valid[r] ? static_cast<uint8_t *>(p.v_base[t.layer]) + ri.off_v[r] * EB : nullptr;
  }
  return rp;
}

template <int PDT>
struct PageRing {
  static constexpr int EB = Chunk<PDT>::kElemBytes;
  static constexpr int NH = EB / 2;              // 16-byte pieces per 8-element chunk
  static constexpr int kSlotBytes = 4 * NH * 32 * 16;
  uint32_t base;  // this warp's ring in shared memory
  int depth;
  Cursor cur;     // next pass to issue
  int slot;

  __device__ __forceinline__ uint32_t piece(int s, int rh, int half, int lane) const {
    return base + s * kSlotBytes + (((rh * NH + half) * 32 + lane) << 4);
  }
  __device__ __forceinline__ void begin(const Params &p) {
    cur.begin(p);
    slot = 0;
  }
  // start the copies of the next pass's page chunks (rows g, g+8; chunks lo, hi)
  __device__ __forceinline__ void issue(const Params &p, const RowPtrs &rp, int lane) {
    if (cur.kv < 2 && p.accumulate) {
      const Chunks c = chunks_of(p, cur, lane & 3, cur.kv == 0 ? p.k_shead_i : p.v_shead_i);
      if (c.hok) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint8_t *row = cur.kv == 0 ? rp.k[r] : rp.v[r];
          if (row == nullptr) continue;
#pragma unroll
          for (int half = 0; half < NH; ++half) {
            cp_async_16(piece(slot, 2 * r, half, lane), row + c.e_lo * EB + 16 * half);
            cp_async_16(piece(slot, 2 * r + 1, half, lane), row + c.e_hi * EB + 16 * half);
          }
        }
      }
    }
    cp_async_commit();
    if (cur.kv < 2) cur.next(p);
    if (++slot == depth) slot = 0;
  }
};

// Expand, RoPE, scale and write back one pass.  `pg` holds the current page chunks when
// accumulating.  The pass's B fragments come from shared memory at `bsm` (a per-warp slot the
// caller staged) when BS, otherwise from global memory at `bfrag`.
template <int R16, int PDT, bool BS>
__device__ __forceinline__ void expand_pass(const uint4 *__restrict__ bfrag, uint32_t bsm,
                                            const uint32_t (&cf)[R16][4], const float (&cs)[2][8],
                                            const float (&sn)[2][8], bool rope, int e_lo, int e_hi,
                                            uint8_t *const (&rows)[2], const float (&om)[2],
                                            const bool (&valid)[2], bool accumulate, int lane,
                                            Chunk<PDT> (&pg)[2][2]) {
  constexpr int EB = Chunk<PDT>::kElemBytes;
  float acc[8][4];
#pragma unroll
  for (int ks = 0; ks < R16; ++ks) {
    uint4 b[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      b[c] = BS ? lds128(bsm + static_cast<uint32_t>(((ks * 4 + c) * 32 + lane) * 16))
                : ldg128_nc(bfrag + (ks * 4 + c) * 32 + lane);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (ks == 0) {
        mma16816_zc(acc[2 * c], cf[ks][0], cf[ks][1], cf[ks][2], cf[ks][3], b[c].x, b[c].y);
        mma16816_zc(acc[2 * c + 1], cf[ks][0], cf[ks][1], cf[ks][2], cf[ks][3], b[c].z, b[c].w);
      } else {
        mma16816(acc[2 * c], cf[ks][0], cf[ks][1], cf[ks][2], cf[ks][3], b[c].x, b[c].y);
        mma16816(acc[2 * c + 1], cf[ks][0], cf[ks][1], cf[ks][2], cf[ks][3], b[c].z, b[c].w);
      }
    }
  }
  // C fragment: acc[jt][2r + b] = row r (g or g+8), chunk lo (jt < 4) / hi, elements 2(jt%4)+b
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (!valid[r]) continue;
    uint64_t lo[4], hi[4];
#pragma unroll
    for (int jt = 0; jt < 4; ++jt) {
      lo[jt] = f2pack(acc[jt][2 * r], acc[jt][2 * r + 1]);
      hi[jt] = f2pack(acc[jt + 4][2 * r], acc[jt + 4][2 * r + 1]);
    }
    if (rope) {
      // lo' = lo*cos - hi*sin, hi' = hi*cos + lo*sin  (rotate-half, rope.py:9-25)
#pragma unroll
      for (int jt = 0; jt < 4; ++jt) {
        const uint64_t c2 = f2pack(cs[r][2 * jt], cs[r][2 * jt + 1]);
        const uint64_t s2 = f2pack(sn[r][2 * jt], sn[r][2 * jt + 1]);
        const uint64_t ns2 = f2pack(-sn[r][2 * jt], -sn[r][2 * jt + 1]);
        const uint64_t a = lo[jt], b = hi[jt];
        lo[jt] = fma2(a, c2, mul2(b, ns2));
        hi[jt] = fma2(b, c2, mul2(a, s2));
      }
    }
    const uint64_t m2 = f2pack(om[r], om[r]);
    uint64_t o_lo[4], o_hi[4];
    if (accumulate) {
#pragma unroll
      for (int jt = 0; jt < 4; ++jt) {
        o_lo[jt] = fma2(lo[jt], m2, pg[r][0].pair(jt));
        o_hi[jt] = fma2(hi[jt], m2, pg[r][1].pair(jt));
      }
    } else {
#pragma unroll
      for (int jt = 0; jt < 4; ++jt) {
        o_lo[jt] = mul2(lo[jt], m2);
        o_hi[jt] = mul2(hi[jt], m2);
      }
    }
    Chunk<PDT> w0, w1;
    w0.set_pairs(o_lo);
    w1.set_pairs(o_hi);
    w0.store(rows[r] + e_lo * EB);
    w1.store(rows[r] + e_hi * EB);
  }
}

template <int R16>
__device__ __forceinline__ void load_rope(const Params &p, const RowInfo &ri, int f0,
                                          float (&cs)[2][8], float (&sn)[2][8]) {
  const int half = p.hd / 2;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t base = static_cast<int64_t>(ri.valid[r] ? ri.pos[r] : 0) * half + f0;
    const float4 c0 = __ldg(reinterpret_cast<const float4 *>(p.rope_cos + base));
    const float4 c1 = __ldg(reinterpret_cast<const float4 *>(p.rope_cos + base + 4));
    const float4 s0 = __ldg(reinterpret_cast<const float4 *>(p.rope_sin + base));
    const float4 s1 = __ldg(reinterpret_cast<const float4 *>(p.rope_sin + base + 4));
    cs[r][0] = c0.x; cs[r][1] = c0.y; cs[r][2] = c0.z; cs[r][3] = c0.w;
    cs[r][4] = c1.x; cs[r][5] = c1.y; cs[r][6] = c1.z; cs[r][7] = c1.w;
    sn[r][0] = s0.x; sn[r][1] = s0.y; sn[r][2] = s0.z; sn[r][3] = s0.w;
    sn[r][4] = s1.x; sn[r][5] = s1.y; sn[r][6] = s1.z; sn[r][7] = s1.w;
  }
}

// A CTA-wide ring of B-fragment slots, one pass (16 B x 4 x R16 per lane) per slot.  A
// producer thread fills the slots with the passes of the CTA's tiles in the order the
// epilogue consumes them, as far ahead as the ring allows; every epilogue warp reads a slot
// and releases it (empty: kEpiWarps arrivals).  Fetching the fragments inside the pass
// (mma.sync operands straight from L2) left every pass's MMAs waiting on L2 latency.
struct BRing {
  uint8_t *base;
  uint64_t *full, *empty;
  int slot;
  uint32_t phase;
};

// All expand passes of one tile (K then V), consuming the page ring whose first `depth`
// passes the caller has already issued.  With BS the passes' B fragments come from the
// CTA's B ring; returns false when a slot never filled (abort raised).
template <int R16, int PDT, int DEPTH, bool BS = false>
__device__ __forceinline__ bool phase2(const Params &p, const Tile &t, const RowInfo &ri,
                                       const RowPtrs &rp, PageRing<PDT> &ring,
                                       const uint32_t (&ck)[R16][4], const uint32_t (&cv)[R16][4],
                                       const float (&om_k)[2], const float (&om_v)[2], int lane,
                                       BRing *br = nullptr, int n_bslots = 0, volatile int *abort = nullptr) {
  const uint8_t *img = p.packed + t.layer * p.packed_stride;
  const uint4 *bfk = reinterpret_cast<const uint4 *>(img + p.bk_off);
  const uint4 *bfv = reinterpret_cast<const uint4 *>(img + p.bv_off);
  const int q = lane & 3;
  const bool acc = p.accumulate != 0;
  constexpr uint32_t kBBytes = 16u * 4 * 32 * R16;
  float cs[2][8], sn[2][8];
  int cur_ip = -1;
  Cursor c;
  c.begin(p);
  int slot = 0;
  while (c.kv < 2) {
    const bool is_k = c.kv == 0;
    const Chunks ch = chunks_of(p, c, q, is_k ? p.k_shead_i : p.v_shead_i);
    const bool rope = is_k && p.has_rope;
    if (rope && c.ip != cur_ip) {
      const int f0 = p.hd >= 64 ? 32 * c.ip + 8 * q : (p.hd == 32 ? 8 * (q & 1) : 0);
      load_rope<R16>(p, ri, f0, cs, sn);
      cur_ip = c.ip;
    }
    const uint4 *bf = (is_k ? bfk : bfv) + ch.pk * R16 * 4 * 32;
    Cursor nx = c;
    nx.next(p);
    if (!BS && nx.kv < 2 && lane < 16 * R16) {
      // pull the next pass's B fragments into L1 (16 lines of 128 B per k-step block)
      const uint8_t *nb = reinterpret_cast<const uint8_t *>(
          (nx.kv == 0 ? bfk : bfv) + chunks_of(p, nx, 0, 0).pk * R16 * 4 * 32);
      asm volatile("prefetch.global.L1 [%0];" ::"l"(nb + lane * 128));
    }
    if (BS) {
      const bool ok = mbar_wait_bounded(&br->full[br->slot], br->phase, abort);
      if (!__all_sync(0xffffffffu, ok)) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort = 1;
        cp_async_wait<0>();
        return false;
      }
    }
    cp_async_wait<DEPTH - 1>();
    Chunk<PDT> pg[2][2];
    const bool v2[2] = {ri.valid[0] && ch.hok, ri.valid[1] && ch.hok};
    if (acc) {
#pragma unroll
      for (int r = 0; r < 2; ++r)
        if (v2[r]) {
          pg[r][0].lds(ring.piece(slot, 2 * r, 0, lane));
          pg[r][1].lds(ring.piece(slot, 2 * r + 1, 0, lane));
        }
    }
    const uint32_t bsm = BS ? smem_u32(br->base) + static_cast<uint32_t>(br->slot) * kBBytes : 0u;
    if (is_k)
      expand_pass<R16, PDT, BS>(bf, bsm, ck, cs, sn, rope, ch.e_lo, ch.e_hi, rp.k, om_k, v2, acc, lane, pg);
    else
      expand_pass<R16, PDT, BS>(bf, bsm, cv, cs, sn, false, ch.e_lo, ch.e_hi, rp.v, om_v, v2, acc, lane, pg);
    if (BS) {  // the slot's fragments went into this pass's MMAs: release it
      __syncwarp();
      if (lane == 0) mbar_arrive(&br->empty[br->slot]);
      if (++br->slot == n_bslots) {
        br->slot = 0;
        br->phase ^= 1u;
      }
    }
    // the chunks read from this slot have been consumed: refill it with the pass DEPTH ahead
    ring.issue(p, rp, lane);
    if (++slot == DEPTH) slot = 0;
    c.next(p);
  }
  cp_async_wait<0>();
  return true;
}

// Validity, RoPE position and page offsets of rows g and g+8 of warp `warp` in tile t;
// range errors are recorded in the status word and the row is skipped.
__device__ __forceinline__ RowInfo make_row_info(const Params &p, const Tile &t, int warp, int g) {
  RowInfo ri;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int tok = t.c0 + 16 * warp + g + 8 * r;
    const int64_t grow = static_cast<int64_t>(t.row0 - t.c0) + tok;
    bool v = tok < t.len;
    if (v && grow >= p.x_rows) {
      record_error(p.status, DKV_ERR_INVALID_ARGUMENT);
      v = false;
    }
    int pos = tok;
    ri.off_k[r] = ri.off_v[r] = 0;
    ri.xs[r] = 1.f;
    ri.ss[r] = 0.f;
    if (v) {
      if (p.positions) pos = __ldg(p.positions + grow);
      if (p.has_rope && (pos < 0 || pos >= p.rope_max_pos)) {
        record_error(p.status, DKV_ERR_ROPE_RANGE);
        v = false;
      }
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
          ri.off_k[r] = static_cast<int64_t>(bid) * p.k_sblock + static_cast<int64_t>(slot) * p.k_sslot;
          ri.off_v[r] = static_cast<int64_t>(bid) * p.v_sblock + static_cast<int64_t>(slot) * p.v_sslot;
        }
      }
      if (p.x_scale) ri.xs[r] = __ldg(p.x_scale + t.layer * p.xs_stride + grow);
      if (p.x_sumsq) ri.ss[r] = __ldg(p.x_sumsq + t.layer * p.xsq_stride + grow);
    }
    ri.valid[r] = v;
    ri.pos[r] = pos;
  }
  return ri;
}

// TMA producer run by one thread: walks the same (tile, k-slab) sequence the warps consume
// and keeps every ring slot filled.  The X slab comes by a 3-D tensor copy (128-B swizzle),
// the matching packed-A slab by a contiguous bulk copy; both complete on full[stage].
template <int A_STAGE, int STAGES = kStages>
struct Producer {
  int64_t tile;
  int kc, layer, row0, stage;
  uint32_t phase, issued, parity;

  __device__ void init(const Params &p) {
    tile = static_cast<int64_t>(blockIdx.x) - gridDim.x;
    kc = p.kc;
    stage = 0;
    phase = issued = parity = 0;
  }
  __device__ bool advance(const Params &p) {
    if (kc < p.kc) return true;
    for (;;) {
      tile += gridDim.x;
      if (tile >= p.n_tiles) return false;
      Tile t;
      if (decode_tile(p, tile, t)) {
        kc = 0;
        layer = t.layer;
        row0 = t.row0;
        return true;
      }
    }
  }
  // 1: issued one item; 0: nothing left; -1: gave up waiting for a free slot
  __device__ int issue(const Params &p, uint8_t *sx, uint8_t *sa, uint64_t *full, uint64_t *empty,
                       volatile int *abort) {
    if (!advance(p)) return 0;
    if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort)) return -1;
    mbar_arrive_expect_tx(&full[stage], kXStageBytes + A_STAGE);
    tma_load_3d(sx + stage * kXStageBytes, &p.x_map, &full[stage], kc * p.stage_k, row0, layer);
    bulk_load(sa + stage * A_STAGE,
              p.packed + layer * p.packed_stride + p.a_off + static_cast<int64_t>(kc) * A_STAGE,
              A_STAGE, &full[stage]);
    issued |= 1u << stage;
    parity = (parity & ~(1u << stage)) | (phase << stage);
    ++kc;
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
    return 1;
  }
  // never let the CTA exit with a copy still landing in its shared memory
  __device__ void drain(const Params &p, uint64_t *full) const {
    for (int s = 0; s < STAGES; ++s) {
      if (!(issued & (1u << s))) continue;
      const long long t0 = clock64();
      while (!mbar_try_wait(&full[s], (parity >> s) & 1)) {
        if (clock64() - t0 > kWaitLimitCycles) {
          record_error(p.status, DKV_ERR_TIMEOUT);
          break;
        }
      }
    }
  }
};

// Depth of the per-warp page ring: as deep as shared memory allows next to the X / A ring.
template <int R16, int PDT>
struct RingDepth {
  static constexpr int slot = PageRing<PDT>::kSlotBytes;
  static constexpr int value = (R16 <= 2) ? (PDT == DKV_F32 ? 2 : 4)
                               : (R16 == 3) ? (PDT == DKV_F32 ? 2 : 4)
                                            : (PDT == DKV_F32 ? 1 : 2);
};

template <int XT, int R16, bool NORM, int PDT>
__global__ void __launch_bounds__(kThreads, 1) patch_kernel(const __grid_constant__ Params p) {
  constexpr int NT1 = 4 * R16;  // phase-1 n-tiles: K codes then V codes, 8 columns each
  constexpr int SROW = XT == 0 ? 256 : 128;
  constexpr int A_STAGE = 2 * 16 * R16 * SROW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *sx = smem;                          // [kStages][128 rows][128 B], 128-B swizzled
  uint8_t *sa = smem + kStages * kXStageBytes;  // [kStages][n1 rows][SROW]
  constexpr int DEPTH = RingDepth<R16, PDT>::value;
  constexpr int RING_BYTES = DEPTH * PageRing<PDT>::kSlotBytes;
  uint8_t *sp = sa + kStages * A_STAGE;  // [warps][DEPTH] page-chunk slots
  uint64_t *full = reinterpret_cast<uint64_t *>(sp + kConsumerWarps * RING_BYTES);
  uint64_t *empty = full + kStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // lane 0 of warp 0 drives the TMA ring, kStages (tile, k-slab) items ahead
  const bool is_prod = threadIdx.x == 0;
  Producer<A_STAGE> prod;
  if (is_prod) {
    prefetch_tensormap(&p.x_map);
    prod.init(p);
    for (int i = 0; i < kStages; ++i) {
      const int r = prod.issue(p, sx, sa, full, empty, abort_flag);
      if (r < 0) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      if (r <= 0) break;
    }
  }
  __syncwarp();

  // ------------------------------- consumers --------------------------------
  const int g = lane >> 2, q = lane & 3;
  int stage = 0;
  uint32_t phase = 0;
  // ldmatrix addressing of this lane inside a stage
  const int mat = lane >> 3;
  const int xrow = 16 * warp + (lane & 7) + ((mat & 1) << 3);
  const int xsw = xrow & 7;
  const int bsw = (g & 1) << 2;
  PageRing<PDT> ring;
  ring.base = smem_u32(sp) + warp * RING_BYTES;
  ring.depth = DEPTH;

  for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
    Tile t;
    if (!decode_tile(p, tile, t)) continue;

    // ---- per-row metadata (rows g and g+8 of this warp) ----
    const RowInfo ri = make_row_info(p, t, warp, g);
    const RowPtrs rp = row_ptrs<PDT>(p, t, ri);

    // ---- phase 1: codes = x . A^T (and sum x^2) over the streamed stages ----
    float acc[NT1][4];
#pragma unroll
    for (int j = 0; j < NT1; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    float dg[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) dg[j][0] = dg[j][1] = dg[j][2] = dg[j][3] = 0.f;

    const int pf_at = p.kc > p.prefetch_lead ? p.kc - p.prefetch_lead : 0;
    for (int kc = 0; kc < p.kc; ++kc) {
      if (kc == pf_at && lane < 16) {
        // warm L2 with this warp's page rows before the read-add-write pass
        const int tok = t.c0 + 16 * warp + lane;
        if (tok < t.len) {
          const int bi = tok / p.block_size;
          const int64_t tlen = p.table_lens ? __ldg(p.table_lens + t.seq) : p.table_stride;
          if (bi < tlen) {
            const int bid = __ldg(p.block_tables + static_cast<int64_t>(t.seq) * p.table_stride + bi);
            if (bid >= 0 && bid < p.k_nblocks && bid < p.v_nblocks) {
              const int slot = tok % p.block_size;
              constexpr int EB = Chunk<PDT>::kElemBytes;
              const uint32_t row_bytes = static_cast<uint32_t>(p.d_kv * EB);
              if (p.do_k && p.k_shead == p.hd) {
                const uint8_t *a = static_cast<const uint8_t *>(p.k_base[t.layer]) +
                                   (static_cast<int64_t>(bid) * p.k_sblock + static_cast<int64_t>(slot) * p.k_sslot) * EB;
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(row_bytes) : "memory");
              }
              if (p.do_v && p.v_shead == p.hd) {
                const uint8_t *a = static_cast<const uint8_t *>(p.v_base[t.layer]) +
                                   (static_cast<int64_t>(bid) * p.v_sblock + static_cast<int64_t>(slot) * p.v_sslot) * EB;
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(row_bytes) : "memory");
              }
            }
          }
        }
      }
      if (kc == p.kc - 1) {
        // start streaming the first page chunks of phase 2 under the last X slab
        ring.begin(p);
        for (int i = 0; i < DEPTH; ++i) ring.issue(p, rp, lane);
      }
      if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort_flag = 1;
        cp_async_wait<0>();
        if (is_prod) prod.drain(p, full);
        return;
      }
      const uint32_t xb = smem_u32(sx + stage * kXStageBytes) + xrow * 128;
      const uint32_t ab = smem_u32(sa + stage * A_STAGE);
      if (XT == 0) {
        // fp8 e4m3: one ldmatrix.x4 gives 16 rows x 32 k; k is permuted consistently in A
#pragma unroll
        for (int grp = 0; grp < 4; ++grp) {
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4(r0, r1, r2, r3, xb + (((2 * grp + (mat >> 1)) ^ xsw) << 4));
          uint32_t a[2][4];
          a[0][0] = e4m3x2_to_f16x2(r0);
          a[0][2] = e4m3x2_to_f16x2(r0 >> 16);
          a[0][1] = e4m3x2_to_f16x2(r1);
          a[0][3] = e4m3x2_to_f16x2(r1 >> 16);
          a[1][0] = e4m3x2_to_f16x2(r2);
          a[1][2] = e4m3x2_to_f16x2(r2 >> 16);
          a[1][1] = e4m3x2_to_f16x2(r3);
          a[1][3] = e4m3x2_to_f16x2(r3 >> 16);
#pragma unroll
          for (int j = 0; j < NT1; ++j) {
            const uint4 bb = lds128(ab + (8 * j + g) * SROW + (((4 * grp + q) ^ bsw) << 4));
            mma16816(acc[j], a[0][0], a[0][1], a[0][2], a[0][3], bb.x, bb.y);
            mma16816(acc[j], a[1][0], a[1][1], a[1][2], a[1][3], bb.z, bb.w);
          }
          if (NORM && !p.x_sumsq) {
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              mma16816(dg[0], a[kk][0], a[kk][1], a[kk][2], a[kk][3], a[kk][0], a[kk][2]);
              mma16816(dg[1], a[kk][0], a[kk][1], a[kk][2], a[kk][3], a[kk][1], a[kk][3]);
            }
          }
        }
      } else {
        // f16: two ldmatrix.x4 per 32 k, standard fragment order
#pragma unroll
        for (int grp = 0; grp < 2; ++grp) {
          uint32_t a[2][4];
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            ldmatrix_x4(a[kk][0], a[kk][1], a[kk][2], a[kk][3],
                        xb + (((4 * grp + 2 * kk + (mat >> 1)) ^ xsw) << 4));
#pragma unroll
          for (int j = 0; j < NT1; ++j) {
            const uint4 bb = lds128(ab + (8 * j + g) * SROW + (((4 * grp + q) ^ bsw) << 4));
            mma16816(acc[j], a[0][0], a[0][1], a[0][2], a[0][3], bb.x, bb.y);
            mma16816(acc[j], a[1][0], a[1][1], a[1][2], a[1][3], bb.z, bb.w);
          }
          if (NORM && !p.x_sumsq) {
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
              mma16816(dg[0], a[kk][0], a[kk][1], a[kk][2], a[kk][3], a[kk][0], a[kk][2]);
              mma16816(dg[1], a[kk][0], a[kk][1], a[kk][2], a[kk][3], a[kk][1], a[kk][3]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1;
      }
      if (warp == 0) {
        // refill the slot just released by all warps with the item kStages ahead
        if (is_prod && prod.issue(p, sx, sa, full, empty, abort_flag) < 0) {
          record_error(p.status, DKV_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        __syncwarp();
      }
    }

    // ---- per-row scales: dequant * RMSNorm * LoRA scale ----
    const float *hdr = reinterpret_cast<const float *>(p.packed + t.layer * p.packed_stride);
    float rs[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) rs[r] = ri.xs[r];
    if (NORM) {
      const int src = 4 * g + (g >> 1);
      const float s0 = __shfl_sync(0xffffffffu, (g & 1) ? dg[0][1] : dg[0][0], src);
      const float s1 = __shfl_sync(0xffffffffu, (g & 1) ? dg[1][3] : dg[1][2], src);
      const float ss[2] = {p.x_sumsq ? ri.ss[0] : s0, p.x_sumsq ? ri.ss[1] : s1};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const float xs = ri.xs[r];
        rs[r] = xs * rsqrtf(xs * xs * ss[r] * p.inv_d + p.norm_eps);
      }
    }

    // codes -> f16 A fragments with a per-row power-of-two scale (K then V)
    uint32_t ck[R16][4], cv[R16][4];
    float om_k[2], om_v[2];
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const float cm = hdr[kv];  // s * 2^-ea
      float mrow[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 2 * R16; ++j) {
        const int jj = kv * 2 * R16 + j;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          acc[jj][2 * r] *= cm * rs[r];
          acc[jj][2 * r + 1] *= cm * rs[r];
          mrow[r] = fmaxf(mrow[r], fmaxf(fabsf(acc[jj][2 * r]), fabsf(acc[jj][2 * r + 1])));
        }
      }
      float e2[2], oms[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float m = mrow[r];
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        int e = (m > 0.f && isfinite(m)) ? 14 - ilogbf(m) : 0;
        e = max(-120, min(120, e));
        e2[r] = exp2i(e);
        oms[r] = hdr[2 + kv] * exp2i(-e);
      }
#pragma unroll
      for (int ks = 0; ks < R16; ++ks) {
        const int j0 = kv * 2 * R16 + 2 * ks, j1 = j0 + 1;
        const uint32_t f0 = pack_f16x2(acc[j0][0] * e2[0], acc[j0][1] * e2[0]);
        const uint32_t f1 = pack_f16x2(acc[j0][2] * e2[1], acc[j0][3] * e2[1]);
        const uint32_t f2 = pack_f16x2(acc[j1][0] * e2[0], acc[j1][1] * e2[0]);
        const uint32_t f3 = pack_f16x2(acc[j1][2] * e2[1], acc[j1][3] * e2[1]);
        if (kv == 0) {
          ck[ks][0] = f0; ck[ks][1] = f1; ck[ks][2] = f2; ck[ks][3] = f3;
        } else {
          cv[ks][0] = f0; cv[ks][1] = f1; cv[ks][2] = f2; cv[ks][3] = f3;
        }
      }
      if (kv == 0) { om_k[0] = oms[0]; om_k[1] = oms[1]; }
      else { om_v[0] = oms[0]; om_v[1] = oms[1]; }
    }

    // ---- phase 2: dK / dV, RoPE, page read-add-write ----
    phase2<R16, PDT, DEPTH>(p, t, ri, rp, ring, ck, cv, om_k, om_v, lane);
  }
  if (is_prod) prod.drain(p, full);
}

// ----------------------------------------------------------------------------
// tcgen05 variant (rank <= 32): codes on the 5th-generation tensor cores
// ----------------------------------------------------------------------------
// Warp roles (12 warps):
//   0-7  epilogue: per tile, read the codes out of tensor memory (warps 0-3, one TMEM lane
//        quarter each), then all 8 run phase 2 exactly as the mma.sync kernel does;
//   8    TMA producer (lane 0): X slab + packed-A slab per stage, STAGES-deep ring;
//   9    MMA issuer (lane 0) and owner of the 512-column TMEM allocation;
//   10,11 spare.
// Per stage the issuer runs K=32 tcgen05.mma steps for codes (M=128 tokens, N = codes
// columns, e4m3 x e4m3 or f16 x f16 -> fp32 in TMEM) and, with RMSNorm, for X.X^T whose
// diagonal is sum(x^2).  Accumulators are double-buffered across tiles when they fit, so
// the tensor cores and the X stream work on tile i+1 while the epilogue patches tile i.
constexpr int kTcWarps = 12;  // 8 epilogue, TMA producer, MMA issuer, B-fragment producer, idle
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kEpiWarps = 8;
constexpr int kBProdWarp = 10;
constexpr int kBSlots = 8;  // passes of B fragments in flight or waiting in shared memory

template <int XT, int R16, bool NORM>
struct TcCfg {
  static constexpr int RPAD = 16 * R16;
  static constexpr int TERMS = XT == 0 ? 3 : 1;
  static constexpr int N1 = TERMS * 2 * RPAD;  // codes columns: K terms, then V terms
  static constexpr int STAGES = R16 == 1 ? 4 : 3;
  static constexpr int A_STAGE = N1 * 128;
  static constexpr int DIAG = N1 <= 128 ? 128 : 256;  // column of the X.X^T accumulator
  static constexpr int BUF = NORM ? DIAG + 128 : (N1 <= 128 ? 128 : 256);
  static constexpr int NBUF = BUF <= 256 ? 2 : 1;
  static constexpr int CROW = 4 * RPAD + 16;  // bytes per row of the f16 codes tile in smem
  static constexpr uint32_t IDESC_CODES = umma_idesc(0, 128, N1);
  static constexpr uint32_t IDESC_DIAG = umma_idesc(0, 128, 128);
};

template <int XT, int R16, bool NORM, int PDT>
struct TcSmem {
  using C = TcCfg<XT, R16, NORM>;
  static constexpr int DEPTH = RingDepth<R16, PDT>::value;
  static constexpr int RING = DEPTH * PageRing<PDT>::kSlotBytes;
  static constexpr int X_OFF = 0;
  static constexpr int A_OFF = X_OFF + C::STAGES * kXStageBytes;
  static constexpr int P_OFF = A_OFF + C::STAGES * C::A_STAGE;
  static constexpr int CODES_OFF = P_OFF + kEpiWarps * RING;
  static constexpr int OM_OFF = CODES_OFF + 2 * 128 * C::CROW;
  // the CTA's B-fragment ring (kBSlots passes), when it fits next to the other rings
  static constexpr int BSLOT = 16 * 4 * 32 * R16;
  static constexpr int B_OFF = OM_OFF + 2 * 2 * 128 * 4;
  static constexpr int BASE_BARS = 2 * C::STAGES + 4 + 1 + 4;
  static constexpr bool BSMEM =
      1024 + B_OFF + kBSlots * BSLOT + (BASE_BARS + 2 * kBSlots) * 8 + 16 <= 227 * 1024;
  static constexpr int BAR_OFF = B_OFF + (BSMEM ? kBSlots * BSLOT : 0);
  static constexpr int N_BARS = BASE_BARS + (BSMEM ? 2 * kBSlots : 0);
  static constexpr int MISC_OFF = BAR_OFF + N_BARS * 8;
  static constexpr int BYTES = MISC_OFF + 16;
};

template <int XT, int R16, bool NORM>
__device__ __forceinline__ void issue_stage_mmas(uint32_t d_codes, uint32_t d_diag, uint32_t xs,
                                                 uint32_t as, bool first, bool diag) {
  using C = TcCfg<XT, R16, NORM>;
  const uint64_t adesc = umma_desc_k_sw128(xs);
  const uint64_t bdesc = umma_desc_k_sw128(as);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {  // 4 x 32 bytes of K per 128-byte swizzled row
    const uint32_t acc = (first && kk == 0) ? 0u : 1u;
    const uint64_t a = adesc + static_cast<uint64_t>(2 * kk), b = bdesc + static_cast<uint64_t>(2 * kk);
    if (XT == 0) {
      umma_e4m3(d_codes, a, b, C::IDESC_CODES, acc);
      if (NORM && diag) umma_e4m3(d_diag, a, a, C::IDESC_DIAG, acc);
    } else {
      umma_f16(d_codes, a, b, C::IDESC_CODES, acc);
      if (NORM && diag) umma_f16(d_diag, a, a, C::IDESC_DIAG, acc);
    }
  }
}

// TMEM -> shared-memory codes of one tile, one lane quarter and one projection per warp: warp
// w reads rows 32 (w & 3) + lane, the K codes for w < 4 and the V codes for w >= 4; combines
// the e4m3 terms, applies the dequantisation / RMSNorm / LoRA scales and stores f16 codes with
// a per-row power-of-two exponent.  Returns false (abort raised) when the accumulator never
// became ready.
template <int XT, int R16, bool NORM>
__device__ __forceinline__ bool tc_readout(const Params &p, const Tile &t, int b, int64_t use, uint8_t *codes,
                                           float *om, uint32_t tmem, uint64_t *tfull, uint64_t *tempty,
                                           volatile int *abort_flag, int warp, int lane) {
  using C = TcCfg<XT, R16, NORM>;
  constexpr int RPAD = C::RPAD;
  const int qw = warp & 3, kv = warp >> 2;
  const bool ok = mbar_wait_bounded(&tfull[b], static_cast<uint32_t>(use & 1), abort_flag);
  if (!__all_sync(0xffffffffu, ok)) {
    record_error(p.status, DKV_ERR_TIMEOUT);
    *abort_flag = 1;
    return false;
  }
  tc_fence_after();
  const int row = 32 * qw + lane;
  const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * qw) << 16) + b * C::BUF;
  const int tok = t.c0 + row;
  const int64_t grow = static_cast<int64_t>(t.row0) + row;
  float xs = 1.f;
  if (p.x_scale && tok < t.len && grow < p.x_rows) xs = __ldg(p.x_scale + t.layer * p.xs_stride + grow);
  float rs = xs;
  if (NORM) {
    float ss = 0.f;
    if (p.x_sumsq) {  // warp-uniform: written with the stored activations
      if (tok < t.len && grow < p.x_rows) ss = __ldg(p.x_sumsq + t.layer * p.xsq_stride + grow);
    } else {  // the diagonal of the X.X^T accumulator
      float d0[16], d1[16];
      tmem_ld16(taddr + C::DIAG + 32 * qw, d0);
      tmem_ld16(taddr + C::DIAG + 32 * qw + 16, d1);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        ss = (i == lane) ? d0[i] : ss;
        ss = (16 + i == lane) ? d1[i] : ss;
      }
    }
    rs = xs * rsqrtf(xs * xs * ss * p.inv_d + p.norm_eps);
  }
  const float *hdr = reinterpret_cast<const float *>(p.packed + t.layer * p.packed_stride);
  {
    float c[RPAD];
#pragma unroll
    for (int h = 0; h < R16; ++h) {
      float v0[16], v1[16], v2[16];
      const uint32_t col = taddr + kv * C::TERMS * RPAD + 16 * h;
      tmem_ld16(col, v0);
      if (C::TERMS == 3) {
        tmem_ld16(col + RPAD, v1);
        tmem_ld16(col + 2 * RPAD, v2);
      }
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float x = v0[i];
        if (C::TERMS == 3) x = fmaf(v2[i], 0.00390625f, fmaf(v1[i], 0.0625f, x));
        c[16 * h + i] = x;
      }
    }
    const float cm = hdr[kv] * rs;
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < RPAD; ++i) {
      c[i] *= cm;
      m = fmaxf(m, fabsf(c[i]));
    }
    int e = (m > 0.f && isfinite(m)) ? 14 - ilogbf(m) : 0;
    e = max(-120, min(120, e));
    const float e2 = exp2i(e);
    uint32_t w[RPAD / 2];
#pragma unroll
    for (int i = 0; i < RPAD / 2; ++i) w[i] = pack_f16x2(c[2 * i] * e2, c[2 * i + 1] * e2);
    uint4 *dst = reinterpret_cast<uint4 *>(codes + row * C::CROW + kv * RPAD * 2);
#pragma unroll
    for (int i = 0; i < RPAD / 8; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    om[kv * 128 + row] = hdr[2 + kv] * exp2i(-e);
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(&tempty[b]);
  return true;
}

template <int XT, int R16, bool NORM, int PDT>
__global__ void __launch_bounds__(kTcThreads, 1) patch_kernel_tc(const __grid_constant__ Params p) {
  using C = TcCfg<XT, R16, NORM>;
  using S = TcSmem<XT, R16, NORM, PDT>;
  constexpr int RPAD = C::RPAD, STAGES = C::STAGES, NBUF = C::NBUF, DEPTH = S::DEPTH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t *sx = smem + S::X_OFF;
  uint8_t *sa = smem + S::A_OFF;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + S::BAR_OFF);
  uint64_t *empty = full + STAGES;
  uint64_t *tfull = empty + STAGES;  // [2]
  uint64_t *tempty = tfull + 2;      // [2]
  uint64_t *done = tempty + 2;
  uint64_t *cready = done + 1;   // [2] codes buffer written by all epilogue warps
  uint64_t *cfree = cready + 2;  // [2] codes buffer read by all epilogue warps
  uint64_t *bfull = cfree + 2;       // [kBSlots] B ring slot filled (BSMEM)
  uint64_t *bempty = bfull + kBSlots; // [kBSlots] B ring slot read by every epilogue warp
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + S::MISC_OFF);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + S::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);  // every epilogue warp reads its share of the codes
    }
    mbar_init(done, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&cready[b], kEpiWarps);
      mbar_init(&cfree[b], kEpiWarps);
    }
    if (S::BSMEM)
      for (int i = 0; i < kBSlots; ++i) {
        mbar_init(&bfull[i], 1);
        mbar_init(&bempty[i], kEpiWarps);
      }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t *>(tmem_slot);

  if (warp == 8) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      prefetch_tensormap(&p.x_map);
      Producer<C::A_STAGE, STAGES> prod;
      prod.init(p);
      for (;;) {
        const int r = prod.issue(p, sx, sa, full, empty, abort_flag);
        if (r < 0) {
          record_error(p.status, DKV_ERR_TIMEOUT);
          *abort_flag = 1;
        }
        if (r <= 0) break;
      }
      prod.drain(p, full);
    }
  } else if (warp == 9) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t j = 0;  // tiles done by this CTA
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        Tile t;
        if (!decode_tile(p, tile, t)) continue;
        const int b = static_cast<int>(j % NBUF);
        const int64_t use = j / NBUF;
        if (use > 0 && !mbar_wait_bounded(&tempty[b], static_cast<uint32_t>((use - 1) & 1), abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_codes = tmem + b * C::BUF;
        const uint32_t d_diag = d_codes + C::DIAG;
        for (int kc = 0; kc < p.kc; ++kc) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_stage_mmas<XT, R16, NORM>(d_codes, d_diag, smem_u32(sx + stage * kXStageBytes),
                                          smem_u32(sa + stage * C::A_STAGE), kc == 0, p.x_sumsq == nullptr);
          umma_commit(&empty[stage]);  // the slot is free once these MMAs have read it
          if (++stage == STAGES) {
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
  } else if (warp < kEpiWarps) {
    // -------------------------------- epilogue --------------------------------
    // The codes of tile j+1 are read out of TMEM (all 8 warps, one lane quarter and projection
    // each) right after this warp has loaded its fragments of tile j, while tile j's first page
    // copies are in flight; codes_ready / codes_free (8 arrivals each, one pair per codes buffer)
    // replace a per-tile barrier of all epilogue warps.
    const int g = lane >> 2;
    uint8_t *codes_base = smem + S::CODES_OFF;
    float *om_base = reinterpret_cast<float *>(smem + S::OM_OFF);
    PageRing<PDT> ring;
    ring.base = smem_u32(smem + S::P_OFF) + warp * S::RING;
    ring.depth = DEPTH;
    BRing bring{smem + S::B_OFF, bfull, bempty, 0, 0u};
    auto next_valid = [&](int64_t tile, Tile &t) -> int64_t {
      for (; tile < p.n_tiles; tile += gridDim.x)
        if (decode_tile(p, tile, t)) return tile;
      return p.n_tiles;
    };
    auto wait_all = [&](uint64_t *bar, uint32_t parity) -> bool {
      const bool ok = mbar_wait_bounded(bar, parity, abort_flag);
      if (__all_sync(0xffffffffu, ok)) return true;
      record_error(p.status, DKV_ERR_TIMEOUT);
      *abort_flag = 1;
      return false;
    };
    Tile tc;
    int64_t tile = next_valid(blockIdx.x, tc);
    bool ok = true;
    if (tile < p.n_tiles) {
      ok = tc_readout<XT, R16, NORM>(p, tc, 0, 0, codes_base, om_base, tmem, tfull, tempty, abort_flag, warp, lane);
      if (ok) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&cready[0]);
      }
    }
    int64_t j = 0;
    while (ok && tile < p.n_tiles) {
      const int par = static_cast<int>(j & 1);
      const RowInfo ri = make_row_info(p, tc, warp, g);
      const RowPtrs rp = row_ptrs<PDT>(p, tc, ri);
      ring.begin(p);
      for (int i = 0; i < DEPTH; ++i) ring.issue(p, rp, lane);  // page chunks of phase 2
      if (!wait_all(&cready[par], static_cast<uint32_t>((j >> 1) & 1))) break;
      const uint8_t *codes = codes_base + par * 128 * C::CROW;
      const float *om = om_base + par * 2 * 128;
      // A fragments of this warp's 16 rows, K and V codes
      uint32_t ck[R16][4], cv[R16][4];
      {
        const int frow = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
        const uint32_t fbase = smem_u32(codes) + frow * C::CROW + (lane >> 4) * 16;
#pragma unroll
        for (int ks = 0; ks < R16; ++ks) {
          ldmatrix_x4(ck[ks][0], ck[ks][1], ck[ks][2], ck[ks][3], fbase + ks * 32);
          ldmatrix_x4(cv[ks][0], cv[ks][1], cv[ks][2], cv[ks][3], fbase + RPAD * 2 + ks * 32);
        }
      }
      const float om_k[2] = {om[16 * warp + g], om[16 * warp + g + 8]};
      const float om_v[2] = {om[128 + 16 * warp + g], om[128 + 16 * warp + g + 8]};
      __syncwarp();
      if (lane == 0) mbar_arrive(&cfree[par]);
      // readout of the next tile into the other codes buffer, once every warp has read tile j-1
      Tile tn;
      const int64_t ntile = next_valid(tile + gridDim.x, tn);
      if (ntile < p.n_tiles) {
        const int np1 = static_cast<int>((j + 1) & 1);
        if (j >= 1 && !wait_all(&cfree[np1], static_cast<uint32_t>(((j - 1) >> 1) & 1))) break;
        if (!tc_readout<XT, R16, NORM>(p, tn, static_cast<int>((j + 1) % NBUF), (j + 1) / NBUF,
                                       codes_base + np1 * 128 * C::CROW, om_base + np1 * 2 * 128, tmem, tfull,
                                       tempty, abort_flag, warp, lane))
          break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&cready[np1]);
      }
      if (!phase2<R16, PDT, DEPTH, S::BSMEM>(p, tc, ri, rp, ring, ck, cv, om_k, om_v, lane, &bring, kBSlots,
                                               abort_flag))
        break;
      tile = ntile;
      tc = tn;
      ++j;
    }
    cp_async_wait<0>();
  } else if (S::BSMEM && warp == kBProdWarp) {
    // --------------------------- B-fragment producer ---------------------------
    // Walks the tiles and passes in the epilogue's order and fills each ring slot as soon as
    // all epilogue warps have released it.
    if (lane == 0) {
      constexpr uint32_t kBBytes = S::BSLOT;
      int slot = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, parity = 0;  // slots with a copy issued, and its phase (drain below)
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < p.n_tiles && ok; tile += gridDim.x) {
        Tile t;
        if (!decode_tile(p, tile, t)) continue;
        const uint8_t *img = p.packed + t.layer * p.packed_stride;
        const uint4 *bfk = reinterpret_cast<const uint4 *>(img + p.bk_off);
        const uint4 *bfv = reinterpret_cast<const uint4 *>(img + p.bv_off);
        Cursor c;
        c.begin(p);
        while (c.kv < 2) {
          if (!mbar_wait_bounded(&bempty[slot], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bfull[slot], kBBytes);
          bulk_load(smem + S::B_OFF + slot * S::BSLOT,
                    (c.kv == 0 ? bfk : bfv) + chunks_of(p, c, 0, 0).pk * R16 * 4 * 32, kBBytes, &bfull[slot]);
          issued |= 1u << slot;
          parity = (parity & ~(1u << slot)) | (phase << slot);
          c.next(p);
          if (++slot == kBSlots) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && !*abort_flag) {
        record_error(p.status, DKV_ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // never exit with a copy still landing in shared memory
      for (int i = 0; i < kBSlots; ++i) {
        if (!(issued & (1u << i))) continue;
        const long long t0 = clock64();
        while (!mbar_try_wait(&bfull[i], (parity >> i) & 1u)) {
          if (clock64() - t0 > kWaitLimitCycles) {
            record_error(p.status, DKV_ERR_TIMEOUT);
            break;
          }
        }
      }
    }
  }

  // ------------------------------- teardown -------------------------------
  __syncthreads();
  if (warp == 9) {
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
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensormap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

template <int XT, int R16, bool NORM, int PDT>
int launch_tc(const Params &p, cudaStream_t st, int grid) {
  using S = TcSmem<XT, R16, NORM, PDT>;
  const size_t smem = 1024 + S::BYTES;
  auto kern = patch_kernel_tc<XT, R16, NORM, PDT>;
  static bool attr_set = false;
  if (!attr_set) {
    DKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
    attr_set = true;
  }
  kern<<<grid, kTcThreads, smem, st>>>(p);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

template <int XT, int R16, bool NORM, int PDT>
int launch_t(const Params &p, cudaStream_t st, int grid) {
  constexpr int SROW = XT == 0 ? 256 : 128;
  constexpr int A_STAGE = 2 * 16 * R16 * SROW;
  constexpr int RING_BYTES = RingDepth<R16, PDT>::value * PageRing<PDT>::kSlotBytes;
  const size_t smem = 1024 + kStages * (kXStageBytes + A_STAGE) + kConsumerWarps * RING_BYTES +
                      2 * kStages * 8 + 16;
  auto kern = patch_kernel<XT, R16, NORM, PDT>;
  DKV_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
  kern<<<grid, kThreads, smem, st>>>(p);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

template <int XT, int R16, bool NORM>
int launch_p(const Params &p, int pdt, cudaStream_t st, int grid) {
  if (R16 <= 2) {
    constexpr int RT = R16 <= 2 ? R16 : 2;
    switch (pdt) {
      case DKV_BF16: return launch_tc<XT, RT, NORM, DKV_BF16>(p, st, grid);
      case DKV_F16: return launch_tc<XT, RT, NORM, DKV_F16>(p, st, grid);
      case DKV_F32: return launch_tc<XT, RT, NORM, DKV_F32>(p, st, grid);
      default: return DKV_ERR_UNSUPPORTED;
    }
  }
  switch (pdt) {
    case DKV_BF16: return launch_t<XT, R16, NORM, DKV_BF16>(p, st, grid);
    case DKV_F16: return launch_t<XT, R16, NORM, DKV_F16>(p, st, grid);
    case DKV_F32: return launch_t<XT, R16, NORM, DKV_F32>(p, st, grid);
    default: return DKV_ERR_UNSUPPORTED;
  }
}
template <int XT, int R16>
int launch_n(const Params &p, bool norm, int pdt, cudaStream_t st, int grid) {
  return norm ? launch_p<XT, R16, true>(p, pdt, st, grid)
              : launch_p<XT, R16, false>(p, pdt, st, grid);
}
template <int XT>
int launch_r(const Params &p, int r16, bool norm, int pdt, cudaStream_t st, int grid) {
  switch (r16) {
    case 1: return launch_n<XT, 1>(p, norm, pdt, st, grid);
    case 2: return launch_n<XT, 2>(p, norm, pdt, st, grid);
    case 3: return launch_n<XT, 3>(p, norm, pdt, st, grid);
    case 4: return launch_n<XT, 4>(p, norm, pdt, st, grid);
    default: return DKV_ERR_UNSUPPORTED;
  }
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  }
  return n;
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace exact
}  // namespace dkv

using namespace dkv;
using namespace dkv::exact;

extern "C" int dkv_exact_packed_bytes(const dkv_exact_geometry *geom, int64_t *bytes_per_layer) {
  if (geom == nullptr || bytes_per_layer == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  Geo g;
  if (!make_geo(*geom, g)) return DKV_ERR_UNSUPPORTED;
  *bytes_per_layer = g.total;
  return DKV_OK;
}

extern "C" int dkv_pack_exact_factors(const dkv_exact_geometry *geom,
                                      const dkv_lora_factors *factors, void *packed,
                                      int64_t packed_layer_stride, dkv_stream_t stream) {
  if (geom == nullptr || factors == nullptr || packed == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  Geo g;
  if (!make_geo(*geom, g)) return DKV_ERR_UNSUPPORTED;
  if (factors->rank_k != geom->rank_k || factors->rank_v != geom->rank_v)
    return DKV_ERR_INVALID_ARGUMENT;
  if (factors->n_layers <= 0 || factors->n_layers > 65535) return DKV_ERR_INVALID_ARGUMENT;
  if (factors->n_layers > 1 && packed_layer_stride < g.total) return DKV_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(packed) & 255u) || (packed_layer_stride & 255))
    return DKV_ERR_ALIGNMENT;
  const int dt = factors->dtype;
  if (dt != DKV_F32 && dt != DKV_F16 && dt != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  if (factors->norm_weight != nullptr && factors->norm_dtype != DKV_F32 &&
      factors->norm_dtype != DKV_F16 && factors->norm_dtype != DKV_BF16)
    return DKV_ERR_UNSUPPORTED;
  PackParams pp;
  pp.g = g;
  pp.f = *factors;
  pp.packed = static_cast<uint8_t *>(packed);
  pp.pstride = packed_layer_stride;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  pack_kernel<<<dim3(factors->n_layers, 4), 256, 0, st>>>(pp);
  DKV_CUDA_CHECK(cudaGetLastError());
  return DKV_OK;
}

static int check_pages(const dkv_paged_cache &c, const Geo &g) {
  if (c.dtype != DKV_BF16 && c.dtype != DKV_F16 && c.dtype != DKV_F32) return DKV_ERR_UNSUPPORTED;
  if (c.n_heads != g.n_kv || c.head_dim != g.hd) return DKV_ERR_LAYOUT;
  if (c.block_size <= 0 || c.num_blocks <= 0) return DKV_ERR_LAYOUT;
  const int64_t vec = c.dtype == DKV_F32 ? 4 : 8;  // elements per 16 bytes
  if (c.stride_block % vec || c.stride_slot % vec || c.stride_head % vec) return DKV_ERR_ALIGNMENT;
  return DKV_OK;
}

extern "C" int dkv_exact_patch_paged(const dkv_exact_patch_args *a, dkv_stream_t stream) {
  if (a == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  Geo g;
  if (!make_geo(a->geom, g)) return DKV_ERR_UNSUPPORTED;
  const dkv_seq_batch &s = a->seqs;
  if (a->n_layers <= 0 || a->n_layers > DKV_MAX_LAYERS) return DKV_ERR_INVALID_ARGUMENT;
  if (s.n_seqs < 0 || s.max_seq_len < 0) return DKV_ERR_INVALID_ARGUMENT;
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
  const int esz = g.x_dtype == DKV_E4M3 ? 1 : 2;
  if (!aligned16(a->x) || (a->x_row_stride * esz) % 16 || (a->x_layer_stride * esz) % 16)
    return DKV_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(a->packed) & 255u) || (a->packed_layer_stride & 255))
    return DKV_ERR_ALIGNMENT;
  if (a->n_layers > 1 && a->packed_layer_stride < g.total) return DKV_ERR_INVALID_ARGUMENT;
  const bool rope = a->rope_cos != nullptr && a->rope_sin != nullptr;
  if (rope && (a->rope_max_pos <= 0 || !aligned16(a->rope_cos) || !aligned16(a->rope_sin)))
    return DKV_ERR_ALIGNMENT;
  if (a->x_rows <= 0 || a->x_rows > 0x7fffffffLL) return DKV_ERR_INVALID_ARGUMENT;

  Params p;
  memset(&p, 0, sizeof(p));
  auto enc = tensormap_encoder();
  if (enc == nullptr) {
    note_cuda_error(cudaErrorNotSupported, "cuTensorMapEncodeTiled entry point");
    return DKV_ERR_CUDA;
  }
  {
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(g.d_model), static_cast<cuuint64_t>(a->x_rows),
                          static_cast<cuuint64_t>(a->n_layers)};
    int64_t lstride = a->n_layers > 1 ? a->x_layer_stride : a->x_rows * a->x_row_stride;
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(a->x_row_stride * esz),
                             static_cast<cuuint64_t>(lstride * esz)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / esz), static_cast<cuuint32_t>(kMTile), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(&p.x_map,
                     esz == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                     const_cast<void *>(a->x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return DKV_ERR_ALIGNMENT;
  }
  p.packed = static_cast<const uint8_t *>(a->packed);
  p.packed_stride = a->packed_layer_stride;
  p.x_scale = a->x_scale;
  p.xs_stride = a->x_scale_layer_stride;
  p.x_sumsq = a->apply_norm ? a->x_sumsq : nullptr;
  p.xsq_stride = a->x_sumsq_layer_stride;
  p.rope_cos = rope ? a->rope_cos : nullptr;
  p.rope_sin = rope ? a->rope_sin : nullptr;
  p.rope_max_pos = rope ? a->rope_max_pos : 0;
  p.has_rope = rope ? 1 : 0;
  p.norm_eps = a->norm_eps;
  p.inv_d = 1.0f / static_cast<float>(g.d_model);
  p.d_model = g.d_model;
  p.n_kv = g.n_kv;
  p.hd = g.hd;
  p.d_kv = g.d_kv;
  p.r16 = g.r16;
  p.n_passes = g.n_passes;
  p.nip = g.hd >= 64 ? g.hd / 64 : 1;
  p.nh = g.hd >= 64 ? g.n_kv : g.n_passes;
  p.kc = g.kc;
  p.stage_k = g.stage_k;
  p.a_off = g.a_off;
  p.bk_off = g.bk_off;
  p.bv_off = g.bv_off;
  p.accumulate = a->accumulate ? 1 : 0;
  p.do_k = (g.rank_k > 0 || !p.accumulate) ? 1 : 0;
  p.do_v = (g.rank_v > 0 || !p.accumulate) ? 1 : 0;
  p.n_layers = a->n_layers;
  p.cu_seqlens = s.cu_seqlens;
  p.block_tables = s.block_tables;
  p.table_lens = s.table_lens;
  p.positions = s.positions;
  p.table_stride = s.table_stride;
  p.n_seqs = s.n_seqs;
  p.max_chunks = ceil_div(s.max_seq_len, kMTile);
  p.block_size = kp.block_size;
  static int lead = -1;
  if (lead < 0) {
    const char *env = getenv("DKV_PREFETCH_LEAD");
    lead = env ? atoi(env) : 8;
  }
  p.prefetch_lead = lead;
  if (kp.stride_head * g.n_kv >= (1LL << 30) || vp.stride_head * g.n_kv >= (1LL << 30))
    return DKV_ERR_LAYOUT;
  p.k_shead_i = static_cast<int32_t>(kp.stride_head);
  p.v_shead_i = static_cast<int32_t>(vp.stride_head);
  p.k_sblock = kp.stride_block;
  p.k_sslot = kp.stride_slot;
  p.k_shead = kp.stride_head;
  p.k_nblocks = kp.num_blocks;
  p.v_sblock = vp.stride_block;
  p.v_sslot = vp.stride_slot;
  p.v_shead = vp.stride_head;
  p.v_nblocks = vp.num_blocks;
  p.status = a->status;
  p.n_tiles = static_cast<int64_t>(a->n_layers) * s.n_seqs * p.max_chunks;
  p.x_rows = a->x_rows;
  for (int l = 0; l < a->n_layers; ++l) {
    p.k_base[l] = a->k_pages[l].base;
    p.v_base[l] = a->v_pages[l].base;
    if (p.k_base[l] == nullptr || p.v_base[l] == nullptr) return DKV_ERR_INVALID_ARGUMENT;
    if (!aligned16(p.k_base[l]) || !aligned16(p.v_base[l])) return DKV_ERR_ALIGNMENT;
  }
  if (!p.do_k && !p.do_v) return DKV_OK;
  const int64_t want = static_cast<int64_t>(sm_count());
  const int grid = static_cast<int>(p.n_tiles < want ? p.n_tiles : want);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool norm = a->apply_norm != 0;
  if (g.x_dtype == DKV_E4M3) return launch_r<0>(p, g.r16, norm, kp.dtype, st, grid);
  return launch_r<1>(p, g.r16, norm, kp.dtype, st, grid);
}
