// First-order causal attention — the O(n^2) core of the analytic route (Route A,
// src/deltakv/patches/analytic.py:38-105 attention_first_order):
//
//   S = Q K^T / sqrt(hd) + causal,  A = softmax(S),  dS = (dQ K^T + Q dK^T) / sqrt(hd)
//   dA = A (.) (dS - rowsum(A (.) dS))          (softmax_jacobian_product, analytic.py:25-35)
//   ctx = A V,   dctx = dA V + A dV
//
// per query head h with its GQA key/value head h / (H / Hkv) (analytic.py:142-153), without
// materialising the [H, n, n] matrices: one flash-style pass over the causal keys with an
// online softmax, since dA V = (sum_k p_k dS_k v_k - (sum_k p_k dS_k / l) sum_k p_k v_k) / l
// needs only per-row running sums.  fp32-level arithmetic (the reference runs the route in the
// model dtype, fp32 for its toy): head_dim 64 / 128 on tensor cores in a three-term bf16 split
// (afo_tc_kernel below), 16 / 32 in fp32 SIMT (afo_kernel).  A CTA takes 64 query rows of one
// head with Q and dQ resident in shared memory and streams blocks of 32 keys of K, dK, V, dV.
#include "dkv_common.cuh"

namespace dkv {
namespace afo {

constexpr int kRows = 64;  // query rows per CTA
constexpr int kKeys = 32;  // keys per staged block
constexpr int kThreads = 256;

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
  int kv_vec;  // fp32 K / dK / V / dV with 16-byte aligned rows: staged as float4, one block ahead
};

// SIMT form.  One pass over the causal keys with online softmax.  Thread (ty, tx) = (tid / 16, tid % 16)
// owns query rows 4 ty .. 4 ty + 3: in the score phase keys 2 tx, 2 tx + 1 of the block (a
// 4 x 2 micro-tile of S and dS), in the output phase head_dim columns tx + 16 j.  Per row the
// 16 threads of a half-warp share the online statistics m (max), l (sum of p = exp(S - m)),
// t (sum of p dS) and the three accumulators
//   O = sum p v,  OS = sum p dS v,  OD = sum p dv
// rescaled by exp(m_old - m_new) as m grows; at the end ctx = O / l and
// dctx = (OS - (t / l) O) / l + OD / l.
template <int DT, int HD>
__global__ void __launch_bounds__(kThreads, HD <= 64 ? 2 : 1) afo_kernel(const Args a) {
  constexpr int CPT = HD / 16;  // output columns per thread
  extern __shared__ __align__(16) float sm[];
  float *Qt = sm;                       // [HD][kRows]  (q * scale)^T
  float *dQt = Qt + HD * kRows;         // [HD][kRows]
  float *Kt = dQt + HD * kRows;         // [HD][kKeys]
  float *dKt = Kt + HD * kKeys;         // [HD][kKeys]
  float *Vs = dKt + HD * kKeys;         // [kKeys][HD]
  float *dVs = Vs + kKeys * HD;         // [kKeys][HD]
  float *Pt = dVs + kKeys * HD;         // [kKeys][kRows]  p
  float *PDt = Pt + kKeys * kRows;      // [kKeys][kRows]  p dS
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int h = blockIdx.y, hk = h / (a.n_heads / a.n_kv);
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kRows;  // the longest (latest) rows first
  for (int e = tid; e < kRows * HD; e += kThreads) {
    const int r = e / HD, d = e - r * HD;
    const int row = q0 + r;
    float x = 0.f, dx = 0.f;
    if (row < a.n) {
      const int64_t o = static_cast<int64_t>(row) * a.q_row + static_cast<int64_t>(h) * HD + d;
      x = ld<DT>(a.q, o) * a.scale;  // the 1/sqrt(hd) of S and dS folded into Q and dQ
      dx = ld<DT>(a.dq, o) * a.scale;
    }
    Qt[d * kRows + r] = x;
    dQt[d * kRows + r] = dx;
  }
  float m[4], l[4], t[4], O[4][CPT], OS[4][CPT], OD[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -INFINITY;
    l[i] = t[i] = 0.f;
#pragma unroll
    for (int j = 0; j < CPT; ++j) O[i][j] = OS[i][j] = OD[i][j] = 0.f;
  }
  const int last_key = min(q0 + kRows, a.n);
  const int n_blocks = (last_key + kKeys - 1) / kKeys;
  for (int kb = 0; kb < n_blocks; ++kb) {
    const int k0 = kb * kKeys;
    __syncthreads();  // the previous block's tiles are consumed
    for (int e = tid; e < kKeys * HD; e += kThreads) {
      const int c = e / HD, d = e - c * HD;
      const int key = k0 + c;
      float kv = 0.f, dkv = 0.f, vv = 0.f, dvv = 0.f;
      if (key < a.n) {
        const int64_t o = static_cast<int64_t>(key) * a.kv_row + static_cast<int64_t>(hk) * HD + d;
        kv = ld<DT>(a.k, o);
        dkv = ld<DT>(a.dk, o);
        vv = ld<DT>(a.v, o);
        dvv = ld<DT>(a.dv, o);
      }
      Kt[d * kKeys + c] = kv;
      dKt[d * kKeys + c] = dkv;
      Vs[e] = vv;
      dVs[e] = dvv;
    }
    __syncthreads();
    // scores: S and dS for rows 4 ty + i, keys 2 tx + c
    float S[4][2], dS[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) S[i][0] = S[i][1] = dS[i][0] = dS[i][1] = 0.f;
#pragma unroll 4
    for (int d = 0; d < HD; ++d) {
      const float4 qv = *reinterpret_cast<const float4 *>(Qt + d * kRows + 4 * ty);
      const float4 dqv = *reinterpret_cast<const float4 *>(dQt + d * kRows + 4 * ty);
      const float2 kv = *reinterpret_cast<const float2 *>(Kt + d * kKeys + 2 * tx);
      const float2 dkv = *reinterpret_cast<const float2 *>(dKt + d * kKeys + 2 * tx);
      const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, dqa[4] = {dqv.x, dqv.y, dqv.z, dqv.w};
      const float ka[2] = {kv.x, kv.y}, dka[2] = {dkv.x, dkv.y};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          S[i][c] = fmaf(qa[i], ka[c], S[i][c]);
          dS[i][c] = fmaf(dqa[i], ka[c], dS[i][c]);
          dS[i][c] = fmaf(qa[i], dka[c], dS[i][c]);
        }
    }
    // online softmax over this block (causal: key <= row; keys past n are masked too)
    float corr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = q0 + 4 * ty + i;
      float bm = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int key = k0 + 2 * tx + c;
        if (key > row || key >= a.n) S[i][c] = -INFINITY;
        bm = fmaxf(bm, S[i][c]);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
      const float mn = fmaxf(m[i], bm);
      corr[i] = mn == -INFINITY ? 1.f : expf(m[i] - mn);
      float ls = 0.f, ts = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const float p = S[i][c] == -INFINITY ? 0.f : expf(S[i][c] - mn);
        const float pd = p * dS[i][c];
        ls += p;
        ts += pd;
        Pt[(2 * tx + c) * kRows + 4 * ty + i] = p;
        PDt[(2 * tx + c) * kRows + 4 * ty + i] = pd;
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        ls += __shfl_xor_sync(0xffffffffu, ls, o);
        ts += __shfl_xor_sync(0xffffffffu, ts, o);
      }
      m[i] = mn;
      l[i] = fmaf(l[i], corr[i], ls);
      t[i] = fmaf(t[i], corr[i], ts);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < CPT; ++j) {
        O[i][j] *= corr[i];
        OS[i][j] *= corr[i];
        OD[i][j] *= corr[i];
      }
    __syncthreads();  // P / PdS complete
    const int kmax = min(kKeys, last_key - k0);
    for (int c = 0; c < kmax; ++c) {
      const float4 pv = *reinterpret_cast<const float4 *>(Pt + c * kRows + 4 * ty);
      const float4 pdv = *reinterpret_cast<const float4 *>(PDt + c * kRows + 4 * ty);
      const float pa[4] = {pv.x, pv.y, pv.z, pv.w}, pda[4] = {pdv.x, pdv.y, pdv.z, pdv.w};
#pragma unroll
      for (int j = 0; j < CPT; ++j) {
        const float vv = Vs[c * HD + tx + 16 * j], dvv = dVs[c * HD + tx + 16 * j];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          O[i][j] = fmaf(pa[i], vv, O[i][j]);
          OS[i][j] = fmaf(pda[i], vv, OS[i][j]);
          OD[i][j] = fmaf(pa[i], dvv, OD[i][j]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + 4 * ty + i;
    if (row >= a.n) continue;
    const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
    const float tb = t[i] * inv;
    float *o = a.dctx + static_cast<int64_t>(row) * a.out_row + static_cast<int64_t>(h) * HD;
    float *c = a.ctx ? a.ctx + static_cast<int64_t>(row) * a.out_row + static_cast<int64_t>(h) * HD : nullptr;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      o[tx + 16 * j] = fmaf(OS[i][j] - tb * O[i][j], inv, OD[i][j] * inv);
      if (c) c[tx + 16 * j] = O[i][j] * inv;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Tensor-core form (head_dim 64 / 128): the same single pass, with every product on mma.sync
// bf16 tensor cores in a three-term split — x = hi + lo with hi = bf16(x), lo = bf16(x - hi),
// x y ~ hi_x hi_y + hi_x lo_y + lo_x hi_y (the lo_x lo_y term is below 2^-16 relative), fp32
// accumulation — so scores keep ~2^-16 relative accuracy.  8 warps per CTA of 64 query rows:
// warp w computes S and dS for rows 16 (w & 3) .. + 15 over each 32-key block (the two warps of
// a row group duplicate this) and accumulates O, OS, OD for its half of head_dim (w >> 2).  The
// score fragments become the A fragments of the output products in registers (FlashAttention-2
// layout reuse); K / dK come as B fragments by ldmatrix, V / dV by ldmatrix.trans.
template <int HD>
struct TcLayout {
  static constexpr int LD = HD + 8;  // bf16 per smem row (16-byte pad: conflict-free ldmatrix)
  static constexpr int Q_ROWS = kRows, K_ROWS = kKeys;
  static constexpr int bytes() { return (4 * Q_ROWS + 8 * K_ROWS) * LD * 2; }
};

__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16 &h, __nv_bfloat16 &l) {
  h = __float2bfloat16_rn(x);
  l = __float2bfloat16_rn(x - __bfloat162float(h));
}
// hi / lo bf16x2 pairs of two fp32 values (lower element in the low half)
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
  hi = pack_bf16x2(a, b);
  const float ah = __uint_as_float(hi << 16), bh = __uint_as_float(hi & 0xffff0000u);
  lo = pack_bf16x2(a - ah, b - bh);
}
__device__ __forceinline__ void mma3(float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                                     uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma16816_bf16(c, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
  mma16816_bf16(c, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
  mma16816_bf16(c, al[0], al[1], al[2], al[3], bh0, bh1);
}

template <int DT, int HD>
__global__ void __launch_bounds__(kThreads, 1) afo_tc_kernel(const Args a) {
  using Lt = TcLayout<HD>;
  constexpr int LD = Lt::LD;
  constexpr int NT = HD / 16;  // 8-column output n-tiles in this warp's half of head_dim
  extern __shared__ __align__(16) __nv_bfloat16 smb[];
  __nv_bfloat16 *Qh = smb, *Ql = Qh + kRows * LD, *dQh = Ql + kRows * LD, *dQl = dQh + kRows * LD;
  __nv_bfloat16 *Kh = dQl + kRows * LD, *Kl = Kh + kKeys * LD, *dKh = Kl + kKeys * LD, *dKl = dKh + kKeys * LD;
  __nv_bfloat16 *Vh = dKl + kKeys * LD, *Vl = Vh + kKeys * LD, *dVh = Vl + kKeys * LD, *dVl = dVh + kKeys * LD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  const int rg = warp & 3, half = warp >> 2;
  const int h = blockIdx.y, hk = h / (a.n_heads / a.n_kv);
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kRows;  // the longest (latest) rows first
  for (int e = tid; e < kRows * HD; e += kThreads) {
    const int r = e / HD, d = e - r * HD;
    const int row = q0 + r;
    float x = 0.f, dx = 0.f;
    if (row < a.n) {
      const int64_t o = static_cast<int64_t>(row) * a.q_row + static_cast<int64_t>(h) * HD + d;
      x = ld<DT>(a.q, o) * a.scale;
      dx = ld<DT>(a.dq, o) * a.scale;
    }
    split_bf16(x, Qh[r * LD + d], Ql[r * LD + d]);
    split_bf16(dx, dQh[r * LD + d], dQl[r * LD + d]);
  }
  const int r0 = q0 + 16 * rg + g, r1 = r0 + 8;  // this lane's two rows
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, t[2] = {0.f, 0.f};
  float O[NT][4], OS[NT][4], OD[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) O[j][c] = OS[j][c] = OD[j][c] = 0.f;
  const int last_key = min(q0 + kRows, a.n);
  const int n_blocks = (last_key + kKeys - 1) / kKeys;
  // ldmatrix lane addressing
  const int a_row = 16 * rg + (lane & 15), a_col = (lane >> 4) * 8;                 // A: rows x k
  const int b_key = (lane & 7) + ((lane >> 4) << 3), b_col = ((lane >> 3) & 1) * 8;  // B from K rows
  const int v_key = (lane & 7) + (((lane >> 3) & 1) << 3), v_col = (lane >> 4) * 8;  // B from V rows (trans)
  // fp32 inputs with 16-byte rows: each thread holds NV float4 of K, dK, V and dV of the next
  // key block in registers, loaded before the current block's products and split into the
  // shared tiles after them, so the global loads overlap the tensor-core work
  // (head_dim <= 64: at 128 the four register blocks would not fit next to the accumulators)
  constexpr bool kPF = HD <= 64;
  constexpr int NV = kPF ? kKeys * HD / 4 / kThreads : 1;
  const bool vec = kPF && a.kv_vec;
  float4 pk[NV], pdk[NV], pv[NV], pdv[NV];
  auto fetch = [&](int kbase) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e4 = tid + i * kThreads, c = e4 / (HD / 4), d4 = e4 - c * (HD / 4);
      const int key = kbase + c;
      pk[i] = pdk[i] = pv[i] = pdv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (key < a.n) {
        const int64_t o = static_cast<int64_t>(key) * a.kv_row + static_cast<int64_t>(hk) * HD + 4 * d4;
        pk[i] = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.k) + o));
        pdk[i] = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.dk) + o));
        pv[i] = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.v) + o));
        pdv[i] = __ldg(reinterpret_cast<const float4 *>(static_cast<const float *>(a.dv) + o));
      }
    }
  };
  auto put4 = [&](__nv_bfloat16 *hi, __nv_bfloat16 *lo, int off, const float4 &x) {
    uint32_t h01, l01, h23, l23;
    split2(x.x, x.y, h01, l01);
    split2(x.z, x.w, h23, l23);
    *reinterpret_cast<uint2 *>(hi + off) = make_uint2(h01, h23);
    *reinterpret_cast<uint2 *>(lo + off) = make_uint2(l01, l23);
  };
  if constexpr (kPF) {
    if (vec) fetch(0);
  }
  for (int kb = 0; kb < n_blocks; ++kb) {
    const int k0 = kb * kKeys;
    __syncthreads();
    if (vec) {
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int e4 = tid + i * kThreads, c = e4 / (HD / 4), d4 = e4 - c * (HD / 4);
        const int off = c * LD + 4 * d4;
        put4(Kh, Kl, off, pk[i]);
        put4(dKh, dKl, off, pdk[i]);
        put4(Vh, Vl, off, pv[i]);
        put4(dVh, dVl, off, pdv[i]);
      }
    } else
    for (int e = tid; e < kKeys * HD; e += kThreads) {
      const int c = e / HD, d = e - c * HD;
      const int key = k0 + c;
      float kv = 0.f, dkv = 0.f, vv = 0.f, dvv = 0.f;
      if (key < a.n) {
        const int64_t o = static_cast<int64_t>(key) * a.kv_row + static_cast<int64_t>(hk) * HD + d;
        kv = ld<DT>(a.k, o);
        dkv = ld<DT>(a.dk, o);
        vv = ld<DT>(a.v, o);
        dvv = ld<DT>(a.dv, o);
      }
      split_bf16(kv, Kh[c * LD + d], Kl[c * LD + d]);
      split_bf16(dkv, dKh[c * LD + d], dKl[c * LD + d]);
      split_bf16(vv, Vh[c * LD + d], Vl[c * LD + d]);
      split_bf16(dvv, dVh[c * LD + d], dVl[c * LD + d]);
    }
    __syncthreads();
    if constexpr (kPF) {
      if (vec && kb + 1 < n_blocks) fetch(k0 + kKeys);
    }
    // scores of 4 n-tiles (32 keys): S and dS
    float S[4][4], dS[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) S[j][c] = dS[j][c] = 0.f;
#pragma unroll 2
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t qh[4], ql[4], dqh[4], dql[4];
      const int ao = a_row * LD + 16 * ks + a_col;
      ldmatrix_x4(qh[0], qh[1], qh[2], qh[3], smem_u32(Qh + ao));
      ldmatrix_x4(ql[0], ql[1], ql[2], ql[3], smem_u32(Ql + ao));
      ldmatrix_x4(dqh[0], dqh[1], dqh[2], dqh[3], smem_u32(dQh + ao));
      ldmatrix_x4(dql[0], dql[1], dql[2], dql[3], smem_u32(dQl + ao));
#pragma unroll
      for (int np = 0; np < 2; ++np) {  // n-tiles 2 np, 2 np + 1
        const int bo = (16 * np + b_key) * LD + 16 * ks + b_col;
        uint32_t kh[4], kl[4], dkh[4], dkl[4];
        ldmatrix_x4(kh[0], kh[1], kh[2], kh[3], smem_u32(Kh + bo));
        ldmatrix_x4(kl[0], kl[1], kl[2], kl[3], smem_u32(Kl + bo));
        ldmatrix_x4(dkh[0], dkh[1], dkh[2], dkh[3], smem_u32(dKh + bo));
        ldmatrix_x4(dkl[0], dkl[1], dkl[2], dkl[3], smem_u32(dKl + bo));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = 2 * np + u;
          mma3(S[j], qh, ql, kh[2 * u], kh[2 * u + 1], kl[2 * u], kl[2 * u + 1]);
          mma3(dS[j], dqh, dql, kh[2 * u], kh[2 * u + 1], kl[2 * u], kl[2 * u + 1]);
          mma3(dS[j], qh, ql, dkh[2 * u], dkh[2 * u + 1], dkl[2 * u], dkl[2 * u + 1]);
        }
      }
    }
    // online softmax: lane holds rows r0 (c = 0, 1) and r1 (c = 2, 3), keys k0 + 8 j + 2 q + (c & 1)
    float corr[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int row = hr ? r1 : r0;
      float bm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int key = k0 + 8 * j + 2 * q + c;
          if (key > row || key >= a.n) S[j][2 * hr + c] = -INFINITY;
          bm = fmaxf(bm, S[j][2 * hr + c]);
        }
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 2));
      const float mn = fmaxf(m[hr], bm);
      corr[hr] = mn == -INFINITY ? 1.f : expf(m[hr] - mn);
      float ls = 0.f, ts = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float sv = S[j][2 * hr + c];
          const float pv = sv == -INFINITY ? 0.f : expf(sv - mn);
          const float pd = pv * dS[j][2 * hr + c];
          S[j][2 * hr + c] = pv;  // S now holds p
          dS[j][2 * hr + c] = pd;  // dS now holds p dS
          ls += pv;
          ts += pd;
        }
      ls += __shfl_xor_sync(0xffffffffu, ls, 1);
      ls += __shfl_xor_sync(0xffffffffu, ls, 2);
      ts += __shfl_xor_sync(0xffffffffu, ts, 1);
      ts += __shfl_xor_sync(0xffffffffu, ts, 2);
      m[hr] = mn;
      l[hr] = fmaf(l[hr], corr[hr], ls);
      t[hr] = fmaf(t[hr], corr[hr], ts);
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      O[j][0] *= corr[0], O[j][1] *= corr[0], O[j][2] *= corr[1], O[j][3] *= corr[1];
      OS[j][0] *= corr[0], OS[j][1] *= corr[0], OS[j][2] *= corr[1], OS[j][3] *= corr[1];
      OD[j][0] *= corr[0], OD[j][1] *= corr[0], OD[j][2] *= corr[1], OD[j][3] *= corr[1];
    }
    // outputs: two 16-key k-steps; P / PdS fragments straight from the score accumulators
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t ph[4], pl[4], pdh[4], pdl[4];
      split2(S[2 * kk][0], S[2 * kk][1], ph[0], pl[0]);
      split2(S[2 * kk][2], S[2 * kk][3], ph[1], pl[1]);
      split2(S[2 * kk + 1][0], S[2 * kk + 1][1], ph[2], pl[2]);
      split2(S[2 * kk + 1][2], S[2 * kk + 1][3], ph[3], pl[3]);
      split2(dS[2 * kk][0], dS[2 * kk][1], pdh[0], pdl[0]);
      split2(dS[2 * kk][2], dS[2 * kk][3], pdh[1], pdl[1]);
      split2(dS[2 * kk + 1][0], dS[2 * kk + 1][1], pdh[2], pdl[2]);
      split2(dS[2 * kk + 1][2], dS[2 * kk + 1][3], pdh[3], pdl[3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        const int vo = (16 * kk + v_key) * LD + half * (HD / 2) + 16 * np + v_col;
        uint32_t vh[4], vl[4], dvh[4], dvl[4];
        ldmatrix_x4_trans(vh[0], vh[1], vh[2], vh[3], smem_u32(Vh + vo));
        ldmatrix_x4_trans(vl[0], vl[1], vl[2], vl[3], smem_u32(Vl + vo));
        ldmatrix_x4_trans(dvh[0], dvh[1], dvh[2], dvh[3], smem_u32(dVh + vo));
        ldmatrix_x4_trans(dvl[0], dvl[1], dvl[2], dvl[3], smem_u32(dVl + vo));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int j = 2 * np + u;
          mma3(O[j], ph, pl, vh[2 * u], vh[2 * u + 1], vl[2 * u], vl[2 * u + 1]);
          mma3(OS[j], pdh, pdl, vh[2 * u], vh[2 * u + 1], vl[2 * u], vl[2 * u + 1]);
          mma3(OD[j], ph, pl, dvh[2 * u], dvh[2 * u + 1], dvl[2 * u], dvl[2 * u + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = hr ? r1 : r0;
    if (row >= a.n) continue;
    const float inv = l[hr] > 0.f ? 1.f / l[hr] : 0.f;
    const float tb = t[hr] * inv;
    float *o = a.dctx + static_cast<int64_t>(row) * a.out_row + static_cast<int64_t>(h) * HD + half * (HD / 2);
    float *cx = a.ctx ? a.ctx + static_cast<int64_t>(row) * a.out_row + static_cast<int64_t>(h) * HD + half * (HD / 2)
                      : nullptr;
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col = 8 * j + 2 * q + c;
        o[col] = fmaf(OS[j][2 * hr + c] - tb * O[j][2 * hr + c], inv, OD[j][2 * hr + c] * inv);
        if (cx) cx[col] = O[j][2 * hr + c] * inv;
      }
  }
}

template <int HD>
constexpr int smem_bytes() {
  return (2 * HD * kRows + 2 * HD * kKeys + 2 * kKeys * HD + 2 * kKeys * kRows) * 4;
}

template <int DT>
int launch(const Args &a, cudaStream_t st) {
  dim3 grid(static_cast<unsigned>((a.n + kRows - 1) / kRows), static_cast<unsigned>(a.n_heads));
#define DKV_AFO(HD)                                                                                   \
  if (a.hd == HD) {                                                                                   \
    static unsigned long long set_on = 0; /* the attribute once per device: later launches make */  \
    int dev = 0;                          /* no other runtime-API call (graph-capturable)          */  \
    DKV_CUDA_CHECK(cudaGetDevice(&dev));                                                              \
    if (dev >= 64 || !((set_on >> dev) & 1ull)) {                                                     \
      DKV_CUDA_CHECK(cudaFuncSetAttribute(afo_kernel<DT, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          smem_bytes<HD>()));                                         \
      if (dev < 64) set_on |= 1ull << dev;                                                            \
    }                                                                                                 \
    afo_kernel<DT, HD><<<grid, kThreads, smem_bytes<HD>(), st>>>(a);                                  \
    DKV_CUDA_CHECK(cudaGetLastError());                                                               \
    return DKV_OK;                                                                                    \
  }
  DKV_AFO(16)
  DKV_AFO(32)
#undef DKV_AFO
#define DKV_AFO_TC(HD)                                                                                   \
  if (a.hd == HD) {                                                                                      \
    static unsigned long long set_on = 0; /* the attribute once per device (as above) */               \
    int dev = 0;                                                                                         \
    DKV_CUDA_CHECK(cudaGetDevice(&dev));                                                                 \
    if (dev >= 64 || !((set_on >> dev) & 1ull)) {                                                        \
      DKV_CUDA_CHECK(cudaFuncSetAttribute(afo_tc_kernel<DT, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          TcLayout<HD>::bytes()));                                       \
      if (dev < 64) set_on |= 1ull << dev;                                                               \
    }                                                                                                    \
    afo_tc_kernel<DT, HD><<<grid, kThreads, TcLayout<HD>::bytes(), st>>>(a);                              \
    DKV_CUDA_CHECK(cudaGetLastError());                                                                  \
    return DKV_OK;                                                                                       \
  }
  DKV_AFO_TC(64)
  DKV_AFO_TC(128)
#undef DKV_AFO_TC
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
  const auto al16 = [](const void *ptr) { return reinterpret_cast<uintptr_t>(ptr) % 16 == 0; };
  const int kv_vec = dtype == DKV_F32 && kv_row_stride % 4 == 0 && al16(k) && al16(dk) && al16(v) && al16(dv);
  afo::Args a{q, dq, k, dk, v, dv, q_row_stride, kv_row_stride, ctx, dctx, out_row_stride,
              n_tokens, n_heads, n_kv_heads, head_dim, scale, kv_vec};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DKV_F32) return afo::launch<DKV_F32>(a, st);
  if (dtype == DKV_BF16) return afo::launch<DKV_BF16>(a, st);
  return afo::launch<DKV_F16>(a, st);
}
