// Subspace correction of a KIVI int4 KV cache, batched over (layer, projection) problems.
//
// Reference: deltakv.patches.subspace.subspace_correct (src/deltakv/patches/subspace.py:45-106)
// applied to a cache whose reused KV is stored KIVI int4 and whose corrected KV is written back
// in the same format (the multi-adapter maintenance step: every adapter view patches the
// shared int4 prefix):
//   reused = dequant(base);  R = fresh - reused
//   rhs = R B;  codes = rhs (B^T B + 1e-6 I)^-1;  fitted = codes B^T
//   orth_mu = mean_P(R - fitted);  w = min(||R|| / mean ||R||, 1)
//   corr = reused + fitted + w orth_mu;  corr[P] = fresh[P];  out = quant(corr)
// All problems of a call share d; each has its own token count, probes, basis (rank <= 64)
// and caches.  Launches (all problems at once; the two passes once per grouping mode):
//   flags   probe flags, deduplicated probe list and count
//   pack    basis -> split bf16 terms in pass1's MMA fragment order, and an fp32 row copy
//   pass1   per warp of 32 tokens: dequant, R, ||R||, rhs = R B (mma.sync on split bf16
//           terms, fp32 accumulate), per-tile column sums
//   psum    sums over the probes of R and of rhs
//   solve   one CTA per problem: G^-1 = (B^T B + 1e-6 I)^-1 in fp64, orth_mu, subspace,
//           mean ||R||
//   fitb    B G^-1 (= B G^-T, G symmetric) -> split bf16 terms in pass2's MMA fragment
//           order, so that fitted = codes B^T = rhs (B G^-1)^T needs no per-token solve
//   pass2   per warp of 32 tokens: fitted = rhs (B G^-1)^T (mma.sync on split bf16 terms),
//           corr, requantise — group extrema gathered through the warp's scratch: V groups
//           from the 4 lanes of a row, K groups from the 8 row-lanes of the warp (a warp
//           tile is exactly one K group); V probe rows are left to vprobe
//   vprobe  the V problems' probe rows requantised from fresh (per-token groups are a row's own)
// Both passes walk the channels in blocks of 32.  Per block, each warp stages its codes (one
// 16-B row per lane), the K group's scale / zero and its fresh rows (pass1) with cp.async two
// blocks ahead; the basis fragments, the same for the CTA's four warps, arrive once per CTA
// by bulk copy (cp.async.bulk, an mbarrier per slot) into a ring of kBSlots blocks that
// every warp releases after reading.  Codes are decoded without per-code shifts and
// dequantised with one fma (kivi::code_pairs), and requantised words are packed with
// cvt.pack.sat (kivi::quant_word).
// Lane (g, q) of a warp owns rows g + 8i (i = 0..3) and, in every block of 32 channels, the
// 8 contiguous channels 8q..8q+7: pass1 forms its R directly as MMA A fragments by
// permuting k inside the block (both operands use the same permutation, which leaves R B
// unchanged), and pass2's basis image permutes output columns so that the accumulator
// fragments land on those same 8 channels.
// Precision: the reference computes in fp32.  Every tensor-core operand here is carried as
// two bf16 terms (x = hi + lo to 2^-16 |x|) and each product as ah bh + ah bl + al bh in fp32
// accumulation (the dropped al bl is below 2^-16 of the product), so R B and rhs (B G^-1)^T
// are within ~2^-15 relative of their fp32 values; G = B^T B and its inverse are formed in
// fp64 from the fp32 basis.  The corrected values then differ from an fp32 evaluation by
// ~1e-5 of the fitted part, ~1e-6 of an int4 step here, and the requantised codes and fp16
// scale / zero agree with an fp32 evaluation except where a value lies that close to a
// rounding tie.  For the same reason pass2 quantises with the group's reciprocal alone
// (kivi::quant_word): it departs from the IEEE quotient only within 4e-6 of a tie, inside the
// window the upstream differences already leave, and an exact-quotient fix-up near ties cost
// 8 % of the route's time for no measurable change in its output.
#include <algorithm>
#include <cstring>
#include <vector>

#include "dkv_common.cuh"
#include "kivi_math.cuh"

namespace dkv {
namespace ksub {

constexpr int kWT = 32;  // tokens per warp tile (one K group)
constexpr int kWarps = 4;
constexpr int kThreads = 32 * kWarps;
constexpr int kTM = kWT * kWarps;  // tokens per CTA
constexpr int kCB = 32;            // channels per block
constexpr int kMaxRank = 64;
constexpr int kPsumCtas = 8;  // fewest probe-sum CTAs (of 8 warps) per problem

struct Prob {
  union {
    const uint8_t *codes;  // int4: the base codes
    const void *reused;    // dense: the reused rows (fresh dtype)
  };
  union {
    const __half *scale;  // int4: the base scales
    const float *tw;      // dense: the caller's token weights (or null)
  };
  const __half *zero;
  union {
    int64_t crs;  // int4: bytes per code row
    int64_t rrs;  // dense: elements per reused row
  };
  union {
    int64_t szrs;  // int4: elements per scale / zero row
    int64_t odt;   // dense: output dtype
  };
  union {
    uint8_t *o_codes;  // int4: the corrected codes
    void *out;         // dense: the corrected rows (output dtype odt)
  };
  __half *o_scale, *o_zero;
  union {
    int64_t o_crs;  // int4: bytes per output code row
    int64_t ors;    // dense: elements per output row
  };
  int64_t o_szrs;
  const void *fresh;
  int64_t frs;
  int64_t n;
  const int32_t *probes;
  int64_t n_probes;
  float *sub_out, *mu_out;
  // workspace
  float *rhs, *dist, *part, *sums, *ginv, *mu, *subv;
  uint32_t *flag;
  int32_t *uprobe, *ucount;
  __nv_bfloat16 *b1, *b1l, *b2;  // MMA B operands: high and low bf16 terms
  float *bb;                           // the basis as [d][RP] fp32 rows (zero past the rank)
  const float *basis;
  int64_t tile0;
  int r, mode;
};

constexpr int kMaxProblems = 112;

// The problem table travels in the kernel parameters (read through the constant cache).
struct Batch {
  int n_probs;
  int64_t d, n_tiles;
  int32_t *status;
  Prob probs[kMaxProblems];
};
static_assert(sizeof(Batch) <= 32000, "kernel parameter limit");

// sums (zeroed per call): [0, RP) sum_P rhs, [RP, RP + d) sum_P R
// part: [ceil(n/32) tiles][RP + 1]: per-tile column sums of rhs, then the tile's sum of ||R||
__device__ __forceinline__ int find_prob(const Batch &b, int64_t tile) {
  int lo = 0, hi = b.n_probs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.probs[mid].tile0 <= tile) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// 8 consecutive fresh values (16 B of bf16/f16, 32 B of f32)
template <int FDT>
__device__ __forceinline__ void load8(const void *base, int64_t off, float (&v)[8]) {
  if (FDT == DKV_F32) {
    const float4 *p = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + off);
    const float4 a = p[0], c = p[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = c.x, v[5] = c.y, v[6] = c.z, v[7] = c.w;
  } else {
    const uint4 a = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(base) + off);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = FDT == DKV_BF16 ? bf16lo(w[j]) : f16lo(w[j]);
      v[2 * j + 1] = FDT == DKV_BF16 ? bf16hi(w[j]) : f16hi(w[j]);
    }
  }
}

// 8 staged values (one 16-B chunk, or two for f32) -> floats
template <int FDT>
__device__ __forceinline__ void unpack8(const uint4 &u0, const uint4 &u1, float (&f)[8]) {
  if (FDT == DKV_F32) {
    f[0] = __uint_as_float(u0.x), f[1] = __uint_as_float(u0.y), f[2] = __uint_as_float(u0.z);
    f[3] = __uint_as_float(u0.w), f[4] = __uint_as_float(u1.x), f[5] = __uint_as_float(u1.y);
    f[6] = __uint_as_float(u1.z), f[7] = __uint_as_float(u1.w);
  } else {
    const uint32_t w4[4] = {u0.x, u0.y, u0.z, u0.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] = FDT == DKV_BF16 ? bf16lo(w4[j]) : f16lo(w4[j]);
      f[2 * j + 1] = FDT == DKV_BF16 ? bf16hi(w4[j]) : f16hi(w4[j]);
    }
  }
}

// 8 halves (16 B) -> floats
__device__ __forceinline__ void halves8(const __half *p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4 *>(p);
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = f16lo(w[j]);
    v[2 * j + 1] = f16hi(w[j]);
  }
}

// ---------------------------------------------------------------------------------------
__global__ void flags_kernel(const __grid_constant__ Batch b) {
  const Prob &P = b.probs[blockIdx.y];
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < P.n_probes;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = P.probes[i];
    if (t < 0 || t >= P.n) {
      record_error(b.status, DKV_ERR_INVALID_ARGUMENT);
      continue;
    }
    if (atomicExch(&P.flag[t], 1u) == 0u) P.uprobe[atomicAdd(P.ucount, 1)] = static_cast<int32_t>(t);
  }
}

// basis value B[c][k] (zero beyond the problem's rank)
__device__ __forceinline__ float basis_at(const Prob &P, int64_t c, int k) {
  return (k < P.r && P.basis != nullptr) ? P.basis[c * P.r + k] : 0.f;
}

// b1 / b1l (pass1 B operand, high / low bf16 terms): [block][n-tile][lane][8]:
//     B[32 block + 8q + j][8 nt + g]
// b2 (pass2 B operand, written by fitb): [block][k-step][n-tile][lane][high 4, low 4]:
//     (B G^-1)[ch][16 ks + 2q + {0, 1, 8, 9}], ch = 32 block + 8 (g >> 1) + 2 nt + (g & 1);
//     one block's fragments are contiguous (RP / 16 x 2 KB), the unit of pass2's bulk copies
// bb: [d][RP] fp32 rows
__global__ void pack_kernel(const __grid_constant__ Batch b, int rp) {
  const Prob &P = b.probs[blockIdx.y];
  const int64_t total = b.d * rp;
  const int nt_n = rp / 8;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    {
      const int64_t c = e / rp;
      const int k = static_cast<int>(e - c * rp);
      P.bb[e] = basis_at(P, c, k);
    }
    {
      const int j = static_cast<int>(e & 7);
      const int lane = static_cast<int>((e >> 3) & 31);
      const int64_t rest = e >> 8;
      const int nt = static_cast<int>(rest % nt_n);
      const int64_t blk = rest / nt_n;
      const int g = lane >> 2, q = lane & 3;
      const float x = basis_at(P, kCB * blk + 8 * q + j, 8 * nt + g);
      const __nv_bfloat16 hi = __float2bfloat16_rn(x);
      P.b1[e] = hi;
      P.b1l[e] = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hi)));
    }
  }
}

// ---------------------------------------------------------------------------------------
// pass 1
// ---------------------------------------------------------------------------------------
constexpr int kP1Stages = 3;  // per-warp staging depth (blocks in flight)
// the dense form stages two rows per token (fresh and reused): two blocks deep keeps the
// shared memory of five CTAs per SM
template <bool DENSE>
constexpr int p1_stages() {
  return DENSE ? 2 : kP1Stages;
}
constexpr int kBSlots = 4;    // CTA-wide ring of basis fragment blocks (both passes)

// Bounded wait on a phase without the abort word (draining copies already issued).
__device__ __forceinline__ void mbar_wait_drain(uint64_t *bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity) && clock64() - t0 < kWaitLimitCycles) {
  }
}

// r = hi + lo: hi = RN_bf16(r), lo = RN_bf16(r - hi) for a pair, as packed bf16 words
__device__ __forceinline__ void split2(uint64_t r2, uint32_t &hi, uint32_t &lo) {
  float x, y;
  f2unpack(r2, x, y);
  hi = pack_bf16x2(x, y);
  f2unpack(sub2(r2, f2pack(bf16lo(hi), bf16hi(hi))), x, y);
  lo = pack_bf16x2(x, y);
}

// one block's per-warp operands: fresh (16 or 32 B per lane and row, copied by that lane),
// the codes (row r's 16 B, copied by lane r) and, for K, the group's scale / zero (16 B per
// 8 channels, copied by lanes 0-7)
template <int FDT, bool DENSE>
struct P1Stage {
  static constexpr int kFB = FDT == DKV_F32 ? 2 : 1;
  uint4 fr[4][kFB][32];
  uint32_t cd[kWT][4];
  uint4 sz[2][4];
};
template <int FDT>
struct P1Stage<FDT, true> {  // dense caches: the reused rows staged like the fresh ones
  static constexpr int kFB = FDT == DKV_F32 ? 2 : 1;
  uint4 fr[4][kFB][32];
  uint4 rr[4][kFB][32];
};
// V: the rows' scale / zero, 4 blocks (8 B per row) per buffer, two buffers
struct P1VStage {
  uint2 s[2][kWT], z[2][kWT];
};

template <int RP>
constexpr int p1_bq_bytes() {  // one block's basis fragments: high terms, then low terms
  return (RP / 8) * 32 * 16 * 2;
}
template <int RP, int FDT, int MODE, bool DENSE = false>
constexpr int p1_smem_bytes() {
  return kBSlots * p1_bq_bytes<RP>() + kWarps * p1_stages<DENSE>() * static_cast<int>(sizeof(P1Stage<FDT, DENSE>)) +
         (MODE == DKV_KIVI_PER_TOKEN && !DENSE ? kWarps * static_cast<int>(sizeof(P1VStage)) : 0) +
         2 * kBSlots * 8 + 16;
}

// CTAs per SM that pass1 is compiled for (its register budget; measured per rank tile)
template <int RP, int MODE>
constexpr int p1_min_blocks() {
  return RP == 16 ? 5 : RP == 32 ? 4 : 3;
}

template <int RP, int FDT, int MODE, bool DENSE = false>
__global__ void __launch_bounds__(kThreads, p1_min_blocks<RP, MODE>())
    pass1_kernel(const __grid_constant__ Batch b, int64_t tile_lo) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const Prob &P = b.probs[find_prob(b, tile_lo + blockIdx.x)];
  const int64_t tile_t0 = (tile_lo + blockIdx.x - P.tile0) * kTM;
  const int64_t t0 = tile_t0 + warp * kWT;
  const int64_t n = P.n;
  constexpr int NT = RP / 8;
  constexpr bool kmode = MODE == DKV_KIVI_PER_CHANNEL;
  constexpr int BQ = p1_bq_bytes<RP>();
  const int n_blocks = static_cast<int>(b.d / kCB);
  // shared: [fragment ring][per-warp stage rings][V rows][barriers, abort]
  using Stage = P1Stage<FDT, DENSE>;
  extern __shared__ __align__(16) unsigned char p1_smem[];
  unsigned char *const bq_ring = p1_smem;
  unsigned char *sp = p1_smem + kBSlots * BQ;
  constexpr int S1 = p1_stages<DENSE>();
  Stage *const ring = reinterpret_cast<Stage *>(sp) + warp * S1;
  sp += kWarps * S1 * sizeof(Stage);
  P1VStage *const vst = reinterpret_cast<P1VStage *>(sp) + warp;
  if constexpr (!kmode && !DENSE) sp += kWarps * sizeof(P1VStage);
  uint64_t *const bq_full = reinterpret_cast<uint64_t *>(sp);
  uint64_t *const bq_empty = bq_full + kBSlots;
  volatile int *const abort_flag = reinterpret_cast<volatile int *>(bq_empty + kBSlots);

  // the warps with tokens (every tile has at least one token, so warp 0 is one of them)
  const int active = static_cast<int>((n - tile_t0 + kWT - 1) / kWT < kWarps ? (n - tile_t0 + kWT - 1) / kWT : kWarps);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBSlots; ++s) {
      mbar_init(&bq_full[s], 1);
      mbar_init(&bq_empty[s], active);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (t0 >= n) return;

  // basis fragments: two bulk copies per block (high, low terms) by lane 0 of warp 0 into the
  // CTA-wide ring; every warp with tokens releases a slot after reading it
  const bool producer = warp == 0 && lane == 0;
  int bq_issued = 0;
  auto bq_issue = [&]() -> bool {
    const int blk = bq_issued, s = blk % kBSlots;
    if (blk >= kBSlots && !mbar_wait_bounded(&bq_empty[s], ((blk / kBSlots) - 1) & 1, abort_flag)) return false;
    mbar_arrive_expect_tx(&bq_full[s], BQ);
    const int64_t off = static_cast<int64_t>(blk) * (BQ / 2);
    bulk_load(bq_ring + s * BQ, reinterpret_cast<const unsigned char *>(P.b1) + off, BQ / 2, &bq_full[s]);
    bulk_load(bq_ring + s * BQ + BQ / 2, reinterpret_cast<const unsigned char *>(P.b1l) + off, BQ / 2, &bq_full[s]);
    ++bq_issued;
    return true;
  };
  bool ok = true;
  if (producer)
    while (bq_issued < kBSlots - 1 && bq_issued < n_blocks) bq_issue();

  float acc[2][NT][4];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int i = 0; i < NT; ++i) acc[m][i][0] = acc[m][i][1] = acc[m][i][2] = acc[m][i][3] = 0.f;
  float d2[4] = {0.f, 0.f, 0.f, 0.f};
  int64_t row[4];
  bool rv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    row[i] = t0 + g + 8 * i;
    rv[i] = row[i] < n;
  }
  const int64_t krow = t0 / kivi::kG;
  const int64_t my_row = t0 + lane;
  const bool my_valid = my_row < n;
  const uint8_t *const my_codes = DENSE ? nullptr : P.codes + (my_valid ? my_row : t0) * P.crs;
  // V: the rows' scale / zero staged 4 blocks at a time where the rows allow 8-B copies,
  // otherwise read directly
  const bool vstage = !DENSE && !kmode && n_blocks % 4 == 0 && P.szrs % 4 == 0;
  constexpr int kFB = Stage::kFB;
  constexpr int kEs = FDT == DKV_F32 ? 4 : 2;
  // per-warp staging ring (cp.async, S1 - 1 blocks ahead)
  auto issue = [&](int cb) {
    if (cb < n_blocks) {
      Stage &S = ring[cb % S1];
      const int64_t c = static_cast<int64_t>(cb) * kCB + 8 * q;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t rr = rv[i] ? row[i] : t0;
        const unsigned char *fp = static_cast<const unsigned char *>(P.fresh) + (rr * P.frs + c) * kEs;
#pragma unroll
        for (int f = 0; f < kFB; ++f) cp_async16(&S.fr[i][f][lane], fp + 16 * f, rv[i] ? 16u : 0u);
        if constexpr (DENSE) {
          const unsigned char *rp = static_cast<const unsigned char *>(P.reused) + (rr * P.rrs + c) * kEs;
#pragma unroll
          for (int f = 0; f < kFB; ++f) cp_async16(&S.rr[i][f][lane], rp + 16 * f, rv[i] ? 16u : 0u);
        }
      }
      if constexpr (!DENSE) {
        cp_async16(&S.cd[lane][0], my_codes + static_cast<int64_t>(cb) * (kCB / 2), my_valid ? 16u : 0u);
        if constexpr (kmode) {
          if (lane < 8)
            cp_async16(&S.sz[lane >> 2][lane & 3],
                       (lane < 4 ? P.scale : P.zero) + krow * P.szrs + static_cast<int64_t>(cb) * kCB +
                           8 * (lane & 3),
                       16u);
        } else {
          if (vstage && cb % 4 == 0) {
            const int buf = (cb >> 2) & 1;
            const int64_t off = (my_valid ? my_row : t0) * P.szrs + cb;
            cp_async8(&vst->s[buf][lane], P.scale + off, my_valid ? 8u : 0u);
            cp_async8(&vst->z[buf][lane], P.zero + off, my_valid ? 8u : 0u);
          }
        }
      }
    }
    cp_async_commit();  // possibly empty: keeps the group count per block fixed
  };
#pragma unroll
  for (int s0 = 0; s0 < S1 - 1; ++s0) issue(s0);

  const uint64_t rs_lo = kivi::pair_rescale(0), rs_hi = kivi::pair_rescale(1);
  int cb = 0;
  for (; cb < n_blocks; ++cb) {
    __syncwarp();  // every lane is done with the slot the next copy overwrites
    if (warp == 0) {  // the producer's outcome, for the whole warp (exits stay warp-uniform)
      int pok = 1;
      if (producer && bq_issued < n_blocks) pok = bq_issue() ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, pok, 0)) {
        ok = false;
        break;
      }
    }
    issue(cb + S1 - 1);
    cp_async_wait<S1 - 1>();
    __syncwarp();  // the other lanes' copies of this block are visible
    const Stage &S = ring[cb % S1];
    uint64_t ks2[4], kz2[4];  // K: this lane's channels' rescaled scale and zero, in pairs
    if constexpr (kmode && !DENSE) {
      const uint4 sv = S.sz[0][q], zv = S.sz[1][q];
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        ks2[p] = mul2(f2pack(f16lo(sw[p]), f16hi(sw[p])), (p & 1) ? rs_hi : rs_lo);
        kz2[p] = f2pack(f16lo(zw[p]), f16hi(zw[p]));
      }
    }
    uint32_t a[2][2][4], al[2][2][4];  // [m-tile][k-step][reg]: R's high and low bf16 terms
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint64_t r2[4] = {0, 0, 0, 0};
      if (rv[i]) {
        float f[8];
        unpack8<FDT>(S.fr[i][0][lane], S.fr[i][kFB - 1][lane], f);
        if constexpr (DENSE) {
          float x[8];
          unpack8<FDT>(S.rr[i][0][lane], S.rr[i][kFB - 1][lane], x);
          uint64_t dd2 = 0;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            r2[p] = sub2(f2pack(f[2 * p], f[2 * p + 1]), f2pack(x[2 * p], x[2 * p + 1]));
            dd2 = fma2(r2[p], r2[p], dd2);
          }
          float e0, e1;
          f2unpack(dd2, e0, e1);
          d2[i] += e0 + e1;
        } else {
          uint64_t raw[4];
          kivi::code_pairs(S.cd[g + 8 * i][q], raw);
          uint64_t vs_lo = 0, vs_hi = 0, vz2 = 0;
          if constexpr (!kmode) {
            float vs, vz;
            if (vstage) {
              const int buf = (cb >> 2) & 1;
              vs = __half2float(reinterpret_cast<const __half *>(&vst->s[buf][g + 8 * i])[cb & 3]);
              vz = __half2float(reinterpret_cast<const __half *>(&vst->z[buf][g + 8 * i])[cb & 3]);
            } else {
              vs = __half2float(P.scale[row[i] * P.szrs + cb]);
              vz = __half2float(P.zero[row[i] * P.szrs + cb]);
            }
            vs_lo = mul2(f2pack(vs, vs), rs_lo);
            vs_hi = mul2(f2pack(vs, vs), rs_hi);
            vz2 = f2pack(vz, vz);
          }
          uint64_t dd2 = 0;
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const uint64_t reused2 =
                fma2(raw[p], kmode ? ks2[p] : ((p & 1) ? vs_hi : vs_lo), kmode ? kz2[p] : vz2);
            r2[p] = sub2(f2pack(f[2 * p], f[2 * p + 1]), reused2);
            dd2 = fma2(r2[p], r2[p], dd2);
          }
          float e0, e1;
          f2unpack(dd2, e0, e1);
          d2[i] += e0 + e1;
        }
      }
      const int m = i >> 1, h = i & 1;
      split2(r2[0], a[m][0][h], al[m][0][h]);
      split2(r2[1], a[m][0][2 + h], al[m][0][2 + h]);
      split2(r2[2], a[m][1][h], al[m][1][h]);
      split2(r2[3], a[m][1][2 + h], al[m][1][2 + h]);
    }
    const int slot = cb % kBSlots;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bq_full[slot], (cb / kBSlots) & 1, abort_flag))) {
      ok = false;
      break;
    }
    const uint4 *const bq = reinterpret_cast<const uint4 *>(bq_ring + slot * BQ) + lane;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const uint4 bv = bq[nt * 32], bl = bq[(NT + nt) * 32];
#pragma unroll
      for (int m = 0; m < 2; ++m) {  // R B ~ Rh Bh + Rh Bl + Rl Bh, small terms first
        mma16816_bf16(acc[m][nt], al[m][0][0], al[m][0][1], al[m][0][2], al[m][0][3], bv.x, bv.y);
        mma16816_bf16(acc[m][nt], al[m][1][0], al[m][1][1], al[m][1][2], al[m][1][3], bv.z, bv.w);
        mma16816_bf16(acc[m][nt], a[m][0][0], a[m][0][1], a[m][0][2], a[m][0][3], bl.x, bl.y);
        mma16816_bf16(acc[m][nt], a[m][1][0], a[m][1][1], a[m][1][2], a[m][1][3], bl.z, bl.w);
        mma16816_bf16(acc[m][nt], a[m][0][0], a[m][0][1], a[m][0][2], a[m][0][3], bv.x, bv.y);
        mma16816_bf16(acc[m][nt], a[m][1][0], a[m][1][1], a[m][1][2], a[m][1][3], bv.z, bv.w);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bq_empty[slot]);
  }
  cp_async_wait<0>();
  if (!ok) {
    record_error(b.status, DKV_ERR_TIMEOUT);
    *abort_flag = 1;
  }
  // copies this CTA issued and warp 0 has not waited for complete before the CTA exits
  if (producer)
    for (int blk = cb; blk < bq_issued; ++blk) mbar_wait_drain(&bq_full[blk % kBSlots], (blk / kBSlots) & 1);
  if (!ok) return;

  // ||R|| per row (4 lanes per row) and the tile's sum
  float dsum = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v = d2[i];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    const float dd = sqrtf(v);
    if (q == 0 && rv[i]) P.dist[row[i]] = dd;
    if (rv[i]) dsum += dd;
  }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
  float *part = P.part + (t0 / kWT) * (RP + 1);
  if (lane == 0) part[RP] = dsum;
  // rhs rows and the tile's column sums
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float s0 = 0.f, s1 = 0.f;
    const int col = 8 * nt + 2 * q;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (rv[2 * m]) {
        *reinterpret_cast<float2 *>(P.rhs + row[2 * m] * RP + col) = make_float2(acc[m][nt][0], acc[m][nt][1]);
        s0 += acc[m][nt][0];
        s1 += acc[m][nt][1];
      }
      if (rv[2 * m + 1]) {
        *reinterpret_cast<float2 *>(P.rhs + row[2 * m + 1] * RP + col) = make_float2(acc[m][nt][2], acc[m][nt][3]);
        s0 += acc[m][nt][2];
        s1 += acc[m][nt][3];
      }
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (g == 0) {
      part[col] = s0;
      part[col + 1] = s1;
    }
  }
}

// ---------------------------------------------------------------------------------------
// psum: sums over the (deduplicated) probes of R and of rhs.  `ctas` CTAs of 8 warps per
// problem; warp w takes probes w, w + 8 ctas, ...; a probe row is read 256 channels at a
// time with 16-byte loads (8 channels per lane), the CTA's warps are summed in shared memory
// and one atomic per channel and CTA goes to the problem's sums.
// ---------------------------------------------------------------------------------------
template <int RP, int FDT, bool DENSE = false>
__global__ void __launch_bounds__(256) psum_kernel(const __grid_constant__ Batch b, int ctas) {
  __shared__ float red[8][256];
  const Prob &P = b.probs[blockIdx.y];
  const int cnt = *P.ucount;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wstep = 8 * ctas;
  const int w0 = blockIdx.x * 8 + warp;
  const bool kmode = P.mode == DKV_KIVI_PER_CHANNEL;
  for (int64_t c0 = 0; c0 < b.d; c0 += 256) {
    const int64_t c = c0 + 8 * lane;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (c < b.d) {
      for (int i = w0; i < cnt; i += wstep) {
        const int64_t t = P.uprobe[i];
        float f[8];
        load8<FDT>(P.fresh, t * P.frs + c, f);
        if constexpr (DENSE) {
          float x[8];
          load8<FDT>(P.reused, t * P.rrs + c, x);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += f[j] - x[j];
        } else {
          float sc[8], zr[8];
          const uint32_t w = *reinterpret_cast<const uint32_t *>(P.codes + t * P.crs + c / 2);
          if (kmode) {
            halves8(P.scale + (t / kivi::kG) * P.szrs + c, sc);
            halves8(P.zero + (t / kivi::kG) * P.szrs + c, zr);
          } else {
            const float vs = __half2float(P.scale[t * P.szrs + c / kivi::kG]);
            const float vz = __half2float(P.zero[t * P.szrs + c / kivi::kG]);
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[j] = vs, zr[j] = vz;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += f[j] - kivi::deq((w >> (4 * j)) & 0xFu, sc[j], zr[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) red[warp][8 * lane + j] = acc[j];
    __syncthreads();
    {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += red[w][threadIdx.x];
      if (c0 + threadIdx.x < b.d) atomicAdd(&P.sums[RP + c0 + threadIdx.x], sum);
    }
    __syncthreads();
  }
  // rhs rows: lanes 0 .. RP/4 - 1 take 4 codes each
  float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane < RP / 4)
    for (int i = w0; i < cnt; i += wstep) {
      const float4 x = reinterpret_cast<const float4 *>(P.rhs + static_cast<int64_t>(P.uprobe[i]) * RP)[lane];
      acc4.x += x.x, acc4.y += x.y, acc4.z += x.z, acc4.w += x.w;
    }
  if (lane < RP / 4) {
    red[warp][4 * lane] = acc4.x, red[warp][4 * lane + 1] = acc4.y;
    red[warp][4 * lane + 2] = acc4.z, red[warp][4 * lane + 3] = acc4.w;
  }
  __syncthreads();
  if (threadIdx.x < RP) {
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) sum += red[w][threadIdx.x];
    atomicAdd(&P.sums[threadIdx.x], sum);
  }
}

// ---------------------------------------------------------------------------------------
// solve: one CTA per problem
// ---------------------------------------------------------------------------------------
template <int RP>
__global__ void __launch_bounds__(256) solve_kernel(const __grid_constant__ Batch b) {
  extern __shared__ double Mdyn[];  // [r][2r + 1]: [G | I]
  __shared__ float cp[RP], ca[RP], colsum[RP + 1];
  __shared__ float wsum[8][RP + 1];
  __shared__ double fac[RP];
  __shared__ double piv_val;
  __shared__ int piv_row;
  const Prob &P = b.probs[blockIdx.x];
  const int r = P.r;
  const int ldm = 2 * r + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float np = static_cast<float>(*P.ucount);
  const int64_t tiles = (P.n + kWT - 1) / kWT;
  for (int e = threadIdx.x; e < RP * RP; e += blockDim.x) P.ginv[e] = 0.f;
  if (threadIdx.x < RP) cp[threadIdx.x] = ca[threadIdx.x] = 0.f;
  // column sums of rhs and the sum of ||R|| from the per-tile partials: warp w takes tiles
  // w, w + 8, ..., lanes the columns
  {
    float acc[3] = {0.f, 0.f, 0.f};
    for (int64_t t = warp; t < tiles; t += 8) {
      const float *row = P.part + t * (RP + 1);
#pragma unroll
      for (int u = 0; u < 3; ++u)
        if (lane + 32 * u <= RP) acc[u] += row[lane + 32 * u];
    }
#pragma unroll
    for (int u = 0; u < 3; ++u)
      if (lane + 32 * u <= RP) wsum[warp][lane + 32 * u] = acc[u];
    __syncthreads();
    for (int k = threadIdx.x; k <= RP; k += blockDim.x) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) sum += wsum[w][k];
      colsum[k] = sum;
    }
  }
  __syncthreads();
  if (r > 0) {
    // G = B^T B + 1e-6 I: 64-channel tiles of B staged in shared memory as fp64 (exact:
    // fp32 values), fp64 accumulation; the tile area is the not yet used part of Mdyn past
    // [G | I].  Thread (bi, bj) of a 16 x 16 grid owns the BS x BS block of G at rows BS bi,
    // columns BS bj (BS = RP / 16), so each staged value it reads feeds BS products.
    double *tile = Mdyn + r * ldm;  // [64][RP]
    constexpr int BS = RP / 16;
    const int bi = threadIdx.x >> 4, bj = threadIdx.x & 15;
    double accg[BS][BS];
#pragma unroll
    for (int u = 0; u < BS; ++u)
#pragma unroll
      for (int v = 0; v < BS; ++v) accg[u][v] = 0.0;
    for (int64_t c0 = 0; c0 < b.d; c0 += 64) {
      for (int e = threadIdx.x; e < 64 * RP; e += blockDim.x) {
        const int64_t c = c0 + e / RP;
        tile[e] = c < b.d ? static_cast<double>(P.bb[c * RP + e % RP]) : 0.0;
      }
      __syncthreads();
      for (int cc = 0; cc < 64; ++cc) {
        const double *tr = tile + cc * RP;
        double xi[BS], xj[BS];
#pragma unroll
        for (int u = 0; u < BS; ++u) {
          xi[u] = tr[BS * bi + u];
          xj[u] = tr[BS * bj + u];
        }
#pragma unroll
        for (int u = 0; u < BS; ++u)
#pragma unroll
          for (int v = 0; v < BS; ++v) accg[u][v] = fma(xi[u], xj[v], accg[u][v]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < BS; ++u)
#pragma unroll
      for (int v = 0; v < BS; ++v) {
        const int i = BS * bi + u, j = BS * bj + v;
        if (i < r && j < r) {
          Mdyn[i * ldm + j] = accg[u][v] + (i == j ? 1e-6 : 0.0);
          Mdyn[i * ldm + r + j] = (i == j) ? 1.0 : 0.0;
        }
      }
    __syncthreads();
    // Gauss-Jordan with partial pivoting on [G | I]; three barriers per column
    const int jj = threadIdx.x & 127, i0 = threadIdx.x >> 7;
    for (int col = 0; col < r; ++col) {
      if (warp == 0) {
        // pivot: the first row of largest |G[i][col]|, i >= col (warp arg-max)
        double bv = -1.0;
        int bi = r;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = col + lane + 32 * u;
          if (i < r) {
            const double v = fabs(Mdyn[i * ldm + col]);
            if (v > bv) {
              bv = v;
              bi = i;
            }
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
          }
        }
        const int pr = bi < r ? bi : col;
        // column multipliers after the row swap
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = lane + 32 * u;
          if (i < r) fac[i] = Mdyn[(i == pr ? col : (i == col ? pr : i)) * ldm + col];
        }
        if (lane == 0) {
          piv_row = pr;
          piv_val = Mdyn[pr * ldm + col];
        }
      }
      __syncthreads();
      const int pr = piv_row;
      const double inv = 1.0 / piv_val;
      if (i0 == 0 && jj < 2 * r) {
        const double top = Mdyn[col * ldm + jj], prow = Mdyn[pr * ldm + jj];
        Mdyn[col * ldm + jj] = prow * inv;
        if (pr != col) Mdyn[pr * ldm + jj] = top;
      }
      __syncthreads();
      if (jj < 2 * r && jj >= col) {
        const double pv = Mdyn[col * ldm + jj];
        for (int i = i0; i < r; i += 2)
          if (i != col) Mdyn[i * ldm + jj] -= fac[i] * pv;
      }
      __syncthreads();
    }
    for (int e = threadIdx.x; e < r * r; e += blockDim.x)
      P.ginv[(e / r) * RP + e % r] = static_cast<float>(Mdyn[(e / r) * ldm + r + e % r]);
    if (threadIdx.x < r) {
      const int j = threadIdx.x;
      double sp = 0.0, sa = 0.0;
      for (int i = 0; i < r; ++i) {
        sp += static_cast<double>(P.sums[i]) * Mdyn[i * ldm + r + j];
        sa += static_cast<double>(colsum[i]) * Mdyn[i * ldm + r + j];
      }
      cp[j] = np > 0 ? static_cast<float>(sp / np) : 0.f;
      ca[j] = P.n > 0 ? static_cast<float>(sa / static_cast<double>(P.n)) : 0.f;
    }
    __syncthreads();
  }
  for (int64_t c = threadIdx.x; c < b.d; c += blockDim.x) {
    float fp = 0.f, fa = 0.f;
    for (int i = 0; i < r; ++i) {
      const float bv = P.bb[c * RP + i];
      fp = fmaf(cp[i], bv, fp);
      fa = fmaf(ca[i], bv, fa);
    }
    const float meanR = np > 0 ? P.sums[RP + c] / np : 0.f;
    P.mu[c] = meanR - fp;
    P.subv[c] = fa;
    if (P.mu_out) P.mu_out[c] = meanR - fp;
    if (P.sub_out) P.sub_out[c] = fa;
  }
  if (threadIdx.x == 0) P.subv[b.d] = fmaxf(P.n > 0 ? colsum[RP] / static_cast<float>(P.n) : 0.f, 1e-8f);
}

// ---------------------------------------------------------------------------------------
// fitb: pass2's B operand, B G^-1 as high / low bf16 terms in the b2 fragment order (per
// fragment 16 B: the 4 high terms, then the 4 low terms); one CTA per 32-channel block
// ---------------------------------------------------------------------------------------
template <int RP>
__global__ void __launch_bounds__(256) fitb_kernel(const __grid_constant__ Batch b) {
  __shared__ float Gf[RP][RP + 1];
  __shared__ float Bs[kCB][RP + 1];
  const Prob &P = b.probs[blockIdx.y];
  const int64_t blk = blockIdx.x;
  for (int e = threadIdx.x; e < RP * RP; e += blockDim.x) Gf[e / RP][e % RP] = P.ginv[e];  // zero past r
  for (int e = threadIdx.x; e < kCB * RP; e += blockDim.x)
    Bs[e / RP][e % RP] = P.bb[(blk * kCB + e / RP) * RP + e % RP];
  __syncthreads();
  constexpr int KS = RP / 16;
  for (int f = threadIdx.x; f < KS * 512; f += blockDim.x) {
    const int x = f & 3, lane = (f >> 2) & 31, nt = (f >> 7) & 3, ks = f >> 9;
    const int g = lane >> 2, q = lane & 3;
    const int cl = 8 * (g >> 1) + 2 * nt + (g & 1);
    const int k = 16 * ks + 2 * q + (x & 1) + 8 * (x >> 1);
    float acc = 0.f;
#pragma unroll 8
    for (int j = 0; j < RP; ++j) acc = fmaf(Gf[k][j], Bs[cl][j], acc);
    const __nv_bfloat16 hi = __float2bfloat16_rn(acc);
    __nv_bfloat16 *o = P.b2 + blk * (KS * 1024) + (f >> 2) * 8 + x;
    o[0] = hi;
    o[4] = __float2bfloat16_rn(__fsub_rn(acc, __bfloat162float(hi)));
  }
}

// ---------------------------------------------------------------------------------------
// pass 2
// ---------------------------------------------------------------------------------------
constexpr int kP2Stages = 3;  // per-warp staging depth of codes and K scale / zero (blocks)

// one block's per-warp operands: the codes (row r's 16 B, copied by lane r) and, for K, the
// group's scale / zero (16 B per 8 channels, copied by lanes 0-7) and the fresh values of the
// lane's first two probe rows (16 or 32 B each)
template <int FDT, bool K>
struct P2Stage {
  static constexpr int kFB = FDT == DKV_F32 ? 2 : 1;
  uint32_t cd[kWT][4];
  uint4 sz[2][4];
  uint4 pf[2][kFB][32];
};
template <int FDT>
struct P2Stage<FDT, false> {  // V: probe rows are not read here
  static constexpr int kFB = FDT == DKV_F32 ? 2 : 1;
  uint32_t cd[kWT][4];
  uint4 sz[2][4];
};
// per-warp scratch: group extrema partials, then the groups' (zero, 1 / scale)
constexpr int kRedK = 136;  // K: floats per q-row, [g][j] (lo, hi) pairs + 8 floats of pad
constexpr int kRedV = 40;   // V: floats per g-row, [q][i] (lo, hi) pairs + 8 floats of pad
struct P2Scratch {
  float red[4 * kRedK];
  float pz[32], pinv[32];
};
// V: the rows' scale / zero, 8 blocks (16 B per row) per buffer, two buffers
struct P2VStage {
  uint4 s[2][kWT], z[2][kWT];
};

template <int RP>
constexpr int p2_bq_bytes() {  // one block's (B G^-1) fragments, high and low terms
  return (RP / 16) * 4 * 32 * 16;
}
// shared memory besides orth_mu [d]: fragment ring, per-warp rings and scratch, V rows,
// barriers and the abort word
template <int RP, int FDT, int MODE>
constexpr int p2_smem_fixed() {
  return kBSlots * p2_bq_bytes<RP>() +
         kWarps * (kP2Stages * static_cast<int>(sizeof(P2Stage<FDT, MODE == DKV_KIVI_PER_CHANNEL>)) +
                   static_cast<int>(sizeof(P2Scratch))) +
         (MODE == DKV_KIVI_PER_TOKEN ? kWarps * static_cast<int>(sizeof(P2VStage)) : 0) + 2 * kBSlots * 8 + 16;
}

// CTAs per SM that pass2 is compiled for (its register budget; measured per rank tile)
template <int RP, int MODE>
constexpr int p2_min_blocks() {
  return RP == 16 ? 5 : RP == 32 ? 4 : 3;
}

template <int RP, int FDT, int MODE>
__global__ void __launch_bounds__(kThreads, p2_min_blocks<RP, MODE>())
    pass2_kernel(const __grid_constant__ Batch b, int64_t tile_lo) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const Prob &P = b.probs[find_prob(b, tile_lo + blockIdx.x)];
  const int64_t tile_t0 = (tile_lo + blockIdx.x - P.tile0) * kTM;
  const int64_t t0 = tile_t0 + warp * kWT;
  const int64_t n = P.n;
  constexpr int KS = RP / 16;
  constexpr bool kmode = MODE == DKV_KIVI_PER_CHANNEL;
  constexpr int BQ = p2_bq_bytes<RP>();
  const int n_blocks = static_cast<int>(b.d / kCB);
  // shared: [fragment ring][per-warp stage rings][per-warp scratch][V rows][barriers, abort][orth_mu]
  extern __shared__ __align__(16) unsigned char p2_smem[];
  unsigned char *const bq_ring = p2_smem;
  unsigned char *sp = p2_smem + kBSlots * BQ;
  using Stage = P2Stage<FDT, kmode>;
  constexpr int kFB = Stage::kFB;
  constexpr int kEs = FDT == DKV_F32 ? 4 : 2;
  Stage *const ring = reinterpret_cast<Stage *>(sp) + warp * kP2Stages;
  sp += kWarps * kP2Stages * sizeof(Stage);
  P2Scratch &X = reinterpret_cast<P2Scratch *>(sp)[warp];
  sp += kWarps * sizeof(P2Scratch);
  P2VStage *const vst = reinterpret_cast<P2VStage *>(sp) + warp;
  if constexpr (!kmode) sp += kWarps * sizeof(P2VStage);
  uint64_t *const bq_full = reinterpret_cast<uint64_t *>(sp);
  uint64_t *const bq_empty = bq_full + kBSlots;
  volatile int *const abort_flag = reinterpret_cast<volatile int *>(bq_empty + kBSlots);
  float *const mu_s = reinterpret_cast<float *>(sp + 2 * kBSlots * 8 + 16);

  // the warps with tokens (every tile has at least one token, so warp 0 is one of them)
  const int active = static_cast<int>((n - tile_t0 + kWT - 1) / kWT < kWarps ? (n - tile_t0 + kWT - 1) / kWT : kWarps);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBSlots; ++s) {
      mbar_init(&bq_full[s], 1);
      mbar_init(&bq_empty[s], active);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int64_t e = threadIdx.x; e < b.d / 4; e += kThreads)
    reinterpret_cast<float4 *>(mu_s)[e] = reinterpret_cast<const float4 *>(P.mu)[e];
  __syncthreads();
  if (t0 >= n) return;

  // (B G^-1) fragments: one bulk copy per block by lane 0 of warp 0 into the CTA-wide ring;
  // every warp with tokens releases a slot after reading it
  const bool producer = warp == 0 && lane == 0;
  const unsigned char *const bq_src = reinterpret_cast<const unsigned char *>(P.b2);
  int bq_issued = 0;
  auto bq_issue = [&]() -> bool {
    const int blk = bq_issued, s = blk % kBSlots;
    if (blk >= kBSlots && !mbar_wait_bounded(&bq_empty[s], ((blk / kBSlots) - 1) & 1, abort_flag)) return false;
    mbar_arrive_expect_tx(&bq_full[s], BQ);
    bulk_load(bq_ring + s * BQ, bq_src + static_cast<int64_t>(blk) * BQ, BQ, &bq_full[s]);
    ++bq_issued;
    return true;
  };
  bool ok = true;
  if (producer)
    while (bq_issued < kBSlots - 1 && bq_issued < n_blocks) bq_issue();

  const float mean_dist = P.subv[b.d];
  int64_t row[4];
  bool rv[4], fl[4];
  float w[4];
  int pslot[4];  // K: the row's slot among the lane's prefetched probe rows (-1: read directly)
  int n_pf = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    row[i] = t0 + g + 8 * i;
    rv[i] = row[i] < n;
    fl[i] = rv[i] && P.flag[row[i]] != 0u;
    w[i] = rv[i] ? fminf(P.dist[row[i]] / mean_dist, 1.f) : 0.f;
    pslot[i] = -1;
    if (kmode && fl[i] && n_pf < 2) pslot[i] = n_pf++;
  }
  // V: a probe row's groups are the fresh row's alone; vprobe_kernel writes them, and here
  // the row is skipped (the owner lane of row g + 8q checks its own flag)
  const bool own_probe = !kmode && t0 + g + 8 * q < n && P.flag[t0 + g + 8 * q] != 0u;
  const bool full = t0 + kWT <= n;
  // A fragments: the row's rhs at this lane's positions k = 16 ks + 2q + {0, 1, 8, 9}, as
  // high and low bf16 terms
  uint32_t a[2][KS][4], al[2][KS][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = i >> 1, h = i & 1;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
      if (rv[i]) {
        const float *rr = P.rhs + row[i] * RP + 16 * ks + 2 * q;
        lo = *reinterpret_cast<const float2 *>(rr);
        hi = *reinterpret_cast<const float2 *>(rr + 8);
      }
      split_bf16x2(lo.x, lo.y, a[m][ks][h], al[m][ks][h]);
      split_bf16x2(hi.x, hi.y, a[m][ks][2 + h], al[m][ks][2 + h]);
    }
  }

  const int64_t krow = t0 / kivi::kG;
  const int64_t my_row = t0 + lane;
  const bool my_valid = my_row < n;
  const uint8_t *const my_codes = P.codes + (my_valid ? my_row : t0) * P.crs;
  // V: the rows' scale / zero staged 8 blocks at a time where the rows allow 16-B copies,
  // otherwise read directly
  const bool vstage = !kmode && n_blocks % 8 == 0 && P.szrs % 8 == 0;
  // per-warp staging ring (cp.async, kP2Stages - 1 blocks ahead)
  auto issue = [&](int cb) {
    if (cb < n_blocks) {
      Stage &S = ring[cb % kP2Stages];
      cp_async16(&S.cd[lane][0], my_codes + static_cast<int64_t>(cb) * (kCB / 2), my_valid ? 16u : 0u);
      if constexpr (kmode) {
        if (lane < 8)
          cp_async16(&S.sz[lane >> 2][lane & 3],
                     (lane < 4 ? P.scale : P.zero) + krow * P.szrs + static_cast<int64_t>(cb) * kCB + 8 * (lane & 3),
                     16u);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (pslot[i] >= 0) {
            const unsigned char *fp = static_cast<const unsigned char *>(P.fresh) +
                                      (row[i] * P.frs + static_cast<int64_t>(cb) * kCB + 8 * q) * kEs;
#pragma unroll
            for (int f = 0; f < kFB; ++f) cp_async16(&S.pf[pslot[i]][f][lane], fp + 16 * f, 16u);
          }
      } else {
        if (vstage && cb % 8 == 0) {
          const int buf = (cb >> 3) & 1;
          const int64_t off = (my_valid ? my_row : t0) * P.szrs + cb;
          cp_async16(&vst->s[buf][lane], P.scale + off, my_valid ? 16u : 0u);
          cp_async16(&vst->z[buf][lane], P.zero + off, my_valid ? 16u : 0u);
        }
      }
    }
    cp_async_commit();  // possibly empty: keeps the group count per block fixed
  };
#pragma unroll
  for (int s0 = 0; s0 < kP2Stages - 1; ++s0) issue(s0);

  const uint64_t rs_lo = kivi::pair_rescale(0), rs_hi = kivi::pair_rescale(1);
  int cb = 0;
  for (; cb < n_blocks; ++cb) {
    __syncwarp();  // every lane is done with the slot the next copy overwrites
    if (warp == 0) {  // the producer's outcome, for the whole warp (exits stay warp-uniform)
      int pok = 1;
      if (producer && bq_issued < n_blocks) pok = bq_issue() ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, pok, 0)) {
        ok = false;
        break;
      }
    }
    issue(cb + kP2Stages - 1);
    cp_async_wait<kP2Stages - 1>();
    __syncwarp();  // the other lanes' copies of this block are visible
    const int slot = cb % kBSlots;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bq_full[slot], (cb / kBSlots) & 1, abort_flag))) {
      ok = false;
      break;
    }
    const Stage &S = ring[cb % kP2Stages];
    const uint4 *const bq = reinterpret_cast<const uint4 *>(bq_ring + slot * BQ) + lane;
    const int64_t c = static_cast<int64_t>(cb) * kCB + 8 * q;
    float acc[2][4][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const uint4 f = bq[(ks * 4 + nt) * 32];  // high terms (x, y), low terms (z, w)
#pragma unroll
        for (int m = 0; m < 2; ++m) {  // rhs (B G^-1)^T ~ ah bh + ah bl + al bh, small terms first
          if (ks == 0)
            mma16816_bf16_zc(acc[m][nt], al[m][ks][0], al[m][ks][1], al[m][ks][2], al[m][ks][3], f.x, f.y);
          else
            mma16816_bf16(acc[m][nt], al[m][ks][0], al[m][ks][1], al[m][ks][2], al[m][ks][3], f.x, f.y);
          mma16816_bf16(acc[m][nt], a[m][ks][0], a[m][ks][1], a[m][ks][2], a[m][ks][3], f.z, f.w);
          mma16816_bf16(acc[m][nt], a[m][ks][0], a[m][ks][1], a[m][ks][2], a[m][ks][3], f.x, f.y);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bq_empty[slot]);

    uint64_t mu2[4];
    {
      const float4 *mp = reinterpret_cast<const float4 *>(mu_s + c);
      const float4 x = mp[0], y = mp[1];
      mu2[0] = f2pack(x.x, x.y), mu2[1] = f2pack(x.z, x.w), mu2[2] = f2pack(y.x, y.y), mu2[3] = f2pack(y.z, y.w);
    }
    uint64_t ks2[4], kz2[4];  // K: this lane's channels' rescaled scale and zero, in pairs
    if constexpr (kmode) {
      const uint4 sv = S.sz[0][q], zv = S.sz[1][q];
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        ks2[p] = mul2(f2pack(f16lo(sw[p]), f16hi(sw[p])), (p & 1) ? rs_hi : rs_lo);
        kz2[p] = f2pack(f16lo(zw[p]), f16hi(zw[p]));
      }
    }
    // corrected values of rows g + 8i, channels 8q + 2p + {0, 1}: (reused + fitted) + w orth_mu,
    // each operation rounded as the reference's fp32 form
    uint64_t v2[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = i >> 1, h = i & 1;
      bool taken = false;  // K: a probe row takes its fresh values
      if constexpr (kmode) {
        if (fl[i]) {
          taken = true;
          float f[8];
          if (pslot[i] >= 0) {
            if (FDT == DKV_F32) {
              const uint4 u0 = S.pf[pslot[i]][0][lane], u1 = S.pf[pslot[i]][kFB - 1][lane];
              f[0] = __uint_as_float(u0.x), f[1] = __uint_as_float(u0.y), f[2] = __uint_as_float(u0.z);
              f[3] = __uint_as_float(u0.w), f[4] = __uint_as_float(u1.x), f[5] = __uint_as_float(u1.y);
              f[6] = __uint_as_float(u1.z), f[7] = __uint_as_float(u1.w);
            } else {
              const uint4 u = S.pf[pslot[i]][0][lane];
              const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                f[2 * j] = FDT == DKV_BF16 ? bf16lo(w4[j]) : f16lo(w4[j]);
                f[2 * j + 1] = FDT == DKV_BF16 ? bf16hi(w4[j]) : f16hi(w4[j]);
              }
            }
          } else {
            load8<FDT>(P.fresh, row[i] * P.frs + c, f);
          }
#pragma unroll
          for (int p = 0; p < 4; ++p) v2[i][p] = f2pack(f[2 * p], f[2 * p + 1]);
        }
      }
      if (!taken) {
        uint64_t raw[4];
        kivi::code_pairs(S.cd[g + 8 * i][q], raw);
        uint64_t vs_lo = 0, vs_hi = 0, vz2 = 0;
        if constexpr (!kmode) {
          float vs = 0.f, vz = 0.f;
          if (vstage) {
            const int buf = (cb >> 3) & 1;
            vs = __half2float(reinterpret_cast<const __half *>(&vst->s[buf][g + 8 * i])[cb & 7]);
            vz = __half2float(reinterpret_cast<const __half *>(&vst->z[buf][g + 8 * i])[cb & 7]);
          } else if (rv[i]) {
            vs = __half2float(P.scale[row[i] * P.szrs + cb]);
            vz = __half2float(P.zero[row[i] * P.szrs + cb]);
          }
          vs_lo = mul2(f2pack(vs, vs), rs_lo);
          vs_hi = mul2(f2pack(vs, vs), rs_hi);
          vz2 = f2pack(vz, vz);
        }
        const uint64_t w2 = f2pack(w[i], w[i]);
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const uint64_t r2 = fma2(raw[p], kmode ? ks2[p] : ((p & 1) ? vs_hi : vs_lo), kmode ? kz2[p] : vz2);
          v2[i][p] = add2(add2(r2, f2pack(acc[m][p][2 * h], acc[m][p][2 * h + 1])), mul2(w2, mu2[p]));
        }
      }
    }
    // requantise: group extrema partials go through the warp's scratch to the lane that owns
    // the group, which forms its fp16 scale / zero and publishes (zero, 1 / scale)
    if constexpr (!kmode) {
      // V: group = (row g + 8i, the block's 32 channels) over the lanes q; lane q owns row i = q
      float lo[4], hi[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x[8];
#pragma unroll
        for (int p = 0; p < 4; ++p) f2unpack(v2[i][p], x[2 * p], x[2 * p + 1]);
        lo[i] = kivi::fmin8(x);
        hi[i] = kivi::fmax8(x);
      }
      float *const wr = X.red + g * kRedV + q * 8;
      *reinterpret_cast<float4 *>(wr) = make_float4(lo[0], hi[0], lo[1], hi[1]);
      *reinterpret_cast<float4 *>(wr + 4) = make_float4(lo[2], hi[2], lo[3], hi[3]);
      __syncwarp();
      const float2 *const rd = reinterpret_cast<const float2 *>(X.red + g * kRedV) + q;
      const float2 e0 = rd[0], e1 = rd[4], e2 = rd[8], e3 = rd[12];
      const float glo = fminf(kivi::fmin3(e0.x, e1.x, e2.x), e3.x);
      const float ghi = fmaxf(kivi::fmax3(e0.y, e1.y, e2.y), e3.y);
      __half s16, z16;
      kivi::group_params(glo, ghi, s16, z16);
      const float s_own = __half2float(s16);
      const int64_t orow = t0 + g + 8 * q;
      if (orow < n && !own_probe) {
        P.o_scale[orow * P.o_szrs + cb] = s16;
        P.o_zero[orow * P.o_szrs + cb] = z16;
      }
      X.pz[4 * g + q] = __half2float(z16);
      X.pinv[4 * g + q] = s_own > 0.f ? __frcp_rn(s_own) : 0.f;
      __syncwarp();
      const float4 zz = *reinterpret_cast<const float4 *>(&X.pz[4 * g]);
      const float4 ii = *reinterpret_cast<const float4 *>(&X.pinv[4 * g]);
      const float zr[4] = {zz.x, zz.y, zz.z, zz.w}, ir[4] = {ii.x, ii.y, ii.z, ii.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t z2 = f2pack(zr[i], zr[i]), i2 = f2pack(ir[i], ir[i]);
        const uint64_t zp[4] = {z2, z2, z2, z2}, ip[4] = {i2, i2, i2, i2};
        const uint32_t word = kivi::quant_word(v2[i], zp, ip);
        if (rv[i] && !fl[i]) *reinterpret_cast<uint32_t *>(P.o_codes + row[i] * P.o_crs + c / 2) = word;
      }
    } else {
      // K: group = (the warp tile's 32 rows, channel 8q + j) over the lanes g; lane g owns j = g
      float lo[8], hi[8];
      if (full) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          float x0[4], x1[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) f2unpack(v2[i][p], x0[i], x1[i]);
          lo[2 * p] = fminf(kivi::fmin3(x0[0], x0[1], x0[2]), x0[3]);
          hi[2 * p] = fmaxf(kivi::fmax3(x0[0], x0[1], x0[2]), x0[3]);
          lo[2 * p + 1] = fminf(kivi::fmin3(x1[0], x1[1], x1[2]), x1[3]);
          hi[2 * p + 1] = fmaxf(kivi::fmax3(x1[0], x1[1], x1[2]), x1[3]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          lo[j] = INFINITY;
          hi[j] = -INFINITY;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (rv[i]) {
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              float x0, x1;
              f2unpack(v2[i][p], x0, x1);
              lo[2 * p] = fminf(lo[2 * p], x0);
              hi[2 * p] = fmaxf(hi[2 * p], x0);
              lo[2 * p + 1] = fminf(lo[2 * p + 1], x1);
              hi[2 * p + 1] = fmaxf(hi[2 * p + 1], x1);
            }
          }
      }
      float *const wr = X.red + q * kRedK + g * 16;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        *reinterpret_cast<float4 *>(wr + 4 * jj) = make_float4(lo[2 * jj], hi[2 * jj], lo[2 * jj + 1], hi[2 * jj + 1]);
      __syncwarp();
      const float2 *const rd = reinterpret_cast<const float2 *>(X.red + q * kRedK) + g;
      float2 e[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) e[s] = rd[8 * s];
      const float glo =
          fminf(kivi::fmin3(kivi::fmin3(e[0].x, e[1].x, e[2].x), kivi::fmin3(e[3].x, e[4].x, e[5].x), e[6].x), e[7].x);
      const float ghi =
          fmaxf(kivi::fmax3(kivi::fmax3(e[0].y, e[1].y, e[2].y), kivi::fmax3(e[3].y, e[4].y, e[5].y), e[6].y), e[7].y);
      __half s16, z16;
      kivi::group_params(glo, ghi, s16, z16);
      const float s_own = __half2float(s16);
      P.o_scale[krow * P.o_szrs + c + g] = s16;
      P.o_zero[krow * P.o_szrs + c + g] = z16;
      X.pz[8 * q + g] = __half2float(z16);
      X.pinv[8 * q + g] = s_own > 0.f ? __frcp_rn(s_own) : 0.f;
      __syncwarp();
      const float4 za = *reinterpret_cast<const float4 *>(&X.pz[8 * q]);
      const float4 zb = *reinterpret_cast<const float4 *>(&X.pz[8 * q + 4]);
      const float4 ia = *reinterpret_cast<const float4 *>(&X.pinv[8 * q]);
      const float4 ib = *reinterpret_cast<const float4 *>(&X.pinv[8 * q + 4]);
      const uint64_t zp[4] = {f2pack(za.x, za.y), f2pack(za.z, za.w), f2pack(zb.x, zb.y), f2pack(zb.z, zb.w)};
      const uint64_t ip[4] = {f2pack(ia.x, ia.y), f2pack(ia.z, ia.w), f2pack(ib.x, ib.y), f2pack(ib.z, ib.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t word = kivi::quant_word(v2[i], zp, ip);
        if (rv[i]) *reinterpret_cast<uint32_t *>(P.o_codes + row[i] * P.o_crs + c / 2) = word;
      }
    }
  }
  cp_async_wait<0>();
  if (!ok) {
    record_error(b.status, DKV_ERR_TIMEOUT);
    *abort_flag = 1;
  }
  // copies this CTA issued and warp 0 has not waited for complete before the CTA exits
  if (producer)
    for (int blk = cb; blk < bq_issued; ++blk) mbar_wait_drain(&bq_full[blk % kBSlots], (blk / kBSlots) & 1);
}

// ---------------------------------------------------------------------------------------
// Dense caches (dkv_subspace_correct on f32 / f16 / bf16 rows): the same pipeline with the
// reused rows read directly — pass1<..., DENSE>, psum<..., DENSE>, solve, fitb, then dpass2
// (corr = (reused + fitted) + w orth_mu for the non-probe rows, stored in the output dtype)
// and dprobe (the probe rows take the fresh values, corr[P] = fresh[P]).
// ---------------------------------------------------------------------------------------
// 8 values to a row of the output dtype (16-B aligned: 32 B for f32, 16 B otherwise)
__device__ __forceinline__ void store8(void *base, int dt, int64_t off, const float (&v)[8]) {
  if (dt == DKV_F32) {
    float4 *o = reinterpret_cast<float4 *>(static_cast<float *>(base) + off);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 u;
    if (dt == DKV_BF16) {
      u.x = pack_bf16x2(v[0], v[1]), u.y = pack_bf16x2(v[2], v[3]);
      u.z = pack_bf16x2(v[4], v[5]), u.w = pack_bf16x2(v[6], v[7]);
    } else {
      u.x = pack_f16x2(v[0], v[1]), u.y = pack_f16x2(v[2], v[3]);
      u.z = pack_f16x2(v[4], v[5]), u.w = pack_f16x2(v[6], v[7]);
    }
    *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(base) + off) = u;
  }
}

// one block's per-warp operands in dpass2: the reused rows (16 or 32 B per lane and row)
template <int FDT>
struct D2Stage {
  static constexpr int kFB = FDT == DKV_F32 ? 2 : 1;
  uint4 rr[4][kFB][32];
};
template <int RP, int FDT>
constexpr int d2_smem_fixed() {  // everything but orth_mu [d]
  return kBSlots * p2_bq_bytes<RP>() + kWarps * kP2Stages * static_cast<int>(sizeof(D2Stage<FDT>)) +
         2 * kBSlots * 8 + 16;
}

template <int RP, int FDT>
__global__ void __launch_bounds__(kThreads, p2_min_blocks<RP, DKV_KIVI_PER_TOKEN>())
    dpass2_kernel(const __grid_constant__ Batch b) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
  const Prob &P = b.probs[find_prob(b, blockIdx.x)];
  const int64_t tile_t0 = (blockIdx.x - P.tile0) * kTM;
  const int64_t t0 = tile_t0 + warp * kWT;
  const int64_t n = P.n;
  constexpr int KS = RP / 16;
  constexpr int BQ = p2_bq_bytes<RP>();
  const int n_blocks = static_cast<int>(b.d / kCB);
  using Stage = D2Stage<FDT>;
  constexpr int kFB = Stage::kFB;
  constexpr int kEs = FDT == DKV_F32 ? 4 : 2;
  // shared: [fragment ring][per-warp stage rings][barriers, abort][orth_mu]
  extern __shared__ __align__(16) unsigned char d2_smem[];
  unsigned char *const bq_ring = d2_smem;
  Stage *const ring = reinterpret_cast<Stage *>(d2_smem + kBSlots * BQ) + warp * kP2Stages;
  unsigned char *const sp = d2_smem + kBSlots * BQ + kWarps * kP2Stages * sizeof(Stage);
  uint64_t *const bq_full = reinterpret_cast<uint64_t *>(sp);
  uint64_t *const bq_empty = bq_full + kBSlots;
  volatile int *const abort_flag = reinterpret_cast<volatile int *>(bq_empty + kBSlots);
  float *const mu_s = reinterpret_cast<float *>(sp + 2 * kBSlots * 8 + 16);

  const int active = static_cast<int>((n - tile_t0 + kWT - 1) / kWT < kWarps ? (n - tile_t0 + kWT - 1) / kWT : kWarps);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBSlots; ++s) {
      mbar_init(&bq_full[s], 1);
      mbar_init(&bq_empty[s], active);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int64_t e = threadIdx.x; e < b.d / 4; e += kThreads)
    reinterpret_cast<float4 *>(mu_s)[e] = reinterpret_cast<const float4 *>(P.mu)[e];
  __syncthreads();
  if (t0 >= n) return;

  const bool producer = warp == 0 && lane == 0;
  const unsigned char *const bq_src = reinterpret_cast<const unsigned char *>(P.b2);
  int bq_issued = 0;
  auto bq_issue = [&]() -> bool {
    const int blk = bq_issued, s = blk % kBSlots;
    if (blk >= kBSlots && !mbar_wait_bounded(&bq_empty[s], ((blk / kBSlots) - 1) & 1, abort_flag)) return false;
    mbar_arrive_expect_tx(&bq_full[s], BQ);
    bulk_load(bq_ring + s * BQ, bq_src + static_cast<int64_t>(blk) * BQ, BQ, &bq_full[s]);
    ++bq_issued;
    return true;
  };
  bool ok = true;
  if (producer)
    while (bq_issued < kBSlots - 1 && bq_issued < n_blocks) bq_issue();

  const float mean_dist = P.subv[b.d];
  int64_t row[4];
  bool st[4];  // rows this lane stores (valid, not a probe)
  float w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    row[i] = t0 + g + 8 * i;
    const bool rv = row[i] < n;
    st[i] = rv && P.flag[row[i]] == 0u;
    w[i] = !rv ? 0.f : P.tw != nullptr ? P.tw[row[i]] : fminf(P.dist[row[i]] / mean_dist, 1.f);
  }
  // A fragments: the row's rhs at this lane's positions k = 16 ks + 2q + {0, 1, 8, 9}, as
  // high and low bf16 terms
  uint32_t a[2][KS][4], al[2][KS][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = i >> 1, h = i & 1;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
      if (row[i] < n) {
        const float *rr = P.rhs + row[i] * RP + 16 * ks + 2 * q;
        lo = *reinterpret_cast<const float2 *>(rr);
        hi = *reinterpret_cast<const float2 *>(rr + 8);
      }
      split_bf16x2(lo.x, lo.y, a[m][ks][h], al[m][ks][h]);
      split_bf16x2(hi.x, hi.y, a[m][ks][2 + h], al[m][ks][2 + h]);
    }
  }
  // per-warp staging ring: each lane copies and reads back only its own reused chunks
  auto issue = [&](int blk) {
    if (blk < n_blocks) {
      Stage &S = ring[blk % kP2Stages];
      const int64_t c = static_cast<int64_t>(blk) * kCB + 8 * q;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const unsigned char *rp =
            static_cast<const unsigned char *>(P.reused) + ((st[i] ? row[i] : t0) * P.rrs + c) * kEs;
#pragma unroll
        for (int f = 0; f < kFB; ++f) cp_async16(&S.rr[i][f][lane], rp + 16 * f, st[i] ? 16u : 0u);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s0 = 0; s0 < kP2Stages - 1; ++s0) issue(s0);

  int cb = 0;
  for (; cb < n_blocks; ++cb) {
    if (warp == 0) {
      int pok = 1;
      if (producer && bq_issued < n_blocks) pok = bq_issue() ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, pok, 0)) {
        ok = false;
        break;
      }
    }
    issue(cb + kP2Stages - 1);
    cp_async_wait<kP2Stages - 1>();
    const int slot = cb % kBSlots;
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bq_full[slot], (cb / kBSlots) & 1, abort_flag))) {
      ok = false;
      break;
    }
    const Stage &S = ring[cb % kP2Stages];
    const uint4 *const bq = reinterpret_cast<const uint4 *>(bq_ring + slot * BQ) + lane;
    const int64_t c = static_cast<int64_t>(cb) * kCB + 8 * q;
    float acc[2][4][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const uint4 f = bq[(ks * 4 + nt) * 32];  // high terms (x, y), low terms (z, w)
#pragma unroll
        for (int m = 0; m < 2; ++m) {  // rhs (B G^-1)^T ~ ah bh + ah bl + al bh, small terms first
          if (ks == 0)
            mma16816_bf16_zc(acc[m][nt], al[m][ks][0], al[m][ks][1], al[m][ks][2], al[m][ks][3], f.x, f.y);
          else
            mma16816_bf16(acc[m][nt], al[m][ks][0], al[m][ks][1], al[m][ks][2], al[m][ks][3], f.x, f.y);
          mma16816_bf16(acc[m][nt], a[m][ks][0], a[m][ks][1], a[m][ks][2], a[m][ks][3], f.z, f.w);
          mma16816_bf16(acc[m][nt], a[m][ks][0], a[m][ks][1], a[m][ks][2], a[m][ks][3], f.x, f.y);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bq_empty[slot]);
    uint64_t mu2[4];
    {
      const float4 *mp = reinterpret_cast<const float4 *>(mu_s + c);
      const float4 x = mp[0], y = mp[1];
      mu2[0] = f2pack(x.x, x.y), mu2[1] = f2pack(x.z, x.w), mu2[2] = f2pack(y.x, y.y), mu2[3] = f2pack(y.z, y.w);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (!st[i]) continue;
      const int m = i >> 1, h = i & 1;
      float x[8], v[8];
      unpack8<FDT>(S.rr[i][0][lane], S.rr[i][kFB - 1][lane], x);
      const uint64_t w2 = f2pack(w[i], w[i]);
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const uint64_t c2 = add2(add2(f2pack(x[2 * p], x[2 * p + 1]), f2pack(acc[m][p][2 * h], acc[m][p][2 * h + 1])),
                                 mul2(w2, mu2[p]));
        f2unpack(c2, v[2 * p], v[2 * p + 1]);
      }
      store8(P.out, P.odt, row[i] * P.ors + c, v);
    }
  }
  cp_async_wait<0>();
  if (!ok) {
    record_error(b.status, DKV_ERR_TIMEOUT);
    *abort_flag = 1;
  }
  if (producer)
    for (int blk = cb; blk < bq_issued; ++blk) mbar_wait_drain(&bq_full[blk % kBSlots], (blk / kBSlots) & 1);
}

// corr[P] = fresh[P]: one warp per unique probe row
template <int FDT>
__global__ void __launch_bounds__(128) dprobe_kernel(const __grid_constant__ Batch b) {
  const Prob &P = b.probs[blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = *P.ucount;
  for (int k = blockIdx.x * 4 + warp; k < count; k += gridDim.x * 4) {
    const int64_t t = P.uprobe[k];
    for (int64_t c = 8 * lane; c < b.d; c += 256) {
      float f[8];
      load8<FDT>(P.fresh, t * P.frs + c, f);
      store8(P.out, P.odt, t * P.ors + c, f);
    }
  }
}

// ---------------------------------------------------------------------------------------
// vprobe: the probe rows of the V (per-token) problems.  There corr = fresh, and a per-token
// group holds one row's channels only, so each probe row is requantised from its fresh values
// alone (pass2 leaves these rows untouched): one warp per row, one lane per 32-channel group,
// with the IEEE quotient (kivi::quant_one)
// ---------------------------------------------------------------------------------------
template <int FDT>
__global__ void __launch_bounds__(128) vprobe_kernel(const __grid_constant__ Batch b, int first_v) {
  const Prob &P = b.probs[first_v + blockIdx.y];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = *P.ucount;
  const int n_blocks = static_cast<int>(b.d / kCB);
  for (int k = blockIdx.x * 4 + warp; k < count; k += gridDim.x * 4) {
    const int64_t t = P.uprobe[k];
    for (int cb = lane; cb < n_blocks; cb += 32) {
      float x[kCB];
#pragma unroll
      for (int j = 0; j < kCB; j += 8) {
        float f[8];
        load8<FDT>(P.fresh, t * P.frs + static_cast<int64_t>(cb) * kCB + j, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[j + e] = f[e];
      }
      float lo = x[0], hi = x[0];
#pragma unroll
      for (int j = 1; j < kCB; ++j) {
        lo = fminf(lo, x[j]);
        hi = fmaxf(hi, x[j]);
      }
      __half s16, z16;
      kivi::group_params(lo, hi, s16, z16);
      const float sf = __half2float(s16), zf = __half2float(z16);
      uint32_t wd[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t word = 0u;
#pragma unroll
        for (int j = 7; j >= 0; --j) word = (word << 4) | kivi::quant_one(x[8 * w + j], sf, zf);
        wd[w] = word;
      }
      *reinterpret_cast<uint4 *>(P.o_codes + t * P.o_crs + static_cast<int64_t>(cb) * (kCB / 2)) =
          make_uint4(wd[0], wd[1], wd[2], wd[3]);
      P.o_scale[t * P.o_szrs + cb] = s16;
      P.o_zero[t * P.o_szrs + cb] = z16;
    }
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
inline int64_t al(int64_t x) { return (x + 255) / 256 * 256; }

struct Layout {
  int64_t zero_begin, zero_end, total;
  std::vector<int64_t> flag, ucount, sums, uprobe, rhs, dist, part, ginv, mu, subv, b1, b1l, b2, bb;
};

inline int padded_rank(const dkv_kivi_subspace_problem *p, int np) {
  int rmax = 0;
  for (int i = 0; i < np; ++i) rmax = p[i].rank > rmax ? p[i].rank : rmax;
  const int rp = (rmax + 15) / 16 * 16;
  return rp < 16 ? 16 : rp;
}

inline Layout layout(const dkv_kivi_subspace_problem *p, int np, int64_t d, int rp) {
  Layout L;
  int64_t o = 0;
  L.zero_begin = o;
  for (int i = 0; i < np; ++i) {
    const int64_t n = p[i].base.n_tokens;
    L.flag.push_back(o);
    o = al(o + n * 4);
    L.ucount.push_back(o);
    o = al(o + 4);
    L.sums.push_back(o);
    o = al(o + (rp + d) * 4);
  }
  L.zero_end = o;
  for (int i = 0; i < np; ++i) {
    const int64_t n = p[i].base.n_tokens;
    const int64_t npr = p[i].n_probes > 0 ? p[i].n_probes : 1;
    L.uprobe.push_back(o);
    o = al(o + npr * 4);
    L.rhs.push_back(o);
    o = al(o + n * rp * 4);
    L.dist.push_back(o);
    o = al(o + n * 4);
    L.part.push_back(o);
    o = al(o + ((n + kWT - 1) / kWT) * (rp + 1) * 4);
    L.ginv.push_back(o);
    o = al(o + static_cast<int64_t>(rp) * rp * 4);
    L.mu.push_back(o);
    o = al(o + d * 4);
    L.subv.push_back(o);
    o = al(o + (d + 1) * 4);
    L.b1.push_back(o);
    o = al(o + rp * d * 2);
    L.b1l.push_back(o);
    o = al(o + rp * d * 2);
    L.b2.push_back(o);
    o = al(o + rp * d * 4);
    L.bb.push_back(o);
    o = al(o + rp * d * 4);
  }
  L.total = o;
  return L;
}

bool a16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_cache(const dkv_kivi_cache &c, int64_t n, int64_t d) {
  if (c.codes == nullptr || c.scale == nullptr || c.zero == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  if (c.n_tokens != n || c.d != d) return DKV_ERR_INVALID_ARGUMENT;
  if (c.mode != DKV_KIVI_PER_TOKEN && c.mode != DKV_KIVI_PER_CHANNEL) return DKV_ERR_INVALID_ARGUMENT;
  if (!a16(c.codes) || !a16(c.scale) || !a16(c.zero) || c.code_row_stride % 16) return DKV_ERR_ALIGNMENT;
  if (c.mode == DKV_KIVI_PER_CHANNEL && c.sz_row_stride % 8) return DKV_ERR_ALIGNMENT;  // 16-B scale rows
  if (c.code_row_stride < d / 2) return DKV_ERR_LAYOUT;
  if (c.mode == DKV_KIVI_PER_TOKEN ? c.sz_row_stride < d / 32 : c.sz_row_stride < d) return DKV_ERR_LAYOUT;
  return DKV_OK;
}

int validate(const dkv_kivi_subspace_problem *p, int np, int64_t &d, int &fdt) {
  if (p == nullptr || np <= 0 || np > kMaxProblems) return DKV_ERR_INVALID_ARGUMENT;
  d = p[0].base.d;
  fdt = p[0].fresh_dtype;
  if (d <= 0 || d % kCB) return DKV_ERR_UNSUPPORTED;
  if (fdt != DKV_F32 && fdt != DKV_F16 && fdt != DKV_BF16) return DKV_ERR_UNSUPPORTED;
  const int esz = fdt == DKV_F32 ? 4 : 2;
  for (int i = 0; i < np; ++i) {
    const dkv_kivi_subspace_problem &q = p[i];
    if (q.base.d != d || q.fresh_dtype != fdt) return DKV_ERR_INVALID_ARGUMENT;
    if (q.rank < 0 || q.rank > kMaxRank) return DKV_ERR_INVALID_ARGUMENT;
    if (q.rank > 0 && q.basis == nullptr) return DKV_ERR_INVALID_ARGUMENT;
    const int64_t n = q.base.n_tokens;
    if (n < 0 || n > 0x7fffffffLL) return DKV_ERR_INVALID_ARGUMENT;
    if (n == 0) continue;
    int rc = check_cache(q.base, n, d);
    if (rc) return rc;
    rc = check_cache(q.out, n, d);
    if (rc) return rc;
    if (q.out.mode != q.base.mode) return DKV_ERR_INVALID_ARGUMENT;
    if (q.fresh == nullptr || !a16(q.fresh) || (q.fresh_row_stride * esz) % 16 || q.fresh_row_stride < d)
      return DKV_ERR_ALIGNMENT;
    if (q.n_probes < 0 || q.n_probes > n || (q.n_probes > 0 && q.probe_index == nullptr))
      return DKV_ERR_INVALID_ARGUMENT;
  }
  return DKV_OK;
}

template <int RP, int FDT>
int launch(const Batch &b, int np, int n_kprob, int64_t max_probes, int64_t k_tiles, cudaStream_t st) {
  if (max_probes > 0) {
    const int bx = static_cast<int>((max_probes + 255) / 256 < 64 ? (max_probes + 255) / 256 : 64);
    flags_kernel<<<dim3(bx, np), 256, 0, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  {
    const int64_t total = b.d * RP;
    const int bx = static_cast<int>((total + 255) / 256 < 256 ? (total + 255) / 256 : 256);
    pack_kernel<<<dim3(bx, np), 256, 0, st>>>(b, RP);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  // the table holds the K (per-channel) problems first (tiles [0, k_tiles)), then the V ones
  if (k_tiles > 0) {
    constexpr int sm = p1_smem_bytes<RP, FDT, DKV_KIVI_PER_CHANNEL>();
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass1_kernel<RP, FDT, DKV_KIVI_PER_CHANNEL>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass1_kernel<RP, FDT, DKV_KIVI_PER_CHANNEL>,
                                        cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared));
    pass1_kernel<RP, FDT, DKV_KIVI_PER_CHANNEL><<<static_cast<unsigned>(k_tiles), kThreads, sm, st>>>(b, 0);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (b.n_tiles > k_tiles) {
    constexpr int sm = p1_smem_bytes<RP, FDT, DKV_KIVI_PER_TOKEN>();
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass1_kernel<RP, FDT, DKV_KIVI_PER_TOKEN>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass1_kernel<RP, FDT, DKV_KIVI_PER_TOKEN>,
                                        cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared));
    pass1_kernel<RP, FDT, DKV_KIVI_PER_TOKEN><<<static_cast<unsigned>(b.n_tiles - k_tiles), kThreads, sm, st>>>(
        b, k_tiles);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (max_probes > 0) {
    // about four CTAs per SM in all, at least kPsumCtas per problem
    const int ctas = std::max(kPsumCtas, std::min(64, 4 * 148 / np));
    psum_kernel<RP, FDT><<<dim3(ctas, np), 256, 0, st>>>(b, ctas);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  const int solve_smem = kMaxRank * (2 * kMaxRank + 1) * 8 + 64 * RP * 8;
  DKV_CUDA_CHECK(cudaFuncSetAttribute(solve_kernel<RP>, cudaFuncAttributeMaxDynamicSharedMemorySize, solve_smem));
  solve_kernel<RP><<<np, 256, solve_smem, st>>>(b);
  DKV_CUDA_CHECK(cudaGetLastError());
  fitb_kernel<RP><<<dim3(static_cast<unsigned>(b.d / kCB), np), 256, 0, st>>>(b);
  DKV_CUDA_CHECK(cudaGetLastError());
  if (k_tiles > 0) {
    const int sm = static_cast<int>(b.d * 4) + p2_smem_fixed<RP, FDT, DKV_KIVI_PER_CHANNEL>();
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass2_kernel<RP, FDT, DKV_KIVI_PER_CHANNEL>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass2_kernel<RP, FDT, DKV_KIVI_PER_CHANNEL>,
                                        cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared));
    pass2_kernel<RP, FDT, DKV_KIVI_PER_CHANNEL><<<static_cast<unsigned>(k_tiles), kThreads, sm, st>>>(b, 0);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (b.n_tiles > k_tiles) {
    const int sm = static_cast<int>(b.d * 4) + p2_smem_fixed<RP, FDT, DKV_KIVI_PER_TOKEN>();
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass2_kernel<RP, FDT, DKV_KIVI_PER_TOKEN>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    DKV_CUDA_CHECK(cudaFuncSetAttribute(pass2_kernel<RP, FDT, DKV_KIVI_PER_TOKEN>,
                                        cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared));
    pass2_kernel<RP, FDT, DKV_KIVI_PER_TOKEN><<<static_cast<unsigned>(b.n_tiles - k_tiles), kThreads, sm, st>>>(
        b, k_tiles);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (max_probes > 0 && np > n_kprob) {
    const int bx = static_cast<int>((max_probes + 3) / 4 < 64 ? (max_probes + 3) / 4 : 64);
    vprobe_kernel<FDT><<<dim3(bx, np - n_kprob), 128, 0, st>>>(b, n_kprob);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  return DKV_OK;
}

template <int FDT>
int launch_rp(int rp, const Batch &b, int np, int n_kprob, int64_t max_probes, int64_t k_tiles, cudaStream_t st) {
  switch (rp) {
    case 16: return launch<16, FDT>(b, np, n_kprob, max_probes, k_tiles, st);
    case 32: return launch<32, FDT>(b, np, n_kprob, max_probes, k_tiles, st);
    case 48: return launch<48, FDT>(b, np, n_kprob, max_probes, k_tiles, st);
    case 64: return launch<64, FDT>(b, np, n_kprob, max_probes, k_tiles, st);
    default: return DKV_ERR_UNSUPPORTED;
  }
}

// ---------------------------------------------------------------------------------------
// dense caches: one problem per call (dkv_subspace_correct), d a multiple of 32 and 16-byte
// rows; other shapes stay on the general kernels of subspace.cu
// ---------------------------------------------------------------------------------------
template <int RP, int FDT>
int launch_dense(const Batch &b, int64_t max_probes, cudaStream_t st) {
  if (max_probes > 0) {
    const int bx = static_cast<int>((max_probes + 255) / 256 < 64 ? (max_probes + 255) / 256 : 64);
    flags_kernel<<<dim3(bx, b.n_probs), 256, 0, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  {
    const int64_t total = b.d * RP;
    const int bx = static_cast<int>((total + 255) / 256 < 256 ? (total + 255) / 256 : 256);
    pack_kernel<<<dim3(bx, b.n_probs), 256, 0, st>>>(b, RP);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  const unsigned tiles = static_cast<unsigned>(b.n_tiles);
  {
    constexpr int sm = p1_smem_bytes<RP, FDT, DKV_KIVI_PER_TOKEN, true>();
    auto fn = pass1_kernel<RP, FDT, DKV_KIVI_PER_TOKEN, true>;
    DKV_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    DKV_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared));
    fn<<<tiles, kThreads, sm, st>>>(b, 0);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (max_probes > 0) {
    // about four CTAs per SM in all, at least kPsumCtas per problem
    const int ctas = std::max(kPsumCtas, std::min(64, 4 * 148 / b.n_probs));
    psum_kernel<RP, FDT, true><<<dim3(ctas, b.n_probs), 256, 0, st>>>(b, ctas);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  const int solve_smem = kMaxRank * (2 * kMaxRank + 1) * 8 + 64 * RP * 8;
  DKV_CUDA_CHECK(cudaFuncSetAttribute(solve_kernel<RP>, cudaFuncAttributeMaxDynamicSharedMemorySize, solve_smem));
  solve_kernel<RP><<<b.n_probs, 256, solve_smem, st>>>(b);
  DKV_CUDA_CHECK(cudaGetLastError());
  fitb_kernel<RP><<<dim3(static_cast<unsigned>(b.d / kCB), b.n_probs), 256, 0, st>>>(b);
  DKV_CUDA_CHECK(cudaGetLastError());
  {
    const int sm = static_cast<int>(b.d * 4) + d2_smem_fixed<RP, FDT>();
    auto fn = dpass2_kernel<RP, FDT>;
    DKV_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, sm));
    DKV_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared));
    fn<<<tiles, kThreads, sm, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  if (max_probes > 0) {
    const int bx = static_cast<int>((max_probes + 3) / 4 < 64 ? (max_probes + 3) / 4 : 64);
    dprobe_kernel<FDT><<<dim3(bx, b.n_probs), 128, 0, st>>>(b);
    DKV_CUDA_CHECK(cudaGetLastError());
  }
  return DKV_OK;
}

template <int FDT>
int launch_dense_rp(int rp, const Batch &b, int64_t max_probes, cudaStream_t st) {
  switch (rp) {
    case 16: return launch_dense<16, FDT>(b, max_probes, st);
    case 32: return launch_dense<32, FDT>(b, max_probes, st);
    case 48: return launch_dense<48, FDT>(b, max_probes, st);
    case 64: return launch_dense<64, FDT>(b, max_probes, st);
    default: return DKV_ERR_UNSUPPORTED;
  }
}

inline int dense_rp(int rank) { return rank <= 16 ? 16 : (rank + 15) / 16 * 16; }

bool dense_applies(const dkv_subspace_args &a) {
  if (a.n_tokens <= 0 || a.n_tokens > 0x7fffffffLL || a.d <= 0 || a.d % kCB) return false;
  if (a.rank < 0 || a.rank > kMaxRank) return false;
  auto esz = [](int dt) { return dt == DKV_F32 ? 4 : (dt == DKV_F16 || dt == DKV_BF16) ? 2 : 0; };
  const int ke = esz(a.kv_dtype), oe = esz(a.out_dtype);
  if (ke == 0 || oe == 0) return false;
  if (!a16(a.reused) || !a16(a.fresh) || !a16(a.corrected)) return false;
  if ((a.reused_row_stride * ke) % 16 || (a.fresh_row_stride * ke) % 16 || (a.out_row_stride * oe) % 16) return false;
  return a.reused_row_stride >= a.d && a.fresh_row_stride >= a.d && a.out_row_stride >= a.d;
}

// problems of one dense batch: all dense-applicable, one d and fresh dtype, at most
// kMaxProblems; their padded rank
bool dense_batch_ok(const dkv_subspace_args *a, int np, int &rp) {
  if (a == nullptr || np <= 0 || np > kMaxProblems) return false;
  rp = 16;
  for (int i = 0; i < np; ++i) {
    if (!dense_applies(a[i]) || a[i].d != a[0].d || a[i].kv_dtype != a[0].kv_dtype) return false;
    rp = std::max(rp, dense_rp(a[i].rank));
  }
  return true;
}

inline Layout dense_layout(const dkv_subspace_args *a, int np, int rp) {
  std::vector<dkv_kivi_subspace_problem> q(np);
  for (int i = 0; i < np; ++i) {
    memset(&q[i], 0, sizeof(q[i]));
    q[i].base.n_tokens = a[i].n_tokens;
    q[i].n_probes = a[i].n_tokens;  // unique probe rows never exceed the token count
  }
  return layout(q.data(), np, a[0].d, rp);
}

// The dense form over `np` problems: DKV_ERR_UNSUPPORTED when one of them is not a shape or
// layout it takes (the caller then runs them on the general kernels).
int dense_correct(const dkv_subspace_args *a, int np, uint8_t *ws, int64_t ws_bytes, cudaStream_t st) {
  int rp = 16;
  if (!dense_batch_ok(a, np, rp)) return DKV_ERR_UNSUPPORTED;
  const Layout L = dense_layout(a, np, rp);
  if (ws == nullptr || ws_bytes < L.total || !a16(ws)) return DKV_ERR_UNSUPPORTED;
  int64_t max_probes = 0, tiles = 0;
  for (int i = 0; i < np; ++i) {
    if (a[i].n_probes < 0 || (a[i].n_probes > 0 && a[i].probe_index == nullptr)) return DKV_ERR_INVALID_ARGUMENT;
    if (a[i].rank > 0 && a[i].basis == nullptr) return DKV_ERR_INVALID_ARGUMENT;
    max_probes = std::max<int64_t>(max_probes, a[i].n_probes);
  }
  static thread_local Batch b;
  memset(&b, 0, sizeof(b));
  for (int i = 0; i < np; ++i) {
    Prob &P = b.probs[i];
    P.fresh = a[i].fresh;
    P.frs = a[i].fresh_row_stride;
    P.n = a[i].n_tokens;
    P.probes = a[i].probe_index;
    P.n_probes = a[i].n_probes;
    P.sub_out = a[i].subspace_out;
    P.mu_out = a[i].orth_mu_out;
    P.mode = DKV_KIVI_PER_TOKEN;
    // the reference applies the column-space fit only with a basis and at least one probe
    P.r = (a[i].n_probes > 0 && a[i].basis != nullptr) ? a[i].rank : 0;
    P.basis = a[i].basis;
    P.flag = reinterpret_cast<uint32_t *>(ws + L.flag[i]);
    P.ucount = reinterpret_cast<int32_t *>(ws + L.ucount[i]);
    P.sums = reinterpret_cast<float *>(ws + L.sums[i]);
    P.uprobe = reinterpret_cast<int32_t *>(ws + L.uprobe[i]);
    P.rhs = reinterpret_cast<float *>(ws + L.rhs[i]);
    P.dist = reinterpret_cast<float *>(ws + L.dist[i]);
    P.part = reinterpret_cast<float *>(ws + L.part[i]);
    P.ginv = reinterpret_cast<float *>(ws + L.ginv[i]);
    P.mu = reinterpret_cast<float *>(ws + L.mu[i]);
    P.subv = reinterpret_cast<float *>(ws + L.subv[i]);
    P.b1 = reinterpret_cast<__nv_bfloat16 *>(ws + L.b1[i]);
    P.b1l = reinterpret_cast<__nv_bfloat16 *>(ws + L.b1l[i]);
    P.b2 = reinterpret_cast<__nv_bfloat16 *>(ws + L.b2[i]);
    P.bb = reinterpret_cast<float *>(ws + L.bb[i]);
    P.reused = a[i].reused;
    P.rrs = a[i].reused_row_stride;
    P.out = a[i].corrected;
    P.ors = a[i].out_row_stride;
    P.odt = a[i].out_dtype;
    P.tw = a[i].token_weights;
    P.tile0 = tiles;
    tiles += (P.n + kTM - 1) / kTM;
  }
  if (tiles > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  DKV_CUDA_CHECK(cudaMemsetAsync(ws + L.zero_begin, 0, L.zero_end - L.zero_begin, st));
  b.n_probs = np;
  b.d = a[0].d;
  b.n_tiles = tiles;
  b.status = nullptr;
  switch (a[0].kv_dtype) {
    case DKV_BF16: return launch_dense_rp<DKV_BF16>(rp, b, max_probes, st);
    case DKV_F16: return launch_dense_rp<DKV_F16>(rp, b, max_probes, st);
    default: return launch_dense_rp<DKV_F32>(rp, b, max_probes, st);
  }
}

int dense_correct(const dkv_subspace_args *a, uint8_t *ws, int64_t ws_bytes, cudaStream_t st) {
  return dense_correct(a, 1, ws, ws_bytes, st);
}

int64_t dense_workspace_bytes(int64_t n, int64_t d, int rank) {
  if (n <= 0 || d <= 0 || d % kCB || rank < 0 || rank > kMaxRank) return 0;
  dkv_subspace_args a;
  memset(&a, 0, sizeof(a));
  a.n_tokens = n;
  a.d = d;
  return dense_layout(&a, 1, dense_rp(rank)).total;
}

}  // namespace ksub
}  // namespace dkv

using namespace dkv;
using namespace dkv::ksub;

extern "C" int dkv_subspace_correct_batched_workspace_bytes(const dkv_subspace_args *args, int32_t n,
                                                           int64_t *bytes) {
  int rp = 16;
  if (bytes == nullptr || !dense_batch_ok(args, n, rp)) return DKV_ERR_UNSUPPORTED;
  *bytes = dense_layout(args, n, rp).total;
  return DKV_OK;
}

extern "C" int dkv_subspace_correct_batched(const dkv_subspace_args *args, int32_t n, void *workspace,
                                            int64_t workspace_bytes, dkv_stream_t stream) {
  return dense_correct(args, n, static_cast<uint8_t *>(workspace), workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int dkv_kivi_subspace_workspace_bytes(const dkv_kivi_subspace_problem *problems, int32_t n_problems,
                                                 int64_t *bytes) {
  if (bytes == nullptr) return DKV_ERR_INVALID_ARGUMENT;
  int64_t d;
  int fdt;
  const int rc = validate(problems, n_problems, d, fdt);
  if (rc) return rc;
  *bytes = layout(problems, n_problems, d, padded_rank(problems, n_problems)).total;
  return DKV_OK;
}

extern "C" int dkv_kivi_subspace_correct(const dkv_kivi_subspace_problem *problems, int32_t n_problems,
                                         void *workspace, int64_t workspace_bytes, int32_t *status,
                                         dkv_stream_t stream) {
  int64_t d;
  int fdt;
  int rc = validate(problems, n_problems, d, fdt);
  if (rc) return rc;
  const int rp = padded_rank(problems, n_problems);
  const Layout L = layout(problems, n_problems, d, rp);
  if (workspace == nullptr || workspace_bytes < L.total || !a16(workspace)) return DKV_ERR_WORKSPACE;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  static thread_local Batch b;  // ~30 KB: not on the caller's stack
  memset(&b, 0, sizeof(b));
  // the table holds the K (per-channel) problems first, then the V ones: one launch per mode
  std::vector<int> order;
  for (int pass = 0; pass < 2; ++pass)
    for (int i = 0; i < n_problems; ++i)
      if ((problems[i].base.mode == DKV_KIVI_PER_CHANNEL) == (pass == 0)) order.push_back(i);
  int64_t tiles = 0, max_probes = 0, k_tiles = 0;
  int n_kprob = 0;
  for (int slot = 0; slot < n_problems; ++slot) {
    const int i = order[slot];
    const dkv_kivi_subspace_problem &q = problems[i];
    Prob &P = b.probs[slot];
    P.codes = static_cast<const uint8_t *>(q.base.codes);
    P.scale = static_cast<const __half *>(q.base.scale);
    P.zero = static_cast<const __half *>(q.base.zero);
    P.crs = q.base.code_row_stride;
    P.szrs = q.base.sz_row_stride;
    P.o_codes = static_cast<uint8_t *>(q.out.codes);
    P.o_scale = static_cast<__half *>(q.out.scale);
    P.o_zero = static_cast<__half *>(q.out.zero);
    P.o_crs = q.out.code_row_stride;
    P.o_szrs = q.out.sz_row_stride;
    P.fresh = q.fresh;
    P.frs = q.fresh_row_stride;
    P.n = q.base.n_tokens;
    P.probes = q.probe_index;
    P.n_probes = q.n_probes;
    P.sub_out = q.subspace_out;
    P.mu_out = q.orth_mu_out;
    P.mode = q.base.mode;
    // the reference applies the column-space fit only with a basis and at least one probe
    P.r = (q.n_probes > 0 && q.basis != nullptr) ? q.rank : 0;
    P.basis = q.basis;
    P.flag = reinterpret_cast<uint32_t *>(ws + L.flag[i]);
    P.ucount = reinterpret_cast<int32_t *>(ws + L.ucount[i]);
    P.sums = reinterpret_cast<float *>(ws + L.sums[i]);
    P.uprobe = reinterpret_cast<int32_t *>(ws + L.uprobe[i]);
    P.rhs = reinterpret_cast<float *>(ws + L.rhs[i]);
    P.dist = reinterpret_cast<float *>(ws + L.dist[i]);
    P.part = reinterpret_cast<float *>(ws + L.part[i]);
    P.ginv = reinterpret_cast<float *>(ws + L.ginv[i]);
    P.mu = reinterpret_cast<float *>(ws + L.mu[i]);
    P.subv = reinterpret_cast<float *>(ws + L.subv[i]);
    P.b1 = reinterpret_cast<__nv_bfloat16 *>(ws + L.b1[i]);
    P.b1l = reinterpret_cast<__nv_bfloat16 *>(ws + L.b1l[i]);
    P.b2 = reinterpret_cast<__nv_bfloat16 *>(ws + L.b2[i]);
    P.bb = reinterpret_cast<float *>(ws + L.bb[i]);
    P.tile0 = tiles;
    tiles += (P.n + kTM - 1) / kTM;
    if (P.mode == DKV_KIVI_PER_CHANNEL) {
      k_tiles = tiles;
      ++n_kprob;
    }
    if (P.n_probes > max_probes) max_probes = P.n_probes;
  }
  if (tiles > 0x7fffffffLL) return DKV_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DKV_CUDA_CHECK(cudaMemsetAsync(ws + L.zero_begin, 0, L.zero_end - L.zero_begin, st));
  b.n_probs = n_problems;
  b.d = d;
  b.n_tiles = tiles;
  b.status = status;
  switch (fdt) {
    case DKV_BF16: rc = launch_rp<DKV_BF16>(rp, b, n_problems, n_kprob, max_probes, k_tiles, st); break;
    case DKV_F16: rc = launch_rp<DKV_F16>(rp, b, n_problems, n_kprob, max_probes, k_tiles, st); break;
    default: rc = launch_rp<DKV_F32>(rp, b, n_problems, n_kprob, max_probes, k_tiles, st); break;
  }
  return rc;
}
