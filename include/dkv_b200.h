/*
 * dkv_b200.h — C ABI of the B200 (sm_100a) KV-cache patch kernels.
 *
 * Every entry point is stream-ordered on the caller's stream, allocates nothing,
 * synchronises nothing, and returns an int status (DKV_OK = 0, negative on error).
 * All pointers are device pointers unless a field says "host".  Tensors are
 * described by a base pointer plus element strides; no framework types appear.
 *
 * Reference interfaces replaced (file:line within adityaraj-09/DeltaKV):
 *   dkv_scatter_paged      deltakv.paged.scatter_into_paged          src/deltakv/paged.py:8-43
 *   dkv_gather_paged       deltakv.paged.gather_from_paged           src/deltakv/paged.py:46-70
 *   dkv_pack_exact_factors LowRankFactors.codes/.apply operands      src/deltakv/deltas/factors.py:61-67
 *   dkv_subspace_correct   deltakv.patches.subspace.subspace_correct src/deltakv/patches/subspace.py:45-106
 *   dkv_subspace_correct_batched  the per-layer loop over it in apply_probe_to_cache
 *                          src/deltakv/patches/probe.py:112-165
 *   dkv_subspace_probe_residual  the probe residual R[P] whose SVD is svd_basis's input
 *                          src/deltakv/patches/subspace.py:37-42,69-73
 *   dkv_kivi_*             KIVI int4 cache (the reference has only the fake-quant
 *                          metrics._minmax_quantize, src/deltakv/metrics.py:115-132)
 *   dkv_exact_patch_paged  exact_kv_patch + LowRankKVPatch.materialize + scatter_into_paged,
 *                          as driven by DeltaKVEngine._patch (exact branch) and
 *                          DeltaKVConnector.patch_paged
 *                          src/deltakv/patches/exact.py:14-94, patches/tensors.py:105-123,
 *                          patches/compose.py:29-34, engine.py:263-288, connectors/vllm.py:70-81
 *
 * The reference has no FFI of its own (it is pure Python/PyTorch); these are the
 * entry points its Python operators bind through ctypes.
 */
#ifndef DKV_B200_H
#define DKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t; NULL selects the legacy default stream. */
typedef struct CUstream_st *dkv_stream_t;

/* ---- status codes ------------------------------------------------------- */
#define DKV_OK 0
#define DKV_ERR_INVALID_ARGUMENT (-1)
#define DKV_ERR_BLOCK_TABLE_SHORT (-2) /* "block_table shorter than prefix" (paged.py:27-28) */
#define DKV_ERR_LAYOUT (-3)            /* "unsupported paged KV layout" (paged.py:36-37)   */
#define DKV_ERR_UNSUPPORTED (-4)       /* shape / dtype combination not built             */
#define DKV_ERR_ALIGNMENT (-5)         /* pointer or stride alignment (TMA needs 16 B)    */
#define DKV_ERR_ROPE_RANGE (-6)        /* "seq_len exceeds RoPE cache" (rope.py:48-49)     */
#define DKV_ERR_BASIS_DIM (-7)         /* "basis d != kv d" (subspace.py:76-77)            */
#define DKV_ERR_CUDA (-8)              /* a CUDA runtime call failed                      */
#define DKV_ERR_TIMEOUT (-9)           /* a bounded device-side wait gave up              */
#define DKV_ERR_PAGE_RANGE (-10)       /* block id outside [0, num_blocks)                */
#define DKV_ERR_WORKSPACE (-11)        /* workspace too small                             */

/* ---- element types ------------------------------------------------------ */
#define DKV_F32 0
#define DKV_F16 1
#define DKV_BF16 2
#define DKV_E4M3 3 /* float8 e4m3fn */
#define DKV_I32 4
#define DKV_U8 5

/* Upper bound on layers covered by one dkv_exact_patch_paged launch. */
#define DKV_MAX_LAYERS 128

/* Human-readable text of a status code (static storage). */
const char *dkv_status_string(int status);
/* ABI version: bumped when a struct below changes.  2: dkv_exact_patch_args ends with x_sumsq and
   x_sumsq_layer_stride (a caller built against version 1 passes a shorter struct). */
int dkv_abi_version(void);
/* Text of the last CUDA runtime failure behind a DKV_ERR_CUDA on this thread ("" if none). */
const char *dkv_last_cuda_error(void);

/*
 * A paged KV cache of one layer for one of K or V.  Element (block, slot, head, dim)
 * lives at base + block*stride_block + slot*stride_slot + head*stride_head + dim
 * (strides in elements, dim stride 1).  The three layouts the reference accepts
 * (paged.py:18-37) — [nb,bs,h,d], [2,nb,bs,h,d][kv], [nb,2,bs,h,d][:,kv] — are all
 * this struct with different base/strides.  A dense [seq, h, d] tensor is the case
 * num_blocks=1, block_size=seq, block table {0}.
 */
typedef struct dkv_paged_cache {
  void *base;
  int32_t dtype; /* DKV_F32 / DKV_F16 / DKV_BF16 */
  int32_t block_size;
  int32_t n_heads;
  int32_t head_dim;
  int64_t num_blocks;
  int64_t stride_block;
  int64_t stride_slot;
  int64_t stride_head;
} dkv_paged_cache;

/*
 * A batch of sequences.  Token i of sequence b is row cu_seqlens[b] + i of the
 * token-major inputs, sits in block block_tables[b*table_stride + i/block_size]
 * at slot i % block_size (paged.py:39-43), and has RoPE position positions[row]
 * (or i when positions is NULL, rope.py:59-60).
 */
typedef struct dkv_seq_batch {
  const int32_t *cu_seqlens;   /* [n_seqs+1], non-decreasing, cu_seqlens[0] = 0          */
  const int32_t *block_tables; /* [n_seqs, table_stride]                                  */
  const int32_t *table_lens;   /* [n_seqs] valid entries per row, or NULL = table_stride  */
  const int32_t *positions;    /* [total rows] or NULL                                    */
  int64_t table_stride;
  int32_t n_seqs;
  int32_t max_seq_len; /* host-known bound on any sequence length (grid sizing)           */
} dkv_seq_batch;

/*
 * pages[block, slot] += delta[row]  (additive, in place), rounding once from
 * fp32(page) + fp32(delta) to the page dtype — bit-identical to the reference's
 * `pages[bid,:span] = pages[bid,:span] + delta[start:end]` (paged.py:43).
 * delta element (row, head, dim) at delta + row*delta_stride_row + head*delta_stride_head + dim.
 * Device-side range errors are written to *status (first error wins; may be NULL).
 */
int dkv_scatter_paged(const void *delta, int32_t delta_dtype, int64_t delta_stride_row,
                      int64_t delta_stride_head, const dkv_paged_cache *cache,
                      const dkv_seq_batch *seqs, int32_t *status, dkv_stream_t stream);

/* out[row] = pages[block, slot]  (paged.py:46-70), converted to out_dtype. */
int dkv_gather_paged(const dkv_paged_cache *cache, const dkv_seq_batch *seqs, void *out,
                     int32_t out_dtype, int64_t out_stride_row, int64_t out_stride_head,
                     int32_t *status, dkv_stream_t stream);

/*
 * Per-layer sums of the measured patch error (compose.py:147-163 measured_error): for layer l
 * (pages[l], same geometry as pages[0]) and every token of `seqs`,
 *   sums[2l]   += sum (page - fresh)^2,   sums[2l+1] += sum fresh^2
 * with fresh element (l, row, head, dim) at fresh + l*fresh_layer_stride + row*fresh_row_stride
 * + head*fresh_head_stride + dim.  The caller zeroes sums; the per-layer error is
 * (sqrt(sK0) + sqrt(sV0)) / (sqrt(sK1) + sqrt(sV1) + 1e-8) over a K call and a V call.
 */
int dkv_paged_error_sums(const dkv_paged_cache *pages, int32_t n_layers, const void *fresh,
                         int32_t fresh_dtype, int64_t fresh_layer_stride, int64_t fresh_row_stride,
                         int64_t fresh_head_stride, const dkv_seq_batch *seqs, double *sums,
                         int32_t *status, dkv_stream_t stream);

/* The same walk with four sums per layer for compare_kv (metrics.py:60-81):
   sums[4l] += sum (page - fresh)^2, sums[4l+1] += sum fresh^2, sums[4l+2] += sum page*fresh,
   sums[4l+3] += sum page^2 — relative L2 = sqrt(s0) / (sqrt(s1) + 1e-8) and cosine =
   s2 / max(sqrt(s3) sqrt(s1), 1e-8).  The caller zeroes sums. */
int dkv_paged_compare_sums(const dkv_paged_cache *pages, int32_t n_layers, const void *fresh,
                           int32_t fresh_dtype, int64_t fresh_layer_stride, int64_t fresh_row_stride,
                           int64_t fresh_head_stride, const dkv_seq_batch *seqs, double *sums,
                           int32_t *status, dkv_stream_t stream);

/*
 * Stored-activation writer.  The reference keeps HiddenSnapshot.h in the model dtype
 * (model.py:157-164; config.py:31 names float16 storage but nothing applies it).  This
 * quantises rows of x (F32/F16/BF16) into out (DKV_F16 with a power-of-two row scale, or
 * DKV_E4M3 with scale = max|x|/448): out[r,c] = x[r,c]/scale[r]; columns
 * [cols, out_cols) are zero-filled so rows can be padded to 16 bytes.
 */
int dkv_quantize_rows(const void *x, int32_t x_dtype, int64_t rows, int64_t cols,
                      int64_t x_row_stride, void *out, int32_t out_dtype, int64_t out_row_stride,
                      int64_t out_cols, float *scale, dkv_stream_t stream);
/* The same, also writing sumsq[r] = sum of the squared stored codes of row r (fp32): with
   the codes' scale, RMSNorm's sum(x^2) = scale^2 * sumsq, which dkv_exact_patch_args.x_sumsq
   takes so the patch forms no X.X^T product. */
int dkv_quantize_rows_sumsq(const void *x, int32_t x_dtype, int64_t rows, int64_t cols,
                            int64_t x_row_stride, void *out, int32_t out_dtype, int64_t out_row_stride,
                            int64_t out_cols, float *scale, float *sumsq, dkv_stream_t stream);

/* ---- exact / zeroth-order patch (fused) --------------------------------- */

/*
 * LoRA factors of the k_proj / v_proj maps of n_layers layers (PEFT convention,
 * factors.py:11-75): A [rank, d_model], B [n_kv*head_dim, rank], dW = scale*B@A.
 * Layer l's A starts at a + l*a_layer_stride (elements), row-major contiguous.
 * rank = 0 (or NULL pointers) means that projection has no delta (exact.py:46-53).
 * norm_weight (optional, [n_layers, d_model] via norm_layer_stride) is the attn RMSNorm
 * weight; when given it is folded into A so that the patch consumes pre-norm X
 * (model.py:48-56,310-314).
 */
typedef struct dkv_lora_factors {
  const void *a_k, *b_k, *a_v, *b_v;
  int32_t dtype; /* DKV_F32 / DKV_F16 / DKV_BF16 for all four */
  int32_t rank_k, rank_v;
  int32_t n_layers;
  float scale_k, scale_v;
  int64_t a_k_layer_stride, b_k_layer_stride, a_v_layer_stride, b_v_layer_stride;
  const void *norm_weight;
  int32_t norm_dtype;
  int64_t norm_layer_stride;
} dkv_lora_factors;

/* Geometry shared by packing and patching. */
typedef struct dkv_exact_geometry {
  int32_t d_model;
  int32_t n_kv_heads;
  int32_t head_dim; /* 16, 32 or a multiple of 64 up to 256 */
  int32_t x_dtype;  /* DKV_E4M3 or DKV_F16: the stored-activation format */
  int32_t rank_k;   /* 0..64 */
  int32_t rank_v;   /* 0..64 */
} dkv_exact_geometry;

/* Bytes of the packed-factor image of one layer (a multiple of 256). */
int dkv_exact_packed_bytes(const dkv_exact_geometry *geom, int64_t *bytes_per_layer);

/*
 * Convert factors to the kernel's tensor-core operand image: f16 with per-matrix
 * power-of-two scaling, RMSNorm weight folded into A, fragment-ordered.  `packed`
 * receives n_layers images, image l at packed + l*packed_layer_stride bytes.
 */
int dkv_pack_exact_factors(const dkv_exact_geometry *geom, const dkv_lora_factors *factors,
                           void *packed, int64_t packed_layer_stride, dkv_stream_t stream);

typedef struct dkv_exact_patch_args {
  dkv_exact_geometry geom;
  /* stored activations X: element (layer l, row t, k) at x + l*x_layer_stride + t*x_row_stride + k
     (elements of x_dtype); rows are the tokens of `seqs`. Base 16-B aligned, strides*elem % 16 == 0. */
  const void *x;
  int64_t x_layer_stride, x_row_stride, x_rows;
  /* optional per-token dequantisation scale (fp32), element (l, t) at x_scale + l*x_scale_layer_stride + t */
  const float *x_scale;
  int64_t x_scale_layer_stride;
  int32_t apply_norm; /* 1: X is pre-norm; RMSNorm(x)*w is applied (w folded into packed) */
  float norm_eps;
  /* packed factor images (dkv_pack_exact_factors), layer l at packed + l*packed_layer_stride */
  const void *packed;
  int64_t packed_layer_stride;
  /* RoPE tables [rope_max_pos, head_dim/2] fp32 (cos, sin of position*inv_freq) or NULL: no RoPE on K */
  const float *rope_cos, *rope_sin;
  int32_t rope_max_pos;
  int32_t n_layers; /* <= DKV_MAX_LAYERS */
  dkv_seq_batch seqs;
  /* per-layer caches: K and V pages of layer l (host arrays of n_layers entries); only
     base differs between layers, the rest is taken from k_pages[0] / v_pages[0] */
  const dkv_paged_cache *k_pages;
  const dkv_paged_cache *v_pages;
  int32_t accumulate; /* 1: pages += delta (read-add-write); 0: pages = delta */
  int32_t *status;    /* optional device status word */
  /* optional, with apply_norm: per-row sum of the squared stored codes (fp32, (l, t) at
     x_sumsq + l*x_sumsq_layer_stride + t), as dkv_quantize_rows_sumsq writes it beside the
     codes; the RMSNorm then uses it instead of forming X.X^T's diagonal on the tensor
     cores.  The sums must come from the same codes as x: nothing checks that, and stale
     sums silently give a wrong norm.  Ignored without apply_norm.  NULL: formed here. */
  const float *x_sumsq;
  int64_t x_sumsq_layer_stride;
} dkv_exact_patch_args;

/*
 * For every layer l and token t of every sequence:
 *   x  = dequant(X[l,t]) (optionally RMSNorm(x)*w_l)
 *   dK = RoPE_pos(t)( scale_k * (x @ A_k^T) @ B_k^T ),  dV = scale_v * (x @ A_v^T) @ B_v^T
 *   K_pages[l][block(t), slot(t)] (+)= dK,  V_pages[l][...] (+)= dV
 * in one persistent launch: X streamed by TMA, both products on tensor cores with the
 * rank-r codes kept in registers, RoPE and the page read-add-write fused.
 */
int dkv_exact_patch_paged(const dkv_exact_patch_args *args, dkv_stream_t stream);

/* ---- dense-delta patch (RL step: full-rank dW on k_proj / v_proj) ------------------ */

/*
 * The reference expresses a dense weight delta through the exact route with
 * LowRankFactors(A = dW, B = I, scale = 1) (patches/exact.py:14-63, factors.py:61-67):
 * dK = RoPE(x @ dW_K^T), dV = x @ dW_V^T.  Here dW_K and dW_V are packed once per delta
 * into one bf16 operand and the patch is one tensor-core GEMM launch per call.
 */
typedef struct dkv_dense_geometry {
  int32_t d_model;    /* multiple of 64 */
  int32_t n_kv_heads;
  int32_t head_dim;   /* 32, 64 or 128 */
} dkv_dense_geometry;

/*
 * dW_K, dW_V [n_kv*head_dim, d_model] row-major (either may be NULL: zero delta), layer l
 * at dw + l*layer_stride elements.  Optional RMSNorm weight [n_layers, d_model] is folded in
 * (dW . diag(w)), so the patch consumes pre-norm X with x_scale = 1/rms(x)
 * (dkv_row_inv_rms).  scale_k / scale_v multiply the deltas.
 */
typedef struct dkv_dense_delta {
  const void *dw_k, *dw_v;
  int32_t dtype; /* DKV_F32 / DKV_F16 / DKV_BF16 */
  int32_t n_layers;
  int64_t dw_k_layer_stride, dw_v_layer_stride;
  const void *norm_weight;
  int32_t norm_dtype;
  int64_t norm_layer_stride;
  float scale_k, scale_v;
} dkv_dense_delta;

/* packed: n_layers bf16 images [2*n_kv*head_dim, d_model] (K rows, then V rows), layer l at
   packed + l*packed_layer_stride elements (>= 2*n_kv*head_dim*d_model, multiple of 8). */
int dkv_pack_dense_delta(const dkv_dense_geometry *geom, const dkv_dense_delta *dw, void *packed,
                         int64_t packed_layer_stride, dkv_stream_t stream);

typedef struct dkv_dense_patch_args {
  dkv_dense_geometry geom;
  /* stored activations X, bf16: element (l, t, k) at x + l*x_layer_stride + t*x_row_stride + k */
  const void *x;
  int64_t x_layer_stride, x_row_stride, x_rows;
  /* optional per-token multiplier of the product (fp32, (l, t) at x_scale + l*x_scale_layer_stride + t) */
  const float *x_scale;
  int64_t x_scale_layer_stride;
  const void *packed; /* dkv_pack_dense_delta output */
  int64_t packed_layer_stride;
  const float *rope_cos, *rope_sin; /* [rope_max_pos, head_dim/2] or NULL: no RoPE on K */
  int32_t rope_max_pos;
  int32_t n_layers;
  int32_t do_k, do_v; /* which projections to patch */
  dkv_seq_batch seqs;
  const dkv_paged_cache *k_pages; /* per layer, bf16 or f16; layouts as for the exact patch */
  const dkv_paged_cache *v_pages;
  int32_t accumulate;
  int32_t *status;
} dkv_dense_patch_args;

/*
 * For every layer l and token t:  dK = RoPE_pos(t)(x_scale * X[l,t] @ W_K^T),
 * dV = x_scale * X[l,t] @ W_V^T, pages (+)= dK / dV — a persistent tcgen05 GEMM (bf16 in,
 * fp32 accumulate in tensor memory) with RoPE and the paged read-add-write in its epilogue.
 */
int dkv_dense_patch_paged(const dkv_dense_patch_args *args, dkv_stream_t stream);

/* out[r] = 1/sqrt(mean_c(x[r,c]^2) + eps) (fp32), the RMSNorm row factor (model.py:48-56). */
int dkv_row_inv_rms(const void *x, int32_t x_dtype, int64_t rows, int64_t cols, int64_t x_row_stride,
                    float eps, float *out, dkv_stream_t stream);

/* ---- KIVI-style int4 KV cache ---------------------------------------------- */

#define DKV_KIVI_PER_CHANNEL 0 /* K: groups of 32 consecutive tokens of one channel */
#define DKV_KIVI_PER_TOKEN 1   /* V: groups of 32 consecutive channels of one token */

/*
 * One int4 K or V tensor of n_tokens x d (d % 32 == 0): codes [n_tokens, d/2] bytes (even
 * channel in the low nibble; per-token rows 16-B aligned), fp16 scale and zero per group —
 * PER_TOKEN: [n_tokens, d/32], PER_CHANNEL: [ceil(n_tokens/32), d] (row stride
 * sz_row_stride elements, shared by scale and zero).  x = q*scale + zero with
 * scale = max(hi-lo, 1e-8)/15 and zero = lo rounded to fp16 before q = clamp(rint((x-zero)/
 * scale), 0, 15); a partial last K group covers the remaining tokens.  This format is this
 * library's; the reference's int4 arithmetic is the fake-quant metrics._minmax_quantize.
 */
typedef struct dkv_kivi_cache {
  void *codes;
  void *scale, *zero;
  int64_t code_row_stride; /* bytes */
  int64_t sz_row_stride;   /* elements */
  int64_t n_tokens, d;
  int32_t mode;
} dkv_kivi_cache;

/* out = int4(x);  x is F32/F16/BF16 [n_tokens, d] with row stride x_row_stride elements. */
int dkv_kivi_quantize(const void *x, int32_t x_dtype, int64_t x_row_stride, const dkv_kivi_cache *out,
                      dkv_stream_t stream);
/* x = dequant(in) */
int dkv_kivi_dequantize(const dkv_kivi_cache *in, void *x, int32_t x_dtype, int64_t x_row_stride,
                        dkv_stream_t stream);
/* out = int4(dequant(base) + delta) — the int4 form of a KV patch; out may be base itself. */
int dkv_kivi_patch(const dkv_kivi_cache *base, const void *delta, int32_t delta_dtype,
                   int64_t delta_row_stride, const dkv_kivi_cache *out, dkv_stream_t stream);

/* out[i, :] = fresh[rows[i], :] - dequant(base)[rows[i], :] as fp32 (the probe residual of
   the subspace route's K basis, subspace.py:86-93, read straight from the int4 cache). */
int dkv_kivi_probe_residual(const dkv_kivi_cache *base, const void *fresh, int32_t fresh_dtype,
                            int64_t fresh_row_stride, const int32_t *rows, int64_t n_rows, float *out,
                            int64_t out_row_stride, int32_t *status, dkv_stream_t stream);

/* The same for many caches at once (all layers of an adapter view): job j reads jobs[j].base,
   jobs[j].fresh and its own probe rows (n_rows each) and writes
   out + j * out_job_stride (fp32 [n_rows, d], row stride out_row_stride).  All jobs share d
   (a multiple of 32) and the fresh dtype; 16-byte aligned fresh rows and out. */
typedef struct dkv_kivi_probe_job {
  dkv_kivi_cache base;
  const void *fresh;
  int64_t fresh_row_stride; /* elements */
  const int32_t *rows;
} dkv_kivi_probe_job;
int dkv_kivi_probe_residual_batched(const dkv_kivi_probe_job *jobs, int32_t n_jobs, int32_t fresh_dtype,
                                    int64_t n_rows, float *out, int64_t out_job_stride, int64_t out_row_stride,
                                    int32_t *status, dkv_stream_t stream);

/* ---- subspace route -------------------------------------------------------- */

/* ---- probe scoring and the residual gate ------------------------------------------ */

/* out[t] (+)= || scale * x[t] @ A^T ||  for A [rank, d] fp32 row-major (rank <= 64): the per-token
   adapter activation of lora_activation_scores (patches/exact.py:111-115); summed over the
   projections of a layer it is weight_axis_scores (patches/probe.py:30-47). */
int dkv_lora_scores(const void *x, int32_t x_dtype, int64_t rows, int64_t d, int64_t x_row_stride,
                    const float *a, int32_t rank, float scale, float *out, int32_t accumulate,
                    dkv_stream_t stream);

/* out[i] = || a[r_i] - b[r_i] || (fp32), r_i = rows[i] or i when rows is NULL: the per-token
   residual estimates of residual_gate (patches/probe.py:85-109). */
int dkv_row_diff_norms(const void *a, const void *b, int32_t dtype, int64_t n_rows, int64_t cols,
                       int64_t a_row_stride, int64_t b_row_stride, const int32_t *rows, int64_t n_out,
                       float *out, int32_t *status, dkv_stream_t stream);

/*
 * Analytic route (Route A, patches/analytic.py).  First-order causal attention without the
 * [H, n, n] matrices (attention_first_order's core, analytic.py:85-99): for each query head h
 * and its GQA kv head h / (n_heads / n_kv_heads), with S = q k^T * scale (causal),
 * A = softmax(S), dS = (dq k^T + q dk^T) * scale, dA = A (.) (dS - rowsum(A (.) dS)):
 *   dctx = dA v + A dv,  ctx = A v (ctx may be NULL).
 * q, dq: [n, n_heads, head_dim] (row stride q_row_stride elements); k, dk, v, dv:
 * [n, n_kv_heads, head_dim] (kv_row_stride); dtype F32, BF16 or F16; outputs fp32
 * [n, n_heads, head_dim] with row stride out_row_stride; head_dim 16/32/64/128.  head_dim 64
 * and 128 run on tensor cores in a three-term bf16 split (fp32-level accuracy, ~5e-6
 * relative), 16 and 32 in fp32 SIMT arithmetic.
 */
int dkv_attn_first_order(const void *q, const void *dq, int64_t q_row_stride, const void *k, const void *dk,
                         const void *v, const void *dv, int64_t kv_row_stride, int32_t dtype, int32_t n_tokens,
                         int32_t n_heads, int32_t n_kv_heads, int32_t head_dim, float scale, float *ctx,
                         float *dctx, int64_t out_row_stride, dkv_stream_t stream);
/* y = RMSNorm(x) and its first-order image dy under dx (rmsnorm_first_order,
   analytic.py:245-262); fp32 rows of d elements. */
int dkv_rmsnorm_first_order(const float *x, const float *dx, const float *w, float eps, int64_t rows, int32_t d,
                            int64_t x_row_stride, int64_t dx_row_stride, float *y, float *dy,
                            int64_t y_row_stride, int64_t dy_row_stride, dkv_stream_t stream);
/* h = silu(g) u, dh = silu'(g) dg u + silu(g) du, elementwise over n fp32 values
   (mlp_first_order's SwiGLU, analytic.py:108-138). */
int dkv_swiglu_first_order(const float *g, const float *u, const float *dg, const float *du, int64_t n, float *h,
                           float *dh, dkv_stream_t stream);
/* In place: x = x cos + rotate_half(x) sin at positions 0..rows-1 (rope.py:9-63) for fp32
   x [rows, heads, head_dim] (row stride elements); cos/sin are half-width [table_rows, head_dim/2]. */
int dkv_rope_rows(float *x, int64_t rows, int32_t heads, int32_t head_dim, int64_t row_stride,
                  const float *cos_half, const float *sin_half, int64_t table_rows, dkv_stream_t stream);

/* Eigendecomposition of `batch` symmetric k x k fp64 matrices (k <= 96; matrix b at
   a + b * a_stride, row-major, only its symmetric part is used) by parallel cyclic Jacobi:
   evals [batch, k] descending, evecs [batch, k, k] row-major with column j the unit
   eigenvector of evals[b, j], info[b] = 0 converged, 1 not converged within max_sweeps,
   2 non-finite input.  The Rayleigh-Ritz step of the K basis that stands in for svd_basis
   (patches/subspace.py:37-42) on the device. */
int dkv_sym_eig_batched(const double *a, int64_t batch, int32_t k, int64_t a_stride, int32_t max_sweeps,
                        double *evals, double *evecs, int32_t *info, dkv_stream_t stream);

/* Block subspace iteration on a symmetric positive semi-definite fp64 matrix g [d, d]
   (row-major, exactly symmetric): `iters` steps of q <- orth(g q) by Cholesky QR, q [d, k]
   row-major (k <= 96, k <= d) holding the start block on entry and the orthonormal result on
   return; then, if t is not NULL, t [k, k] = q^T g q (the Rayleigh quotient) and y = g q.
   Workspace: y [d, k], w [2, k, k] (fp64).  status (device int32, zeroed here) gets bit 0 when
   a Cholesky pivot is not finite or falls below 1e-12 of the first (the block lost rank);
   the result is then not usable.  The top-k eigen-subspace of the Gram matrix dX^T dX that
   stands in for the SVD of rank_truncate (patches/analytic.py:14-22). */
int dkv_gram_subspace_iterate(const double *g, int32_t d, double *q, int32_t k, int32_t iters, double *y,
                              double *w, double *t, int32_t *status, dkv_stream_t stream);

/* c[i] = op(a[i]) b[i] for i < batch, fp32 in and out, on the tensor cores with every operand
   split into two bf16 terms (products lo*hi + hi*lo + hi*hi, fp32 accumulation; within ~1e-5
   relative of an fp32 product).  a[i] is [m, k] row-major (lda) or, with trans_a, stored
   [k, m] row-major (lda) and used transposed; b[i] is [k, n], c[i] is [m, n], row-major.
   n is a multiple of 16, at most 96 (pad with zero columns); a and b 16-byte aligned, c 8-byte;
   lda, ldb and the batch strides of a and b multiples of 4, ldc and c's batch stride even;
   k % 4 == 0 (m % 4 == 0 with trans_a).  The thin products X Q, X^T (X Q) of the subspace
   iteration and the Rayleigh-Ritz step that stand in for svd_basis (patches/subspace.py:37-42),
   X the probe residual of one layer. */
int dkv_split_gemm_batched(const float *a, int64_t a_batch_stride, int64_t lda, int32_t trans_a, const float *b,
                           int64_t b_batch_stride, int64_t ldb, float *c, int64_t c_batch_stride, int64_t ldc,
                           int64_t batch, int32_t m, int32_t n, int32_t k, dkv_stream_t stream);

/*
 * Subspace correction of a KIVI int4 cache (the multi-adapter maintenance step): for each
 * problem (one layer's K or V of one adapter view), reused = dequant(base), then exactly
 * subspace_correct (patches/subspace.py:45-106) — R = fresh - reused, codes =
 * solve(B^T B + 1e-6 I, (R B)^T)^T, orth_mu = mean_P(R - codes B^T),
 * w = min(||R|| / mean ||R||, 1), corr = reused + codes B^T + w orth_mu, corr[P] = fresh[P] —
 * and out = KIVI-quantised corr (same grouping as base; out may be base itself).  Without a
 * basis, or with no probe, corr = reused + w mean_P(R) as in the reference.  Probe indices
 * are deduplicated.  All problems of one call share d (a multiple of 64) and the fresh
 * dtype; at most 112 problems, ranks <= 64.  The basis products run on tensor cores with
 * bf16 operands (the basis, R and the codes rounded to bf16) and fp32 accumulation.
 */
typedef struct dkv_kivi_subspace_problem {
  dkv_kivi_cache base; /* reused KV, int4 */
  dkv_kivi_cache out;  /* corrected KV, int4, same mode and size */
  const void *fresh;   /* [n_tokens, d], row stride fresh_row_stride elements */
  int32_t fresh_dtype; /* DKV_F32 / DKV_F16 / DKV_BF16 */
  int64_t fresh_row_stride;
  const int32_t *probe_index;
  int64_t n_probes;
  const float *basis; /* [d, rank] fp32 row-major, or NULL */
  int32_t rank;
  float *subspace_out, *orth_mu_out; /* optional [d] fp32 */
} dkv_kivi_subspace_problem;

int dkv_kivi_subspace_workspace_bytes(const dkv_kivi_subspace_problem *problems, int32_t n_problems,
                                      int64_t *bytes);
int dkv_kivi_subspace_correct(const dkv_kivi_subspace_problem *problems, int32_t n_problems,
                              void *workspace, int64_t workspace_bytes, int32_t *status,
                              dkv_stream_t stream);

/*
 * One subspace_correct problem (subspace.py:45-106) on [n_tokens, d] views of the reused
 * and fresh K or V (d = n_kv*head_dim; row strides in elements):
 *   R = fresh - reused; codes = (R B)(B^T B + 1e-6 I)^-1; fitted = codes B^T;
 *   subspace = mean(codes) B^T; orth_mu = mean_P(R - fitted);
 *   w_j = token_weights[j] or min(||R_j|| / mean ||R||, 1);
 *   corrected = reused + fitted + w * orth_mu, corrected[P] = fresh[P].
 * rank = 0 (basis NULL) is the reference's unstructured branch: corrected = reused +
 * w * mean_P(R), subspace = 0.  basis is fp32 [d, rank] row-major, rank <= 64.
 * subspace_out / orth_mu_out (fp32 [d]) may be NULL.  Scratch: workspace of at least
 * dkv_subspace_workspace_bytes(n_tokens, d, rank); nothing in it needs clearing.
 * probe_index entries must lie in [0, n_tokens) (checked by the Python drop-in; the kernels
 * skip others).  These calls have no status word: a device-side wait that gives up (bounded,
 * ~1-2 s; it happens only on a broken device) leaves the outputs undefined unreported.
 */
typedef struct dkv_subspace_args {
  const void *reused, *fresh;
  int32_t kv_dtype; /* DKV_F32 / DKV_F16 / DKV_BF16 */
  int64_t n_tokens, d;
  int64_t reused_row_stride, fresh_row_stride;
  const int32_t *probe_index;
  int64_t n_probes;
  const float *basis;
  int32_t rank;
  const float *token_weights;
  void *corrected;
  int32_t out_dtype;
  int64_t out_row_stride;
  float *subspace_out, *orth_mu_out;
  void *workspace;
  int64_t workspace_bytes;
} dkv_subspace_args;

int dkv_subspace_workspace_bytes(int64_t n_tokens, int64_t d, int32_t rank, int64_t *bytes);
int dkv_subspace_correct(const dkv_subspace_args *args, dkv_stream_t stream);
/*
 * n independent dkv_subspace_correct problems in one set of launches — the reference's
 * per-layer K / V loop of apply_probe_to_cache (src/deltakv/patches/probe.py:112-165) as one
 * call.  Every problem: n_tokens > 0, d a multiple of 32 and the same for all, the same
 * kv_dtype, 16-byte aligned reused / fresh / corrected with rows of a multiple of 16 bytes,
 * rank <= 64; at most 112 problems.  Otherwise both functions return DKV_ERR_UNSUPPORTED and
 * nothing runs (call dkv_subspace_correct per problem instead).  Each problem's own
 * workspace fields are ignored: the call uses `workspace`, at least
 * dkv_subspace_correct_batched_workspace_bytes(args, n) bytes, 16-byte aligned.
 */
int dkv_subspace_correct_batched_workspace_bytes(const dkv_subspace_args *args, int32_t n, int64_t *bytes);
int dkv_subspace_correct_batched(const dkv_subspace_args *args, int32_t n, void *workspace,
                                 int64_t workspace_bytes, dkv_stream_t stream);
/*
 * dkv_subspace_correct without a caller workspace and without any allocation.  It has no
 * counterpart in the reference; it exists for callers that cannot allocate device memory
 * when they need a correction (a serving framework that owns all device memory through its
 * own pool, a plugin handed only its input and output buffers, a thread that must not
 * wait on the allocator).  The scratch is one fixed 16 MiB device array inside this
 * library, present on every GPU that loads it until the process exits; args->workspace
 * and args->workspace_bytes are ignored.
 *   - Limit: the scratch of one of the two forms must fit in 16 MiB.  The tensor-core form
 *     (d a multiple of 32, 16-byte rows) needs about 4*r + 12 + (r + 1)/8 bytes per token
 *     plus about 12*(r + 1)*d bytes (r = rank rounded up to a multiple of 16): about 58K tokens
 *     at rank 64 and 212K at rank 16 for d = 1024; the general form needs 4*r + 5 bytes per
 *     token plus a few KB: about 64K tokens at rank 64 and 240K at rank 16.  A problem
 *     between the two limits runs on the general kernels; larger problems are rejected
 *     with DKV_ERR_WORKSPACE before anything is launched.  (dkv_subspace_workspace_bytes
 *     reports the larger of the two needs.)
 *   - The first call made while a given device is current looks up the array's device
 *     address (cudaGetSymbolAddress) and caches it; make that first call before any
 *     stream capture on that device.
 *   - All calls on a device share the one array and each leaves its contents behind (the
 *     entry point clears what must start at zero itself).  Calls whose work overlaps on
 *     the GPU — on different streams, or from different host threads — race on it:
 *     order them on one stream.
 */
int dkv_subspace_correct_noalloc(const dkv_subspace_args *args, dkv_stream_t stream);
/* out[i, :] = fresh[probe_index[i], :] - reused[probe_index[i], :] as fp32 [n_probes, d]. */
int dkv_subspace_probe_residual(const void *reused, const void *fresh, int32_t kv_dtype,
                                int64_t reused_row_stride, int64_t fresh_row_stride,
                                int64_t n_tokens, int64_t d, const int32_t *probe_index,
                                int64_t n_probes, float *out, dkv_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DKV_B200_H */
