/*
 * h3b.h -- C ABI of libh3b.so, the sm_100a (B200) kernels of the X-MinimaxH3
 * DiT-block hot path: per-token INT8 activation quantization (optionally fused
 * with RMSNorm + AdaLN and the ConvRot rotation), tcgen05 INT8 GEMMs with a
 * fused dequant / bias / gated-residual epilogue, the W4A8 weight decode, and
 * the SageAttention-style quantized attention with its Sparge block mask.
 *
 * Conventions (mirroring the comfy_kitchen launchers each entry replaces):
 *  - plain pointers to device memory and int64 sizes; no framework types;
 *  - the caller allocates every output and workspace; nothing here allocates
 *    device memory;
 *  - every launch is asynchronous on the caller's `stream` (a cudaStream_t,
 *    0 = legacy default stream);
 *  - every entry returns an int status: H3B_OK or a negative H3B_ERR_* code,
 *    with a message for the calling thread in h3b_last_error().  Nothing
 *    throws across this boundary (the reference launchers could, e.g.
 *    comfy_kitchen backends/cuda/ops/int8_linear.cu:1311-1322).
 *  - kernels that wait on hardware barriers give up after a bounded time and
 *    record a code in a per-device status word read by h3b_device_status().
 *  - dtype codes: 0 = float32, 1 = float16, 2 = bfloat16 (comfy_kitchen
 *    backends/eager/quantization.py:34-42); bf16 is the only activation dtype
 *    the kernels take.
 * Head dimension is 128 throughout the attention entries (the reference's
 * NHD Sparge helpers require it: model/sparge_nhd.py:176-177).
 */
#ifndef H3B_H_
#define H3B_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3B_OK 0
#define H3B_ERR_INVALID_ARGUMENT -1
#define H3B_ERR_UNSUPPORTED -2
#define H3B_ERR_CUDA -3
#define H3B_ERR_NO_DEVICE -4
/* device status codes (h3b_device_status) */
#define H3B_STATUS_GEMM_TIMEOUT -101
#define H3B_STATUS_ATTN_TIMEOUT -102
#define H3B_STATUS_SELFTEST_TIMEOUT -103

/* ---------------------------------------------------------------- library */

/* Version string of this build. */
const char* h3b_version(void);

/* Message describing the last failing call on this thread ("" if none). */
const char* h3b_last_error(void);

/* Reads the device status word of `device` (0 = no kernel has reported a
 * problem) into *status; clears it when `reset` is non-zero.  Synchronizes
 * the device. */
int h3b_device_status(int device, int* status, int reset);

/* Exercises the kernels' bounded-wait failure path on purpose: one warp waits on a
 * hardware barrier that nothing will release, with the same wait routine the GEMM and
 * attention kernels use but a limit of `limit_ns` (at most 1 s); it gives up, records
 * H3B_STATUS_SELFTEST_TIMEOUT in the device status word and returns.  The CUDA context
 * stays usable.  For tests of the failure handling; no counterpart in the reference
 * (whose kernels do not bound their waits). */
int h3b_selftest_bounded_wait(int64_t limit_ns, void* stream);

/* ---------------------------------------------------------------- quantization */

/* Per-row dynamic INT8 quantization: scale[r] = max(|x[r,:]|)/127 (at least
 * 1e-30), q = rint(bf16(x / bf16(scale))) clamped to [-128, 127].
 * x: bf16 [rows, x_row_stride] (first `cols` columns used), q: int8 [rows, cols],
 * scales: f32 [rows].  cols % 16 == 0, cols <= 16384.
 * Replaces launch_quantize_int8_rowwise_kernel
 * (comfy_kitchen backends/cuda/ops/int8_linear.cu:1035-1084). */
int h3b_quantize_int8_rowwise(const void* x, int64_t rows, int64_t cols, int64_t x_row_stride, void* q,
                              void* scales, void* stream);

/* Fused input activation + ConvRot (normalized regular-Hadamard rotation of
 * every 256-column group, fp32) + per-row INT8 quantization.
 * input_act: 0 none, 1 gelu_tanh, 2 swiglu (x row = [gate | up], 2*cols wide).
 * x: bf16 [rows, x_row_stride]; q: int8 [rows, cols]; scales: f32 [rows].
 * group_size must be 256; cols % 256 == 0, cols <= 16384.
 * Replaces launch_quantize_int8_rowwise_convrot64 / _convrot_kernel
 * (int8_linear.cu:1086-1160, 1294-1408). */
int h3b_quantize_int8_rowwise_convrot(const void* x, int64_t rows, int64_t cols, int64_t x_row_stride,
                                      int group_size, int input_act, void* q, void* scales, void* stream);

/* RMSNorm(norm_weight, eps) + AdaLN modulation n*bf16(1+scale)+shift with the
 * reference's bf16 materialization points, then (convrot_group_size 256) the
 * ConvRot rotation or (0) nothing, then per-row INT8 quantization.
 * x: bf16 [rows, cols] (row stride x_row_stride); norm_weight: bf16 [cols];
 * scale_table / shift_table: bf16 [table_rows, cols]; segment_rows: int32
 * [rows] giving each token's table row, or NULL for row 0.
 * Replaces rms_adaln (model/kernels.py:7594-7642 -> backends/original/kernels/
 * fused_norm_rope.py:12-45, 398-429) followed by the quantizer above. */
int h3b_rms_adaln_quantize_int8(const void* x, int64_t rows, int64_t cols, int64_t x_row_stride,
                                const void* norm_weight, const void* scale_table, const void* shift_table,
                                const int32_t* segment_rows, float eps, int convrot_group_size, void* q,
                                void* scales, void* stream);

/* ---------------------------------------------------------------- GEMM */

/* D[m, n] = bf16( float(sum_k A[m,k] * B[n,k]) * xs[m] * ws[n] + bias[n] ),
 * int32 accumulation on tcgen05 (kind::i8) with TMEM accumulators.
 * A: int8 [M, K] row-major; B: int8 [N, K] row-major (K-major weights);
 * xs: f32 [M]; ws: f32 [N] or [1] (ws_numel 1 = scalar); bias: f32 [N] or NULL;
 * D: bf16 with row stride out_row_stride (elements).  out_dtype must be 2.
 * K % 16 == 0; A, B 16-byte aligned.
 * Replaces launch_cutlass_int8_dequant / _strided
 * (comfy_kitchen backends/cuda/ops/cutlass_gemm_int8.cu:612-666). */
int h3b_int8_gemm_dequant(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                          const void* bias, void* D, int64_t M, int64_t N, int64_t K, int64_t out_row_stride,
                          int out_dtype, void* stream);

/* The QKV projection with the q/k head norm and RoPE in its epilogue: D as
 * h3b_int8_gemm_dequant computes it, and on the Q heads (columns [q_offset,
 * q_offset + H*128)) and K heads ([k_offset, k_offset + H*128)) of every row the
 * transform of h3b_qk_rmsnorm_rope applied before the store -- bit-identical to
 * those two calls in sequence, without the second pass over the rows.
 * cos_table / sin_table: bf16 [M, rot_dim/2], row m for GEMM row m.
 * Returns H3B_ERR_UNSUPPORTED with nothing launched unless the shape runs the 2-SM
 * kernel (ceil(M/256) * ceil(N/256) >= the SM count), rot_dim is 96 or 128, the
 * offsets are multiples of 128 with both head ranges disjoint and inside N, and D,
 * the norm weights and the cos/sin tables are 16-byte aligned with
 * out_row_stride % 8 == 0; the caller then makes the two calls.  Replaces the QKV
 * projection followed by apply_qknorm_rope (model/layers.py:277-295, 72-149). */
int h3b_int8_gemm_dequant_qk_rope(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                                  const void* bias, void* D, int64_t M, int64_t N, int64_t K,
                                  int64_t out_row_stride, int64_t H, int64_t q_offset, int64_t k_offset,
                                  const void* q_weight, const void* k_weight, const void* cos_table,
                                  const void* sin_table, int rot_dim, float eps, void* stream);

/* FC1 of the GELU MLP with the first half of FC2's input quantizer in its
 * epilogue: the bf16 values h3b_int8_gemm_dequant would store go through tanh-GELU
 * and the ConvRot-256 rotation (every 256-column group), and are stored as bf16
 * rotated values in D; amax[m * amax_row_stride + 2 t + h] receives the fp32 absmax
 * of row m's rotated values in columns 256 t + 64 j + 32 h + [0, 32), j = 0..3 (256-column
 * tile t, half h; N / 128 entries per row, their max is the row's absmax).  Then
 * h3b_quantize_rotated_int8 forms the codes and row scales, bit-identical to
 * h3b_int8_gemm_dequant followed by h3b_quantize_int8_rowwise_convrot(input_act = 1).
 * Returns H3B_ERR_UNSUPPORTED with nothing launched unless the shape runs the 2-SM
 * kernel (ceil(M/256) * ceil(N/256) >= the SM count), N % 256 == 0, N <= 16384, D, ws
 * and bias are 16-byte aligned with out_row_stride % 8 == 0 and amax_row_stride >= N / 128; the
 * caller then makes those two calls.  Replaces the FC1 projection followed by the
 * FC2 input quantizer with input_act gelu_tanh (model/fused_mlp.py:269-426 feeding
 * comfy_kitchen int8_linear.cu:943-1030). */
int h3b_int8_gemm_gelu_convrot(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                               const void* bias, void* D, int64_t M, int64_t N, int64_t K, int64_t out_row_stride,
                               void* amax, int64_t amax_row_stride, void* stream);

/* Codes and row scales from rotated bf16 rows (the output of
 * h3b_int8_gemm_gelu_convrot): scale[r] = max(min(absmax, bf16 max) / 127, 1e-30)
 * with absmax the max of amax[r * amax_row_stride + c], c < amax_cols, and
 * q[r, k] = clamp(rint(bf16(rot[r, k] / bf16(scale[r]))), -128, 127).
 * rot: bf16 [rows, rot_row_stride]; q: int8 [rows, cols]; scales: f32 [rows].
 * cols % 8 == 0, cols <= 16384, rot and q 16-byte aligned, rot_row_stride % 8 == 0. */
int h3b_quantize_rotated_int8(const void* rot, int64_t rows, int64_t cols, int64_t rot_row_stride, const void* amax,
                              int64_t amax_row_stride, int64_t amax_cols, void* q, void* scales, void* stream);

/* As h3b_int8_gemm_dequant, but the bf16 result y[m,n] is added into a bf16
 * residual stream in place: residual[m,n] = bf16(residual + y * gate[n])
 * (gate: bf16 [N]).  Replaces int8_linear followed by residual.addcmul_
 * (model/fused_mlp.py:393-425; model/layers.py:944-960). */
int h3b_int8_gemm_gated_residual(const void* A, const void* B, const void* xs, const void* ws,
                                 int64_t ws_numel, const void* bias, const void* gate, void* residual,
                                 int64_t M, int64_t N, int64_t K, int64_t residual_row_stride, void* stream);

/* Raw int32 accumulators acc[m, n] = sum_k A[m,k] * B[n,k] (same tcgen05
 * pipeline), for bit-exact verification.  acc: int32 [M, N]. */
int h3b_int8_gemm_i32(const void* A, const void* B, void* acc, int64_t M, int64_t N, int64_t K, void* stream);

/* ---------------------------------------------------------------- W4A8 */

/* Grouped packed-int4 -> int8 grid: out[n,k] = clamp(rint(level * s_rel[n, k/G]), +-127)
 * with level = codebook[c] or c - 8, c the nibble (even column = low nibble).
 * qweight: int8 [N, K/2]; s_rel: [N, K/G] f32 (s_rel_kind 0) or e4m3 bytes (1);
 * codebook: f32 [16] or NULL; out: int8 [N, K].  G in {4, 8, 16, 32, ...}, K % 32 == 0.
 * Replaces launch_dequant_int4_grouped_to_int8(_e4m3)
 * (comfy_kitchen backends/cuda/ops/w4a8_gemm.cu:94-123). */
int h3b_dequant_int4_grouped_to_int8(const void* qweight, const void* s_rel, int s_rel_kind,
                                     const void* codebook, void* out, int64_t N, int64_t K, int64_t G,
                                     void* stream);

/* The activations of the W4A8 group correction (asymmetric int4 weights carry a
 * per-group offset, applied as out += sx @ correction): sx[m, g] = bf16(bf16(sum of
 * the G codes xq[m, g*G .. g*G+G-1]) * bf16(xs[m])) for g < K/G; columns [K/G,
 * sx_row_stride) are written 0.  xq: int8 [M, K] (the linear's quantized input),
 * xs: f32 [M]; sx: bf16 [M, sx_row_stride].  Replaces the eager group sum of
 * comfy_kitchen backends/cuda/__init__.py:2294-2296. */
int h3b_w4a8_group_sums(const void* xq, const void* xs, int64_t M, int64_t K, int64_t G, void* sx,
                        int64_t sx_row_stride, void* stream);

/* D[m, n] = bf16(float(D[m, n]) + sum_k A[m, k] * B[n, k]) on tcgen05 (kind::f16,
 * bf16 operands, fp32 accumulation in tensor memory), in place.  A: bf16 [M, K],
 * B: bf16 [N, K] (both rows of K contiguous, K % 8 == 0), D: bf16 with row stride
 * out_row_stride (even).  With A = the group sums above and B = correction^T this is
 * the W4A8 group correction; replaces out.addmm_(sx, correction) (comfy_kitchen
 * backends/cuda/__init__.py:2297). */
int h3b_bf16_gemm_accumulate(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                             int64_t out_row_stride, void* stream);

/* The block's AdaLN projection: out[r, n] = bf16(sum_k t[r, k] * w[n, k] + b[n]) with
 * fp32 products and sums, for 1..8 rows of t.  w: bf16 [N, K] row-major, t: bf16
 * [rows, K], b: bf16 [N] or NULL, out: bf16 [rows, N]; K a multiple of 8, w and t
 * 16-byte aligned.  Replaces the engine's adaln_projector linear over the timestep
 * rows (model/layers.py:1083-1085; the base linear of model/lora.py:524-570). */
int h3b_adaln_projection(const void* w, const void* t, const void* b, int64_t rows, int64_t N, int64_t K,
                         void* out, void* stream);

/* ---------------------------------------------------------------- attention preparation */

/* Bytes of workspace h3b_key_mean needs for L tokens and H heads. */
int64_t h3b_key_mean_workspace_bytes(int64_t L, int64_t H);

/* Per-(head, channel) mean of K over all L tokens (double accumulation, fixed
 * order: 1024-token chunks, then chunk sums), rounded to bf16.
 * k: bf16 NHD rows [L, H*128] with row stride k_row_stride; mean: bf16 [H, 128].
 * Replaces hnd_compatible_key_mean_nhd (model/sparge_nhd.py:26-48). */
int h3b_key_mean(const void* k, int64_t L, int64_t H, int64_t k_row_stride, void* mean, void* workspace,
                 int64_t workspace_bytes, void* stream);

/* h3b_key_mean for callers that cannot allocate device memory (no counterpart
 * in the reference, which always allocates its temporaries with torch): the
 * same result, with the scratch taken from a fixed 8 MiB array inside the
 * library instead of a caller workspace.  Limit: ceil(L/1024) * H * 128 <=
 * 2^20 (e.g. L <= 262,144 at H = 32); larger calls return H3B_ERR_UNSUPPORTED.
 * The first call on each device looks the array up (cudaGetSymbolAddress) and
 * should come before any stream capture.  Calls share the array: calls whose
 * kernels overlap on the GPU race; ordered calls are independent. */
int h3b_key_mean_no_alloc(const void* k, int64_t L, int64_t H, int64_t k_row_stride, void* mean, void* stream);

/* Sparge per-block preparation of Q (block 128) or K (block 64, with `mean`
 * for K mean-smoothing value = bf16(x - mean)):
 *   pooled  bf16 [H, nb, 128]  = bf16(sum(value)/valid_rows)
 *   similar u8   [H, nb]       = mean cosine Gram of fp16-normalised rows > thr[h]
 *   qi8     int8 [H, Lpad, 128] = trunc(value/s + 0.5*sign(value/s)), padded rows 0
 *   scale   f32  [H, nb]       = max|value| / 127 + 1e-7
 * x: bf16 NHD [L, H*128] rows of stride x_row_stride; nb = ceil(L/block),
 * Lpad >= nb*block (rows beyond nb*block are not written); thr: f32 [H].
 * block 32 gives the per-warp Q groups of Sage's per_warp granularity (32-row
 * groups; model/kernels.py:5571-5573), whose pooled / similar outputs go unused.
 * Replaces pool_sim_quant_nhd (model/sparge_nhd.py:51-227). */
int h3b_pool_sim_quant(const void* x, int64_t L, int64_t H, int64_t x_row_stride, const void* mean,
                       int block, const void* thr, void* pooled, void* similar, void* qi8, void* scale,
                       int64_t Lpad, void* stream);

/* Sage per_thread INT8 quantization (qk_quant_gran 3): kind 0 quantizes Q in
 * 128-row blocks of 32 scale groups (row r of a block in group (r/32)*8 + r%8),
 * kind 1 quantizes K in 64-row blocks of 4 groups (row r in group (r%8)/2) after
 * the bf16 mean smoothing bf16(k - mean) (mean: bf16 [H, 128], or NULL for none).
 * Per group: scale = max|v|/127 + 1e-7 over its rows, code = trunc(v/scale +
 * 0.5*sign(v)).  x: bf16 NHD [L, H*128] rows of stride x_row_stride; qi8: int8
 * [H, Lpad, 128] (rows past the last block untouched, the last block's rows >= L
 * code 0); scale: f32 [H, ceil(L/128)*32] (Q) or [H, ceil(L/64)*4] (K).
 * Replaces sageattention's per_thread_int8 / quant_query_per_thread_int8_kernel and
 * quantize_key_sub_mean_per_thread_int8 (model/sage_fused_quant.py:20-162,
 * 165-283; model/kernels.py:7664-7727). */
int h3b_quantize_per_thread_int8(const void* x, int64_t L, int64_t H, int64_t x_row_stride, const void* mean,
                                 int kind, void* qi8, void* scale, int64_t Lpad, void* stream);

/* h3b_pool_sim_quant over one slab of `rows` tokens of a longer sequence, writing
 * into that sequence's arrays: pooled / similar / scale point at the slab's first
 * block of head 0 with `blocks_per_head` blocks between heads, qi8 at the slab's
 * first row of head 0 with `Lpad` rows between heads.  The slab starts on a block
 * boundary.  Replaces the per-slab get_pool_sim_triton_simmean_fuse_quant of the
 * compact K/V builder (model/kernels.py:2733-2751). */
int h3b_pool_sim_quant_slab(const void* x, int64_t rows, int64_t H, int64_t x_row_stride, const void* mean,
                            int block, const void* thr, void* pooled, void* similar, void* qi8, void* scale,
                            int64_t blocks_per_head, int64_t Lpad, void* stream);

/* Per-head RMSNorm (weight, eps) of Q and K followed by split-half partial
 * RoPE over the first rot_dim channels, in place on bf16 projection rows:
 * qkv [L, row_stride], Q heads at column q_offset, K heads at k_offset (128
 * channels per head); q_weight / k_weight bf16 [128]; cos_table / sin_table
 * bf16 [L, rot_dim/2] (the packed split-half rotation of the token).
 * n = bf16(x * inv_rms * w); out_d = bf16(n_d cos - n_{d+r} sin),
 * out_{d+r} = bf16(n_d sin + n_{d+r} cos), r = rot_dim/2.
 * Replaces apply_qknorm_rope / rms_rope_split_half_ (model/layers.py:72-149,
 * comfy_kitchen backends/cuda/ops/rms_rope.cu:38-384). */
int h3b_qk_rmsnorm_rope(void* qkv, int64_t L, int64_t H, int64_t row_stride, int64_t q_offset, int64_t k_offset,
                        const void* q_weight, const void* k_weight, const void* cos_table, const void* sin_table,
                        int rot_dim, float eps, void* stream);

/* V -> FP8 E4M3 per-(head, channel) scaled by 2.25/absmax, transposed to
 * vt [H, 128, Lpad] (token index innermost, rows >= L zero); vscale: f32
 * [H, 128] = absmax/2.25.  v: bf16 NHD [L, H*128], row stride v_row_stride.
 * Lpad % 128 == 0.  Replaces prepare_sage_fp8_hnd_direct / write_sage_fp8_slab
 * (model/compact_fp8.py:205-300); the sm89 16-row MMA permutation is not applied. */
int h3b_value_fp8(const void* v, int64_t L, int64_t H, int64_t v_row_stride, int64_t Lpad, void* vt,
                  void* vscale, void* stream);

/* V -> FP8 E4M3 for one slab of `rows` tokens with a per-(head, channel) absmax
 * the caller gathered over the whole sequence beforehand: codes of v * (2.25 /
 * absmax) written transposed at vt (the slab's first token column of head 0,
 * channel 0; `vt_row_pitch` bytes between channel rows), in ceil(rows/128)
 * 128-token tiles (tokens past `rows` in the last tile are zero); vscale (f32
 * [H, 128], may be NULL) receives max(absmax / 2.25, 1e-12).  absmax: f32 [H, 128].
 * Replaces _write_compact_value_fp8 / write_sage_fp8_slab (model/kernels.py:
 * 2491-2526, model/compact_fp8.py:205-300). */
int h3b_value_fp8_given_absmax(const void* v, int64_t rows, int64_t H, int64_t v_row_stride, const void* absmax,
                               void* vt, int64_t vt_row_pitch, void* vscale, void* stream);

/* ---------------------------------------------------------------- block-sparse mask */

/* Parameters of the block-sparse selector (model/kernels.py:3668-3941). */
typedef struct h3b_mask_params {
  int mode;                     /* 0 fixed Top-K: count = (int64)(budget[h]*Kb)
                                   1 top-CDF: smallest-rank prefix with cumulative
                                     probability <= budget[h] */
  const float* budget;          /* device memory, f32 [H]: Top-K fraction or CDF threshold */
  int64_t protected_key_blocks; /* first blocks always kept (protected prefix) */
  int keep_first_column;        /* always keep K block 0 */
  int keep_diagonal;            /* always keep K blocks 2i, 2i+1 for Q block i */
  int temporal_radius;          /* < 0 off; else the temporal correspondence rail */
  int temporal_spatial_radius;
  int64_t frames, frame_tokens, protected_tokens, query_tokens;
  /* device memory, int64 [query_tokens], or NULL: the position in the video of
     each query row of a chunk of selected queries (model/kernels.py:5247-5254);
     the rail then takes query block i's centre from entry min(128 i + 64,
     query_tokens - 1).  NULL: the queries are the whole video in order. */
  const int64_t* query_indices;
  int64_t protected_query_blocks; /* first query blocks kept dense over every key
                                     (model/kernels.py:2423-2426) */
} h3b_mask_params;

/* Pooled scores softmax(bf16(pq . pk) * 128^-0.5, non-similar K -> -inf) per
 * (head, Q block), selection, and the mandatory rails (non-similar K columns
 * and Q rows kept dense).  pooled_q: bf16 [H, Qb, 128], similar_q: u8 [H, Qb],
 * pooled_k: bf16 [H, Kb, 128], similar_k: u8 [H, Kb].  Output bitmap: uint32
 * [H, Qb, ceil(Kb/32)], bit j%32 of word j/32 set when K block j is kept.
 * Kb <= 16384 (1,048,576 key tokens). */
int h3b_block_mask(const void* pooled_q, const void* similar_q, int64_t Qb, const void* pooled_k,
                   const void* similar_k, int64_t Kb, int64_t H, const h3b_mask_params* params, void* bitmap,
                   void* stream);

/* Bitmap -> the Sparge delta-LUT ABI: lut int32 [rows, Kb] (first entry absolute,
 * then deltas; unused tail zero), valid int32 [rows].
 * Replaces parallel_block_map_lut (model/sparse_lut.py:144-192). */
int h3b_bitmap_to_lut(const void* bitmap, int64_t rows, int64_t Kb, void* lut, void* valid, void* stream);

/* ---------------------------------------------------------------- Ulysses layouts */

/* The send buffer of the token -> head all-to-all over P ranks, from this rank's rows:
 * dst[p][l][j][:] = src[l][head_order[p*H/P + j]][:] (head_order NULL: head p*H/P + j),
 * 128 bf16 channels per head.  src: bf16 rows [rows, src_row_stride] whose first H*128
 * columns are the heads (e.g. the K slot of the QKV projection rows); dst: bf16
 * [P, rows, H/P, 128].  head_order: device int64 [H], a permutation.  No counterpart in
 * the reference (single-GPU); replaces a gather and a transposed copy in torch. */
int h3b_ulysses_pack(const void* src, int64_t rows, int64_t H, int64_t src_row_stride, const int64_t* head_order,
                     int64_t P, void* dst, void* stream);

/* The inverse for the head -> token all-to-all's result: dst[l][head_order[p*H/P + j]][:]
 * = src[p][l][j][:], writing token rows [rows, dst_row_stride] in head index order.
 * src: bf16 [P, rows, H/P, 128]. */
int h3b_ulysses_unpack(const void* src, int64_t rows, int64_t H, const int64_t* head_order, int64_t P, void* dst,
                       int64_t dst_row_stride, void* stream);

/* ---------------------------------------------------------------- attention */

/* O = softmax(Q K^T * sm_scale) V with INT8 Q.K^T (tcgen05 kind::i8), fp32
 * online softmax, P and V in FP8 E4M3 (tcgen05 kind::f8f6f4), fp32 output
 * accumulation.  Visits only the K blocks whose bit is set in `bitmap`
 * ([H, ceil(Lq/128), ceil(Kb/32)] words) or all of them when bitmap is NULL.
 * q: int8 [H, Lqpad, 128] with q_scale f32 [H, nqs]:
 *   q_gran 0: one scale per q_block (32, 64 or 128) rows, nqs = ceil(Lq/q_block)
 *             (Sparge per-block 128; per_warp 32);
 *   q_gran 1: Sage per_thread, row i in group (i/32)*8 + i%8, nqs = ceil(Lq/128)*32
 *             (q_block ignored);
 * k: int8 [H, Lkpad, 128] with k_scale f32:
 *   k_gran 0: [H, ceil(Lk/64)], one scale per 64-key block;
 *   k_gran 1: [H, ceil(Lk/64)*4], Sage per_thread, key j in group (j%64 %8)/2 of its
 *             block (k_scale 16-byte aligned);
 * vt: e4m3 [H, 128, Lkpad], v_scale f32 [H, 128];
 * out: bf16 NHD rows [Lq, H*128] with row stride out_row_stride.
 * Lqpad % 128 == 0, Lkpad % 128 == 0.
 * Replaces sageattn qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf (its
 * qk_quant_gran 1 / 2 / 3) and the Sparge block-sparse variant
 * (model/kernels.py:7645-7661, 7728-7742, 5575-5588, 3981-3997). */
int h3b_attention(const void* q, const void* q_scale, int q_gran, int q_block, int64_t Lq, int64_t Lqpad,
                  const void* k, const void* k_scale, int k_gran, int64_t Lk, int64_t Lkpad, const void* vt,
                  const void* v_scale, int64_t H, const void* bitmap, float sm_scale, void* out,
                  int64_t out_row_stride, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
