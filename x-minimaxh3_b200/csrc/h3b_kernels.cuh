// h3b_kernels.cuh -- argument structs and host launchers shared between the
// kernel translation units and the C ABI (capi.cu).
#pragma once

#include "h3b_common.cuh"

namespace h3b {

struct QuantArgs {
  const uint16_t* x;          // bf16 [rows, x_stride]
  int64_t x_stride;           // elements between rows of x
  int K;                      // quantized width
  int act;                    // 0 none, 1 gelu_tanh, 2 swiglu ([gate | up], 2K wide)
  int8_t* q;                  // [rows, K]
  float* scales;              // [rows]
  const uint16_t* norm_w;     // fused RMSNorm + AdaLN: bf16 [K]
  const uint16_t* scale_tab;  // bf16 [R, K]
  const uint16_t* shift_tab;  // bf16 [R, K]
  const int32_t* seg_row;     // [rows] or null (table row 0)
  float eps;
};
cudaError_t launch_quant(const QuantArgs& a, int64_t rows, int mode, bool rms, cudaStream_t s);
// Codes and row scales of rotated bf16 rows [rows, K] whose absmax is spread over
// amax[row * amax_stride + c], c < amax_cols (the GELU + ConvRot GEMM epilogue's output)
cudaError_t launch_quant_rotated(const uint16_t* rot, int64_t rot_stride, const float* amax, int64_t amax_stride,
                                 int amax_cols, int K, int64_t rows, int8_t* q, float* scales, cudaStream_t s);
int quant_threads_for(int K);

// kEpiQkRope64 / 48: the store epilogue of the QKV projection with the per-head q/k
// RMSNorm and split-half RoPE (rotary half-width 64 or 48) applied before the store
// kEpiAddF32: bf16 x bf16 operands (kind::f16, K in bytes = 2 x elements), the fp32
// product added into the bf16 output in place: D = bf16(float(D) + acc)
// kEpiGeluRot: the store epilogue's bf16 values through tanh-GELU and the 256-point
// ConvRot transform (one group per 256-column tile), stored as bf16, with the fp32
// absmax of each (row, tile, half) written to amax[m * amax_stride + 2 * tile + half];
// half h covers the tile's columns 64 j + 32 h + [0, 32), j = 0..3
enum EpiKind : int { kEpiStore = 0, kEpiResidual = 1, kEpiInt32 = 2, kEpiQkRope64 = 3, kEpiQkRope48 = 4,
                     kEpiAddF32 = 5, kEpiGeluRot = 6 };
struct GemmArgs {
  int M, N, K;
  const float* xs;
  const float* ws;
  int ws_scalar;
  const float* bias;
  uint16_t* out;      // bf16 output or residual (in place)
  int32_t* out_i32;   // raw accumulators
  int64_t out_stride;
  const uint16_t* gate;
  // q/k norm + RoPE epilogue: q heads at output columns [q_off, q_off + qk_width),
  // k heads at [k_off, k_off + qk_width), 128 columns each; cos/sin bf16 [rows, half]
  // for the GEMM's row 0 onwards
  int64_t q_off, k_off, qk_width;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const uint16_t* cos_t;
  const uint16_t* sin_t;
  float qk_eps;
  // GELU + ConvRot epilogue: per-(row, half-tile) absmax of the rotated values
  float* amax;
  int64_t amax_stride;
};
// True when an M x N GEMM runs the 2-SM kernel (the only one with the q/k epilogue).
bool gemm_uses_pair_kernel(int64_t M, int64_t N);
// 0 ok, 1 tensor-map encoding failed, 2 CUDA launch error (*err), 4 the q/k epilogue
// was asked for a shape that does not run the 2-SM kernel
int launch_gemm(const void* A, const void* B, GemmArgs a, int kind, cudaStream_t s, cudaError_t* err);
bool make_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                  uint64_t rows, uint64_t stride_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw);

// sx[m, g] = bf16(bf16(sum of xq[m, g*G .. g*G+G-1]) * bf16(xs[m])) for g < K/G, columns
// [K/G, sx_stride) zero: the W4A8 group-correction activations
cudaError_t launch_adaln_projection(const uint16_t* w, const uint16_t* t, const uint16_t* b, int64_t rows,
                                    int64_t n, int64_t k, uint16_t* out, cudaStream_t s);
cudaError_t launch_group_sums(const int8_t* xq, const float* xs, int64_t M, int64_t K, int64_t G, uint16_t* sx,
                              int64_t sx_stride, cudaStream_t s);
cudaError_t launch_w4_decode(const void* qw, const void* s_rel, int s_rel_kind, const void* codebook, void* out,
                             int64_t N, int64_t K, int64_t G, cudaStream_t s);

int64_t key_mean_workspace(int64_t L, int64_t H);
cudaError_t launch_key_mean(const void* k, int64_t L, int64_t H, int64_t stride, void* mean, void* ws, cudaStream_t s);
int64_t key_mean_static_capacity();
cudaError_t launch_key_mean_static(const void* k, int64_t L, int64_t H, int64_t stride, void* mean,
                                   cudaStream_t s);

struct PoolArgs {
  const uint16_t* x;
  int64_t L, stride, Lpad;
  int H, blk;
  const uint16_t* mean;  // bf16 [H, 128] or null
  const float* thr;
  uint16_t* pooled;      // [H, nb, 128]
  uint8_t* similar;      // [H, nb]
  int8_t* q;             // [H, Lpad, 128]
  float* scale;          // [H, nb]
  int64_t nb_stride;     // blocks between heads in pooled / similar / scale (0: nb)
};
cudaError_t launch_pool_sim_quant(const PoolArgs& a, cudaStream_t s);
// Sage per_thread INT8: kind 0 Q (128-row blocks, 32 groups), 1 K (64-row blocks,
// 4 groups); scales at a.scale[h * a.nb_stride + block * groups + g]
cudaError_t launch_quant_per_thread(const PoolArgs& a, int kind, cudaStream_t s);
struct QkRopeArgs {
  uint16_t* x;            // bf16 rows [L, stride], q at column q_off, k at k_off (in place)
  int64_t L, stride, q_off, k_off;
  int H, rot_dim;
  const uint16_t* qw;     // bf16 [128]
  const uint16_t* kw;     // bf16 [128]
  const uint16_t* cos_t;  // bf16 [L, rot_dim/2]
  const uint16_t* sin_t;  // bf16 [L, rot_dim/2]
  float eps;
};
cudaError_t launch_qk_rmsnorm_rope(const QkRopeArgs& a, cudaStream_t s);
cudaError_t launch_value_fp8(const void* v, int64_t L, int64_t H, int64_t stride, int64_t Lpad, void* vt,
                             void* vscale, cudaStream_t s);
// E4M3 codes of `rows` tokens with the caller's per-(head, channel) absmax, written
// at vt (token column 0 of the slab, row pitch Lpad) in ceil(rows/128) tiles;
// vscale (optional) receives max(absmax / 2.25, 1e-12)
cudaError_t launch_value_fp8_given_absmax(const void* v, int64_t rows, int64_t H, int64_t stride, int64_t Lpad,
                                          const float* absmax, void* vt, float* vscale, cudaStream_t s);

struct MaskArgs {
  const uint16_t* pq;   // [H, Qb, 128]
  const uint8_t* simq;  // [H, Qb]
  const uint16_t* pk;   // [H, Kb, 128]
  const uint8_t* simk;  // [H, Kb]
  int64_t Qb, Kb;
  int mode;
  const float* budget;  // device [H]
  int64_t protected_kb;
  int first_col, diag;
  int temporal_radius, temporal_spatial_radius;
  int64_t frames, frame_tokens, protected_tokens, query_tokens;
  uint32_t* bitmap;
  const int64_t* q_index;  // [query_tokens] video position of each query, or null (query i at i)
  int64_t protected_qb;    // query blocks kept dense over every key
};
cudaError_t launch_block_mask(const MaskArgs& a, int64_t H, cudaStream_t s);
cudaError_t launch_bitmap_to_lut(const void* bm, int64_t rows, int64_t Kb, void* lut, void* valid, cudaStream_t s);

struct AttnArgs {
  int H;
  int64_t Lq, Lqpad, Lk, Lkpad;
  int Kb, words, q_block, nqs;
  int q_gran;  // 0: q_block-row scale groups; 1: Sage per_thread ((r/32)*8 + r%8)
  int k_gran;  // 0: one scale per 64-key block; 1: Sage per_thread (4 per block)
  const float* q_scale;
  const float* k_scale;
  const float* v_scale;
  const uint32_t* bitmap;
  float scale_log2;  // sm_scale * log2(e)
  uint16_t* out;
  int64_t out_stride;
};
int launch_attention(const void* q, const void* k, const void* vt, const AttnArgs& a, cudaStream_t s,
                     cudaError_t* err);

// Ulysses all-to-all layouts (ulysses.cu): bf16 heads of 128 channels
cudaError_t launch_gather_heads(const void* src, int64_t rows, int64_t H, int64_t src_stride, const int64_t* order,
                                int64_t P, void* dst, cudaStream_t s);
cudaError_t launch_scatter_heads(const void* src, int64_t rows, int64_t H, const int64_t* order, int64_t P,
                                 void* dst, int64_t dst_stride, cudaStream_t s);

}  // namespace h3b
