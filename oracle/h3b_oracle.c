/*
 * h3b_oracle.c -- CPU restatement of the X-MinimaxH3 DiT-block hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path links, loads or calls
 * this file: it is the checker that tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py compare the CUDA library against.  It is pinned
 * against golden vectors produced by the reference's own importable Python code
 * (tests/golden/make_golden.py).
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math (oracle/Makefile).  With
 * contraction off, every "a*b+c" below is two IEEE roundings; every fused
 * multiply-add is an explicit fmaf().  The CUDA kernels are compiled with
 * -fmad=false and use the same explicit fmaf() calls, so the two agree bit for
 * bit wherever the tests demand it.
 *
 * Reference citations are paths inside the X-MinimaxH3 project.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* scalar formats                                                             */
/* ------------------------------------------------------------------------- */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* round-to-nearest-even float -> bf16 (NaN -> canonical quiet NaN) */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static inline float bf16r(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* round-to-nearest-even float -> IEEE half, with subnormals and overflow to inf */
static inline uint16_t f32_to_f16(float f) {
    uint32_t u = f2u(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                                   /* below 2^-14: subnormal */
        /* value = a_float; half subnormal unit = 2^-24 */
        float af = u2f(a);
        float scaled = af * 16777216.0f;                      /* exact: times 2^24 */
        float r = rintf(scaled);                              /* ties to even */
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = ((a >> 23) - 127 + 15);
    uint32_t m = a & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rest = m & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}
static inline float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 0) {
        float v = (float)m * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (m << 13));
    return u2f(sign | ((e - 15 + 127) << 23) | (m << 13));
}

/* float -> FP8 E4M3 (OCP "fn" variant: no inf, 0x7f = NaN), round to nearest
 * even, saturating to +-448 for finite inputs (PTX cvt.rn.satfinite). */
uint8_t h3bo_f32_to_e4m3(float f) {
    uint32_t u = f2u(f);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    float a = fabsf(f);
    if (a != a) return 0x7f;
    if (a >= 464.0f) return sign | 0x7e;       /* 448 is the largest finite; ties at 464 round to 512 -> saturate */
    if (a < 0.015625f) {                        /* below 2^-6: subnormal, unit 2^-9 */
        float r = rintf(a * 512.0f);
        return sign | (uint8_t)r;               /* r may be 8 == 0x08 = 2^-6, the first normal: correct */
    }
    int ex; float fr = frexpf(a, &ex);           /* a = fr * 2^ex, fr in [0.5,1) */
    int E = ex - 1;                              /* a = 1.m * 2^E */
    float mant = fr * 2.0f - 1.0f;               /* exact */
    float mq = rintf(mant * 8.0f);               /* 3 mantissa bits, ties to even */
    if (mq >= 8.0f) { mq = 0.0f; E += 1; }
    uint32_t code = ((uint32_t)(E + 7) << 3) | (uint32_t)mq;
    if (code > 0x7e) code = 0x7e;
    return sign | (uint8_t)code;
}
float h3bo_e4m3_to_f32(uint8_t b) {
    uint32_t e = (b >> 3) & 0xf, m = b & 7;
    float v;
    if ((b & 0x7f) == 0x7f) return NAN;
    if (e == 0) v = (float)m * (1.0f / 512.0f);
    else v = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
    return (b & 0x80) ? -v : v;
}

/* ------------------------------------------------------------------------- */
/* elementary functions shared bit-for-bit with the CUDA kernels              */
/* ------------------------------------------------------------------------- */

/* exp(x) by Cody-Waite argument reduction x = n*ln2 + r (|r| <= ln2/2, ln2 split
 * into a 16-bit-exact high part and a remainder) followed by the degree-7 Taylor
 * polynomial of exp(r) in Horner form with fused multiply-adds, then scaling by
 * 2^n built from exponent bits.  Truncation error r^8/8! < 6e-9, under one ulp.
 * The same sequence of IEEE operations runs in csrc/h3b_math.cuh. */
float h3bo_expf(float x) {
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -103.972084045410156f) return 0.0f;
    const float kLog2e = 1.44269502162933349609375f;
    const float kLn2Hi = 0.693145751953125f;
    const float kLn2Lo = 1.428606765330187045e-06f;
    float n = rintf(x * kLog2e);
    float r = fmaf(-n, kLn2Hi, x);
    r = fmaf(-n, kLn2Lo, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    int n1 = ni / 2, n2 = ni - n1;               /* each half stays a normal power of two */
    float s1 = u2f((uint32_t)(n1 + 127) << 23);
    float s2 = u2f((uint32_t)(n2 + 127) << 23);
    return (p * s1) * s2;
}

/* tanh(x) = sign(x) * (1 - e) / (1 + e), e = exp(-2|x|) */
float h3bo_tanhf(float x) {
    float a = fabsf(x);
    if (a >= 10.0f) return x > 0 ? 1.0f : -1.0f;
    float e = h3bo_expf(-2.0f * a);
    float t = (1.0f - e) / (1.0f + e);
    return x < 0 ? -t : t;
}

/* GELU, tanh approximation (comfy_kitchen int8_linear.cu apply_input_act). */
static inline float act_gelu_tanh(float v) {
    const float kBeta = 0.7978845608028654f;
    const float kKappa = 0.044715f;
    float inner = kBeta * (v + kKappa * v * v * v);
    return 0.5f * v * (1.0f + h3bo_tanhf(inner));
}
/* silu(gate) * up (comfy_kitchen int8_linear.cu load_input_act). */
static inline float act_swiglu(float gate, float up) {
    return (gate / (1.0f + h3bo_expf(-gate))) * up;
}

/* ------------------------------------------------------------------------- */
/* per-token INT8 quantization (comfy_kitchen int8_linear.cu:158-200,        */
/* 257-341, 943-1030)                                                         */
/* ------------------------------------------------------------------------- */

#define BF16_FINITE_MAX 3.38953139e38f

static inline float row_scale_from_absmax(float absmax) {
    float a = fminf(absmax, BF16_FINITE_MAX);
    return fmaxf(a * (1.0f / 127.0f), 1.0e-30f);
}
static inline int8_t quant_code(float v_bf16_exact, float scale_t) {
    float scaled = bf16r(v_bf16_exact / scale_t);
    float q = rintf(scaled);
    q = fminf(127.0f, fmaxf(-128.0f, q));
    return (int8_t)q;
}

/* Plain row quantization: scale = max(|x|)/127 (times 1/127), code =
 * rint(bf16(x / bf16(scale))).  int8_linear.cu:158-200. */
void h3bo_quant_rowwise(const uint16_t* x, int64_t M, int64_t K, int8_t* q, float* scales) {
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * K;
        float amax = 0.0f;
        for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(bf16_to_f32(xr[k])));
        float scale = row_scale_from_absmax(amax);
        float st = bf16r(scale);
        scales[m] = scale;
        for (int64_t k = 0; k < K; ++k) q[m * K + k] = quant_code(bf16_to_f32(xr[k]), st);
    }
}

/* One normalized 256-point regular-Hadamard transform (H4 Kronecker power / 16)
 * as four radix-4 stages of stride 1, 4, 16, 64 with a 1/2 per stage
 * (int8_linear.cu:217-250 and the stage helpers at :664-718). */
void h3bo_fht256(float* v) {
    float t[256];
    float* src = v; float* dst = t;
    for (int stage = 0; stage < 4; ++stage) {
        int s = stage == 0 ? 1 : stage == 1 ? 4 : stage == 2 ? 16 : 64;
        for (int i = 0; i < 256; ++i) {
            int d = (i / s) & 3, base = i - d * s;
            float x0 = src[base], x1 = src[base + s], x2 = src[base + 2 * s], x3 = src[base + 3 * s];
            float y;
            switch (d) {
                case 0: y = x0 + x1 + x2 - x3; break;
                case 1: y = x0 + x1 - x2 + x3; break;
                case 2: y = x0 - x1 + x2 + x3; break;
                default: y = -x0 + x1 + x2 + x3; break;
            }
            dst[i] = 0.5f * y;
        }
        float* tmp = src; src = dst; dst = tmp;
    }
    /* four swaps: result is back in v */
}

/* input activation codes (comfy_kitchen input_act_codes.h): 0 none, 1 gelu_tanh, 2 swiglu */
static inline float load_act(const uint16_t* xrow, int64_t col, int64_t K, int act) {
    if (act == 2) return act_swiglu(bf16_to_f32(xrow[col]), bf16_to_f32(xrow[K + col]));
    float v = bf16_to_f32(xrow[col]);
    return act == 1 ? act_gelu_tanh(v) : v;
}

/* Fused activation + ConvRot + row quantization
 * (quantize_int8_rowwise_convrot64_kernel, int8_linear.cu:943-1030).  For act=2
 * (swiglu) x is [M, 2K] = [gate | up]. */
void h3bo_quant_rowwise_convrot(const uint16_t* x, int64_t M, int64_t K, int act,
                                int8_t* q, float* scales) {
    int64_t in_w = act == 2 ? 2 * K : K;
    float* row = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * in_w;
        for (int64_t k = 0; k < K; ++k) row[k] = load_act(xr, k, K, act);
        float amax = 0.0f;
        for (int64_t g = 0; g < K; g += 256) {
            h3bo_fht256(row + g);
            for (int i = 0; i < 256; ++i) amax = fmaxf(amax, fabsf(row[g + i]));
        }
        float scale = row_scale_from_absmax(amax);
        float st = bf16r(scale);
        scales[m] = scale;
        for (int64_t k = 0; k < K; ++k) q[m * K + k] = quant_code(bf16r(row[k]), st);
    }
    free(row);
}

static float tree_sum(float* v, int n) {   /* n is a power of two; v is clobbered */
    for (int w = n / 2; w >= 1; w /= 2)
        for (int i = 0; i < w; ++i) v[i] = v[i] + v[i + w];
    return v[0];
}
/* Block reduction as the CUDA kernels do it: a shfl_down tree inside each warp
 * of 32 (pairs i, i+w for w = 16..1), then the same tree over the warp sums
 * zero-padded to 32 entries.  n is a multiple of 32, at most 1024. */
static float block_tree_sum(float* v, int n) {
    int nw = n / 32;
    float ws[32];
    for (int w = 0; w < 32; ++w) ws[w] = w < nw ? tree_sum(v + 32 * w, 32) : 0.0f;
    return tree_sum(ws, 32);
}
float h3bo_tree_sum(const float* v, int n) {
    float* t = (float*)malloc(sizeof(float) * (size_t)n);
    memcpy(t, v, sizeof(float) * (size_t)n);
    float r = tree_sum(t, n);
    free(t);
    return r;
}

/* Threads per row used by the CUDA quantizer: 16 per pair of 256-column groups,
 * rounded up to a warp multiple.  Thread t owns chunk t % 16 (16 columns) of the
 * groups 2p and 2p + 1, p = t / 16: chunks 32p + t % 16 and 32p + 16 + t % 16. */
int h3bo_quant_threads(int64_t K) {
    int64_t chunks = K / 16;
    int64_t groups = (chunks + 15) / 16;
    int64_t T = (groups + 1) / 2 * 16;
    return (int)((T + 31) / 32 * 32);
}

/* RMSNorm(weight) followed by AdaLN modulation with bf16 materialization after
 * each step (fused_norm_rope.py:12-45; layers.py:916-941):
 *   n = bf16(x * inv_rms * w); n = bf16(n * bf16(1 + scale)); n = bf16(n + bf16(shift)).
 * inv_rms = 1 / sqrt(sum(x^2)/K + eps).  The sum of squares follows the CUDA
 * kernel's fixed order: thread t of T = h3bo_quant_threads(K) adds the squares of
 * each of its two chunks in column order (two running sums, zero for a chunk past
 * the row), adds the two sums, and the per-thread sums are combined by
 * block_tree_sum. */
void h3bo_rms_adaln_row(const uint16_t* xr, int64_t K, const uint16_t* w, const uint16_t* scale,
                        const uint16_t* shift, float eps, float* out) {
    int T = h3bo_quant_threads(K);
    int64_t chunks = K / 16;
    float* part = (float*)calloc(1024, sizeof(float));
    for (int t = 0; t < T; ++t) {
        float lane[2] = {0.0f, 0.0f};
        for (int l = 0; l < 2; ++l) {
            int64_t c = (int64_t)(t / 16) * 32 + 16 * l + t % 16;
            if (c >= chunks) continue;
            for (int j = 0; j < 16; ++j) {
                float v = bf16_to_f32(xr[c * 16 + j]);
                lane[l] = lane[l] + v * v;
            }
        }
        part[t] = lane[0] + lane[1];
    }
    float ss = block_tree_sum(part, T);
    free(part);
    float inv = 1.0f / sqrtf(ss / (float)K + eps);
    for (int64_t c = 0; c < K; ++c) {
        float v = bf16_to_f32(xr[c]);
        float n = bf16r(v * inv * bf16_to_f32(w[c]));
        float s1 = bf16r(1.0f + bf16_to_f32(scale[c]));
        n = bf16r(n * s1);
        n = bf16r(n + bf16_to_f32(shift[c]));
        out[c] = n;
    }
}

/* rms_adaln fused into the ConvRot quantizer: per row, the modulated bf16 row is
 * rotated and quantized exactly as h3bo_quant_rowwise_convrot (convrot!=0) or
 * h3bo_quant_rowwise (convrot==0).  `seg_row` gives the modulation-table row of
 * each token (segments of layers.py:916-941). */
void h3bo_rms_adaln_quant(const uint16_t* x, int64_t M, int64_t K, const uint16_t* w,
                          const uint16_t* scale_tab, const uint16_t* shift_tab, const int32_t* seg_row,
                          float eps, int convrot, int8_t* q, float* scales) {
    float* row = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t m = 0; m < M; ++m) {
        int r = seg_row ? seg_row[m] : 0;
        h3bo_rms_adaln_row(x + m * K, K, w, scale_tab + (int64_t)r * K, shift_tab + (int64_t)r * K,
                           eps, row);
        float amax = 0.0f;
        if (convrot)
            for (int64_t g = 0; g < K; g += 256) h3bo_fht256(row + g);
        for (int64_t k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(row[k]));
        float s = row_scale_from_absmax(amax);
        float st = bf16r(s);
        scales[m] = s;
        for (int64_t k = 0; k < K; ++k) q[m * K + k] = quant_code(bf16r(row[k]), st);
    }
    free(row);
}

/* ------------------------------------------------------------------------- */
/* W4 decode (w4a8_gemm.cu:36-90; eager w4a8_int8.py:344-363)                */
/* ------------------------------------------------------------------------- */

/* scale_kind: 0 = fp32 s_rel, 1 = e4m3 s_rel (raw bytes) */
void h3bo_w4_decode(const int8_t* qdata, const void* s_rel, int scale_kind, const float* codebook,
                    int64_t N, int64_t K, int64_t G, int8_t* out) {
    int64_t groups = K / G;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            uint8_t byte = (uint8_t)qdata[n * (K / 2) + k / 2];
            uint32_t c = (k & 1) ? (byte >> 4) & 0xf : byte & 0xf;
            float lvl = codebook ? codebook[c] : (float)c - 8.0f;
            float s = scale_kind == 0 ? ((const float*)s_rel)[n * groups + k / G]
                                      : h3bo_e4m3_to_f32(((const uint8_t*)s_rel)[n * groups + k / G]);
            float p = rintf(lvl * s);
            if (p > 127.0f) p = 127.0f;
            if (p < -127.0f) p = -127.0f;
            out[n * K + k] = (int8_t)p;
        }
}

/* ------------------------------------------------------------------------- */
/* INT8 GEMM + dequant epilogue (cutlass_gemm_int8.cu:1-6)                   */
/* ------------------------------------------------------------------------- */

void h3bo_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int64_t K, int32_t* acc) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            int32_t s = 0;
            const int8_t* a = A + m * K; const int8_t* b = B + n * K;
            for (int64_t k = 0; k < K; ++k) s += (int32_t)a[k] * (int32_t)b[k];
            acc[m * N + n] = s;
        }
}

/* D[m,n] = bf16( fma(float(acc)*xs[m], ws[n], bias[n]) ).  ws_numel is 1 (scalar)
 * or N; bias may be NULL.  If `residual` and `gate` are given the result is
 * residual[m,n] = bf16(residual + D * gate[n]) instead (fused_mlp.py:124-143,
 * layers.py:944-960), and `out` may be NULL. */
void h3bo_epilogue(const int32_t* acc, int64_t M, int64_t N, const float* xs, const float* ws,
                   int64_t ws_numel, const float* bias, uint16_t* out, uint16_t* residual,
                   const uint16_t* gate, int64_t out_stride) {
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n) {
            float v = (float)acc[m * N + n] * xs[m];
            float w = ws[ws_numel == 1 ? 0 : n];
            float d = bias ? fmaf(v, w, bias[n]) : v * w;
            uint16_t db = f32_to_bf16(d);
            if (residual) {
                float r = bf16_to_f32(residual[m * out_stride + n]);
                residual[m * out_stride + n] = f32_to_bf16(r + bf16_to_f32(db) * bf16_to_f32(gate[n]));
            } else {
                out[m * out_stride + n] = db;
            }
        }
}

/* ------------------------------------------------------------------------- */
/* Attention preparation                                                      */
/* ------------------------------------------------------------------------- */

/* Per-(head, channel) mean of K over all L tokens, NHD bf16 input [L,H,D].
 * Accumulated in double in the CUDA kernels' order: the sum of each chunk of
 * 1024 consecutive tokens (tokens in order), then the chunk sums in chunk
 * order; divided by L, rounded to float, then to bf16.  For bf16 inputs the
 * double sums are exact in practice, so the order matters only formally. */
#define H3B_KEY_MEAN_CHUNK 1024
void h3bo_key_mean(const uint16_t* k, int64_t L, int64_t H, int64_t D, uint16_t* mean) {
    for (int64_t h = 0; h < H; ++h)
        for (int64_t d = 0; d < D; ++d) {
            double total = 0.0;
            for (int64_t c0 = 0; c0 < L; c0 += H3B_KEY_MEAN_CHUNK) {
                double part = 0.0;
                int64_t c1 = c0 + H3B_KEY_MEAN_CHUNK < L ? c0 + H3B_KEY_MEAN_CHUNK : L;
                for (int64_t l = c0; l < c1; ++l) part += (double)bf16_to_f32(k[(l * H + h) * D + d]);
                total += part;
            }
            mean[h * D + d] = f32_to_bf16((float)(total / (double)L));
        }
}

/* Butterfly sum over 32 lanes as performed by shfl_xor (offsets 16..1). */
static float warp_butterfly_sum(const float* lanes) {
    float v[32];
    memcpy(v, lanes, sizeof(v));
    for (int off = 16; off >= 1; off /= 2) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ off];
        memcpy(v, t, sizeof(v));
    }
    return v[0];
}
/* Sum of 128 values the way a warp does it: lane l owns elements 4l..4l+3, adds
 * them left to right, then the 32 partials are butterfly-reduced. */
static float warp_sum128(const float* x) {
    float lanes[32];
    for (int l = 0; l < 32; ++l) lanes[l] = ((x[4 * l] + x[4 * l + 1]) + x[4 * l + 2]) + x[4 * l + 3];
    return warp_butterfly_sum(lanes);
}

/* Sparge per-block pool / self-similarity / INT8 quantization of one head-major
 * token block (sparge_nhd.py:51-160; sage_fused_quant.py smoothing boundary).
 *   x: NHD bf16 [L,H,128]; mean: bf16 [H,128] or NULL (K mean-smoothing:
 *   value = bf16(x - mean)); blk: 64 or 128 rows; thr: [H] similarity threshold.
 * Outputs (nb = ceil(L/blk), Lpad = nb*blk):
 *   pooled bf16 [H,nb,128] = bf16(sum_rows(value)/valid)
 *   similar u8 [H,nb]      = mean cosine Gram of fp16-normalised rows > thr[h]
 *                            (sum of the Gram = |sum_i n_i|^2; padded rows make it NaN -> 0)
 *   qi8 int8 [H,Lpad,128]  = trunc(v/s + 0.5*sign), s = max|v|/127 + 1e-7; pad rows 0
 *   scale f32 [H,nb]       = s */
void h3bo_pool_sim_quant(const uint16_t* x, int64_t L, int64_t H, const uint16_t* mean, int blk,
                         const float* thr, uint16_t* pooled, uint8_t* similar, int8_t* qi8, float* scale) {
    const int D = 128;
    int64_t nb = (L + blk - 1) / blk;
    float* v = (float*)malloc(sizeof(float) * (size_t)blk * D);
    for (int64_t h = 0; h < H; ++h)
        for (int64_t b = 0; b < nb; ++b) {
            int64_t r0 = b * blk;
            int valid = (int)((L - r0) < blk ? (L - r0) : blk);
            for (int r = 0; r < blk; ++r)
                for (int d = 0; d < D; ++d) {
                    float val = 0.0f;
                    if (r < valid) {
                        val = bf16_to_f32(x[((r0 + r) * H + h) * D + d]);
                        if (mean) val = bf16r(val - bf16_to_f32(mean[h * D + d]));
                    }
                    v[r * D + d] = val;
                }
            /* The CUDA kernel runs four warps per block; warp w takes rows w, w+4, ...
             * in order and the four partial sums are combined as (p0+p2)+(p1+p3). */
            float pp[4][128], sp[4][128];
            memset(pp, 0, sizeof(pp));
            memset(sp, 0, sizeof(sp));
            int nan_seen = valid < blk;
            for (int r = 0; r < valid; ++r) {
                int w = r & 3;
                float sq[128];
                for (int d = 0; d < D; ++d) {
                    pp[w][d] = pp[w][d] + v[r * D + d];
                    sq[d] = v[r * D + d] * v[r * D + d];
                }
                float norm = sqrtf(warp_sum128(sq));
                if (!(norm > 0.0f)) nan_seen = 1;
                for (int d = 0; d < D; ++d) {
                    float nv = f16_to_f32(f32_to_f16(v[r * D + d] / norm));
                    sp[w][d] = sp[w][d] + nv;
                }
            }
            float ssum[128];
            for (int d = 0; d < D; ++d) {
                float s = (pp[0][d] + pp[2][d]) + (pp[1][d] + pp[3][d]);
                pooled[(h * nb + b) * D + d] = f32_to_bf16(s / (float)valid);
                ssum[d] = (sp[0][d] + sp[2][d]) + (sp[1][d] + sp[3][d]);
            }
            float sq2[128];
            for (int d = 0; d < D; ++d) sq2[d] = ssum[d] * ssum[d];
            float g = warp_sum128(sq2);
            float simv = g / (float)(valid * valid);
            similar[h * nb + b] = (uint8_t)(!nan_seen && simv > thr[h]);
            /* quant */
            float amax = 0.0f;
            for (int r = 0; r < valid; ++r)
                for (int d = 0; d < D; ++d) amax = fmaxf(amax, fabsf(v[r * D + d]));
            float s = amax / 127.0f + 1e-7f;
            scale[h * nb + b] = s;
            int64_t Lpad = nb * blk;
            for (int r = 0; r < blk; ++r)
                for (int d = 0; d < D; ++d) {
                    int8_t qv = 0;
                    if (r < valid) {
                        float t = v[r * D + d] / s;
                        t = t + (t >= 0.0f ? 0.5f : -0.5f);
                        float tr = truncf(t);
                        if (tr > 127.0f) tr = 127.0f;
                        if (tr < -127.0f) tr = -127.0f;
                        qv = (int8_t)tr;
                    }
                    qi8[(h * Lpad + r0 + r) * D + d] = qv;
                }
        }
    free(v);
}

/* Sage per_thread INT8 quantization (qk_quant_gran 3), in the scale groups of
 * q_scale_index / k_scale_index below:
 *   kind 0 (Q): 128-row blocks of 32 groups, row i in group (i / 32) * 8 + i % 8
 *              (sageattention's quant_query_per_thread_int8_kernel, BLK = 32 with
 *              8 row classes: the in-tree callers fix its grid and scale shape,
 *              model/sage_fused_quant.py:201-222, kernels.py:7700-7725);
 *   kind 1 (K): 64-row blocks of 4 groups, row j in group (j % 8) / 2, values
 *              bf16(k - mean) (model/sage_fused_quant.py:20-117).
 * Per group: scale = max|v| / 127 + 1e-7 over its valid rows (rows >= L count as
 * 0); code = trunc(v / scale + 0.5 * sign), rows >= L code 0.
 * qi8: [H, Lpad, 128] with Lpad >= the blocks' rows; scale: [H, blocks * groups]. */
void h3bo_quant_per_thread(const uint16_t* x, int64_t L, int64_t H, const uint16_t* mean, int kind,
                           int8_t* qi8, int64_t Lpad, float* scale) {
    const int D = 128;
    const int blk = kind == 0 ? 128 : 64, ng = kind == 0 ? 32 : 4;
    const int64_t nb = (L + blk - 1) / blk;
    float* v = (float*)malloc(sizeof(float) * (size_t)blk * D);
    for (int64_t h = 0; h < H; ++h)
        for (int64_t b = 0; b < nb; ++b) {
            const int64_t r0 = b * blk;
            const int valid = (int)((L - r0) < blk ? (L - r0) : blk);
            float gmax[32];
            for (int g = 0; g < ng; ++g) gmax[g] = 0.0f;
            for (int r = 0; r < blk; ++r) {
                const int g = kind == 0 ? (r / 32) * 8 + (r % 8) : (r % 8) / 2;
                for (int d = 0; d < D; ++d) {
                    float val = 0.0f;
                    if (r < valid) {
                        val = bf16_to_f32(x[((r0 + r) * H + h) * D + d]);
                        if (mean) val = bf16r(val - bf16_to_f32(mean[h * D + d]));
                    }
                    v[r * D + d] = val;
                    gmax[g] = fmaxf(gmax[g], fabsf(val));
                }
            }
            float sc[32];
            for (int g = 0; g < ng; ++g) {
                sc[g] = gmax[g] / 127.0f + 1e-7f;
                scale[h * nb * ng + b * ng + g] = sc[g];
            }
            for (int r = 0; r < blk; ++r) {
                const int g = kind == 0 ? (r / 32) * 8 + (r % 8) : (r % 8) / 2;
                for (int d = 0; d < D; ++d) {
                    int8_t qv = 0;
                    if (r < valid) {
                        float t = v[r * D + d] / sc[g];
                        t = t + (t >= 0.0f ? 0.5f : -0.5f);
                        float tr = truncf(t);
                        if (tr > 127.0f) tr = 127.0f;
                        if (tr < -127.0f) tr = -127.0f;
                        qv = (int8_t)tr;
                    }
                    qi8[(h * Lpad + r0 + r) * D + d] = qv;
                }
            }
        }
    free(v);
}

/* Per-head RMSNorm + split-half partial RoPE, in place (model/layers.py:72-149):
 * n = bf16((x * inv) * w), inv = 1/sqrt(sum(x^2)/128 + eps) with the sum in the
 * warp order of warp_sum128; then for d < r = rot/2:
 * out_d = bf16(n_d c - n_{d+r} s), out_{d+r} = bf16(n_d s + n_{d+r} c); channels
 * >= rot pass through normalised; c, s from the bf16 tables [L, rot/2]. */
static void rms_rope_vec(uint16_t* p, const uint16_t* w, const uint16_t* ct, const uint16_t* st, int rot, float eps) {
    float v[128], sq[128], n[128];
    for (int d = 0; d < 128; ++d) { v[d] = bf16_to_f32(p[d]); sq[d] = v[d] * v[d]; }
    float ss = warp_sum128(sq);
    float inv = 1.0f / sqrtf(ss / 128.0f + eps);
    for (int d = 0; d < 128; ++d) n[d] = bf16r(v[d] * inv * bf16_to_f32(w[d]));
    int half = rot / 2;
    for (int d = 0; d < 128; ++d) {
        float o = n[d];
        if (d < half) {
            float c = bf16_to_f32(ct[d]), s = bf16_to_f32(st[d]);
            o = bf16r(n[d] * c - n[d + half] * s);
        } else if (d < rot) {
            float c = bf16_to_f32(ct[d - half]), s = bf16_to_f32(st[d - half]);
            o = bf16r(n[d - half] * s + n[d] * c);
        }
        p[d] = f32_to_bf16(o);
    }
}
void h3bo_qk_rmsnorm_rope(uint16_t* x, int64_t L, int64_t H, int64_t stride, int64_t q_off, int64_t k_off,
                          const uint16_t* qw, const uint16_t* kw, const uint16_t* ct, const uint16_t* st,
                          int rot, float eps) {
    int half = rot / 2;
    for (int64_t t = 0; t < L; ++t)
        for (int64_t h = 0; h < H; ++h) {
            rms_rope_vec(x + t * stride + q_off + h * 128, qw, ct + t * half, st + t * half, rot, eps);
            rms_rope_vec(x + t * stride + k_off + h * 128, kw, ct + t * half, st + t * half, rot, eps);
        }
}

/* V -> FP8 E4M3 with per-(head, channel) scale absmax/2.25, transposed to
 * [H, 128, Lpad] (compact_fp8.py:205-300, without the sm89 16-row permutation).
 * scaled = float(v) * (2.25 / absmax); an all-zero channel writes zeros, scale 0. */
void h3bo_value_fp8(const uint16_t* v, int64_t L, int64_t H, int64_t Lpad, uint8_t* vt, float* vscale) {
    const int D = 128;
    for (int64_t h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d) {
            float amax = 0.0f;
            for (int64_t l = 0; l < L; ++l) amax = fmaxf(amax, fabsf(bf16_to_f32(v[(l * H + h) * D + d])));
            float mul = amax > 0.0f ? 2.25f / amax : 0.0f;
            vscale[h * D + d] = amax / 2.25f;
            for (int64_t l = 0; l < Lpad; ++l) {
                uint8_t c = 0;
                if (l < L) c = h3bo_f32_to_e4m3(bf16_to_f32(v[(l * H + h) * D + d]) * mul);
                vt[(h * D + d) * Lpad + l] = c;
            }
        }
}

/* ------------------------------------------------------------------------- */
/* Block-sparse mask: pooled scores, softmax, selection, rails, LUT          */
/* (kernels.py:3668-3941; sparse_lut.py:25-74)                               */
/* ------------------------------------------------------------------------- */

/* One row of pooled-score probabilities, bit-identical to the CUDA mask kernel:
 *   score_j = bf16(sum_d fma(pq[d], pk_j[d]))   (d ascending)
 *   x_j = bf16(score_j * 128^-0.5), -inf where K block j is not self-similar
 *   p_j = bf16(exp(x_j - max) / sum) with the sum taken lane-strided over 32
 *   lanes (lane l adds j = l, l+32, ... in order) then butterfly-reduced. */
static void score_row(const uint16_t* pq, const uint16_t* pk_head, const uint8_t* simk, int64_t Kb,
                      uint16_t* p_out) {
    const float kScale = 0.08838834764831845f;
    float* x = (float*)malloc(sizeof(float) * (size_t)Kb);
    float mx = -INFINITY;
    for (int64_t j = 0; j < Kb; ++j) {
        float acc = 0.0f;
        for (int d = 0; d < 128; ++d) acc = fmaf(bf16_to_f32(pq[d]), bf16_to_f32(pk_head[j * 128 + d]), acc);
        float sc = bf16r(bf16r(acc) * kScale);
        if (!simk[j]) sc = -INFINITY;
        x[j] = sc;
        mx = fmaxf(mx, sc);
    }
    float lanes[32];
    for (int l = 0; l < 32; ++l) lanes[l] = 0.0f;
    for (int64_t j = 0; j < Kb; ++j) {
        float e = h3bo_expf(x[j] - mx);
        x[j] = e;
        lanes[j & 31] = lanes[j & 31] + e;
    }
    float sum = warp_butterfly_sum(lanes);
    for (int64_t j = 0; j < Kb; ++j) p_out[j] = f32_to_bf16(x[j] / sum);
    free(x);
}

/* Ranks by (probability desc, index asc).  Returns the selection flags for the
 * first `count` ranks. */
static int cmp_desc_idx(const void* a, const void* b) {
    const uint32_t ka = *(const uint32_t*)a, kb = *(const uint32_t*)b;
    /* key = (prob_bits << 16) | (0xffff - idx): larger key = higher rank */
    return ka < kb ? 1 : ka > kb ? -1 : 0;
}

/* mode 0: fixed Top-K, count = (int64)(topk[h] * Kb) (kernels.py:3206-3253)
 * mode 1: top-CDF, count = #{r : cdf_r <= cdf_thr[h]} with cdf_r the sum of the
 *         sorted probabilities of ranks 0..r (SpargeAttn meansim rule), summed
 *         exactly in 2^-56 fixed point so any summation order gives the same count
 * rails (always): non-similar K column, non-similar Q row, the first
 *   `protected_kb` columns; optional (flags bit0) column 0, (bit1) the diagonal
 *   K blocks covering the Q block's rows; (temporal_radius >= 0) the temporal
 *   correspondence rail of kernels.py:5206-5294 for an (frames x frame_tokens)
 *   video that starts after `protected_tokens` prefix keys; with `q_index`
 *   (a chunk of selected queries, kernels.py:5247-5254) query block i's centre
 *   is q_index[min(128 i + 64, q_tokens - 1)], else that row number itself;
 *   the first `protected_qb` query blocks keep every key block
 *   (kernels.py:2423-2426).
 * Output: bitmap words [H, Qb, ceil(Kb/32)], bit j%32 of word j/32. */
void h3bo_block_mask(const uint16_t* pooled_q, const uint8_t* simq, int64_t Qb, const uint16_t* pooled_k,
                     const uint8_t* simk, int64_t Kb, int64_t H, int mode, const float* budget,
                     int64_t protected_kb, int flags, int temporal_radius, int temporal_spatial_radius,
                     int64_t frames, int64_t frame_tokens, int64_t protected_tokens, int64_t q_tokens,
                     const int64_t* q_index, int64_t protected_qb, uint32_t* bitmap) {
    int64_t words = (Kb + 31) / 32;
    uint16_t* p = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)Kb);
    uint32_t* keys = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)Kb);
    for (int64_t h = 0; h < H; ++h)
        for (int64_t i = 0; i < Qb; ++i) {
            uint32_t* row = bitmap + (h * Qb + i) * words;
            memset(row, 0, sizeof(uint32_t) * (size_t)words);
            int any_sim = 0;
            for (int64_t j = 0; j < Kb; ++j) any_sim |= simk[h * Kb + j];
            if (any_sim) {
                score_row(pooled_q + (h * Qb + i) * 128, pooled_k + h * Kb * 128, simk + h * Kb, Kb, p);
                for (int64_t j = 0; j < Kb; ++j) keys[j] = ((uint32_t)p[j] << 16) | (uint32_t)(0xffff - j);
                qsort(keys, (size_t)Kb, sizeof(uint32_t), cmp_desc_idx);
                int64_t count;
                if (mode == 0) {
                    count = (int64_t)(budget[h] * (float)Kb);
                } else {
                    /* cumulative probability in exact 2^-56 fixed point */
                    uint64_t thr_fx = (uint64_t)(budget[h] * 72057594037927936.0f);
                    uint64_t cdf = 0; count = 0;
                    for (int64_t r = 0; r < Kb; ++r) {
                        cdf += (uint64_t)(bf16_to_f32((uint16_t)(keys[r] >> 16)) * 72057594037927936.0f);
                        if (cdf <= thr_fx) count = r + 1; else break;
                    }
                }
                if (count > Kb) count = Kb;
                for (int64_t r = 0; r < count; ++r) {
                    int64_t j = 0xffff - (int64_t)(keys[r] & 0xffff);
                    row[j / 32] |= 1u << (j % 32);
                }
            }
            for (int64_t j = 0; j < Kb; ++j) {
                int on = !simk[h * Kb + j] || !simq[h * Qb + i] || j < protected_kb || i < protected_qb;
                if ((flags & 1) && j == 0) on = 1;
                if ((flags & 2) && (j == 2 * i || j == 2 * i + 1)) on = 1;
                if (temporal_radius >= 0 && frame_tokens > 0) {
                    int64_t video = frames * frame_tokens;
                    int64_t qc = i * 128 + 64; if (qc > q_tokens - 1) qc = q_tokens - 1;
                    if (q_index) qc = q_index[qc];
                    int64_t qf = qc / frame_tokens, qs = qc % frame_tokens;
                    int64_t kc = j * 64 + 32 - protected_tokens;
                    int valid = kc >= 0 && kc < video;
                    int64_t kcc = kc < 0 ? 0 : (kc > video - 1 ? video - 1 : kc);
                    int64_t kf = kcc / frame_tokens, ks = kcc % frame_tokens;
                    int64_t dist = 96 + (int64_t)temporal_spatial_radius * 64;
                    if (valid && llabs(qf - kf) <= temporal_radius && llabs(qs - ks) <= dist) on = 1;
                }
                if (on) row[j / 32] |= 1u << (j % 32);
            }
        }
    free(p); free(keys);
}

/* Bitmap -> Sparge delta LUT ABI (sparse_lut.py:25-74): per row the selected
 * block indices ascending, first entry absolute, later entries deltas; the
 * unused tail of each full-stride row is zero here (unspecified upstream). */
void h3bo_bitmap_to_lut(const uint32_t* bitmap, int64_t rows, int64_t Kb, int32_t* lut, int32_t* valid) {
    int64_t words = (Kb + 31) / 32;
    for (int64_t r = 0; r < rows; ++r) {
        int32_t n = 0, prev = 0;
        for (int64_t j = 0; j < Kb; ++j)
            if (bitmap[r * words + j / 32] >> (j % 32) & 1u) {
                lut[r * Kb + n] = (int32_t)j - prev;
                prev = (int32_t)j;
                ++n;
            }
        for (int64_t t = n; t < Kb; ++t) lut[r * Kb + t] = 0;
        valid[r] = n;
    }
}

/* ------------------------------------------------------------------------- */
/* Quantized attention reference                                             */
/* ------------------------------------------------------------------------- */

/* O[l,h,:] = sum_j softmax_j(s) * V_j with s_j = S_ij * qs * ks * sm_scale,
 * S = int8 Q . int8 K (exact), V = e4m3(vt) * vscale[h,d].  Only K blocks whose
 * bit is set in `bitmap` (may be NULL = dense) are visited; keys >= Lk are
 * excluded.  Softmax in double.  Output bf16 NHD [Lq, H, 128].
 * q: [H, Lqpad, 128] int8, qscale [H, ceil(Lq/qblk)]; k: [H, Lkpad, 128] int8,
 * kscale [H, ceil(Lk/64)]; vt: [H,128,Lkpad] e4m3 bytes. */
void h3bo_attention(const int8_t* q, const float* qscale, int qblk, int64_t Lq, int64_t Lqpad,
                    const int8_t* k, const float* kscale, int64_t Lk, int64_t Lkpad,
                    const uint8_t* vt, const float* vscale, int64_t H, const uint32_t* bitmap,
                    float sm_scale, uint16_t* out) {
    const int D = 128;
    int64_t Kb = (Lk + 63) / 64, Qb = (Lq + 127) / 128, words = (Kb + 31) / 32;
    int64_t nqs = (Lq + qblk - 1) / qblk;
#pragma omp parallel
    {
        double* s = (double*)malloc(sizeof(double) * (size_t)Lk);
        double* o = (double*)malloc(sizeof(double) * D);
#pragma omp for schedule(dynamic) collapse(2)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t i = 0; i < Lq; ++i) {
                const int8_t* qr = q + (h * Lqpad + i) * D;
                float qs = qscale[h * nqs + i / qblk];
                const uint32_t* brow = bitmap ? bitmap + (h * Qb + i / 128) * words : NULL;
                double mx = -INFINITY;
                for (int64_t j = 0; j < Lk; ++j) {
                    int64_t kb = j / 64;
                    if (brow && !((brow[kb / 32] >> (kb % 32)) & 1u)) { s[j] = -INFINITY; continue; }
                    const int8_t* kr = k + (h * Lkpad + j) * D;
                    int32_t acc = 0;
                    for (int d = 0; d < D; ++d) acc += (int32_t)qr[d] * (int32_t)kr[d];
                    s[j] = (double)acc * (double)qs * (double)kscale[h * Kb + kb] * (double)sm_scale;
                    if (s[j] > mx) mx = s[j];
                }
                for (int d = 0; d < D; ++d) o[d] = 0.0;
                double l = 0.0;
                for (int64_t j = 0; j < Lk; ++j) {
                    if (s[j] == -INFINITY) continue;
                    double pj = exp(s[j] - mx);
                    l += pj;
                    for (int d = 0; d < D; ++d)
                        o[d] += pj * (double)h3bo_e4m3_to_f32(vt[(h * D + d) * Lkpad + j]);
                }
                for (int d = 0; d < D; ++d) {
                    double val = l > 0 ? o[d] / l * (double)vscale[h * D + d] : 0.0;
                    out[(i * H + h) * D + d] = f32_to_bf16((float)val);
                }
            }
        free(s); free(o);
    }
}

/* W4A8 group correction (comfy_kitchen backends/cuda/__init__.py:2294-2297):
 *   sx[m, g] = bf16(bf16(sum of the G codes of group g) * bf16(xs[m]))
 *   out[m, n] = bf16(float(out[m, n]) + sum_g sx[m, g] * corr[g, n])
 * corr: bf16 bits [K/G, N]; the sum over groups in double (the GPU accumulates the
 * exact bf16 products in fp32 inside the tensor core). */
void h3bo_w4a8_correction(const int8_t* xq, const float* xs, int64_t M, int64_t K, int64_t G,
                          const uint16_t* corr, int64_t N, uint16_t* out) {
    const int64_t groups = K / G;
    float* sx = (float*)malloc(sizeof(float) * (size_t)groups);
    for (int64_t m = 0; m < M; ++m) {
        const float xb = bf16r(xs[m]);
        for (int64_t g = 0; g < groups; ++g) {
            int32_t sum = 0;
            for (int64_t k = 0; k < G; ++k) sum += xq[m * K + g * G + k];
            sx[g] = bf16r(bf16r((float)sum) * xb);
        }
        for (int64_t n = 0; n < N; ++n) {
            double dot = 0.0;
            for (int64_t g = 0; g < groups; ++g) dot += (double)sx[g] * (double)bf16_to_f32(corr[g * N + n]);
            out[m * N + n] = f32_to_bf16(bf16_to_f32(out[m * N + n]) + (float)dot);
        }
    }
    free(sx);
}

/* ------------------------------------------------------------------------- */
/* Quantized attention with the kernel's own P arithmetic                    */
/* ------------------------------------------------------------------------- */

/* Scale groups of the Sage quantization granularities (the reference's
 * qk_quant_gran codes, model/kernels.py:4142-4160, 7652-7660):
 *   Q  gran 0: rows [g * q_block, (g+1) * q_block) share a scale (per-block 128 /
 *              64, per_warp 32); index i / q_block, ceil(Lq / q_block) per head;
 *      gran 1: per_thread -- in each 32-row group the rows with equal i % 8 share a
 *              scale; index (i / 32) * 8 + i % 8, ceil(Lq / 128) * 32 per head.
 *   K  gran 0: one scale per 64-key block, index j / 64, ceil(Lk / 64) per head;
 *      gran 1: per_thread -- in each 64-key block the keys with equal (j % 8) / 2
 *              share a scale; index (j / 64) * 4 + (j % 8) / 2, ceil(Lk / 64) * 4
 *              per head (model/sage_fused_quant.py:41-44). */
static inline int64_t q_scale_index(int64_t i, int q_gran, int q_block) {
    return q_gran == 1 ? (i / 32) * 8 + (i % 8) : i / q_block;
}
static inline int64_t k_scale_index(int64_t j, int k_gran) {
    return k_gran == 1 ? (j / 64) * 4 + (j % 8) / 2 : j / 64;
}

/* 2^x on the FMA pipe, the attention kernel's own polynomial (attn.cu exp2_poly2,
 * fitted for that kernel): j = rint(x) through the 1.5 * 2^23 constant, 2^(x - j)
 * by a degree-3 polynomial, j added to the exponent field; x clamped at -125. */
#ifndef H3BO_ATTN_POLY_MASK16
#define H3BO_ATTN_POLY_MASK16 0x08u
#endif
static float attn_exp2_poly(float x) {
    const float kM = 12582912.0f;
    const float P0 = 0.9999280571937561f, P1 = 0.6932609677314758f, P2 = 0.2426111251115799f,
                P3 = 0.05517164617776871f;
    float xp = x > -125.0f ? x : -125.0f;
    if (x != x) xp = -125.0f;
    float t = xp + kM;
    float f = fmaf(t + (-kM), -1.0f, xp);
    float q = fmaf(fmaf(fmaf(P3, f, P2), f, P1), f, P0);
    return u2f(f2u(q) + (f2u(t) << 23));
}

/* 2^x as the kernel's ex2.approx computes it, up to its last-bit error: double
 * exp2 rounded to float (0 for -inf). */
static float attn_exp2(float x) {
    if (x == -INFINITY) return 0.0f;
    return (float)exp2((double)x);
}

/* O = softmax(Q K^T * sm_scale) V in the attention kernel's arithmetic (attn.cu):
 * for each query row, the key blocks its 128-row tile visits (all, or the bitmap's
 * set bits) in ascending order, two per step (the last step may hold one):
 *   v_j   = float(1.5 * 2^23 + S_j), S_j the exact int32 Q.K dot product
 *   c     = max(qs * (sm_scale * log2 e) * ks, 1e-30)      (per scale group)
 *   tmax  = max over the step's groups of (max_j v_j - 1.5 * 2^23) * c
 *   m     = tmax if tmax > m + 2 else m (lazy running max); alpha = 2^(m_old - m)
 *   x_j   = fma(v_j, c, (log2 112 - m) - 1.5 * 2^23 * c)
 *   P_j   = 2^x_j: the polynomial above on the column pairs (2i, 2i + 1) of every 16
 *           columns of a block whose bit i is set in H3BO_ATTN_POLY_MASK16 (the
 *           kernel's kPolyMask16),
 *           ex2 (hardware, modelled by a correctly rounded exp2) on the others
 *   l     = l * alpha + (sum of the step's fp32 P_j in the kernel's order)
 *   O     = O * alpha + sum_j E4M3(P_j) * E4M3(V_j) * (accumulated in double here;
 *           fp32 in tensor memory on the GPU)
 *   out   = bf16(float(O) * (1 / l) * v_scale[d])
 * Keys >= Lk are -inf (P = 0 on ex2 columns, 2^-125 on polynomial columns, as on
 * the GPU).  Rows whose tile visits no block are 0.  The GPU result differs from
 * this only by ex2.approx's last bits and the tensor core's fp32 accumulation. */
void h3bo_attention_kernel(const int8_t* q, const float* qscale, int q_gran, int q_block, int64_t Lq,
                           int64_t Lqpad, const int8_t* k, const float* kscale, int k_gran, int64_t Lk,
                           int64_t Lkpad, const uint8_t* vt, const float* vscale, int64_t H,
                           const uint32_t* bitmap, float sm_scale, uint16_t* out) {
    const int D = 128;
    const float kM = 12582912.0f, kLog2_112 = 6.807354922057604f, kTau = 2.0f;
    const int64_t Kb = (Lk + 63) / 64, Qb = (Lq + 127) / 128, words = (Kb + 31) / 32;
    const int64_t nqs = q_gran == 1 ? Qb * 32 : (Lq + q_block - 1) / q_block;
    const int64_t nks = k_gran == 1 ? Kb * 4 : Kb;
    const float scale_log2 = sm_scale * 1.4426950408889634f;
    float vlut[256];
    for (int i = 0; i < 256; ++i) vlut[i] = h3bo_e4m3_to_f32((uint8_t)i);
#pragma omp parallel
    {
        int64_t* blocks = (int64_t*)malloc(sizeof(int64_t) * (size_t)(Kb + 1));
        double* o = (double*)malloc(sizeof(double) * D);
        float vrow[128];
        uint8_t pq8[128];
#pragma omp for schedule(dynamic) collapse(2)
        for (int64_t h = 0; h < H; ++h)
            for (int64_t i = 0; i < Lq; ++i) {
                const int8_t* qr = q + (h * Lqpad + i) * D;
                const float qs = qscale[h * nqs + q_scale_index(i, q_gran, q_block)];
                const float qsl = qs * scale_log2;
                int64_t nb = 0;
                const uint32_t* brow = bitmap ? bitmap + (h * Qb + i / 128) * words : NULL;
                for (int64_t b = 0; b < Kb; ++b)
                    if (!brow || ((brow[b / 32] >> (b % 32)) & 1u)) blocks[nb++] = b;
                float m = -INFINITY, l = 0.0f;
                for (int d = 0; d < D; ++d) o[d] = 0.0;
                for (int64_t st = 0; st < nb; st += 2) {
                    const int nblk = st + 1 < nb ? 2 : 1;
                    float v[2][64], c[2][4];
                    float tmax = -INFINITY;
                    for (int u = 0; u < nblk; ++u) {
                        const int64_t b = blocks[st + u];
                        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                        for (int g = 0; g < 4; ++g) {
                            const float ks = kscale[h * nks + (k_gran == 1 ? b * 4 + g : b)];
                            float cc = qsl * ks;
                            c[u][g] = cc > 1e-30f ? cc : 1e-30f;
                        }
                        for (int cidx = 0; cidx < 64; ++cidx) {
                            const int64_t j = b * 64 + cidx;
                            if (j >= Lk) { v[u][cidx] = -INFINITY; continue; }
                            const int8_t* kr = k + (h * Lkpad + j) * D;
                            int32_t acc = 0;
                            for (int d = 0; d < D; ++d) acc += (int32_t)qr[d] * (int32_t)kr[d];
                            v[u][cidx] = kM + (float)acc;   /* exact: |acc| < 2^22 */
                            const int g = k_gran == 1 ? (cidx % 8) / 2 : 0;
                            if (v[u][cidx] > mx[g]) mx[g] = v[u][cidx];
                        }
                        for (int g = 0; g < (k_gran == 1 ? 4 : 1); ++g)
                            if (mx[g] != -INFINITY) {
                                const float t = (mx[g] - kM) * c[u][g];
                                if (t > tmax) tmax = t;
                            }
                    }
                    const float m_new = tmax > m + kTau ? tmax : m;
                    float alpha = 1.0f;
                    if (m_new != m) {
                        alpha = attn_exp2(m - m_new);
                        m = m_new;
                        for (int d = 0; d < D; ++d) o[d] = (double)((float)o[d] * alpha);
                    }
                    const float off = kLog2_112 - m;
                    float psum = 0.0f;
                    for (int u = 0; u < nblk; ++u) {
                        const int64_t b = blocks[st + u];
                        float oo[4];
                        for (int g = 0; g < 4; ++g) oo[g] = off - kM * c[u][g];
                        float p[64];
                        for (int cidx = 0; cidx < 64; ++cidx) {
                            const int g = k_gran == 1 ? (cidx % 8) / 2 : 0;
                            const float x = fmaf(v[u][cidx], c[u][g], oo[g]);
                            const int poly = (int)((H3BO_ATTN_POLY_MASK16 >> ((cidx % 16) >> 1)) & 1u);
                            p[cidx] = poly ? attn_exp2_poly(x) : attn_exp2(x);
                        }
                        /* the kernel's order: four fp32 accumulators over packed pairs */
                        float a0x = 0.f, a0y = 0.f, a1x = 0.f, a1y = 0.f;
                        for (int cb = 0; cb < 64; cb += 8) {
                            a0x = a0x + p[cb + 0]; a0y = a0y + p[cb + 1];
                            a1x = a1x + p[cb + 2]; a1y = a1y + p[cb + 3];
                            a0x = a0x + p[cb + 4]; a0y = a0y + p[cb + 5];
                            a1x = a1x + p[cb + 6]; a1y = a1y + p[cb + 7];
                        }
                        const float bsum = (a0x + a1x) + (a0y + a1y);
                        psum = u == 0 ? bsum : psum + bsum;
                        for (int cidx = 0; cidx < 64; ++cidx) {
                            pq8[cidx] = h3bo_f32_to_e4m3(p[cidx]);
                        }
                        for (int cidx = 0; cidx < 64; ++cidx) {
                            const int64_t j = b * 64 + cidx;
                            const float pe = vlut[pq8[cidx]];
                            if (pe == 0.0f) continue;
                            for (int d = 0; d < D; ++d) vrow[d] = vlut[vt[(h * D + d) * Lkpad + j]];
                            for (int d = 0; d < D; ++d) o[d] += (double)pe * (double)vrow[d];
                        }
                    }
                    l = l * alpha + psum;
                }
                uint16_t* dst = out + (i * H + h) * D;
                if (nb == 0) { for (int d = 0; d < D; ++d) dst[d] = 0; continue; }
                const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
                for (int d = 0; d < D; ++d) dst[d] = f32_to_bf16(((float)o[d] * inv_l) * vscale[h * D + d]);
            }
        free(blocks); free(o);
    }
}

/* convenience exports for the Python side */
uint16_t h3bo_f32_to_bf16(float f) { return f32_to_bf16(f); }
uint16_t h3bo_f32_to_f16(float f) { return f32_to_f16(f); }
