// gemm_i8.cu -- INT8 x INT8 -> INT32 GEMM on the sm_100 tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory), with the linear's
// dequant epilogue fused:  D = bf16(float(acc) * xs[m] * ws[n] + bias[n]),
// optionally added into a bf16 residual stream with a per-column gate.
//
// Two kernels.  Large problems (at least one 256 x 256 tile per SM) run the
// 2-SM kernel at the end of this file; the rest run this 1-SM kernel.
// Persistent, warp-specialized CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: A [128 x 128 B] and B [BN x 128 B] tiles into a
//               kStages-deep shared-memory ring (128-byte swizzle, no multicast)
//   warp 1      TMEM allocator + MMA issuer (one thread): 4 x K=32 MMAs per
//               stage into one of two TMEM accumulators (2 x BN columns)
//   warps 2..5  epilogue: tcgen05.ld of 32 columns at a time, dequant, store;
//               the other accumulator is being filled meanwhile
// Tiles are walked M-major (all N tiles of one 128-row band before the next
// band) so the A band and the whole weight matrix stay L2-resident.
#include "h3b_kernels.cuh"
#include "h3b_packed.cuh"

namespace h3b {

constexpr int kBM = 128;
constexpr int kBK = 128;  // bytes of K per stage = one 128-byte swizzle row
constexpr int kGemmThreads = 192;



template <int BN>
struct GemmSmem {
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kTotal = kBarOffset + 256 + 1024;  // barriers + alignment slack
};

// Every loop over the 32 accumulators is fully unrolled (tails guarded per element):
// a loop bounded by N would index r[] and y[] at run time and put them in local memory.
__device__ __forceinline__ void epi_store_chunk(const uint32_t (&r)[32], int m, int n0, const GemmArgs& a,
                                                float xs_m, int kind) {
  const int N = a.N;
  if (kind == kEpiAddF32) {
    uint16_t* dst = a.out + (int64_t)m * a.out_stride + n0;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const int n = n0 + j;
      if (n + 1 < N) {
        const uint32_t o = *reinterpret_cast<const uint32_t*>(dst + j);
        const float y0 = __fadd_rn(__uint_as_float(o << 16), __uint_as_float(r[j]));
        const float y1 = __fadd_rn(__uint_as_float(o & 0xffff0000u), __uint_as_float(r[j + 1]));
        *reinterpret_cast<uint32_t*>(dst + j) =
            (uint32_t)f32_to_bf16_bits(y0) | ((uint32_t)f32_to_bf16_bits(y1) << 16);
      } else if (n < N) {
        dst[j] = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(dst[j]), __uint_as_float(r[j])));
      }
    }
    return;
  }
  if (kind == kEpiInt32) {
    int32_t* dst = a.out_i32 + (int64_t)m * a.out_stride + n0;
    if (n0 + 32 <= N && (a.out_stride % 4) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(dst + j) = make_int4((int)r[j], (int)r[j + 1], (int)r[j + 2], (int)r[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < N) dst[j] = (int)r[j];
    }
    return;
  }
  float y[32];
  const bool full = n0 + 32 <= N;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int n = n0 + j;
    const int nn = n < N ? n : N - 1;
    const float w = a.ws_scalar ? a.ws[0] : __ldg(a.ws + nn);
    const float v = __fmul_rn((float)(int)r[j], xs_m);
    y[j] = a.bias ? fmaf(v, w, __ldg(a.bias + nn)) : __fmul_rn(v, w);
  }
  uint16_t* dst = a.out + (int64_t)m * a.out_stride + n0;
  const bool vec = full && ((a.out_stride & 7) == 0) && ((n0 & 7) == 0) && ((uintptr_t)a.out & 15) == 0;
  if (kind == kEpiStore) {
    if (vec) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 p;
        p.x = (uint32_t)f32_to_bf16_bits(y[j]) | ((uint32_t)f32_to_bf16_bits(y[j + 1]) << 16);
        p.y = (uint32_t)f32_to_bf16_bits(y[j + 2]) | ((uint32_t)f32_to_bf16_bits(y[j + 3]) << 16);
        p.z = (uint32_t)f32_to_bf16_bits(y[j + 4]) | ((uint32_t)f32_to_bf16_bits(y[j + 5]) << 16);
        p.w = (uint32_t)f32_to_bf16_bits(y[j + 6]) | ((uint32_t)f32_to_bf16_bits(y[j + 7]) << 16);
        *reinterpret_cast<uint4*>(dst + j) = p;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < N) dst[j] = f32_to_bf16_bits(y[j]);
    }
  } else {  // gated residual, in place
    if (vec) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 rv = *reinterpret_cast<const uint4*>(dst + j);
        uint4 gv = __ldg(reinterpret_cast<const uint4*>(a.gate + n0 + j));
        uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w}, ow[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float r0 = __uint_as_float(rw[h] << 16), r1 = __uint_as_float(rw[h] & 0xffff0000u);
          float g0 = __uint_as_float(gw[h] << 16), g1 = __uint_as_float(gw[h] & 0xffff0000u);
          float o0 = __fadd_rn(r0, __fmul_rn(bf16r(y[j + 2 * h]), g0));
          float o1 = __fadd_rn(r1, __fmul_rn(bf16r(y[j + 2 * h + 1]), g1));
          ow[h] = (uint32_t)f32_to_bf16_bits(o0) | ((uint32_t)f32_to_bf16_bits(o1) << 16);
        }
        *reinterpret_cast<uint4*>(dst + j) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (n0 + j >= N) continue;
        float rr = bf16_bits_to_f32(dst[j]);
        float g = bf16_bits_to_f32(a.gate[n0 + j]);
        dst[j] = f32_to_bf16_bits(__fadd_rn(rr, __fmul_rn(bf16r(y[j]), g)));
      }
    }
  }
}

// q/k epilogue of one 128-column head [n_h, n_h + 128) of row m, from its four
// 32-column accumulator chunks: the bf16 dequantized values (as the store epilogue
// writes them), then, exactly as qk_rmsnorm_rope_kernel computes them, the head's
// RMSNorm (sum of squares in the order of that kernel's warp butterfly over 32
// four-channel groups) and the split-half RoPE of channels [0, 2 * HALF).
template <int HALF>
__device__ __forceinline__ void qk_head_finish(uint32_t (&yb)[64], float (&s)[16], int m, int n_h,
                                               const uint16_t* normw, const GemmArgs& a) {
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) s[i] = __fadd_rn(s[i], s[i + w]);
  }
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s[0], 0.0078125f), a.qk_eps)));
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(normw + 8 * q));
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint32_t y = yb[4 * q + e];
      const float v0 = __uint_as_float(y << 16), v1 = __uint_as_float(y & 0xffff0000u);
      const float w0 = __uint_as_float(ww[e] << 16), w1 = __uint_as_float(ww[e] & 0xffff0000u);
      yb[4 * q + e] = bf16x2_bits(__fmul_rn(__fmul_rn(v0, inv), w0), __fmul_rn(__fmul_rn(v1, inv), w1));
    }
  }
  const int64_t tok = m < a.M ? m : a.M - 1;  // rows past M (ragged last tile) store nothing
#pragma unroll
  for (int q = 0; q < HALF / 8; ++q) {
    const uint4 cv = __ldg(reinterpret_cast<const uint4*>(a.cos_t + tok * HALF + 8 * q));
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(a.sin_t + tok * HALF + 8 * q));
    const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * q + e, j = i + HALF / 2;  // words of channels (d, d+1) and (d+HALF, d+HALF+1)
      const float n0 = __uint_as_float(yb[i] << 16), n1 = __uint_as_float(yb[i] & 0xffff0000u);
      const float p0 = __uint_as_float(yb[j] << 16), p1 = __uint_as_float(yb[j] & 0xffff0000u);
      const float c0 = __uint_as_float(cw[e] << 16), c1 = __uint_as_float(cw[e] & 0xffff0000u);
      const float s0 = __uint_as_float(sw[e] << 16), s1 = __uint_as_float(sw[e] & 0xffff0000u);
      yb[i] = bf16x2_bits(__fsub_rn(__fmul_rn(n0, c0), __fmul_rn(p0, s0)),
                          __fsub_rn(__fmul_rn(n1, c1), __fmul_rn(p1, s1)));
      yb[j] = bf16x2_bits(__fadd_rn(__fmul_rn(n0, s0), __fmul_rn(p0, c0)),
                          __fadd_rn(__fmul_rn(n1, s1), __fmul_rn(p1, c1)));
    }
  }
  if (m < a.M) {
    uint16_t* dst = a.out + (int64_t)m * a.out_stride + n_h;
#pragma unroll
    for (int q = 0; q < 16; ++q)
      *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(yb[4 * q], yb[4 * q + 1], yb[4 * q + 2], yb[4 * q + 3]);
  }
}

// One 32-column chunk c of a q/k head: bf16 values into yb[16c .. 16c + 15]; the
// sums of squares g of its eight four-channel groups (groups 8c .. 8c + 7 of 32)
// go into s: chunks 0, 1 store g, chunks 2, 3 add it (s[i] = g[i] + g[i + 16],
// the first level of the butterfly tree).
__device__ __forceinline__ void qk_head_chunk(const uint32_t (&r)[32], int c, int n0, const GemmArgs& a, float xs_m,
                                              uint32_t (&yb)[64], float (&s)[16]) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    float y2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int n = n0 + j + e;
      const float w = a.ws_scalar ? a.ws[0] : __ldg(a.ws + n);
      const float v = __fmul_rn((float)(int)r[j + e], xs_m);
      y2[e] = a.bias ? fmaf(v, w, __ldg(a.bias + n)) : __fmul_rn(v, w);
    }
    yb[16 * c + j / 2] = (uint32_t)f32_to_bf16_bits(y2[0]) | ((uint32_t)f32_to_bf16_bits(y2[1]) << 16);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = yb[16 * c + 2 * i], hi = yb[16 * c + 2 * i + 1];
    const float v0 = __uint_as_float(lo << 16), v1 = __uint_as_float(lo & 0xffff0000u);
    const float v2 = __uint_as_float(hi << 16), v3 = __uint_as_float(hi & 0xffff0000u);
    const float g = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(v0, v0), __fmul_rn(v1, v1)), __fmul_rn(v2, v2)),
                              __fmul_rn(v3, v3));
    const int gi = (8 * c + i) & 15;
    s[gi] = c < 2 ? g : __fadd_rn(s[gi], g);
  }
}

template <int BN, int KIND>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs a) {
  using S = GemmSmem<BN>;
  constexpr int kStages = S::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;   // [2]
  uint64_t* tempty = tfull + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // GELU + ConvRot exchange: [quadrant][half][accumulator], "this half's values are in TMEM"
  uint64_t* xbar = reinterpret_cast<uint64_t*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (a.M + kBM - 1) / kBM, num_n = (a.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int num_k = (a.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // TMA producer: the whole warp runs the loop (warp-uniform control flow),
    // one elected lane issues the copies
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
      const int mb = t / num_n, nb = t % num_n;
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait_warp(&empty[stage], phase ^ 1, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) { ok = false; break; }
        if (elect_one()) {
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          // the tensor maps count elements: 128 int8 or 64 bf16 per 128-byte K step
          const int kx = KIND == kEpiAddF32 ? kb * (kBK / 2) : kb * kBK;
          tma_load_2d(sa, &tmA, &full[stage], kx, mb * kBM);
          tma_load_2d(sb, &tmB, &full[stage], kx, nb * BN);
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
    }
    // Drain: every filled stage must have been consumed (its TMA landed and
    // its MMAs finished) before the CTA may exit.  Bounded like every wait.
    for (int s2 = 0; s2 < kStages; ++s2) {
      if (!mbar_wait_warp(&empty[stage], phase ^ 1, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) break;
      if (++stage == kStages) { stage = 0; phase ^= 1; }
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp runs the loop (so descriptors stay in uniform
    // registers), one elected lane issues tcgen05.mma / commit
    constexpr uint32_t idesc = KIND == kEpiAddF32 ? idesc_bf16(kBM, BN) : idesc_i8(kBM, BN);
    const uint32_t smem_base = smem_u32(smem);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      if (!mbar_wait_warp(&tempty[acc], acc_phase ^ 1, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + (uint32_t)(acc * BN);
      bool ok = true;
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait_warp(&full[stage], phase, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_base + (uint32_t)(stage * S::kStageBytes);
        const uint64_t da = sdesc_kmajor_sw128(sa), db = sdesc_kmajor_sw128(sa + S::kABytes);
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            // +32 bytes of K per MMA (32 int8 or 16 bf16): +2 in the descriptor's 16-byte units
            if constexpr (KIND == kEpiAddF32)
              mma_bf16_ss(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
            else
              mma_i8_ss(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&tfull[acc]);
      __syncwarp();
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant (warp % 4)
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int mb = t / num_n, nb = t % num_n;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) break;
      tc_fence_after();
      __syncwarp();
      const int m = mb * kBM + row_in_tile;
      const float xs_m = (KIND != kEpiInt32 && KIND != kEpiAddF32 && m < a.M) ? __ldg(a.xs + m) : 0.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + (uint32_t)(c * 32), r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          tc_fence_before();
          mbar_arrive(&tempty[acc]);
        }
        const int n0 = nb * BN + c * 32;
        if (m < a.M && n0 < a.N) epi_store_chunk(r, m, n0, a, xs_m, KIND);
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ------------------------------------------------------------------ 2-SM variant
// A cluster of two CTAs on two SMs computes 256 x 256 output tiles with
// tcgen05.mma.cta_group::2 (M 256, N 256, K 32): each CTA loads its own 128 rows
// of A and one half (128 rows) of the B tile into its own shared memory, and the
// even CTA's MMA reads both CTAs' operands.  Per 128-deep K step an SM then reads
// 32 KB of operands from shared memory instead of the 1-SM kernel's 48 KB, which
// is what bounds the 1-SM kernel (shared-memory bandwidth, not the tensor pipe).
// Each CTA's tensor memory holds its 128 rows x 256 columns, two accumulators.
//   warp 0      TMA producer in both CTAs (no multicast); both signal the even
//               CTA's full barrier (count 2 + bytes)
//   warp 1      pair TMEM allocation in both CTAs; MMA issuer in the even CTA,
//               whose commits arrive on both CTAs' barriers (empty, tfull)
//   epilogue    in both CTAs (warps 4..11, two per TMEM lane quadrant, for the
//               bf16 kinds; warps 2..5 for the int32 kind, see PairCfg); each
//               warp releases the accumulator on the even CTA's tempty barrier
//               (count: epilogue warps x 2 CTAs)
template <int PBN>
struct PairSmem {
  static constexpr int kStages = PBN == 256 ? 6 : 8;
  static constexpr int kABytes = 128 * kBK;
  static constexpr int kBBytes = (PBN / 2) * kBK;  // this CTA's half of the B tile
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kTotal = kBarOffset + 512 + 1024;  // barriers + alignment slack
};

// ---------------------------------------------------------------- GELU + ConvRot epilogue
// A 256-column tile of FC1 holds one ConvRot group of each of its rows.  The two
// epilogue warps of a TMEM lane quadrant split it: warp hh takes 64-column blocks
// 2hh and 2hh + 1 as the two lanes of packed pairs.  Each value is the store
// epilogue's bf16 output (dequantized, bias added, rounded), then tanh-GELU, then
// the stride-1, -4 and -16 radix-4 stages of the transform, which stay inside a
// 64-column block; the results go back into the warp's own accumulator columns.
// After the partner warp has done the same, warp hh runs the stride-64 stage for
// butterfly positions [32 hh, 32 hh + 32) of the four blocks, stores the rotated
// values as bf16 and the absmax of its 128 fp32 outputs.  Every value passes the
// same butterflies with the same operands as in the standalone quantizer
// (quant_rows_kernel<kConvRot, gelu>), so the codes formed from these values equal
// that kernel's bit for bit.

// bf16(float(acc) * xs * ws[n] (+ bias[n])) on both lanes: the store epilogue's value
__device__ __forceinline__ float2 dequant_bf16x2(uint32_t r0, uint32_t r1, float xs_m, float2 w, float2 b,
                                                 bool has_bias) {
  const float2 v = mul2(make_float2((float)(int)r0, (float)(int)r1), splat2(xs_m));
  return bf16r2(has_bias ? fma2(v, w, b) : mul2(v, w));
}
// four consecutive per-column values (16-byte aligned: n is a multiple of 4)
__device__ __forceinline__ float4 ld_col4(const float* p, int n) {
  return __ldg(reinterpret_cast<const float4*>(p + n));
}

// GELU and the first three transform stages of this warp's two blocks, written back
// over the warp's own accumulator columns
__device__ __forceinline__ void gelu_rot_first_half(uint32_t taddr, int hh, int nbase, float xs_m,
                                                    const GemmArgs& a) {
  const uint32_t tcol = taddr + (uint32_t)(hh * 128);
  const int ncol = nbase + hh * 128;
  float2 v[4][16];  // [16-column chunk of the block][column], lanes = (block 2hh, block 2hh + 1)
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t r0[16], r1[16];
    tmem_ld16(tcol + (uint32_t)(q * 16), r0);
    tmem_ld16(tcol + (uint32_t)(64 + q * 16), r1);
    tmem_wait_ld();
    reg_barrier16(r0);
    reg_barrier16(r1);
#pragma unroll
    for (int j4 = 0; j4 < 16; j4 += 4) {
      const int n = ncol + q * 16 + j4;
      const float4 w0 = a.ws_scalar ? make_float4(a.ws[0], a.ws[0], a.ws[0], a.ws[0]) : ld_col4(a.ws, n);
      const float4 w1 = a.ws_scalar ? w0 : ld_col4(a.ws, n + 64);
      const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 b0 = a.bias ? ld_col4(a.bias, n) : zero;
      const float4 b1 = a.bias ? ld_col4(a.bias, n + 64) : zero;
      const float2 w[4] = {make_float2(w0.x, w1.x), make_float2(w0.y, w1.y), make_float2(w0.z, w1.z),
                           make_float2(w0.w, w1.w)};
      const float2 b[4] = {make_float2(b0.x, b1.x), make_float2(b0.y, b1.y), make_float2(b0.z, b1.z),
                           make_float2(b0.w, b1.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[q][j4 + j] = gelu_tanh2(dequant_bf16x2(r0[j4 + j], r1[j4 + j], xs_m, w[j], b[j], a.bias != nullptr));
    }
    fht16x2(v[q]);  // stride 1 and 4 inside the chunk
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {  // stride 16: the four chunks of the block
    const float2 x[4] = {v[0][j], v[1][j], v[2][j], v[3][j]};
    float2 y[4];
    h4_stage2(x, 1, y, 0);
    v[0][j] = y[0];
    v[1][j] = y[1];
    v[2][j] = y[2];
    v[3][j] = y[3];
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w0[16], w1[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      w0[j] = __float_as_uint(v[q][j].x);
      w1[j] = __float_as_uint(v[q][j].y);
    }
    tmem_st16(tcol + (uint32_t)(q * 16), w0);
    tmem_st16(tcol + (uint32_t)(64 + q * 16), w1);
  }
  tmem_wait_st();
}

// The stride-64 stage for positions [32 hh, 32 hh + 32) of the four blocks, the bf16
// stores and the absmax; releases the accumulator (cluster barrier address tempty)
// after the last TMEM read.
__device__ __forceinline__ void gelu_rot_second_half(uint32_t taddr, int hh, int nb, int m, const GemmArgs& a,
                                                     uint32_t tempty) {
  float amax = 0.0f;
  const bool live = m < a.M;
  uint16_t* dst_row = a.out + (int64_t)(live ? m : 0) * a.out_stride + (int64_t)nb * 256;
#pragma unroll
  for (int sub = 0; sub < 2; ++sub) {
    const int c0 = hh * 32 + sub * 16;
    uint32_t x[4][16];
#pragma unroll
    for (int b = 0; b < 4; ++b) tmem_ld16(taddr + (uint32_t)(b * 64 + c0), x[b]);
    tmem_wait_ld();
#pragma unroll
    for (int b = 0; b < 4; ++b) reg_barrier16(x[b]);
    if (sub == 1) {
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive_cluster(tempty);
    }
    uint32_t packed[4][8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 in[4] = {
          make_float2(__uint_as_float(x[0][2 * i]), __uint_as_float(x[0][2 * i + 1])),
          make_float2(__uint_as_float(x[1][2 * i]), __uint_as_float(x[1][2 * i + 1])),
          make_float2(__uint_as_float(x[2][2 * i]), __uint_as_float(x[2][2 * i + 1])),
          make_float2(__uint_as_float(x[3][2 * i]), __uint_as_float(x[3][2 * i + 1]))};
      float2 y[4];
      h4_stage2(in, 1, y, 0);
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        amax = fmaxf(amax, fmaxf(fabsf(y[b].x), fabsf(y[b].y)));
        packed[b][i] = bf16x2_bits(y[b].x, y[b].y);
      }
    }
    if (live) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint4* d = reinterpret_cast<uint4*>(dst_row + b * 64 + c0);
        d[0] = make_uint4(packed[b][0], packed[b][1], packed[b][2], packed[b][3]);
        d[1] = make_uint4(packed[b][4], packed[b][5], packed[b][6], packed[b][7]);
      }
    }
  }
  if (live) a.amax[(int64_t)m * a.amax_stride + 2 * nb + hh] = amax;
}

// Warp layout of the 2-SM kernel per epilogue kind.  The bf16 epilogues (store,
// gated residual, q/k norm + RoPE) run 8 epilogue warps, two per TMEM lane
// quadrant, each taking one 128-column half of the tile, in warpgroups 1 and 2;
// warpgroup 0 holds the producer and MMA warps (2 and 3 idle).  With one warp per
// quadrant the epilogue is latency-bound and, at K = 4096, slower than the MMAs of
// the next tile.  Registers are split with setmaxnreg: warpgroup 0 drops to
// kQkCtrlRegs, the epilogue warpgroups rise to kQkEpiRegs.  The split must not
// exceed the launch total; the host checks the compiled register count against
// kQkLaunchRegs.  The int32 verification kind keeps 192 threads, one epilogue warp
// per quadrant.
template <int KIND>
struct PairCfg {
  static constexpr bool kQk = KIND == kEpiQkRope64 || KIND == kEpiQkRope48;
  static constexpr bool kWide = kQk || KIND == kEpiResidual || KIND == kEpiStore || KIND == kEpiGeluRot;
  static constexpr int kThreads = kWide ? 384 : kGemmThreads;
  static constexpr int kEpiWarp0 = kWide ? 4 : 2;
  static constexpr int kEpiWarps = kWide ? 8 : 4;
};
constexpr int kQkLaunchRegs = 168;
constexpr int kQkCtrlRegs = 72;
constexpr int kQkEpiRegs = 216;
static_assert(128 * kQkCtrlRegs + 256 * kQkEpiRegs <= 384 * kQkLaunchRegs, "register split too large");

// The pair tile is 256 x PBN; each CTA's tensor memory holds 2 x PBN columns.
template <int PBN, int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<KIND>::kThreads, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmArgs a) {
  using S = PairSmem<PBN>;
  constexpr int kPairStages = S::kStages;
  constexpr int kPairABytes = S::kABytes;
  constexpr int kPairStageBytes = S::kStageBytes;
  constexpr int kPairBarOffset = S::kBarOffset;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairBarOffset);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;  // [2]
  uint64_t* tempty = tfull + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // GELU + ConvRot exchange: [quadrant][half][accumulator], "this half's values are in TMEM"
  uint64_t* xbar = reinterpret_cast<uint64_t*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int num_m = (a.M + 255) / 256, num_n = (a.N + PBN - 1) / PBN;
  const int tiles = num_m * num_n;
  const int num_k = (a.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * PairCfg<KIND>::kEpiWarps);
    }
    if (KIND == kEpiGeluRot)
      for (int b = 0; b < 16; ++b) mbar_init(&xbar[b], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * PBN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and the pair's TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  {
    // the pair allocation must hand both CTAs the same columns; otherwise do no work
    uint32_t leader_base;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(leader_base) : "r"(mapa_shared(smem_u32(tmem_slot), 0)));
    if (leader_base != tmem_base) {
      if (threadIdx.x == 0) record_status(H3B_STATUS_GEMM_TIMEOUT);
      *abort_flag = 1;
    }
  }
  __syncthreads();
  const bool pair_ok = *abort_flag == 0;
  const uint32_t full0 = mapa_shared(smem_u32(full), 0);
  const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);

  if constexpr (PairCfg<KIND>::kWide) {
    if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kQkCtrlRegs));
  }
  if (warp == 0) {
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = pair; ok && pair_ok && t < tiles; t += pairs) {
      const int mb = t / num_n, nb = t % num_n;
      for (int kb = 0; kb < num_k; ++kb) {
        if (!mbar_wait_warp(&empty[stage], phase ^ 1, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) { ok = false; break; }
        if (elect_one()) {
          uint8_t* sa = smem + stage * kPairStageBytes;
          const uint32_t fb = full0 + (uint32_t)(stage * 8);
          mbar_arrive_expect_tx_cluster(fb, kPairStageBytes);
          tma_load_2d_pair(sa, &tmA, fb, kb * kBK, mb * 256 + (int)rank * 128);
          tma_load_2d_pair(sa + kPairABytes, &tmB, fb, kb * kBK, nb * PBN + (int)rank * (PBN / 2));
        }
        __syncwarp();
        if (++stage == kPairStages) { stage = 0; phase ^= 1; }
      }
    }
    // drain: every filled stage consumed before the CTA may exit (bounded)
    for (int s2 = 0; pair_ok && s2 < kPairStages; ++s2) {
      if (!mbar_wait_warp(&empty[stage], phase ^ 1, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) break;
      if (++stage == kPairStages) { stage = 0; phase ^= 1; }
    }
  } else if (warp == 1) {
    if (rank == 0 && pair_ok) {
      constexpr uint32_t idesc = idesc_i8(256, PBN);
      const uint32_t smem_base = smem_u32(smem);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = pair; t < tiles; t += pairs) {
        if (!mbar_wait_warp(&tempty[acc], acc_phase ^ 1, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * PBN);
        bool ok = true;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait_warp(&full[stage], phase, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_base + (uint32_t)(stage * kPairStageBytes);
          const uint64_t da = sdesc_kmajor_sw128(sa), db = sdesc_kmajor_sw128(sa + kPairABytes);
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < kBK / 32; ++k)
              mma_i8_ss_pair(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
            mma_commit_pair(&empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == kPairStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (elect_one()) mma_commit_pair(&tfull[acc], 0x3);
        __syncwarp();
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else if (warp >= PairCfg<KIND>::kEpiWarp0) {
    if constexpr (PairCfg<KIND>::kWide) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kQkEpiRegs));
    // epilogue warps -> TMEM lane quadrant (warp % 4) of this CTA's 128 rows
    const int quad = warp & 3;
    const int row_in_tile = (int)rank * 128 + quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; pair_ok && t < tiles; t += pairs) {
      const int mb = t / num_n, nb = t % num_n;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, H3B_STATUS_GEMM_TIMEOUT)) break;
      tc_fence_after();
      __syncwarp();
      const int m = mb * 256 + row_in_tile;
      const float xs_m = (KIND != kEpiInt32 && m < a.M) ? __ldg(a.xs + m) : 0.0f;
      const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * PBN);
      if constexpr (PairCfg<KIND>::kQk) {
        // this warp's 128-column head of the tile: q/k heads normed and rotated, the rest stored
        static_assert(PBN == 256, "the q/k epilogue splits a 256-column tile between two warps");
        const int hh = (warp - PairCfg<KIND>::kEpiWarp0) >> 2;
        const int n_h = nb * PBN + hh * 128;
        const bool is_q = n_h >= a.q_off && n_h < a.q_off + a.qk_width;
        const bool is_k = n_h >= a.k_off && n_h < a.k_off + a.qk_width;
        uint32_t yb[64];
        float s[16];
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)((hh * 4 + c4) * 32), r);
          tmem_wait_ld();
          if (c4 == 3) {
            // this warp is done with the accumulator: release it on the even CTA
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * 8));
          }
          const int n0 = n_h + c4 * 32;
          if (is_q || is_k)
            qk_head_chunk(r, c4, n0, a, xs_m, yb, s);
          else if (m < a.M && n0 < a.N)
            epi_store_chunk(r, m, n0, a, xs_m, kEpiStore);
        }
        if (is_q || is_k)
          qk_head_finish<KIND == kEpiQkRope64 ? 64 : 48>(yb, s, m, n_h, is_q ? a.q_norm : a.k_norm, a);
      } else if constexpr (KIND == kEpiGeluRot) {
        static_assert(PBN == 256, "one ConvRot group per 256-column tile");
        const int hh = (warp - PairCfg<KIND>::kEpiWarp0) >> 2;
        gelu_rot_first_half(taddr, hh, nb * PBN, xs_m, a);
        // the partner warp's stride-16 results are in its half of the accumulator columns
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&xbar[(quad * 2 + hh) * 2 + acc]);
        if (!mbar_wait_warp(&xbar[(quad * 2 + (hh ^ 1)) * 2 + acc], acc_phase, abort_flag,
                            H3B_STATUS_GEMM_TIMEOUT))
          break;
        tc_fence_after();
        gelu_rot_second_half(taddr, hh, nb, m, a, tempty0 + (uint32_t)(acc * 8));
      } else if constexpr (PairCfg<KIND>::kWide) {
        // this warp's 128-column half of the tile
        const int hh = (warp - PairCfg<KIND>::kEpiWarp0) >> 2;
#pragma unroll 1
        for (int c4 = 0; c4 < 4; ++c4) {
          const int c = hh * 4 + c4;
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)(c * 32), r);
          tmem_wait_ld();
          if (c4 == 3) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * 8));
          }
          const int n0 = nb * PBN + c * 32;
          if (m < a.M && n0 < a.N) epi_store_chunk(r, m, n0, a, xs_m, KIND);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < PBN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)(c * 32), r);
          tmem_wait_ld();
          if (c == PBN / 32 - 1) {
            // this warp is done with the accumulator: release it on the even CTA
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty0 + (uint32_t)(acc * 8));
          }
          const int n0 = nb * PBN + c * 32;
          if (m < a.M && n0 < a.N) epi_store_chunk(r, m, n0, a, xs_m, KIND);
        }
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair's MMAs and both CTAs' epilogues are done
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * PBN);
  }
}

// ------------------------------------------------------------------ host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D byte tensor [rows, cols] with row stride `stride` bytes; box [box_rows, box_cols]
// with 128-byte swizzle (box_cols * elem must be <= 128).
bool make_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                  uint64_t rows, uint64_t stride_bytes, uint32_t box_cols, uint32_t box_rows,
                  CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = get_encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, int KIND>
static cudaError_t launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, cudaStream_t s) {
  using S = GemmSmem<BN>;
  auto k = gemm_i8_kernel<BN, KIND>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
  if (e != cudaSuccess) return e;
  const int tiles = ((a.M + kBM - 1) / kBM) * ((a.N + BN - 1) / BN);
  const int grid = tiles < num_sms() ? tiles : num_sms();
  k<<<grid, kGemmThreads, S::kTotal, s>>>(ta, tb, a);
  return cudaGetLastError();
}

constexpr int kPairBN = 256;

template <int KIND>
static cudaError_t launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                                    cudaStream_t s) {
  auto k = gemm_i8_pair_kernel<kPairBN, KIND>;
  if constexpr (PairCfg<KIND>::kWide) {
    // the register split was planned for kQkLaunchRegs registers per thread at launch
    cudaFuncAttributes fa;
    cudaError_t e0 = cudaFuncGetAttributes(&fa, k);
    if (e0 != cudaSuccess) return e0;
    if (fa.numRegs != kQkLaunchRegs) return cudaErrorInvalidConfiguration;
  }
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PairSmem<kPairBN>::kTotal);
  if (e != cudaSuccess) return e;
  const int tiles = ((a.M + 255) / 256) * ((a.N + kPairBN - 1) / kPairBN);
  const int max_pairs = num_sms() / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  k<<<2 * pairs, PairCfg<KIND>::kThreads, PairSmem<kPairBN>::kTotal, s>>>(ta, tb, a);
  return cudaGetLastError();
}

bool gemm_uses_pair_kernel(int64_t M, int64_t N) {
  return ((M + 255) / 256) * ((N + kPairBN - 1) / kPairBN) >= (int64_t)num_sms();
}

// Returns 0 on success, 1 if a tensor map could not be encoded, 2 on a CUDA error,
// 4 if the q/k epilogue was asked for a shape that runs the 1-SM kernel.
int launch_gemm(const void* A, const void* B, GemmArgs a, int kind, cudaStream_t s, cudaError_t* err) {
  if (kind != kEpiAddF32 && gemm_uses_pair_kernel(a.M, a.N)) {
    // 2-SM kernel: A rows and B rows in boxes of 128 (each CTA's half of a 256 tile)
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K, kBK,
                      128, CU_TENSOR_MAP_SWIZZLE_128B))
      return 1;
    if (!make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, kBK,
                      kPairBN / 2, CU_TENSOR_MAP_SWIZZLE_128B))
      return 1;
    cudaError_t e = kind == kEpiStore       ? launch_gemm_pair<kEpiStore>(ta, tb, a, s)
                    : kind == kEpiResidual  ? launch_gemm_pair<kEpiResidual>(ta, tb, a, s)
                    : kind == kEpiQkRope64  ? launch_gemm_pair<kEpiQkRope64>(ta, tb, a, s)
                    : kind == kEpiQkRope48  ? launch_gemm_pair<kEpiQkRope48>(ta, tb, a, s)
                    : kind == kEpiGeluRot   ? launch_gemm_pair<kEpiGeluRot>(ta, tb, a, s)
                                            : launch_gemm_pair<kEpiInt32>(ta, tb, a, s);
    *err = e;
    return e == cudaSuccess ? 0 : 2;
  }
  if (kind == kEpiQkRope64 || kind == kEpiQkRope48 || kind == kEpiGeluRot) return 4;
  const int tiles256 = ((a.M + kBM - 1) / kBM) * ((a.N + 255) / 256);
  if (kind == kEpiAddF32) {
    // bf16 operands [rows, a.K / 2] (a.K counts bytes); 64 elements = 128 bytes per box row
    const int BNf = (tiles256 >= num_sms() || a.N > 128) ? 256 : 128;
    const uint64_t kel = (uint64_t)a.K / 2;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kel, (uint64_t)a.M, (uint64_t)a.K, kBK / 2, kBM,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return 1;
    if (!make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kel, (uint64_t)a.N, (uint64_t)a.K, kBK / 2,
                      (uint32_t)BNf, CU_TENSOR_MAP_SWIZZLE_128B))
      return 1;
    cudaError_t e = BNf == 256 ? launch_gemm_bn<256, kEpiAddF32>(ta, tb, a, s)
                               : launch_gemm_bn<128, kEpiAddF32>(ta, tb, a, s);
    *err = e;
    return e == cudaSuccess ? 0 : 2;
  }
  const int BN = (tiles256 >= num_sms() || a.N > 128) ? 256 : 128;
  CUtensorMap ta, tb;
  if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K, kBK, kBM,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return 1;
  if (!make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.K, kBK,
                    (uint32_t)BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return 1;
  cudaError_t e;
  if (BN == 256) {
    e = kind == kEpiStore      ? launch_gemm_bn<256, kEpiStore>(ta, tb, a, s)
        : kind == kEpiResidual ? launch_gemm_bn<256, kEpiResidual>(ta, tb, a, s)
                               : launch_gemm_bn<256, kEpiInt32>(ta, tb, a, s);
  } else {
    e = kind == kEpiStore      ? launch_gemm_bn<128, kEpiStore>(ta, tb, a, s)
        : kind == kEpiResidual ? launch_gemm_bn<128, kEpiResidual>(ta, tb, a, s)
                               : launch_gemm_bn<128, kEpiInt32>(ta, tb, a, s);
  }
  *err = e;
  return e == cudaSuccess ? 0 : 2;
}

}  // namespace h3b
