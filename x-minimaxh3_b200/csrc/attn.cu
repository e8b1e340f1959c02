// attn.cu -- SageAttention-style quantized attention for sm_100a, dense or
// driven by a Sparge block bitmap.
//
//   S = Q_i8 . K_i8^T   tcgen05.mma kind::i8, int32 in tensor memory
//   P = exp2(S * qs * ks * scale * log2 e - m) * 112 -> E4M3 (shared memory);
//       exp2 runs on packed f16 pairs (ex2.approx.f16x2: two exponentials per
//       MUFU op; f16 is far finer than the E4M3 result), m is a lazily updated
//       running max: it moves only when a tile's max exceeds it by more than
//       kTau = 2, so P <= 2^kTau * 112 = 448 (the E4M3 maximum) and the O
//       rescale in tensor memory is rare
//   [O | l] += P . [V | 1]   tcgen05.mma kind::f8f6f4, N = 144: the 16 extra
//       columns of ones give the row sum of exactly the E4M3 P that meets V
//   out = O / l * v_scale[d] -> bf16
//
// One CTA per (128-query tile, head), 320 threads:
//   warp 0      TMA producer: the Q tile once, then K/V for each PAIR of selected
//               64-key blocks (K: 2 x [64 x 128 B], 128-byte swizzle; V^T: 2 x
//               [128 x 64 B], 64-byte swizzle) into a 3-stage ring; no multicast
//   warp 1      TMEM allocator + MMA issuer: S for pair i into one of two S
//               buffers, then O += P(i-1) . V(i-1) once the softmax published P(i-1)
//   warps 2..9  softmax, two warps per TMEM lane quadrant: for its 32 query rows
//               warp 2..5 takes key columns 0..63 (block j0), warp 6..9 columns
//               64..127 (block j1); the two exchange only their tile max per row
//               through shared memory (named barrier per quadrant), then each
//               writes its half of the P row (128-byte-swizzled K-major, as the
//               MMA reads it), rescales its half of the O row in TMEM when the
//               running max moves, and normalises its half of the output.
// TMEM: S0 cols 0..127, S1 128..255, [O | l] 256..399.  Blocks are visited in
// ascending order; a trailing unpaired block uses N = 64 / K = 64 MMAs.
#include "h3b_kernels.cuh"

namespace h3b {

constexpr int kAttnThreads = 320;
constexpr int kSoftmaxThreads = 256;
constexpr int kKVStages = 3;
constexpr int kQBytes = 128 * 128;
constexpr int kPBytes = 128 * 128;
// K pair 16 KB, then per V block an [128 x 64 B] tile followed by a 1 KB block
// of E4M3 ones (16 rows): the P.V MMA reads 144 rows = V^T plus the ones.
constexpr int kVTile = 8192 + 1024;
constexpr int kKVBytes = 16384 + 2 * kVTile;
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + kQBytes;            // 2 buffers
constexpr int kOffKV = kOffP + 2 * kPBytes;
constexpr int kOffBar = kOffKV + kKVStages * kKVBytes;
constexpr int kOffXchg = kOffBar + 256;            // float [2 parity][2 halves][128 rows]
constexpr int kAttnSmem = kOffXchg + 2 * 2 * 128 * 4 + 1024;
constexpr float kLog2_112 = 6.807354922057604f;
constexpr float kTau = 2.0f;
constexpr int kON = 144;  // O columns incl. the row-sum block


// Ascending walk over the K blocks of one query tile.
struct BlockIter {
  const uint32_t* row;
  int words, w, Kb, dense_next;
  uint32_t bits;
  __device__ void init(const AttnArgs& a, int h, int qt) {
    Kb = a.Kb;
    dense_next = 0;
    if (a.bitmap) {
      row = a.bitmap + ((int64_t)h * ((a.Lq + 127) / 128) + qt) * a.words;
      words = a.words;
      w = 0;
      bits = words > 0 ? row[0] : 0u;
    } else {
      row = nullptr;
    }
  }
  __device__ int next() {
    if (!row) return dense_next < Kb ? dense_next++ : -1;
    while (bits == 0) {
      if (++w >= words) return -1;
      bits = row[w];
    }
    const int b = __ffs(bits) - 1;
    bits &= bits - 1;
    return w * 32 + b;
  }
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// two floats -> packed f16 pair (lo in bits 0..15), round to nearest
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t ex2_f16x2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
// packed f16 pair -> two E4M3 bytes (satfinite, round to nearest even), lo byte = lo half
__device__ __forceinline__ uint32_t f16x2_to_e4m3x2(uint32_t x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(x));
  return (uint32_t)r;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                  // 1
  uint64_t* kv_full = bars + 1;             // kKVStages
  uint64_t* kv_empty = kv_full + kKVStages; // kKVStages
  uint64_t* s_full = kv_empty + kKVStages;  // 2
  uint64_t* s_free = s_full + 2;            // 2
  uint64_t* p_full = s_free + 2;            // 2
  uint64_t* pv_done = p_full + 2;           // 2 (one per P buffer)
  uint64_t* xbar = pv_done + 2;             // 4: tile-max exchange per lane quadrant (64 threads)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], kSoftmaxThreads);
      mbar_init(&p_full[b], kSoftmaxThreads);
    }
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 64);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // constant E4M3 ones after every V tile (never overwritten by TMA)
  for (int i = threadIdx.x; i < kKVStages * 2 * 64; i += blockDim.x) {
    const int st = i / 128, blk = (i / 64) & 1, w = i & 63;
    reinterpret_cast<uint4*>(smem + kOffKV + st * kKVBytes + 16384 + blk * kVTile + 8192)[w] =
        make_uint4(0x38383838u, 0x38383838u, 0x38383838u, 0x38383838u);
  }
  fence_proxy_async_smem();
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  BlockIter it;
  it.init(a, h, qt);

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(smem + kOffQ, &tmQ, q_full, 0, (int)(h * a.Lqpad + (int64_t)qt * 128));
      int stage = 0;
      uint32_t phase = 0;
      while (true) {
        const int j0 = it.next();
        if (j0 < 0) break;
        const int j1 = it.next();
        if (!mbar_wait(&kv_empty[stage], phase ^ 1, abort_flag, H3B_STATUS_ATTN_TIMEOUT)) break;
        uint8_t* kst = smem + kOffKV + stage * kKVBytes;
        uint8_t* vst = kst + 16384;
        mbar_arrive_expect_tx(&kv_full[stage], j1 >= 0 ? 32768u : 16384u);
        tma_load_2d(kst, &tmK, &kv_full[stage], 0, (int)(h * a.Lkpad + (int64_t)j0 * 64));
        tma_load_2d(vst, &tmV, &kv_full[stage], j0 * 64, h * 128);
        if (j1 >= 0) {
          tma_load_2d(kst + 8192, &tmK, &kv_full[stage], 0, (int)(h * a.Lkpad + (int64_t)j1 * 64));
          tma_load_2d(vst + kVTile, &tmV, &kv_full[stage], j1 * 64, h * 128);
        }
        if (++stage == kKVStages) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, abort_flag, H3B_STATUS_ATTN_TIMEOUT);
      const uint64_t qdesc = sdesc_kmajor_sw128(smem_u32(smem + kOffQ));
      int stage = 0, prev_stage = 0, i = 0;
      uint32_t phase = 0;
      bool prev_has1 = false;
      constexpr uint32_t idesc_pv = idesc_e4m3(128, kON);
      auto issue_pv = [&](int pi) -> bool {
        const int pb = pi & 1;
        if (!mbar_wait(&p_full[pb], (uint32_t)((pi >> 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) return false;
        tc_fence_after();
        const uint32_t pbase = smem_u32(smem + kOffP + pb * kPBytes);
        const uint32_t vbase = smem_u32(smem + kOffKV + prev_stage * kKVBytes + 16384);
        const int ksteps = prev_has1 ? 4 : 2;
        for (int k = 0; k < ksteps; ++k) {
          const uint64_t pd = sdesc_kmajor_sw128(pbase + 32 * k);
          const uint64_t vd = sdesc_kmajor_sw64(vbase + (k >> 1) * kVTile + (k & 1) * 32);
          mma_f8_ss(tmem + 256, pd, vd, idesc_pv, (pi > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&pv_done[pb]);
        mma_commit(&kv_empty[prev_stage]);
        return true;
      };
      while (ok) {
        const int j0 = it.next();
        if (j0 < 0) break;
        const int j1 = it.next();
        const bool has1 = j1 >= 0;
        const int b = i & 1;
        if (!mbar_wait(&kv_full[stage], phase, abort_flag, H3B_STATUS_ATTN_TIMEOUT)) { ok = false; break; }
        if (!mbar_wait(&s_free[b], (uint32_t)(((i >> 1) & 1) ^ 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kbase = smem_u32(smem + kOffKV + stage * kKVBytes);
        const uint32_t idesc_s = has1 ? idesc_i8(128, 128) : idesc_i8(128, 64);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_i8_ss(tmem + (uint32_t)(b * 128), qdesc + (uint64_t)(2 * k),
                    sdesc_kmajor_sw128(kbase + 32 * k), idesc_s, k > 0 ? 1u : 0u);
        mma_commit(&s_full[b]);
        if (i >= 1 && !issue_pv(i - 1)) { ok = false; break; }
        prev_stage = stage;
        prev_has1 = has1;
        if (++stage == kKVStages) { stage = 0; phase ^= 1; }
        ++i;
      }
      if (ok && i >= 1) issue_pv(i - 1);
    }
  } else {
    // softmax warps 2..9: TMEM lane quadrant warp % 4, key-column half (warp - 2) / 4
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int64_t qrow = (int64_t)qt * 128 + r;
    const bool row_ok = qrow < a.Lq;
    const float qs = row_ok ? __ldg(a.q_scale + (int64_t)h * a.nqs + qrow / a.q_block) : 0.f;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + 256;
    float* xchg = reinterpret_cast<float*>(smem + kOffXchg);   // [parity][half][row]
    const int o_c0 = half ? 80 : 0, o_c1 = half ? kON : 80;  // this warp's O columns (16-column chunks)
    float m = -__int_as_float(0x7f800000);
    int i = 0;
    bool ok = true;
    while (true) {
      const int j0 = it.next();
      if (j0 < 0) break;
      const int j1 = it.next();
      const bool has1 = j1 >= 0;
      const int b = i & 1;
      const int jb = half ? j1 : j0;           // this warp's key block (-1: none)
      const bool mine = jb >= 0;
      if (!mbar_wait_warp(&s_full[b], (uint32_t)((i >> 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[64];
      __syncwarp();
      if (mine) {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
        tmem_ld32(tmem + lane_off + b * 128 + half * 64, s0);
        tmem_ld32(tmem + lane_off + b * 128 + half * 64 + 32, s1);
        tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(&s_free[b]);

      const int n = mine ? (int)min((int64_t)64, a.Lk - (int64_t)jb * 64) : 0;
      const float c = mine ? qs * __ldg(a.k_scale + (int64_t)h * a.Kb + jb) * a.scale_log2 : 0.f;
      // tile max of this half on the raw int32 scores (scales are positive)
      int mx = INT_MIN;
      if (n == 64) {
#pragma unroll
        for (int cc = 0; cc < 64; ++cc) mx = max(mx, (int)s[cc]);
      } else {
#pragma unroll
        for (int cc = 0; cc < 64; ++cc)
          if (cc < n) mx = max(mx, (int)s[cc]);
      }
      const float ninf = -__int_as_float(0x7f800000);
      const float hmax = n > 0 ? (float)mx * c : ninf;
      // exchange the half-row maxima with the partner warp of this quadrant
      // (double-buffered slot; bounded mbarrier wait instead of a named barrier)
      xchg[((i & 1) * 2 + half) * 128 + r] = hmax;
      mbar_arrive(&xbar[quad]);
      if (!mbar_wait_warp(&xbar[quad], (uint32_t)(i & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
        ok = false;
        break;
      }
      const float tmax = fmaxf(hmax, xchg[((i & 1) * 2 + (half ^ 1)) * 128 + r]);
      // lazy running max: move it only when this tile exceeds it by more than kTau
      const bool move = tmax > m + kTau;
      const float m_new = move ? tmax : m;
      // tcgen05.ld / st are warp-collective: rescale the whole warp's rows when any
      // lane needs it (lanes whose max did not move scale by exactly 1)
      const bool rescale = __any_sync(0xffffffffu, move && i > 0);
      const float alpha = ex2(m - m_new);
      // x = S*c + log2(112) - m, with float(S) = as_float(S + 0x4B400000) - 12582912
      const float oo = kLog2_112 - m_new - 12582912.0f * c;
      if (mine) {
#pragma unroll
        for (int cc = 0; cc < 64; cc += 2) {
          const float x0 = fmaf(__int_as_float((int)s[cc] + 0x4B400000), c, oo);
          const float x1 = fmaf(__int_as_float((int)s[cc + 1] + 0x4B400000), c, oo);
          uint32_t e = ex2_f16x2(pack_f16x2(x0, x1));
          if (n < 64) {
            if (cc >= n) e &= 0xffff0000u;      // low half: column cc -> +0
            if (cc + 1 >= n) e &= 0x0000ffffu;
          }
          s[cc >> 1] = e;   // packed f16 pair, reuses the first half of s[]
        }
      }

      if (rescale) {
        if (!mbar_wait_warp(&pv_done[(i - 1) & 1], (uint32_t)(((i - 1) >> 1) & 1), abort_flag,
                            H3B_STATUS_ATTN_TIMEOUT)) {
          ok = false;
          break;
        }
        tc_fence_after();
        __syncwarp();
#pragma unroll 1
        for (int cc = o_c0; cc < o_c1; cc += 16) {
          uint32_t o[16];
          tmem_ld16(o_addr + cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st16(o_addr + cc, o);
        }
        tmem_wait_st();
      }
      // P buffer b was last read by PV(i - 2)
      if (i >= 2 &&
          !mbar_wait_warp(&pv_done[b], (uint32_t)(((i - 2) >> 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
        ok = false;
        break;
      }
      if (mine) {
        // this half of the P row -> shared memory, K-major, 128-byte swizzle
        // (16-byte chunk c of the row lives at chunk c ^ (r & 7))
        uint8_t* prow = smem + kOffP + b * kPBytes + r * 128;
#pragma unroll
        for (int cq = 0; cq < 4; ++cq) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = f16x2_to_e4m3x2(s[8 * cq + 2 * e]) | (f16x2_to_e4m3x2(s[8 * cq + 2 * e + 1]) << 16);
          const int chunk = half * 4 + cq;
          *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
      m = m_new;
      ++i;
    }
    // epilogue: this warp's 64 output channels, O / l * v_scale, l from the ones columns
    uint16_t* dst = a.out + (row_ok ? qrow : 0) * a.out_stride + (int64_t)h * 128 + half * 64;
    if (ok && i >= 1) {
      if (mbar_wait_warp(&pv_done[(i - 1) & 1], (uint32_t)(((i - 1) >> 1) & 1), abort_flag,
                         H3B_STATUS_ATTN_TIMEOUT)) {
        tc_fence_after();
        __syncwarp();
        uint32_t lsum[16];
        tmem_ld16(o_addr + 128, lsum);
        tmem_wait_ld();
        const float l = __uint_as_float(lsum[0]);
        const float inv_l = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll 1
        for (int cc = 0; cc < 64; cc += 16) {
          uint32_t o[16];
          tmem_ld16(o_addr + half * 64 + cc, o);
          tmem_wait_ld();
          uint32_t packed[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int d = half * 64 + cc + 2 * e;
            const float v0 = __uint_as_float(o[2 * e]) * inv_l * __ldg(a.v_scale + h * 128 + d);
            const float v1 = __uint_as_float(o[2 * e + 1]) * inv_l * __ldg(a.v_scale + h * 128 + d + 1);
            packed[e] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
          }
          if (row_ok) {
            *reinterpret_cast<uint4*>(dst + cc) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            *reinterpret_cast<uint4*>(dst + cc + 8) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          }
        }
      }
    } else if (row_ok && i == 0) {
      for (int cc = 0; cc < 64; cc += 8) *reinterpret_cast<uint4*>(dst + cc) = make_uint4(0, 0, 0, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int launch_attention(const void* q, const void* k, const void* vt, const AttnArgs& a, cudaStream_t s,
                     cudaError_t* err) {
  CUtensorMap tq, tk, tv;
  if (!make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128, (uint64_t)(a.H * a.Lqpad), 128, 128, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return 1;
  if (!make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 128, (uint64_t)(a.H * a.Lkpad), 128, 128, 64,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return 1;
  if (!make_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)a.Lkpad, (uint64_t)(a.H * 128),
                    (uint64_t)a.Lkpad, 64, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return 1;
  cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e == cudaSuccess) {
    dim3 grid((unsigned)((a.Lq + 127) / 128), (unsigned)a.H);
    attn_kernel<<<grid, kAttnThreads, kAttnSmem, s>>>(tq, tk, tv, a);
    e = cudaGetLastError();
  }
  *err = e;
  return e == cudaSuccess ? 0 : 2;
}

}  // namespace h3b
