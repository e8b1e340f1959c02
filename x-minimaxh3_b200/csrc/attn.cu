// attn.cu -- SageAttention-style quantized attention for sm_100a, dense or
// driven by a Sparge block bitmap.
//
//   S = Q_i8 . K_i8^T   tcgen05.mma kind::i8, int32 in tensor memory
//   P = exp2((S * qs * ks * scale * log2 e) - running max) * 448 -> E4M3 (shared)
//   O += P . V          tcgen05.mma kind::f8f6f4 (E4M3 x E4M3 -> fp32, tensor memory)
//   out = O / rowsum * v_scale[d] -> bf16
//
// One CTA per (128-query tile, head), 192 threads:
//   warp 0      TMA producer: the Q tile once, then K/V for each PAIR of selected
//               64-key blocks (K: 2 x [64 x 128 B], 128-byte swizzle; V^T: 2 x
//               [128 x 64 B], 64-byte swizzle) into a 3-stage ring; no multicast
//   warp 1      TMEM allocator + MMA issuer: S for pair i into one of two S
//               buffers, then O += P(i-1) . V(i-1) once the softmax published P(i-1)
//   warps 2..5  softmax, one query row per thread (its TMEM lane): S row from
//               TMEM, per-block dequant scales, online max / sum, P to shared
//               memory in the 128-byte-swizzled K-major layout the MMA reads,
//               O row rescale in TMEM when the max moves, final normalisation.
// TMEM: S0 cols 0..127, S1 128..255, O 256..383.  Blocks are visited in
// ascending order; a trailing unpaired block uses N = 64 / K = 64 MMAs.
#include "h3b_kernels.cuh"

namespace h3b {

constexpr int kAttnThreads = 192;
constexpr int kKVStages = 3;
constexpr int kQBytes = 128 * 128;
constexpr int kPBytes = 128 * 128;
constexpr int kKVBytes = 32768;  // K pair 16 KB + V pair 16 KB
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + kQBytes;            // 2 buffers
constexpr int kOffKV = kOffP + 2 * kPBytes;
constexpr int kOffBar = kOffKV + kKVStages * kKVBytes;
constexpr int kAttnSmem = kOffBar + 256 + 1024;
constexpr float kLog2_448 = 8.807354922057604f;


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
  uint64_t* pv_done = p_full + 2;           // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);
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
      mbar_init(&s_free[b], 128);
      mbar_init(&p_full[b], 128);
    }
    mbar_init(pv_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
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
          tma_load_2d(vst + 8192, &tmV, &kv_full[stage], j1 * 64, h * 128);
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
      constexpr uint32_t idesc_pv = idesc_e4m3(128, 128);
      auto issue_pv = [&](int pi) -> bool {
        const int pb = pi & 1;
        if (!mbar_wait(&p_full[pb], (uint32_t)((pi >> 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) return false;
        tc_fence_after();
        const uint32_t pbase = smem_u32(smem + kOffP + pb * kPBytes);
        const uint32_t vbase = smem_u32(smem + kOffKV + prev_stage * kKVBytes + 16384);
        const int ksteps = prev_has1 ? 4 : 2;
        for (int k = 0; k < ksteps; ++k) {
          const uint64_t pd = sdesc_kmajor_sw128(pbase + 32 * k);
          const uint64_t vd = sdesc_kmajor_sw64(vbase + (k >> 1) * 8192 + (k & 1) * 32);
          mma_f8_ss(tmem + 256, pd, vd, idesc_pv, (pi > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(pv_done);
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
    // softmax warps 2..5: TMEM lane quadrant warp % 4
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int64_t qrow = (int64_t)qt * 128 + r;
    const bool row_ok = qrow < a.Lq;
    const float qs = row_ok ? __ldg(a.q_scale + (int64_t)h * a.nqs + qrow / a.q_block) : 0.f;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    float m = -__int_as_float(0x7f800000), l = 0.f;
    int i = 0;
    bool ok = true;
    while (true) {
      const int j0 = it.next();
      if (j0 < 0) break;
      const int j1 = it.next();
      const bool has1 = j1 >= 0;
      const int b = i & 1;
      if (!mbar_wait(&s_full[b], (uint32_t)((i >> 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) { ok = false; break; }
      tc_fence_after();
      uint32_t s[128];
      {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[0]);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[32]);
        tmem_ld32(tmem + lane_off + b * 128, s0);
        tmem_ld32(tmem + lane_off + b * 128 + 32, s1);
        if (has1) {
          uint32_t (&s2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[64]);
          uint32_t (&s3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&s[96]);
          tmem_ld32(tmem + lane_off + b * 128 + 64, s2);
          tmem_ld32(tmem + lane_off + b * 128 + 96, s3);
        }
        tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(&s_free[b]);

      const int n0 = (int)min((int64_t)64, a.Lk - (int64_t)j0 * 64);
      const int n1 = has1 ? (int)min((int64_t)64, a.Lk - (int64_t)j1 * 64) : 0;
      const float c0 = qs * __ldg(a.k_scale + (int64_t)h * a.Kb + j0) * a.scale_log2;
      const float c1 = has1 ? qs * __ldg(a.k_scale + (int64_t)h * a.Kb + j1) * a.scale_log2 : 0.f;
      int mx0 = INT_MIN, mx1 = INT_MIN;
#pragma unroll
      for (int c = 0; c < 64; ++c)
        if (c < n0) mx0 = max(mx0, (int)s[c]);
      if (has1) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c < n1) mx1 = max(mx1, (int)s[64 + c]);
      }
      const float ninf = -__int_as_float(0x7f800000);
      float tmax = (float)mx0 * c0;
      if (n1 > 0) tmax = fmaxf(tmax, (float)mx1 * c1);
      const float m_new = fmaxf(m, tmax);
      const float base = m_new == ninf ? 0.f : m_new;
      const float alpha = ex2(m - base);
      // float(S) = as_float(S + 0x4B400000) - 12582912 for |S| < 2^22; fold the
      // subtraction into the FMA constant.
      const float off = kLog2_448 - base;
      const float o0 = off - 12582912.0f * c0, o1 = off - 12582912.0f * c1;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p = c < n0 ? ex2(fmaf(__int_as_float((int)s[c] + 0x4B400000), c0, o0)) : 0.f;
        s[c] = __float_as_uint(p);
        sum += p;
      }
      if (has1) {
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const float p = c < n1 ? ex2(fmaf(__int_as_float((int)s[64 + c] + 0x4B400000), c1, o1)) : 0.f;
          s[64 + c] = __float_as_uint(p);
          sum += p;
        }
      }
      l = l * alpha + sum;

      if (i >= 1) {
        if (!mbar_wait(pv_done, (uint32_t)((i - 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) { ok = false; break; }
        tc_fence_after();
        if (alpha < 1.0f) {
#pragma unroll 1
          for (int c = 0; c < 128; c += 16) {
            uint32_t o[16];
            tmem_ld16(tmem + lane_off + 256 + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(tmem + lane_off + 256 + c, o);
          }
          tmem_wait_st();
        }
      }
      // P row -> shared memory, K-major, 128-byte swizzle (chunk c at c ^ (r & 7))
      uint8_t* prow = smem + kOffP + b * kPBytes + r * 128;
      const int nchunks = has1 ? 8 : 4;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < nchunks) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float* pv = reinterpret_cast<const float*>(&s[16 * c + 4 * e]);
            const uint32_t lo = f32x2_to_e4m3x2(pv[0], pv[1]);
            const uint32_t hi = f32x2_to_e4m3x2(pv[2], pv[3]);
            w[e] = lo | (hi << 16);
          }
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[b]);
      m = m_new;
      ++i;
    }
    // epilogue
    uint16_t* dst = a.out + (row_ok ? qrow : 0) * a.out_stride + (int64_t)h * 128;
    if (ok && i >= 1) {
      if (mbar_wait(pv_done, (uint32_t)((i - 1) & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
        tc_fence_after();
        const float inv_l = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t o[16];
          tmem_ld16(tmem + lane_off + 256 + c, o);
          tmem_wait_ld();
          uint32_t packed[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float v0 = __uint_as_float(o[2 * e]) * inv_l * __ldg(a.v_scale + h * 128 + c + 2 * e);
            const float v1 = __uint_as_float(o[2 * e + 1]) * inv_l * __ldg(a.v_scale + h * 128 + c + 2 * e + 1);
            packed[e] = (uint32_t)f32_to_bf16_bits(v0) | ((uint32_t)f32_to_bf16_bits(v1) << 16);
          }
          if (row_ok) {
            *reinterpret_cast<uint4*>(dst + c) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            *reinterpret_cast<uint4*>(dst + c + 8) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
          }
        }
      }
    } else if (row_ok && i == 0) {
      for (int c = 0; c < 128; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0, 0, 0, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
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
