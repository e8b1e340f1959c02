// attn_prep.cu -- quantized-attention preparation kernels.
//
//  key mean     per-(head, channel) mean of K over the sequence (K smoothing),
//               double accumulation in a fixed order (1024-token chunks, then
//               the chunk sums), replacing hnd_compatible_key_mean_nhd
//               (model/sparge_nhd.py:26-48)
//  pool/sim/quant  Sparge per-block pooled mean, self-similarity flag and
//               per-block INT8 quantization (model/sparge_nhd.py:51-160), on
//               NHD input with any row stride (reads Q/K straight out of the
//               fused QKV projection output)
//  value fp8    per-(head, channel) absmax, V * 2.25/absmax -> E4M3, transposed
//               to [H, 128, Lpad] (model/compact_fp8.py:13-300); also slab by
//               slab with an absmax the caller gathered beforehand (the compact
//               K/V build of model/kernels.py:2491-2526, 2677-2772)
// Every reduction runs in the order the CPU oracle restates, so results are
// bit-identical to it.
#include <mutex>

#include "h3b_kernels.cuh"

namespace h3b {

constexpr int kKeyMeanChunk = 1024;
constexpr int kD = 128;

// ------------------------------------------------------------------ key mean

__global__ void __launch_bounds__(256) key_mean_partial_kernel(const uint16_t* __restrict__ k, int64_t L, int cols,
                                                                int64_t stride, double* __restrict__ part) {
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.x * kKeyMeanChunk;
  const int64_t r1 = r0 + kKeyMeanChunk < L ? r0 + kKeyMeanChunk : L;
  double s = 0.0;
  const uint16_t* p = k + r0 * stride + c;
  int64_t r = r0;
  for (; r + 4 <= r1; r += 4) {
    const float a0 = bf16_bits_to_f32(p[0]), a1 = bf16_bits_to_f32(p[stride]);
    const float a2 = bf16_bits_to_f32(p[2 * stride]), a3 = bf16_bits_to_f32(p[3 * stride]);
    s = __dadd_rn(s, (double)a0);
    s = __dadd_rn(s, (double)a1);
    s = __dadd_rn(s, (double)a2);
    s = __dadd_rn(s, (double)a3);
    p += 4 * stride;
  }
  for (; r < r1; ++r, p += stride) s = __dadd_rn(s, (double)bf16_bits_to_f32(p[0]));
  part[(int64_t)blockIdx.x * cols + c] = s;
}

__global__ void __launch_bounds__(256) key_mean_final_kernel(const double* __restrict__ part, int chunks, int cols,
                                                              int64_t L, uint16_t* __restrict__ mean) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  double s = 0.0;
  for (int i = 0; i < chunks; ++i) s = __dadd_rn(s, part[(int64_t)i * cols + c]);
  mean[c] = f32_to_bf16_bits(__double2float_rn(__ddiv_rn(s, (double)L)));
}

int64_t key_mean_workspace(int64_t L, int64_t H) {
  return ((L + kKeyMeanChunk - 1) / kKeyMeanChunk) * H * kD * (int64_t)sizeof(double);
}

cudaError_t launch_key_mean(const void* k, int64_t L, int64_t H, int64_t stride, void* mean, void* ws,
                            cudaStream_t s) {
  const int cols = (int)(H * kD);
  const int chunks = (int)((L + kKeyMeanChunk - 1) / kKeyMeanChunk);
  dim3 g1(chunks, (cols + 255) / 256);
  key_mean_partial_kernel<<<g1, 256, 0, s>>>(static_cast<const uint16_t*>(k), L, cols, stride,
                                             static_cast<double*>(ws));
  key_mean_final_kernel<<<(cols + 255) / 256, 256, 0, s>>>(static_cast<const double*>(ws), chunks, cols, L,
                                                             static_cast<uint16_t*>(mean));
  return cudaGetLastError();
}

// ------------------------------------------------------------------ key mean, no allocation

// A variant of launch_key_mean for callers that cannot allocate device memory
// (for example a host that hands all of the GPU's memory to its own pool and
// cannot give this library a workspace, or code running where a device
// allocation is not permitted).  Its scratch -- one fp64 partial sum per
// (1024-token chunk, head, channel) -- lives in this fixed, file-scope device
// array instead: 2^20 doubles (8 MiB), held by every GPU that loads the library
// until the process exits.  ceil(L / 1024) * H * 128 must not exceed 2^20
// (e.g. L <= 262,144 tokens at 32 heads).  Every call on a device shares the
// array and nothing is cleared between calls: each call writes every partial
// it reads before reading it, so stale contents are harmless, but two calls
// whose kernels overlap on the GPU (different streams, no ordering) race on it.
constexpr int64_t kKeyMeanScratchDoubles = int64_t(1) << 20;
static __device__ __align__(256) double g_key_mean_scratch[kKeyMeanScratchDoubles];

// Device address of g_key_mean_scratch, looked up once per device with that
// device current (in host code the array's name is only a host-side stand-in).
// The lookup is remembered together with the CUDA context it was made in: after a
// cudaDeviceReset, or under another context on the same device, the module may sit
// at another address, so a changed context means a fresh lookup.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
static std::mutex g_scratch_mu;
static double* g_scratch_ptr[64] = {};
static CUcontext g_scratch_ctx[64] = {};

static CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return c;
}

static cudaError_t key_mean_scratch_for_current_device(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const CUcontext ctx = current_context();  // null until a runtime call made one current
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_key_mean_scratch);  // makes the device's context current
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<double*>(p);
    g_scratch_ctx[dev] = current_context();
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

int64_t key_mean_static_capacity() { return kKeyMeanScratchDoubles; }

cudaError_t launch_key_mean_static(const void* k, int64_t L, int64_t H, int64_t stride, void* mean,
                                   cudaStream_t s) {
  double* scratch = nullptr;
  cudaError_t e = key_mean_scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return e;
  return launch_key_mean(k, L, H, stride, mean, scratch, s);
}

// ------------------------------------------------------------------ pool / sim / quant


__device__ __forceinline__ void load4_row(const PoolArgs& a, int64_t row, int h, int lane, const float (&mean4)[4],
                                          float (&v)[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(a.x + row * a.stride + (int64_t)h * kD + 4 * lane);
  v[0] = __uint_as_float(raw.x << 16);
  v[1] = __uint_as_float(raw.x & 0xffff0000u);
  v[2] = __uint_as_float(raw.y << 16);
  v[3] = __uint_as_float(raw.y & 0xffff0000u);
  if (a.mean) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = bf16r(__fsub_rn(v[i], mean4[i]));
  }
}

// One CTA of four warps per (block, head); lane l owns channels 4l..4l+3 and
// warp w walks rows w, w+4, ... of the block.  With a mean (keys), the first pass
// keeps each row's mean-subtracted bf16 values in shared memory (blk x 256 bytes,
// dynamic) and the quantizing pass reads them back from there (the same thread
// wrote them) instead of reloading and recomputing them.  Without one (queries,
// 128-row blocks) the quantizing pass reloads: the 32 KB a CTA would need costs
// more occupancy than the reload.
__global__ void __launch_bounds__(128) pool_sim_quant_kernel(PoolArgs a) {
  extern __shared__ uint2 rows_s[];  // [blk][32]: lane l's four bf16 of each row
  __shared__ float pp_s[4][kD], sp_s[4][kD];
  __shared__ float amax_s[4];
  __shared__ float scale_s;
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)b * a.blk;
  const int valid = (int)((a.L - r0) < a.blk ? (a.L - r0) : a.blk);
  const int64_t nbs = a.nb_stride ? a.nb_stride : (a.L + a.blk - 1) / a.blk;

  float mean4[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.mean) {
    const uint2 raw = *reinterpret_cast<const uint2*>(a.mean + h * kD + 4 * lane);
    mean4[0] = __uint_as_float(raw.x << 16);
    mean4[1] = __uint_as_float(raw.x & 0xffff0000u);
    mean4[2] = __uint_as_float(raw.y << 16);
    mean4[3] = __uint_as_float(raw.y & 0xffff0000u);
  }

  float pp[4] = {0.f, 0.f, 0.f, 0.f}, sp[4] = {0.f, 0.f, 0.f, 0.f}, amax = 0.f;
#pragma unroll 4
  for (int r = warp; r < valid; r += 4) {
    float v[4];
    load4_row(a, r0 + r, h, lane, mean4, v);
    if (a.mean)
      rows_s[r * 32 + lane] = make_uint2((__float_as_uint(v[0]) >> 16) | (__float_as_uint(v[1]) & 0xffff0000u),
                                       (__float_as_uint(v[2]) >> 16) | (__float_as_uint(v[3]) & 0xffff0000u));
    float sq = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(v[0], v[0]), __fmul_rn(v[1], v[1])), __fmul_rn(v[2], v[2])),
                         __fmul_rn(v[3], v[3]));
    const float norm = __fsqrt_rn(warp_butterfly_sum(sq));
    // v / norm correctly rounded: Markstein's final step from RN(1/norm) where
    // every quotient that survives the f16 rounding keeps an exact residual
    // (norm >= 2^-60); IEEE division for tiny, zero, infinite or NaN norms
    const bool markstein = norm >= 8.673617379884035e-19f && norm <= 3.4e38f;
    const float rn = __frcp_rn(norm);
    float qn[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) qn[i] = markstein ? div_rn_by(v[i], norm, rn) : __fdiv_rn(v[i], norm);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pp[i] = __fadd_rn(pp[i], v[i]);
      sp[i] = __fadd_rn(sp[i], f16r(qn[i]));
      amax = fmaxf(amax, fabsf(v[i]));
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    pp_s[warp][4 * lane + i] = pp[i];
    sp_s[warp][4 * lane + i] = sp[i];
  }
  if (lane == 0) amax_s[warp] = amax;
  __syncthreads();
  if (warp == 0) {
    float s2[4];
    uint16_t pooled[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = 4 * lane + i;
      const float ps = __fadd_rn(__fadd_rn(pp_s[0][d], pp_s[2][d]), __fadd_rn(pp_s[1][d], pp_s[3][d]));
      const float ss = __fadd_rn(__fadd_rn(sp_s[0][d], sp_s[2][d]), __fadd_rn(sp_s[1][d], sp_s[3][d]));
      pooled[i] = f32_to_bf16_bits(__fdiv_rn(ps, (float)valid));
      s2[i] = __fmul_rn(ss, ss);
    }
    *reinterpret_cast<uint2*>(a.pooled + ((int64_t)h * nbs + b) * kD + 4 * lane) =
        make_uint2((uint32_t)pooled[0] | ((uint32_t)pooled[1] << 16), (uint32_t)pooled[2] | ((uint32_t)pooled[3] << 16));
    const float g = warp_butterfly_sum(__fadd_rn(__fadd_rn(__fadd_rn(s2[0], s2[1]), s2[2]), s2[3]));
    const float simv = __fdiv_rn(g, (float)(valid * valid));
    const float am = fmaxf(fmaxf(amax_s[0], amax_s[1]), fmaxf(amax_s[2], amax_s[3]));
    const float sc = __fadd_rn(__fdiv_rn(am, 127.0f), 1e-7f);
    if (lane == 0) {
      a.similar[(int64_t)h * nbs + b] = (uint8_t)(valid == a.blk && simv > a.thr[h]);
      a.scale[(int64_t)h * nbs + b] = sc;
      scale_s = sc;
    }
  }
  __syncthreads();
  const float sc = scale_s;
  // v / sc by Markstein's final step from RN(1/sc): sc >= 1e-7, and the codes
  // depend only on quotients of magnitude >= 0.5, where its residual is exact
  const float rsc = __frcp_rn(sc);
#pragma unroll 4
  for (int r = warp; r < a.blk; r += 4) {
    uint32_t word = 0;
    if (r < valid) {
      float v[4];
      if (a.mean) {
        const uint2 raw = rows_s[r * 32 + lane];
        v[0] = __uint_as_float(raw.x << 16);
        v[1] = __uint_as_float(raw.x & 0xffff0000u);
        v[2] = __uint_as_float(raw.y << 16);
        v[3] = __uint_as_float(raw.y & 0xffff0000u);
      } else {
        load4_row(a, r0 + r, h, lane, mean4, v);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float t = div_rn_by(v[i], sc, rsc);
        t = __fadd_rn(t, t >= 0.0f ? 0.5f : -0.5f);
        // trunc, clamp to [-127, 127], to int: clamping first gives the same code
        // (also for NaN, which both orders send to -127) with one conversion
        const int code = __float2int_rz(fminf(127.0f, fmaxf(-127.0f, t)));
        word |= ((uint32_t)code & 0xffu) << (8 * i);
      }
    }
    *reinterpret_cast<uint32_t*>(a.q + ((int64_t)h * a.Lpad + r0 + r) * kD + 4 * lane) = word;
  }
}

cudaError_t launch_pool_sim_quant(const PoolArgs& a, cudaStream_t s) {
  const int nb = (int)((a.L + a.blk - 1) / a.blk);
  dim3 grid(nb, a.H);
  pool_sim_quant_kernel<<<grid, 128, a.mean ? (size_t)a.blk * 32 * sizeof(uint2) : 0, s>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ Sage per_thread INT8

// Scale groups of Sage's per_thread granularity (qk_quant_gran 3): for Q, 128-row
// blocks of 32 groups, row r of a block in group (r / 32) * 8 + r % 8; for K, 64-row
// blocks of 4 groups, row r in group (r % 8) / 2 -- the rows one sm89 MMA thread
// holds (model/sage_fused_quant.py:41-44 for K; the Q grouping of the grid and scale
// shape at model/sage_fused_quant.py:201-222).  Per group: scale = max|v|/127 + 1e-7,
// code = trunc(v / scale + 0.5 sign); K values are bf16(k - mean).
// One CTA of four warps per (block, head): lane l owns channels 4l..4l+3, warp w the
// rows w, w+4, ...; each row's values stay in shared memory between the two passes.
template <int BLK, int NG>
__device__ __forceinline__ int group_of_row(int r) {
  return NG == 32 ? (r >> 5) * 8 + (r & 7) : (r & 7) >> 1;
}

template <int BLK, int NG>
__global__ void __launch_bounds__(128) quant_per_thread_kernel(PoolArgs a) {
  __shared__ uint2 rows_s[BLK][32];
  __shared__ float ramax_s[BLK];
  __shared__ float gscale_s[NG];
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r0 = (int64_t)b * BLK;
  const int valid = (int)((a.L - r0) < BLK ? (a.L - r0) : BLK);
  float mean4[4] = {0.f, 0.f, 0.f, 0.f};
  if (a.mean) {
    const uint2 raw = *reinterpret_cast<const uint2*>(a.mean + h * kD + 4 * lane);
    mean4[0] = __uint_as_float(raw.x << 16);
    mean4[1] = __uint_as_float(raw.x & 0xffff0000u);
    mean4[2] = __uint_as_float(raw.y << 16);
    mean4[3] = __uint_as_float(raw.y & 0xffff0000u);
  }
#pragma unroll 4
  for (int r = warp; r < BLK; r += 4) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < valid) load4_row(a, r0 + r, h, lane, mean4, v);
    rows_s[r][lane] = make_uint2((__float_as_uint(v[0]) >> 16) | (__float_as_uint(v[1]) & 0xffff0000u),
                                 (__float_as_uint(v[2]) >> 16) | (__float_as_uint(v[3]) & 0xffff0000u));
    float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    if (lane == 0) ramax_s[r] = am;
  }
  __syncthreads();
  if (threadIdx.x < NG) {
    const int g = threadIdx.x;
    float am = 0.f;
    for (int r = 0; r < BLK; ++r)
      if (group_of_row<BLK, NG>(r) == g) am = fmaxf(am, ramax_s[r]);
    const float sc = __fadd_rn(__fdiv_rn(am, 127.0f), 1e-7f);
    gscale_s[g] = sc;
    a.scale[(int64_t)h * a.nb_stride + (int64_t)b * NG + g] = sc;
  }
  __syncthreads();
#pragma unroll 4
  for (int r = warp; r < BLK; r += 4) {
    uint32_t word = 0;
    if (r < valid) {
      const float sc = gscale_s[group_of_row<BLK, NG>(r)];
      const float rsc = __frcp_rn(sc);
      const uint2 raw = rows_s[r][lane];
      const float v[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                          __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float t = div_rn_by(v[i], sc, rsc);
        t = __fadd_rn(t, t >= 0.0f ? 0.5f : -0.5f);
        const int code = __float2int_rz(fminf(127.0f, fmaxf(-127.0f, t)));
        word |= ((uint32_t)code & 0xffu) << (8 * i);
      }
    }
    *reinterpret_cast<uint32_t*>(a.q + ((int64_t)h * a.Lpad + r0 + r) * kD + 4 * lane) = word;
  }
}

cudaError_t launch_quant_per_thread(const PoolArgs& a, int kind, cudaStream_t s) {
  if (kind == 0) {
    dim3 grid((unsigned)((a.L + 127) / 128), a.H);
    quant_per_thread_kernel<128, 32><<<grid, 128, 0, s>>>(a);
  } else {
    dim3 grid((unsigned)((a.L + 63) / 64), a.H);
    quant_per_thread_kernel<64, 4><<<grid, 128, 0, s>>>(a);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ q/k RMSNorm + RoPE

// In place on the projection output rows, per (token, q|k, head):
// n = bf16((x * inv_rms) * w);  for d < rot/2 with its partner e = d + rot/2:
//   out_d = bf16(n_d cos - n_e sin), out_e = bf16(n_d sin + n_e cos)
// (model/layers.py:72-149 split-half partial RoPE after per-head RMSNorm).
// One warp per (token, q|k): lane l owns channels 4l..4l+3 of every head, loads
// its cos/sin values once and walks the heads four at a time, so four
// independent reductions are in flight.
__device__ __forceinline__ void load4_bf16(const uint16_t* p, bool vec, float (&v)[4]) {
  if (vec) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(r.x << 16);
    v[1] = __uint_as_float(r.x & 0xffff0000u);
    v[2] = __uint_as_float(r.y << 16);
    v[3] = __uint_as_float(r.y & 0xffff0000u);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = bf16_bits_to_f32(p[i]);
  }
}

__global__ void __launch_bounds__(256) qk_rmsnorm_rope_kernel(QkRopeArgs a) {
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wid >= 2 * a.L) return;
  const int64_t t = wid >> 1;
  const bool is_k = (wid & 1) != 0;
  uint16_t* row = a.x + t * a.stride + (is_k ? a.k_off : a.q_off) + 4 * lane;
  float wv[4];
  load4_bf16((is_k ? a.kw : a.qw) + 4 * lane, true, wv);
  const int half = a.rot_dim >> 1, d0 = 4 * lane;
  const bool first = d0 < half, rot = d0 < a.rot_dim;
  const int src = first ? lane + (half >> 2) : lane - (half >> 2);
  float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
  if (rot) {
    const int64_t j = t * half + (first ? d0 : d0 - half);
    const bool vec = ((reinterpret_cast<uintptr_t>(a.cos_t) | reinterpret_cast<uintptr_t>(a.sin_t)) & 7) == 0;
    load4_bf16(a.cos_t + j, vec, c);
    load4_bf16(a.sin_t + j, vec, sn);
  }
  for (int h0 = 0; h0 < a.H; h0 += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int h = h0 + u;
      if (h >= a.H) break;  // uniform across the warp
      uint16_t* p = row + (int64_t)h * kD;
      const uint2 raw = *reinterpret_cast<const uint2*>(p);
      const float v[4] = {__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                          __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u)};
      const float sq = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(v[0], v[0]), __fmul_rn(v[1], v[1])),
                                           __fmul_rn(v[2], v[2])),
                                 __fmul_rn(v[3], v[3]));
      const float ss = warp_butterfly_sum(sq);
      // ss / 128 is a scaling by 2^-7: the product rounds the same value the division does
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 0.0078125f), a.eps)));
      // normalized values, rounded to bf16 two at a time; kept as packed bf16 pairs
      const uint32_t n01 = bf16x2_bits(__fmul_rn(__fmul_rn(v[0], inv), wv[0]), __fmul_rn(__fmul_rn(v[1], inv), wv[1]));
      const uint32_t n23 = bf16x2_bits(__fmul_rn(__fmul_rn(v[2], inv), wv[2]), __fmul_rn(__fmul_rn(v[3], inv), wv[3]));
      // the rotation partner of each value, two per shuffle
      const uint32_t p01 = __shfl_sync(0xffffffffu, n01, rot ? src : lane);
      const uint32_t p23 = __shfl_sync(0xffffffffu, n23, rot ? src : lane);
      uint2 outw = make_uint2(n01, n23);
      if (rot) {
        const float n[4] = {__uint_as_float(n01 << 16), __uint_as_float(n01 & 0xffff0000u),
                            __uint_as_float(n23 << 16), __uint_as_float(n23 & 0xffff0000u)};
        const float pt[4] = {__uint_as_float(p01 << 16), __uint_as_float(p01 & 0xffff0000u),
                             __uint_as_float(p23 << 16), __uint_as_float(p23 & 0xffff0000u)};
        float o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          o[i] = first ? __fsub_rn(__fmul_rn(n[i], c[i]), __fmul_rn(pt[i], sn[i]))
                       : __fadd_rn(__fmul_rn(pt[i], sn[i]), __fmul_rn(n[i], c[i]));
        outw = make_uint2(bf16x2_bits(o[0], o[1]), bf16x2_bits(o[2], o[3]));
      }
      *reinterpret_cast<uint2*>(p) = outw;
    }
  }
}

cudaError_t launch_qk_rmsnorm_rope(const QkRopeArgs& a, cudaStream_t s) {
  const int64_t warps = a.L * 2;
  qk_rmsnorm_rope_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(a);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ value fp8

constexpr int kAbsRows = 512;

// Per-column |V| maxima over a band of kAbsRows rows: each thread reads 8
// consecutive columns (one 16-byte load per row) and keeps 8 running maxima.
__global__ void __launch_bounds__(256) value_absmax_kernel(const uint16_t* __restrict__ v, int64_t L, int cols,
                                                            int64_t stride, unsigned int* __restrict__ amax_bits) {
  const int c = 8 * (blockIdx.y * blockDim.x + threadIdx.x);
  if (c >= cols) return;
  const int64_t r0 = (int64_t)blockIdx.x * kAbsRows;
  const int64_t r1 = r0 + kAbsRows < L ? r0 + kAbsRows : L;
  float m[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const uint16_t* p = v + r0 * stride + c;
#pragma unroll 4
  for (int64_t r = r0; r < r1; ++r, p += stride) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      m[2 * j] = fmaxf(m[2 * j], fabsf(__uint_as_float(w[j] << 16)));
      m[2 * j + 1] = fmaxf(m[2 * j + 1], fabsf(__uint_as_float(w[j] & 0xffff0000u)));
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) atomicMax(amax_bits + c + j, __float_as_uint(m[j]));  // non-negative floats order like their bits
}

// One CTA per (128-token tile, head): read V[128 tokens][128 ch] (bf16) into
// shared memory, write vt[h][ch][tile] as E4M3, 128 bytes per channel row.
// vscale (optional): max(amax / 2.25, 1e-12), written by the first tile's CTAs.
__global__ void __launch_bounds__(256) value_fp8_kernel(const uint16_t* __restrict__ v, int64_t L, int H,
                                                         int64_t stride, int64_t Lpad,
                                                         const float* __restrict__ amax, uint8_t* __restrict__ vt,
                                                         float* __restrict__ vscale) {
  __shared__ uint16_t tile[128][kD + 2];
  __shared__ float mul_s[kD];
  const int h = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.x * 128;
  for (int i = threadIdx.x; i < 128 * (kD / 8); i += blockDim.x) {
    const int r = i / (kD / 8), c8 = (i % (kD / 8)) * 8;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (t0 + r < L) raw = *reinterpret_cast<const uint4*>(v + (t0 + r) * stride + (int64_t)h * kD + c8);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      tile[r][c8 + 2 * j] = (uint16_t)(w[j] & 0xffffu);
      tile[r][c8 + 2 * j + 1] = (uint16_t)(w[j] >> 16);
    }
  }
  if (threadIdx.x < kD) {
    const float am = amax[h * kD + threadIdx.x];
    mul_s[threadIdx.x] = am > 0.f ? __fdiv_rn(2.25f, am) : 0.f;
    if (vscale && blockIdx.x == 0) vscale[h * kD + threadIdx.x] = fmaxf(__fdiv_rn(am, 2.25f), 1e-12f);
  }
  __syncthreads();
  // thread -> (channel, half of the 128 tokens): 64 bytes out
  const int d = threadIdx.x >> 1, half = threadIdx.x & 1;
  const float mul = mul_s[d];
  uint32_t out[16];
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      const int r = half * 64 + 4 * w + j;
      const float a0 = (t0 + r < L) ? __fmul_rn(bf16_bits_to_f32(tile[r][d]), mul) : 0.f;
      const float a1 = (t0 + r + 1 < L) ? __fmul_rn(bf16_bits_to_f32(tile[r + 1][d]), mul) : 0.f;
      word |= (uint32_t)f32x2_to_e4m3x2(a0, a1) << (8 * j);
    }
    out[w] = word;
  }
  uint8_t* dst = vt + ((int64_t)h * kD + d) * Lpad + t0 + half * 64;
#pragma unroll
  for (int w = 0; w < 16; w += 4) *reinterpret_cast<uint4*>(dst + 4 * w) = make_uint4(out[w], out[w + 1], out[w + 2], out[w + 3]);
}

__global__ void value_scale_final_kernel(float* vscale, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) vscale[i] = __fdiv_rn(vscale[i], 2.25f);
}

cudaError_t launch_value_fp8(const void* v, int64_t L, int64_t H, int64_t stride, int64_t Lpad, void* vt,
                             void* vscale, cudaStream_t s) {
  const int cols = (int)(H * kD);
  cudaError_t e = cudaMemsetAsync(vscale, 0, sizeof(float) * cols, s);
  if (e != cudaSuccess) return e;
  dim3 g1((unsigned)((L + kAbsRows - 1) / kAbsRows), (cols / 8 + 255) / 256);
  value_absmax_kernel<<<g1, 256, 0, s>>>(static_cast<const uint16_t*>(v), L, cols, stride,
                                         static_cast<unsigned int*>(vscale));
  dim3 g2((unsigned)(Lpad / 128), (unsigned)H);
  value_fp8_kernel<<<g2, 256, 0, s>>>(static_cast<const uint16_t*>(v), L, (int)H, stride, Lpad,
                                      static_cast<const float*>(vscale), static_cast<uint8_t*>(vt), nullptr);
  value_scale_final_kernel<<<(cols + 255) / 256, 256, 0, s>>>(static_cast<float*>(vscale), cols);
  return cudaGetLastError();
}

cudaError_t launch_value_fp8_given_absmax(const void* v, int64_t rows, int64_t H, int64_t stride, int64_t Lpad,
                                          const float* absmax, void* vt, float* vscale, cudaStream_t s) {
  dim3 g((unsigned)((rows + 127) / 128), (unsigned)H);
  value_fp8_kernel<<<g, 256, 0, s>>>(static_cast<const uint16_t*>(v), rows, (int)H, stride, Lpad, absmax,
                                     static_cast<uint8_t*>(vt), vscale);
  return cudaGetLastError();
}

}  // namespace h3b
