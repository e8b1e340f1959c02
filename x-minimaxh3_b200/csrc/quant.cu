// quant.cu -- per-token dynamic INT8 activation quantization for the DiT linears.
//
// Persistent CTAs of T threads (a multiple of 32, at most 512) walk the token
// rows (the next row is loaded while the current one is processed); thread t
// owns two 16-column chunks of the row, chunk t % 16 of the 256-column groups
// 2p and 2p + 1 (p = t / 16), held as the two lanes of packed float pairs, so
// every global access is a 32-byte vector load or a 16-byte vector store and the
// arithmetic runs on packed fp32 pairs.  Variants (template):
//   * plain row quantization        (comfy_kitchen int8_linear.cu:158-200)
//   * ConvRot-256 + row quantization (int8_linear.cu:943-1030), with the
//     optional input activation gelu_tanh / swiglu applied on load
//   * RMSNorm + AdaLN modulation fused in front of either of the above
//     (fused_norm_rope.py:12-45 feeding quantization.py:295-304)
// The 256-point regular-Hadamard transform is done as a 16x16 array: the
// stride-1 and stride-4 radix-4 stages act along a row of 16 (in registers),
// one shared-memory transpose, then the stride-16 and stride-64 stages act
// along a column (in registers).  The operation order inside each radix-4
// butterfly is the reference's, so results equal its fp32 transform bit for bit.
#include "h3b_kernels.cuh"
#include "h3b_packed.cuh"

namespace h3b {

enum QuantMode : int { kPlain = 0, kConvRot = 1 };



// Warp shfl_down tree then the same tree over the (zero padded) warp sums:
// identical to block_tree_sum in the CPU oracle.
__device__ __forceinline__ float block_tree_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float o = __shfl_down_sync(0xffffffffu, v, off);
    v = __fadd_rn(v, o);
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < nw ? red[lane] : 0.0f;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, off));
    if (lane == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float s = lane < nw ? red[lane] : 0.0f;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, off));
    if (lane == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}

// h3b_expf on both lanes.  For rint(x log2 e) = n in [-125, 127] (|x| below ~86)
// h3b_expf's two half scalings of p = 2^f (f in [-0.5, 0.5], so p in [0.7, 1.42])
// are exact and equal one add of n to p's exponent field, which is what this
// computes (rint by adding 1.5 * 2^23, as rintf; n from the sum's bits).  A lane
// outside that range, or NaN, takes h3b_expf itself.
__device__ __forceinline__ float2 h3b_expf_x2(float2 x) {
  const float kLog2e = 1.44269502162933349609375f;
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.428606765330187045e-06f;
  const float2 xc = make_float2(fminf(fmaxf(x.x, -120.0f), 100.0f), fminf(fmaxf(x.y, -120.0f), 100.0f));
  const float2 t = add2(mul2(xc, splat2(kLog2e)), splat2(12582912.0f));
  const float2 n = sub2(t, splat2(12582912.0f));
  float2 r = fma2(n, splat2(-kLn2Hi), xc);
  r = fma2(n, splat2(-kLn2Lo), r);
  float2 p = splat2(1.0f / 5040.0f);
  p = fma2(p, r, splat2(1.0f / 720.0f));
  p = fma2(p, r, splat2(1.0f / 120.0f));
  p = fma2(p, r, splat2(1.0f / 24.0f));
  p = fma2(p, r, splat2(1.0f / 6.0f));
  p = fma2(p, r, splat2(0.5f));
  p = fma2(p, r, splat2(1.0f));
  p = fma2(p, r, splat2(1.0f));
  const int nx = (int)(__float_as_uint(t.x) - 0x4B400000u), ny = (int)(__float_as_uint(t.y) - 0x4B400000u);
  float2 e;
  e.x = (nx >= -125 && nx <= 127 && x.x == x.x) ? __uint_as_float(__float_as_uint(p.x) + ((uint32_t)nx << 23))
                                                 : h3b_expf(x.x);
  e.y = (ny >= -125 && ny <= 127 && x.y == x.y) ? __uint_as_float(__float_as_uint(p.y) + ((uint32_t)ny << 23))
                                                 : h3b_expf(x.y);
  return e;
}
// swiglu on both lanes: the scalar swiglu, lane by lane (IEEE quotient per lane)
__device__ __forceinline__ float2 swiglu2(float2 gate, float2 up) {
  const float2 e = h3b_expf_x2(make_float2(-gate.x, -gate.y));
  const float2 den = add2(splat2(1.0f), e);
  return mul2(make_float2(__fdiv_rn(gate.x, den.x), __fdiv_rn(gate.y, den.y)), up);
}

__device__ __forceinline__ uint4 ldg4(const uint16_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
// 16 bf16 of chunk-lane x (words wx) and lane y (words wy) -> 16 float2
__device__ __forceinline__ void unpack16x2(const uint4 (&wx)[2], const uint4 (&wy)[2], float2 (&v)[16]) {
  const uint32_t qx[8] = {wx[0].x, wx[0].y, wx[0].z, wx[0].w, wx[1].x, wx[1].y, wx[1].z, wx[1].w};
  const uint32_t qy[8] = {wy[0].x, wy[0].y, wy[0].z, wy[0].w, wy[1].x, wy[1].y, wy[1].z, wy[1].w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = make_float2(__uint_as_float(qx[i] << 16), __uint_as_float(qy[i] << 16));
    v[2 * i + 1] = make_float2(__uint_as_float(qx[i] & 0xffff0000u), __uint_as_float(qy[i] & 0xffff0000u));
  }
}
__device__ __forceinline__ void load_pair(const uint16_t* base, int cx, int cy, bool lx, bool ly, uint4 (&wx)[2],
                                          uint4 (&wy)[2]) {
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  wx[0] = lx ? ldg4(base + cx * 16) : z;
  wx[1] = lx ? ldg4(base + cx * 16 + 8) : z;
  wy[0] = ly ? ldg4(base + cy * 16) : z;
  wy[1] = ly ? ldg4(base + cy * 16 + 8) : z;
}

// raw bf16 chunks of one row owned by this thread (prefetched one row ahead)
struct RowRegs {
  uint4 x[2][2];  // [lane][half]
  uint4 u[2][2];  // the `up` half of a swiglu row
};

template <int ACT>
__device__ __forceinline__ void load_row(const QuantArgs& a, int64_t row, int cx, int cy, bool lx, bool ly,
                                         RowRegs& r) {
  const uint16_t* xr = a.x + row * a.x_stride;
  load_pair(xr, cx, cy, lx, ly, r.x[0], r.x[1]);
  if (ACT == 2) load_pair(xr + a.K, cx, cy, lx, ly, r.u[0], r.u[1]);
}

// Persistent: CTA b handles rows b, b + gridDim.x, ...; the next row's loads are
// issued before the current row is processed.
template <int MODE, int ACT, bool RMS>
__global__ void __launch_bounds__(512) quant_rows_kernel(QuantArgs a, int64_t rows) {
  extern __shared__ float2 tile2[];     // (T/16) groups x 16 x 17 float2
  __shared__ float red[33];
  const int t = threadIdx.x;
  const int K = a.K, chunks = K >> 4;
  const int idx = t & 15;                    // place in the group's 16 x 16 array
  const int cx = (t >> 4) * 32 + idx, cy = cx + 16;
  const bool lx = cx < chunks, ly = cy < chunks;
  float2* my_tile = tile2 + (t >> 4) * (16 * 17);

  RowRegs nxt;
  int64_t row = blockIdx.x;
  if (row < rows) load_row<ACT>(a, row, cx, cy, lx, ly, nxt);
  for (; row < rows; row += gridDim.x) {
    const RowRegs cur = nxt;
    if (row + gridDim.x < rows) load_row<ACT>(a, row + gridDim.x, cx, cy, lx, ly, nxt);

    float2 v[16];
    unpack16x2(cur.x[0], cur.x[1], v);
    if (ACT == 2) {
      float2 u[16];
      unpack16x2(cur.u[0], cur.u[1], u);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = swiglu2(v[j], u[j]);
    } else if (ACT == 1) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = gelu_tanh2(v[j]);
    }
    // dead lanes hold zeros (loaded as zero, and every activation maps 0 to 0)

    if (RMS) {
      // sum of squares: each lane in column order, then lane x + lane y, then the block tree
      float2 part2 = splat2(0.0f);
#pragma unroll
      for (int j = 0; j < 16; ++j) part2 = add2(part2, mul2(v[j], v[j]));
      const float ss = block_tree_sum(__fadd_rn(part2.x, part2.y), red);
      const float2 inv = splat2(__fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps))));
      const int r = a.seg_row ? a.seg_row[row] : 0;
      const uint16_t* tabs[3] = {a.norm_w, a.scale_tab + (int64_t)r * K, a.shift_tab + (int64_t)r * K};
#pragma unroll
      for (int h = 0; h < 2; ++h) {  // 8 columns of each lane at a time
        // the tables as bf16 pairs (lane x column, lane y column): pair j is column 8h + j
        uint32_t w[3][8];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const uint4 z = make_uint4(0u, 0u, 0u, 0u);
          const uint4 wx = lx ? ldg4(tabs[k] + cx * 16 + 8 * h) : z;
          const uint4 wy = ly ? ldg4(tabs[k] + cy * 16 + 8 * h) : z;
          const uint32_t qx[4] = {wx.x, wx.y, wx.z, wx.w}, qy[4] = {wy.x, wy.y, wy.z, wy.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            w[k][2 * i] = __byte_perm(qx[i], qy[i], 0x5410);
            w[k][2 * i + 1] = __byte_perm(qx[i], qy[i], 0x7632);
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // bf16(x * inv * w); bf16(n * bf16(1 + scale)) with an fp32 product; bf16(n + shift).
          // The two adds of bf16 operands are packed bf16 adds: for bf16 operands the
          // correctly rounded bf16 sum equals the fp32 sum rounded to bf16 (the fp32 sum is
          // exact unless the exponents differ by more than 16, and then the smaller operand
          // is below half a bf16 step of the larger)
          const float2 n = unpack_bf16x2(pack_bf16x2(mul2(mul2(v[8 * h + j], inv), unpack_bf16x2(w[0][j]))));
          const float2 s1 = unpack_bf16x2(hadd2_bf16(0x3F803F80u, w[1][j]));
          v[8 * h + j] = unpack_bf16x2(hadd2_bf16(pack_bf16x2(mul2(n, s1)), w[2][j]));
        }
      }
      // dead lanes: weight, scale and shift load as 0, so v stays 0
    }

    if (MODE == kConvRot) {
      fht16x2(v);
      __syncthreads();
#pragma unroll
      for (int b = 0; b < 16; ++b) my_tile[idx * 17 + b] = v[b];
      __syncthreads();
      // the thread now holds column idx of both groups' arrays
#pragma unroll
      for (int r = 0; r < 16; ++r) v[r] = my_tile[r * 17 + idx];
      fht16x2(v);
    }

    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fmaxf(fabsf(v[j].x), fabsf(v[j].y)));
    amax = block_max(amax, red);
    const float scale = fmaxf(__fmul_rn(fminf(amax, 3.38953139e38f), 1.0f / 127.0f), 1.0e-30f);
    const float st = bf16r(scale);
    const float2 st2 = splat2(st), rst2 = splat2(__fdiv_rn(1.0f, st));
    if (t == 0) a.scales[row] = scale;

    uint32_t px[4], py[4];
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {
      uint32_t wxv = 0, wyv = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t bx, by;
        codes2(v[4 * w4 + j], st2, rst2, bx, by);
        wxv |= bx << (8 * j);
        wyv |= by << (8 * j);
      }
      px[w4] = wxv;
      py[w4] = wyv;
    }
    int8_t* qr = a.q + row * (int64_t)K;
    if (MODE == kConvRot) {
      // codes are held by column; transpose both groups back through shared memory
      uint8_t* bt = reinterpret_cast<uint8_t*>(my_tile);
      __syncthreads();
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        bt[r * 16 + idx] = (uint8_t)(px[r >> 2] >> (8 * (r & 3)));
        bt[256 + r * 16 + idx] = (uint8_t)(py[r >> 2] >> (8 * (r & 3)));
      }
      __syncthreads();
      const uint4 rx = *reinterpret_cast<const uint4*>(bt + idx * 16);
      const uint4 ry = *reinterpret_cast<const uint4*>(bt + 256 + idx * 16);
      if (lx) *reinterpret_cast<uint4*>(qr + cx * 16) = rx;
      if (ly) *reinterpret_cast<uint4*>(qr + cy * 16) = ry;
    } else {
      if (lx) *reinterpret_cast<uint4*>(qr + cx * 16) = make_uint4(px[0], px[1], px[2], px[3]);
      if (ly) *reinterpret_cast<uint4*>(qr + cy * 16) = make_uint4(py[0], py[1], py[2], py[3]);
    }
  }
}

// ---------------------------------------------------------------- rotated rows -> codes
// The second half of the FC2 input quantizer when FC1's GEMM epilogue has already
// applied tanh-GELU and the ConvRot transform: per row, the absmax is the max of the
// epilogue's per-(row, half-tile) maxima, and the codes are formed from the stored
// bf16 rotated values exactly as quant_rows_kernel forms them from its fp32 ones
// (code of bf16(bf16(v) / bf16(scale))).  One CTA per row at a time (persistent);
// thread t owns the 8-column chunks t, t + 256, ... (16-byte loads, 8-byte stores).
constexpr int kRotThreads = 256;
constexpr int kRotMaxChunks = 8;  // K <= 8 * 8 * 256 = 16384 in registers
__global__ void __launch_bounds__(kRotThreads) quant_rotated_kernel(const uint16_t* __restrict__ rot,
                                                                    int64_t rot_stride, const float* __restrict__ amax,
                                                                    int64_t amax_stride, int amax_cols, int K,
                                                                    int64_t rows, int8_t* __restrict__ q,
                                                                    float* __restrict__ scales) {
  __shared__ float red[33];
  const int t = threadIdx.x;
  const int chunks = K >> 3;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint16_t* src = rot + row * rot_stride;
    uint4 w[kRotMaxChunks];
#pragma unroll
    for (int i = 0; i < kRotMaxChunks; ++i) {
      const int c = t + i * kRotThreads;
      w[i] = c < chunks ? __ldg(reinterpret_cast<const uint4*>(src) + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    float am = 0.0f;
    for (int c = t; c < amax_cols; c += kRotThreads) am = fmaxf(am, __ldg(amax + row * amax_stride + c));
    am = block_max(am, red);
    const float scale = fmaxf(__fmul_rn(fminf(am, 3.38953139e38f), 1.0f / 127.0f), 1.0e-30f);
    const float st = bf16r(scale);
    const float2 st2 = splat2(st), rst2 = splat2(__fdiv_rn(1.0f, st));
    if (t == 0) scales[row] = scale;
    int8_t* dst = q + row * (int64_t)K;
#pragma unroll
    for (int i = 0; i < kRotMaxChunks; ++i) {
      const int c = t + i * kRotThreads;
      if (c >= chunks) continue;
      const uint32_t ww[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
      uint32_t pr[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        pr[j] = codes2_bf16(make_float2(__uint_as_float(ww[j] << 16), __uint_as_float(ww[j] & 0xffff0000u)), st2,
                            rst2);
      // code bytes 0..1 of pairs (0, 1) and (2, 3)
      *reinterpret_cast<uint2*>(dst + c * 8) =
          make_uint2(__byte_perm(pr[0], pr[1], 0x5410u), __byte_perm(pr[2], pr[3], 0x5410u));
    }
  }
}

cudaError_t launch_quant_rotated(const uint16_t* rot, int64_t rot_stride, const float* amax, int64_t amax_stride,
                                 int amax_cols, int K, int64_t rows, int8_t* q, float* scales, cudaStream_t s) {
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quant_rotated_kernel, kRotThreads, 0);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  quant_rotated_kernel<<<grid, kRotThreads, 0, s>>>(rot, rot_stride, amax, amax_stride, amax_cols, K, rows, q, scales);
  return cudaGetLastError();
}

// Threads per row: 16 per pair of 256-column groups (chunk pairs), rounded up to
// a warp multiple; K <= 16384 gives at most 512.
int quant_threads_for(int K) {
  const int chunks = K / 16;
  const int groups = (chunks + 15) / 16;
  const int T = ((groups + 1) / 2) * 16;
  return ((T + 31) / 32) * 32;
}

template <int MODE, int ACT, bool RMS>
static cudaError_t launch_q(const QuantArgs& a, int64_t rows, cudaStream_t s) {
  const int T = quant_threads_for(a.K);
  const size_t smem = (size_t)(T / 16) * 16 * 17 * sizeof(float2);
  auto k = quant_rows_kernel<MODE, ACT, RMS>;
  if (smem > 48 * 1024) {
    cudaError_t e0 = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e0 != cudaSuccess) return e0;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, T, smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t cap = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = (unsigned)(rows < cap ? rows : cap);
  k<<<grid, T, smem, s>>>(a, rows);
  return cudaGetLastError();
}

cudaError_t launch_quant(const QuantArgs& a, int64_t rows, int mode, bool rms, cudaStream_t s) {
  if (rms) {
    return mode == kConvRot ? launch_q<kConvRot, 0, true>(a, rows, s) : launch_q<kPlain, 0, true>(a, rows, s);
  }
  if (mode == kConvRot) {
    switch (a.act) {
      case 1: return launch_q<kConvRot, 1, false>(a, rows, s);
      case 2: return launch_q<kConvRot, 2, false>(a, rows, s);
      default: return launch_q<kConvRot, 0, false>(a, rows, s);
    }
  }
  switch (a.act) {
    case 1: return launch_q<kPlain, 1, false>(a, rows, s);
    case 2: return launch_q<kPlain, 2, false>(a, rows, s);
    default: return launch_q<kPlain, 0, false>(a, rows, s);
  }
}

}  // namespace h3b
