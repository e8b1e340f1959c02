// quant.cu -- per-token dynamic INT8 activation quantization for the DiT linears.
//
// Persistent CTAs of T threads (a multiple of 32, at most 512) walk the token
// rows (the next row is loaded while the current one is processed); thread t
// owns the 16-column chunks c = t, t+T, ... of the row, so every global access
// is a 32-byte vector load or a 16-byte vector store.  Variants (template):
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

namespace h3b {

enum QuantMode : int { kPlain = 0, kConvRot = 1 };


constexpr int kMaxIters = 2;  // chunks per thread; K <= 2 * 512 * 16 = 16384

// One radix-4 butterfly of the regular H4 matrix, outputs in the reference's
// operation order (int8_linear.cu:217-250): y0 = ((x0+x1)+x2)-x3,
// y1 = ((x0+x1)-x2)+x3, y2 = ((x0-x1)+x2)+x3, y3 = ((-x0+x1)+x2)+x3, times 1/2.
// x0+x1 and x0-x1 are shared; (-x0+x1)+x2 == x2-(x0-x1) exactly.
__device__ __forceinline__ void h4_stage(const float* x, int s, float* y, int base) {
  const float x0 = x[base], x1 = x[base + s], x2 = x[base + 2 * s], x3 = x[base + 3 * s];
  const float s01 = __fadd_rn(x0, x1), d01 = __fsub_rn(x0, x1);
  y[base] = __fmul_rn(0.5f, __fsub_rn(__fadd_rn(s01, x2), x3));
  y[base + s] = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(s01, x2), x3));
  y[base + 2 * s] = __fmul_rn(0.5f, __fadd_rn(__fadd_rn(d01, x2), x3));
  y[base + 3 * s] = __fmul_rn(0.5f, __fadd_rn(__fsub_rn(x2, d01), x3));
}

// Two radix-4 stages (stride 1 then 4) over 16 values held by one thread.
__device__ __forceinline__ void fht16(float (&v)[16]) {
  float t[16];
#pragma unroll
  for (int b0 = 0; b0 < 16; b0 += 4) h4_stage(v, 1, t, b0);
#pragma unroll
  for (int b0 = 0; b0 < 4; ++b0) h4_stage(t, 4, v, b0);
}

// exp(x) for x in [-20, 0], the argument range of the GELU's tanh: the IEEE
// operations of h3b_expf on that range without its range branches.  rint(x log2 e)
// is taken by adding and subtracting 1.5 * 2^23 (round half to even, as rintf),
// the integer exponent comes from that sum's low bits, and one power-of-two
// scaling replaces the two half scalings (equal, since every product stays
// normal for n >= -29).  Matches h3b_expf bit for bit on every float of [-20, 0].
__device__ __forceinline__ float expf_neg20(float x) {
  const float kLog2e = 1.44269502162933349609375f;
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.428606765330187045e-06f;
  const float t = __fadd_rn(__fmul_rn(x, kLog2e), 12582912.0f);
  const float n = __fsub_rn(t, 12582912.0f);
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
  const int ni = (int)(__float_as_uint(t) - 0x4B400000u);
  return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
}
// h3b_tanhf without branches: (1 - e) / (1 + e) correctly rounded by Markstein's
// final step from RN(1 / (1 + e)) (equal to IEEE division for every e in
// [2e-9, 1], the range exp(-2|x|) takes for |x| < 10); |x| >= 10 gives +-1.
__device__ __forceinline__ float tanh_gelu(float x) {
  const float a = fabsf(x);
  const float e = expf_neg20(__fmul_rn(-2.0f, a));
  const float num = __fsub_rn(1.0f, e), den = __fadd_rn(1.0f, e);
  float t = div_rn_by(num, den, __frcp_rn(den));
  t = x < 0.0f ? -t : t;
  return a >= 10.0f ? (x > 0.0f ? 1.0f : -1.0f) : t;
}
__device__ __forceinline__ float gelu_tanh(float v) {
  const float kBeta = 0.7978845608028654f;
  const float kKappa = 0.044715f;
  float cube = __fmul_rn(__fmul_rn(__fmul_rn(kKappa, v), v), v);
  float inner = __fmul_rn(kBeta, __fadd_rn(v, cube));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanh_gelu(inner)));
}
// int8 code of a scaled value s: clamp to [-128, 127], round half to even by
// adding 1.5 * 2^23, and take the low byte of the sum's bits -- the code of
// rintf + clamp + (int) (clamping first cannot change the rounded result).
__device__ __forceinline__ uint32_t code_byte(float s) {
  const float c = fminf(127.0f, fmaxf(-128.0f, s));
  return __float_as_uint(__fadd_rn(c, 12582912.0f)) & 0xffu;
}
__device__ __forceinline__ float swiglu(float gate, float up) {
  return __fmul_rn(__fdiv_rn(gate, __fadd_rn(1.0f, h3b_expf(-gate))), up);
}

__device__ __forceinline__ void load16_bf16(const uint16_t* p, float (&v)[16]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  const uint4 b = *reinterpret_cast<const uint4*>(p + 8);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

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

// raw bf16 chunks of one row owned by this thread (prefetched one row ahead)
struct RowRegs {
  uint4 x[kMaxIters][2];
  uint4 u[kMaxIters][2];  // the `up` half of a swiglu row
};

template <int ACT>
__device__ __forceinline__ void load_row(const QuantArgs& a, int64_t row, int t, int T, int chunks, RowRegs& r) {
  const uint16_t* xr = a.x + row * a.x_stride;
#pragma unroll
  for (int i = 0; i < kMaxIters; ++i) {
    const int c = t + i * T;
    if (c < chunks) {
      const uint4* p = reinterpret_cast<const uint4*>(xr + c * 16);
      r.x[i][0] = __ldg(p);
      r.x[i][1] = __ldg(p + 1);
      if (ACT == 2) {
        const uint4* pu = reinterpret_cast<const uint4*>(xr + a.K + c * 16);
        r.u[i][0] = __ldg(pu);
        r.u[i][1] = __ldg(pu + 1);
      }
    }
  }
}

__device__ __forceinline__ void unpack16(const uint4 (&w)[2], float (&v)[16]) {
  const uint32_t q[8] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(q[i] << 16);
    v[2 * i + 1] = __uint_as_float(q[i] & 0xffff0000u);
  }
}

// Persistent: CTA b handles rows b, b + gridDim.x, ...; the next row's loads are
// issued before the current row is processed.
template <int MODE, int ACT, bool RMS>
__global__ void __launch_bounds__(512) quant_rows_kernel(QuantArgs a, int64_t rows) {
  extern __shared__ float tile[];       // (T/16) groups x 16 x 17 floats
  __shared__ float red[33];
  const int T = blockDim.x, t = threadIdx.x;
  const int K = a.K, chunks = K >> 4;
  float* my_tile = tile + (t >> 4) * (16 * 17);
  const int a_idx = t & 15;  // row of the 16x16 group array owned for loads / stores

  RowRegs nxt;
  int64_t row = blockIdx.x;
  if (row < rows) load_row<ACT>(a, row, t, T, chunks, nxt);
  for (; row < rows; row += gridDim.x) {
    const RowRegs cur = nxt;
    if (row + gridDim.x < rows) load_row<ACT>(a, row + gridDim.x, t, T, chunks, nxt);

    float v[kMaxIters][16];
    bool live[kMaxIters];
#pragma unroll
    for (int i = 0; i < kMaxIters; ++i) {
      live[i] = t + i * T < chunks;
      if (live[i]) {
        unpack16(cur.x[i], v[i]);
        if (ACT == 2) {
          float u[16];
          unpack16(cur.u[i], u);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[i][j] = swiglu(v[i][j], u[j]);
        } else if (ACT == 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[i][j] = gelu_tanh(v[i][j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[i][j] = 0.0f;
      }
    }

    if (RMS) {
      float part = 0.0f;
#pragma unroll
      for (int i = 0; i < kMaxIters; ++i)
#pragma unroll
        for (int j = 0; j < 16; ++j) part = __fadd_rn(part, __fmul_rn(v[i][j], v[i][j]));
      const float ss = block_tree_sum(part, red);
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
      const int r = a.seg_row ? a.seg_row[row] : 0;
      const uint16_t* sc = a.scale_tab + (int64_t)r * K;
      const uint16_t* sh = a.shift_tab + (int64_t)r * K;
#pragma unroll
      for (int i = 0; i < kMaxIters; ++i) {
        if (!live[i]) continue;
        const int c0 = (t + i * T) * 16;
        float w[16], s1[16], s2[16];
        load16_bf16(a.norm_w + c0, w);
        load16_bf16(sc + c0, s1);
        load16_bf16(sh + c0, s2);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float n = bf16r(__fmul_rn(__fmul_rn(v[i][j], inv), w[j]));
          n = bf16r(__fmul_rn(n, bf16r(__fadd_rn(1.0f, s1[j]))));
          v[i][j] = bf16r(__fadd_rn(n, s2[j]));
        }
      }
    }

    if (MODE == kConvRot) {
#pragma unroll
      for (int i = 0; i < kMaxIters; ++i) {
        if (i * T >= chunks) break;  // uniform across the block
        fht16(v[i]);
        __syncthreads();
#pragma unroll
        for (int b = 0; b < 16; ++b) my_tile[a_idx * 17 + b] = v[i][b];
        __syncthreads();
        // thread now takes column b = a_idx of its group
#pragma unroll
        for (int r = 0; r < 16; ++r) v[i][r] = my_tile[r * 17 + a_idx];
        fht16(v[i]);
      }
    }

    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxIters; ++i)
      if (live[i])
#pragma unroll
        for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    amax = block_max(amax, red);
    const float scale = fmaxf(__fmul_rn(fminf(amax, 3.38953139e38f), 1.0f / 127.0f), 1.0e-30f);
    const float st = bf16r(scale);
    const float rst = __fdiv_rn(1.0f, st);
    if (t == 0) a.scales[row] = scale;

    int8_t* qr = a.q + row * (int64_t)K;
#pragma unroll
    for (int i = 0; i < kMaxIters; ++i) {
      if (i * T >= chunks) break;
      uint32_t packed[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          word |= code_byte(bf16r(div_rn_by(bf16r(v[i][4 * w + j]), st, rst))) << (8 * j);
        }
        packed[w] = word;
      }
      if (MODE == kConvRot) {
        // codes are held by column; transpose back through shared memory
        uint8_t* bt = reinterpret_cast<uint8_t*>(my_tile);
        __syncthreads();
#pragma unroll
        for (int r = 0; r < 16; ++r) bt[r * 16 + a_idx] = (uint8_t)(packed[r >> 2] >> (8 * (r & 3)));
        __syncthreads();
        const uint4 row16 = *reinterpret_cast<const uint4*>(bt + a_idx * 16);
        if (live[i]) *reinterpret_cast<uint4*>(qr + (t + i * T) * 16) = row16;
      } else if (live[i]) {
        *reinterpret_cast<uint4*>(qr + (t + i * T) * 16) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
    }
  }
}

int quant_threads_for(int K) {
  int chunks = K / 16;
  int T = ((chunks + 31) / 32) * 32;
  return T > 512 ? 512 : T;
}

template <int MODE, int ACT, bool RMS>
static cudaError_t launch_q(const QuantArgs& a, int64_t rows, cudaStream_t s) {
  const int T = quant_threads_for(a.K);
  const size_t smem = (size_t)(T / 16) * 16 * 17 * sizeof(float);
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
