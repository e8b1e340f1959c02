// w4a8.cu -- grouped packed-int4 weights -> the int8 grid the INT8 GEMM consumes.
//
// out[n,k] = clamp(rint(level(c) * s_rel[n, k/G]), -127, 127), level = codebook[c]
// or c - 8, c the 4-bit code (even column in the low nibble); s_rel is fp32 or
// FP8 E4M3 (comfy_kitchen backends/cuda/ops/w4a8_gemm.cu:36-90).  The per-channel
// scale s_channel is applied later in the GEMM epilogue.
//
// Decoding once per call (a memory-bound pass over N*K/2 bytes, ~20 us for a
// 16384 x 4096 layer) and then running the plain tcgen05 INT8 GEMM keeps the
// int8 weight L2-resident for the whole GEMM; decoding inside the GEMM's
// shared-memory pipeline would repeat the decode once per 128-row M tile
// (872 times at M = 111,600).
#include "h3b_kernels.cuh"

namespace h3b {

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(hr));
}

// One thread: 16 packed bytes -> 32 int8 outputs (two 16-byte stores).
template <int SCALE_KIND, bool CODEBOOK>
__global__ void __launch_bounds__(256) w4_decode_kernel(const uint8_t* __restrict__ qw, const void* __restrict__ s_rel,
                                                        const float* __restrict__ codebook, int8_t* __restrict__ out,
                                                        int64_t N, int K, int G) {
  __shared__ float cb[16];
  if (CODEBOOK) {
    if (threadIdx.x < 16) cb[threadIdx.x] = codebook[threadIdx.x];
    __syncthreads();
  }
  const int per_row = K / 32;
  const int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= N * per_row) return;
  const int64_t n = v / per_row;
  const int k0 = (int)(v % per_row) * 32;
  const int groups = K / G;
  const uint4 pk = *reinterpret_cast<const uint4*>(qw + n * (K / 2) + k0 / 2);
  const uint32_t words[4] = {pk.x, pk.y, pk.z, pk.w};
  uint32_t outw[8];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t packed = 0;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const uint32_t byte = (words[w] >> (8 * (2 * half + b))) & 0xffu;
#pragma unroll
        for (int nib = 0; nib < 2; ++nib) {
          const int k = k0 + 8 * w + 4 * half + 2 * b + nib;
          const uint32_t c = nib ? (byte >> 4) : (byte & 0xfu);
          const float lvl = CODEBOOK ? cb[c] : (float)c - 8.0f;
          const int64_t si = n * groups + k / G;
          const float s = SCALE_KIND == 0 ? __ldg(reinterpret_cast<const float*>(s_rel) + si)
                                          : e4m3_to_f32(reinterpret_cast<const uint8_t*>(s_rel)[si]);
          float p = rintf(__fmul_rn(lvl, s));
          p = fminf(127.0f, fmaxf(-127.0f, p));
          packed |= ((uint32_t)(int)p & 0xffu) << (8 * (2 * b + nib));
        }
      }
      outw[2 * w + half] = packed;
    }
  }
  int8_t* dst = out + n * K + k0;
  *reinterpret_cast<uint4*>(dst) = make_uint4(outw[0], outw[1], outw[2], outw[3]);
  *reinterpret_cast<uint4*>(dst + 16) = make_uint4(outw[4], outw[5], outw[6], outw[7]);
}

// ------------------------------------------------------------------ group-correction activations
// The rank-(K/G) correction of asymmetric W4A8 weights (comfy_kitchen
// backends/cuda/__init__.py:2294-2297): sx[m, g] = bf16(bf16(sum_{k in group g} xq[m, k])
// * bf16(xs[m])), the operand of the bf16 GEMM that adds sx @ correction to the output.
// One thread per (row, group column); columns past the last group are written 0 so
// the GEMM's K can be padded to a multiple of 8.
__global__ void __launch_bounds__(256) group_sums_kernel(const int8_t* __restrict__ xq, const float* __restrict__ xs,
                                                         int64_t M, int K, int G, int groups,
                                                         uint16_t* __restrict__ sx, int64_t stride) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * stride) return;
  const int64_t m = i / stride;
  const int g = (int)(i - m * stride);
  uint16_t out = 0;
  if (g < groups) {
    const int8_t* p = xq + m * (int64_t)K + (int64_t)g * G;
    int sum = 0;
    if ((G & 15) == 0 && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
      for (int k = 0; k < G; k += 16) {
        const int4 w = *reinterpret_cast<const int4*>(p + k);
        const int ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          sum += (int)(int8_t)(ws[j] & 0xff) + (int)(int8_t)((ws[j] >> 8) & 0xff) +
                 (int)(int8_t)((ws[j] >> 16) & 0xff) + (int)(int8_t)((ws[j] >> 24) & 0xff);
      }
    } else {
      for (int k = 0; k < G; ++k) sum += p[k];
    }
    const float sb = bf16_bits_to_f32(f32_to_bf16_bits((float)sum));   // int32 -> bf16 (exact to float first)
    const float xb = bf16_bits_to_f32(f32_to_bf16_bits(xs[m]));
    out = f32_to_bf16_bits(__fmul_rn(sb, xb));
  }
  sx[i] = out;
}

cudaError_t launch_group_sums(const int8_t* xq, const float* xs, int64_t M, int64_t K, int64_t G, uint16_t* sx,
                              int64_t sx_stride, cudaStream_t s) {
  const int64_t total = M * sx_stride;
  group_sums_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(xq, xs, M, (int)K, (int)G, (int)(K / G), sx,
                                                                    sx_stride);
  return cudaGetLastError();
}

cudaError_t launch_w4_decode(const void* qw, const void* s_rel, int s_rel_kind, const void* codebook, void* out,
                             int64_t N, int64_t K, int64_t G, cudaStream_t s) {
  const int64_t total = N * (K / 32);
  const int threads = 256;
  const unsigned blocks = (unsigned)((total + threads - 1) / threads);
  const uint8_t* q = static_cast<const uint8_t*>(qw);
  const float* cb = static_cast<const float*>(codebook);
  int8_t* o = static_cast<int8_t*>(out);
  if (s_rel_kind == 0) {
    if (cb) w4_decode_kernel<0, true><<<blocks, threads, 0, s>>>(q, s_rel, cb, o, N, (int)K, (int)G);
    else w4_decode_kernel<0, false><<<blocks, threads, 0, s>>>(q, s_rel, cb, o, N, (int)K, (int)G);
  } else {
    if (cb) w4_decode_kernel<1, true><<<blocks, threads, 0, s>>>(q, s_rel, cb, o, N, (int)K, (int)G);
    else w4_decode_kernel<1, false><<<blocks, threads, 0, s>>>(q, s_rel, cb, o, N, (int)K, (int)G);
  }
  return cudaGetLastError();
}

}  // namespace h3b
