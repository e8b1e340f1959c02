// adaln.cu -- the block's AdaLN projection on the GPU:
//
//   out[r, n] = bf16( sum_k t[r, k] * w[n, k] + b[n] )      (fp32 products and sums)
//
// The engine's adaln_projector is a linear layer over the timestep (or curve) rows
// (model/layers.py:1083-1085, model/lora.py:524-570); its output is split into the
// shift / scale / gate rows of the two AdaLN modulations.  One warp per output
// column n: the lanes stream the bf16 weight row with 16-byte loads (the weight is
// read once from HBM, the few t rows stay in L1), each lane keeps one fp32 partial
// sum per t row, and a butterfly over the warp adds the lanes.  HBM-bound: the
// weight's bytes per call.
#include "h3b_kernels.cuh"

namespace h3b {

constexpr int kAdaRows = 8;     // t rows per call (the H3 block uses at most 3 per timestep)
constexpr int kAdaWarps = 8;    // output columns per CTA

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <int R>
__global__ void __launch_bounds__(32 * kAdaWarps) adaln_gemv_kernel(const uint16_t* __restrict__ w,
                                                                   const uint16_t* __restrict__ t,
                                                                   const uint16_t* __restrict__ b, int64_t n,
                                                                   int64_t k, uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t col = (int64_t)blockIdx.x * kAdaWarps + (threadIdx.x >> 5);
  if (col >= n) return;
  const uint4* wrow = reinterpret_cast<const uint4*>(w + col * k);
  const int64_t chunks = k / 8;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  for (int64_t c = lane; c < chunks; c += 32) {
    float wf[8];
    bf16x8_to_f32(__ldg(wrow + c), wf);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float tf[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(t + r * k) + c), tf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[r] = fmaf(tf[e], wf[e], acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float v = warp_butterfly_sum(acc[r]);
    if (lane == r) {
      if (b) v = __fadd_rn(v, bf16_bits_to_f32(b[col]));
      out[r * n + col] = f32_to_bf16_bits(v);
    }
  }
}

cudaError_t launch_adaln_projection(const uint16_t* w, const uint16_t* t, const uint16_t* b, int64_t rows,
                                    int64_t n, int64_t k, uint16_t* out, cudaStream_t s) {
  const unsigned blocks = (unsigned)((n + kAdaWarps - 1) / kAdaWarps);
  const int threads = 32 * kAdaWarps;
  switch (rows) {
#define H3B_ADA_CASE(R) \
  case R: adaln_gemv_kernel<R><<<blocks, threads, 0, s>>>(w, t, b, n, k, out); break;
    H3B_ADA_CASE(1) H3B_ADA_CASE(2) H3B_ADA_CASE(3) H3B_ADA_CASE(4)
    H3B_ADA_CASE(5) H3B_ADA_CASE(6) H3B_ADA_CASE(7) H3B_ADA_CASE(8)
#undef H3B_ADA_CASE
    default: return cudaErrorInvalidValue;  // the C entry accepts 1..kAdaRows rows
  }
  return cudaGetLastError();
}

}  // namespace h3b
