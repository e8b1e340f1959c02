// ulysses.cu -- layout kernels around the Ulysses all-to-alls of the multi-GPU block.
//
// Token rows are sharded over P ranks; attention needs every token of H/P heads.
// An all-to-all exchanges [P, rows, H/P heads, 128] chunks: chunk p of a rank's send
// buffer holds its own token rows of the heads rank p computes.  These kernels build
// that buffer straight from the projection rows (with an optional head order that
// assigns heads to ranks out of index order, for load balance) and turn the returned
// attention output back into token rows in head index order -- one read and one write
// each, where the torch expression needs a gather and a transposed copy.
#include "h3b_kernels.cuh"

namespace h3b {

// dst[p][l][j][:] = src[l][order[p*hpr + j]][:]  (128 bf16 per head, 16-byte chunks)
__global__ void __launch_bounds__(256) gather_heads_kernel(const uint16_t* __restrict__ src, int64_t rows, int H,
                                                           int64_t src_stride, const int64_t* __restrict__ order,
                                                           int P, uint16_t* __restrict__ dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // 16-byte chunk index over dst
  const int64_t total = rows * H * 16;
  if (i >= total) return;
  const int hpr = H / P;
  const int c = (int)(i & 15);
  const int64_t t = i >> 4;               // (p, l, j) flattened
  const int j = (int)(t % hpr);
  const int64_t pl = t / hpr;
  const int64_t l = pl % rows;
  const int p = (int)(pl / rows);
  const int hd = p * hpr + j;
  const int head = order ? (int)order[hd] : hd;
  const uint4 v = *reinterpret_cast<const uint4*>(src + l * src_stride + (int64_t)head * 128 + c * 8);
  *reinterpret_cast<uint4*>(dst + i * 8) = v;
}

// dst[l][order[p*hpr + j]][:] = src[p][l][j][:]
__global__ void __launch_bounds__(256) scatter_heads_kernel(const uint16_t* __restrict__ src, int64_t rows, int H,
                                                            const int64_t* __restrict__ order, int P,
                                                            uint16_t* __restrict__ dst, int64_t dst_stride) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = rows * H * 16;
  if (i >= total) return;
  const int hpr = H / P;
  const int c = (int)(i & 15);
  const int64_t t = i >> 4;
  const int j = (int)(t % hpr);
  const int64_t pl = t / hpr;
  const int64_t l = pl % rows;
  const int p = (int)(pl / rows);
  const int hd = p * hpr + j;
  const int head = order ? (int)order[hd] : hd;
  const uint4 v = *reinterpret_cast<const uint4*>(src + i * 8);
  *reinterpret_cast<uint4*>(dst + l * dst_stride + (int64_t)head * 128 + c * 8) = v;
}

cudaError_t launch_gather_heads(const void* src, int64_t rows, int64_t H, int64_t src_stride, const int64_t* order,
                                int64_t P, void* dst, cudaStream_t s) {
  const int64_t total = rows * H * 16;
  gather_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      static_cast<const uint16_t*>(src), rows, (int)H, src_stride, order, (int)P, static_cast<uint16_t*>(dst));
  return cudaGetLastError();
}

cudaError_t launch_scatter_heads(const void* src, int64_t rows, int64_t H, const int64_t* order, int64_t P,
                                 void* dst, int64_t dst_stride, cudaStream_t s) {
  const int64_t total = rows * H * 16;
  scatter_heads_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(
      static_cast<const uint16_t*>(src), rows, (int)H, order, (int)P, static_cast<uint16_t*>(dst), dst_stride);
  return cudaGetLastError();
}

}  // namespace h3b
