// capi.cu -- the extern "C" boundary of libh3b.so (declared in include/h3b.h).
// Validates arguments, launches on the caller's stream, converts every failure
// into an int status plus a per-thread message; nothing throws out of here.
#include <climits>
#include <cstdio>
#include <cstring>
#include <string>

#include "h3b_kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
int ok() {
  g_last_error.clear();
  return H3B_OK;
}
int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ok();
  return fail(H3B_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
cudaStream_t st(void* s) { return static_cast<cudaStream_t>(s); }

// The bounded-wait failure path of the kernels, exercised on purpose: one warp
// waits on an mbarrier that nothing arrives at, with the kernels' own wait routine
// and a short limit; it gives up, records `code` in the device status word and
// returns, leaving the context usable.
__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, int code) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    h3b::mbar_init(&bar, 1);
    abort_flag = 0;
    h3b::fence_mbar_init();
  }
  __syncthreads();
  h3b::mbar_wait_for(&bar, 0, &abort_flag, code, limit_ns);
}

}  // namespace

extern "C" {

const char* h3b_version(void) { return "h3b 0.1 sm_100a"; }

const char* h3b_last_error(void) { return g_last_error.c_str(); }

int h3b_device_status(int device, int* status, int reset) {
  if (!status) return fail(H3B_ERR_INVALID_ARGUMENT, "status pointer is null");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, h3b::g_device_status, sizeof(int));
  if (e == cudaSuccess && reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(h3b::g_device_status, &zero, sizeof(int));
  }
  cudaSetDevice(prev);
  return cuda_status(e, "h3b_device_status");
}

int h3b_selftest_bounded_wait(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > 1000000000LL)
    return fail(H3B_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 1 s]");
  bounded_wait_selftest_kernel<<<1, 32, 0, st(stream)>>>((uint64_t)limit_ns, H3B_STATUS_SELFTEST_TIMEOUT);
  return cuda_status(cudaGetLastError(), "selftest_bounded_wait");
}

int h3b_quantize_int8_rowwise(const void* x, int64_t rows, int64_t cols, int64_t x_row_stride, void* q, void* scales,
                              void* stream) {
  if (rows == 0 || cols == 0) return ok();
  if (!x || !q || !scales) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (rows < 0 || cols < 0 || cols % 16 || cols > 16384 || x_row_stride < cols || x_row_stride % 8)
    return fail(H3B_ERR_UNSUPPORTED, "quantize_int8_rowwise: need cols % 16 == 0, cols <= 16384, stride % 8 == 0");
  if (rows > INT_MAX) return fail(H3B_ERR_UNSUPPORTED, "too many rows");
  if (!aligned16(x) || !aligned16(q)) return fail(H3B_ERR_UNSUPPORTED, "x and q must be 16-byte aligned");
  h3b::QuantArgs a{static_cast<const uint16_t*>(x), x_row_stride, (int)cols, 0, static_cast<int8_t*>(q),
                   static_cast<float*>(scales), nullptr, nullptr, nullptr, nullptr, 0.f};
  return cuda_status(h3b::launch_quant(a, rows, 0, false, st(stream)), "quantize_int8_rowwise");
}

int h3b_quantize_int8_rowwise_convrot(const void* x, int64_t rows, int64_t cols, int64_t x_row_stride, int group_size,
                                      int input_act, void* q, void* scales, void* stream) {
  if (rows == 0 || cols == 0) return ok();
  if (!x || !q || !scales) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (group_size != 256) return fail(H3B_ERR_UNSUPPORTED, "ConvRot group size must be 256");
  if (input_act < 0 || input_act > 2) return fail(H3B_ERR_INVALID_ARGUMENT, "input_act must be 0, 1 or 2");
  const int64_t in_w = input_act == 2 ? 2 * cols : cols;
  if (rows < 0 || cols % 256 || cols > 16384 || x_row_stride < in_w || x_row_stride % 8)
    return fail(H3B_ERR_UNSUPPORTED, "quantize_int8_rowwise_convrot: need cols % 256 == 0, cols <= 16384");
  if (rows > INT_MAX) return fail(H3B_ERR_UNSUPPORTED, "too many rows");
  if (!aligned16(x) || !aligned16(q)) return fail(H3B_ERR_UNSUPPORTED, "x and q must be 16-byte aligned");
  h3b::QuantArgs a{static_cast<const uint16_t*>(x), x_row_stride, (int)cols, input_act, static_cast<int8_t*>(q),
                   static_cast<float*>(scales), nullptr, nullptr, nullptr, nullptr, 0.f};
  return cuda_status(h3b::launch_quant(a, rows, 1, false, st(stream)), "quantize_int8_rowwise_convrot");
}

int h3b_rms_adaln_quantize_int8(const void* x, int64_t rows, int64_t cols, int64_t x_row_stride,
                                const void* norm_weight, const void* scale_table, const void* shift_table,
                                const int32_t* segment_rows, float eps, int convrot_group_size, void* q, void* scales,
                                void* stream) {
  if (rows == 0 || cols == 0) return ok();
  if (!x || !q || !scales || !norm_weight || !scale_table || !shift_table)
    return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (convrot_group_size != 0 && convrot_group_size != 256)
    return fail(H3B_ERR_UNSUPPORTED, "convrot_group_size must be 0 or 256");
  if (rows < 0 || cols % (convrot_group_size ? 256 : 16) || cols > 16384 || x_row_stride < cols || x_row_stride % 8)
    return fail(H3B_ERR_UNSUPPORTED, "rms_adaln_quantize_int8: unsupported width or stride");
  if (!aligned16(x) || !aligned16(q) || !aligned16(norm_weight) || !aligned16(scale_table) || !aligned16(shift_table))
    return fail(H3B_ERR_UNSUPPORTED, "operands must be 16-byte aligned");
  h3b::QuantArgs a{static_cast<const uint16_t*>(x), x_row_stride, (int)cols, 0, static_cast<int8_t*>(q),
                   static_cast<float*>(scales), static_cast<const uint16_t*>(norm_weight),
                   static_cast<const uint16_t*>(scale_table), static_cast<const uint16_t*>(shift_table), segment_rows,
                   eps};
  return cuda_status(h3b::launch_quant(a, rows, convrot_group_size ? 1 : 0, true, st(stream)),
                     "rms_adaln_quantize_int8");
}

static int gemm_common(const void* A, const void* B, int64_t M, int64_t N, int64_t K, h3b::GemmArgs& g, int kind,
                       void* stream, const char* what) {
  if (M == 0 || N == 0) return ok();
  if (!A || !B) return fail(H3B_ERR_INVALID_ARGUMENT, "null operand");
  if (M < 0 || N < 0 || K <= 0 || K % 16 || M > INT_MAX || N > INT_MAX || K > INT_MAX)
    return fail(H3B_ERR_UNSUPPORTED, std::string(what) + ": need K % 16 == 0 and sizes < 2^31");
  if (!aligned16(A) || !aligned16(B)) return fail(H3B_ERR_UNSUPPORTED, "A and B must be 16-byte aligned");
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  cudaError_t e = cudaSuccess;
  const int r = h3b::launch_gemm(A, B, g, kind, st(stream), &e);
  if (r == 1) return fail(H3B_ERR_CUDA, std::string(what) + ": cuTensorMapEncodeTiled failed");
  if (r == 4) return fail(H3B_ERR_UNSUPPORTED, std::string(what) + ": the shape does not run the 2-SM kernel");
  return cuda_status(e, what);
}

int h3b_int8_gemm_dequant(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                          const void* bias, void* D, int64_t M, int64_t N, int64_t K, int64_t out_row_stride,
                          int out_dtype, void* stream) {
  if (out_dtype != 2) return fail(H3B_ERR_UNSUPPORTED, "only bf16 output (dtype code 2) is supported");
  if (!xs || !ws || !D) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (ws_numel != 1 && ws_numel != N) return fail(H3B_ERR_INVALID_ARGUMENT, "ws_numel must be 1 or N");
  if (out_row_stride < N) return fail(H3B_ERR_INVALID_ARGUMENT, "out_row_stride < N");
  h3b::GemmArgs g{};
  g.xs = static_cast<const float*>(xs);
  g.ws = static_cast<const float*>(ws);
  g.ws_scalar = ws_numel == 1;
  g.bias = static_cast<const float*>(bias);
  g.out = static_cast<uint16_t*>(D);
  g.out_stride = out_row_stride;
  return gemm_common(A, B, M, N, K, g, 0, stream, "int8_gemm_dequant");
}

int h3b_int8_gemm_dequant_qk_rope(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                                  const void* bias, void* D, int64_t M, int64_t N, int64_t K,
                                  int64_t out_row_stride, int64_t H, int64_t q_offset, int64_t k_offset,
                                  const void* q_weight, const void* k_weight, const void* cos_table,
                                  const void* sin_table, int rot_dim, float eps, void* stream) {
  if (!xs || !ws || !D || !q_weight || !k_weight || !cos_table || !sin_table)
    return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (ws_numel != 1 && ws_numel != N) return fail(H3B_ERR_INVALID_ARGUMENT, "ws_numel must be 1 or N");
  if (out_row_stride < N || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "out_row_stride < N or H <= 0");
  const int64_t W = H * 128;
  if (rot_dim != 96 && rot_dim != 128)
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_dequant_qk_rope: rot_dim must be 96 or 128");
  if (q_offset < 0 || k_offset < 0 || q_offset % 128 || k_offset % 128 || q_offset + W > N || k_offset + W > N ||
      (q_offset < k_offset + W && k_offset < q_offset + W))
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_dequant_qk_rope: head ranges must be disjoint, inside N, at "
                                     "multiples of 128");
  if (!aligned16(D) || out_row_stride % 8 || !aligned16(q_weight) || !aligned16(k_weight) ||
      !aligned16(cos_table) || !aligned16(sin_table))
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_dequant_qk_rope: unaligned operands");
  if (M > 0 && N > 0 && !h3b::gemm_uses_pair_kernel(M, N))
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_dequant_qk_rope: the shape does not run the 2-SM kernel");
  h3b::GemmArgs g{};
  g.xs = static_cast<const float*>(xs);
  g.ws = static_cast<const float*>(ws);
  g.ws_scalar = ws_numel == 1;
  g.bias = static_cast<const float*>(bias);
  g.out = static_cast<uint16_t*>(D);
  g.out_stride = out_row_stride;
  g.q_off = q_offset;
  g.k_off = k_offset;
  g.qk_width = W;
  g.q_norm = static_cast<const uint16_t*>(q_weight);
  g.k_norm = static_cast<const uint16_t*>(k_weight);
  g.cos_t = static_cast<const uint16_t*>(cos_table);
  g.sin_t = static_cast<const uint16_t*>(sin_table);
  g.qk_eps = eps;
  return gemm_common(A, B, M, N, K, g, rot_dim == 128 ? h3b::kEpiQkRope64 : h3b::kEpiQkRope48, stream,
                     "int8_gemm_dequant_qk_rope");
}

int h3b_int8_gemm_gelu_convrot(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                               const void* bias, void* D, int64_t M, int64_t N, int64_t K, int64_t out_row_stride,
                               void* amax, int64_t amax_row_stride, void* stream) {
  if (!xs || !ws || !D || !amax) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (ws_numel != 1 && ws_numel != N) return fail(H3B_ERR_INVALID_ARGUMENT, "ws_numel must be 1 or N");
  if (out_row_stride < N || amax_row_stride < N / 128)
    return fail(H3B_ERR_INVALID_ARGUMENT, "out_row_stride < N or amax_row_stride < N / 128");
  if (N % 256 || N > 16384)
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_gelu_convrot: need N % 256 == 0 and N <= 16384");
  if (!aligned16(D) || out_row_stride % 8 || !aligned16(ws) || (bias && !aligned16(bias)))
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_gelu_convrot: D, ws and bias must be 16-byte aligned, "
                                     "out_row_stride % 8 == 0");
  if (M > 0 && N > 0 && !h3b::gemm_uses_pair_kernel(M, N))
    return fail(H3B_ERR_UNSUPPORTED, "int8_gemm_gelu_convrot: the shape does not run the 2-SM kernel");
  h3b::GemmArgs g{};
  g.xs = static_cast<const float*>(xs);
  g.ws = static_cast<const float*>(ws);
  g.ws_scalar = ws_numel == 1;
  g.bias = static_cast<const float*>(bias);
  g.out = static_cast<uint16_t*>(D);
  g.out_stride = out_row_stride;
  g.amax = static_cast<float*>(amax);
  g.amax_stride = amax_row_stride;
  return gemm_common(A, B, M, N, K, g, h3b::kEpiGeluRot, stream, "int8_gemm_gelu_convrot");
}

int h3b_quantize_rotated_int8(const void* rot, int64_t rows, int64_t cols, int64_t rot_row_stride, const void* amax,
                              int64_t amax_row_stride, int64_t amax_cols, void* q, void* scales, void* stream) {
  if (rows == 0 || cols == 0) return ok();
  if (!rot || !amax || !q || !scales) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (rows < 0 || cols < 0 || amax_cols <= 0 || amax_row_stride < amax_cols || rot_row_stride < cols)
    return fail(H3B_ERR_INVALID_ARGUMENT, "quantize_rotated_int8: bad sizes or strides");
  if (cols % 8 || cols > 16384 || rot_row_stride % 8 || amax_cols > INT_MAX)
    return fail(H3B_ERR_UNSUPPORTED, "quantize_rotated_int8: need cols % 8 == 0, cols <= 16384, stride % 8 == 0");
  if (!aligned16(rot) || !aligned16(q)) return fail(H3B_ERR_UNSUPPORTED, "rot and q must be 16-byte aligned");
  return cuda_status(h3b::launch_quant_rotated(static_cast<const uint16_t*>(rot), rot_row_stride,
                                               static_cast<const float*>(amax), amax_row_stride, (int)amax_cols,
                                               (int)cols, rows, static_cast<int8_t*>(q), static_cast<float*>(scales),
                                               st(stream)),
                     "quantize_rotated_int8");
}

int h3b_int8_gemm_gated_residual(const void* A, const void* B, const void* xs, const void* ws, int64_t ws_numel,
                                 const void* bias, const void* gate, void* residual, int64_t M, int64_t N, int64_t K,
                                 int64_t residual_row_stride, void* stream) {
  if (!xs || !ws || !gate || !residual) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (ws_numel != 1 && ws_numel != N) return fail(H3B_ERR_INVALID_ARGUMENT, "ws_numel must be 1 or N");
  if (residual_row_stride < N) return fail(H3B_ERR_INVALID_ARGUMENT, "residual_row_stride < N");
  if (!aligned16(gate)) return fail(H3B_ERR_UNSUPPORTED, "gate must be 16-byte aligned");
  h3b::GemmArgs g{};
  g.xs = static_cast<const float*>(xs);
  g.ws = static_cast<const float*>(ws);
  g.ws_scalar = ws_numel == 1;
  g.bias = static_cast<const float*>(bias);
  g.out = static_cast<uint16_t*>(residual);
  g.out_stride = residual_row_stride;
  g.gate = static_cast<const uint16_t*>(gate);
  return gemm_common(A, B, M, N, K, g, 1, stream, "int8_gemm_gated_residual");
}

int h3b_int8_gemm_i32(const void* A, const void* B, void* acc, int64_t M, int64_t N, int64_t K, void* stream) {
  if (!acc) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  h3b::GemmArgs g{};
  g.out_i32 = static_cast<int32_t*>(acc);
  g.out_stride = N;
  return gemm_common(A, B, M, N, K, g, 2, stream, "int8_gemm_i32");
}

int h3b_dequant_int4_grouped_to_int8(const void* qweight, const void* s_rel, int s_rel_kind, const void* codebook,
                                     void* out, int64_t N, int64_t K, int64_t G, void* stream) {
  if (N == 0 || K == 0) return ok();
  if (!qweight || !s_rel || !out) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (s_rel_kind != 0 && s_rel_kind != 1) return fail(H3B_ERR_INVALID_ARGUMENT, "s_rel_kind must be 0 or 1");
  if (N < 0 || K % 32 || G < 4 || K % G || (16 % G != 0 && G % 16 != 0) || K > INT_MAX)
    return fail(H3B_ERR_UNSUPPORTED, "w4 decode: need K % 32 == 0, G in {4, 8, 16, 16k} dividing K");
  if (!aligned16(qweight) || !aligned16(out)) return fail(H3B_ERR_UNSUPPORTED, "qweight and out must be aligned");
  return cuda_status(h3b::launch_w4_decode(qweight, s_rel, s_rel_kind, codebook, out, N, K, G, st(stream)),
                     "dequant_int4_grouped_to_int8");
}

int h3b_w4a8_group_sums(const void* xq, const void* xs, int64_t M, int64_t K, int64_t G, void* sx,
                        int64_t sx_row_stride, void* stream) {
  if (M == 0) return ok();
  if (!xq || !xs || !sx) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (M < 0 || K <= 0 || G <= 0 || K % G) return fail(H3B_ERR_INVALID_ARGUMENT, "K must be a positive multiple of G");
  if (sx_row_stride < K / G) return fail(H3B_ERR_INVALID_ARGUMENT, "sx_row_stride < K/G");
  if (K > INT_MAX || M * sx_row_stride > (int64_t)INT_MAX * 256)
    return fail(H3B_ERR_UNSUPPORTED, "w4a8_group_sums: sizes too large");
  return cuda_status(h3b::launch_group_sums(static_cast<const int8_t*>(xq), static_cast<const float*>(xs), M, K, G,
                                            static_cast<uint16_t*>(sx), sx_row_stride, st(stream)),
                     "w4a8_group_sums");
}

int h3b_adaln_projection(const void* w, const void* t, const void* b, int64_t rows, int64_t N, int64_t K,
                         void* out, void* stream) {
  if (N == 0) return ok();
  if (!w || !t || !out) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (rows < 1 || rows > 8) return fail(H3B_ERR_UNSUPPORTED, "adaln_projection: 1..8 rows of t");
  if (N < 0 || K <= 0 || K % 8) return fail(H3B_ERR_INVALID_ARGUMENT, "adaln_projection: K must be a positive multiple of 8");
  if (!aligned16(w) || !aligned16(t)) return fail(H3B_ERR_UNSUPPORTED, "w and t must be 16-byte aligned");
  if (N > (int64_t)INT_MAX * 8) return fail(H3B_ERR_UNSUPPORTED, "adaln_projection: N too large");
  return cuda_status(h3b::launch_adaln_projection(static_cast<const uint16_t*>(w), static_cast<const uint16_t*>(t),
                                                  static_cast<const uint16_t*>(b), rows, N, K,
                                                  static_cast<uint16_t*>(out), st(stream)),
                     "adaln_projection");
}

int h3b_bf16_gemm_accumulate(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                             int64_t out_row_stride, void* stream) {
  if (M == 0 || N == 0) return ok();
  if (!A || !B || !D) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (M < 0 || N < 0 || K <= 0 || K % 8 || M > INT_MAX || N > INT_MAX || K > INT_MAX / 2)
    return fail(H3B_ERR_UNSUPPORTED, "bf16_gemm_accumulate: need K % 8 == 0 and sizes < 2^31");
  if (out_row_stride < N || out_row_stride % 2) return fail(H3B_ERR_INVALID_ARGUMENT, "bad out_row_stride");
  if (!aligned16(A) || !aligned16(B) || (reinterpret_cast<uintptr_t>(D) & 3u))
    return fail(H3B_ERR_UNSUPPORTED, "A, B must be 16-byte and D 4-byte aligned");
  h3b::GemmArgs g{};
  g.out = static_cast<uint16_t*>(D);
  g.out_stride = out_row_stride;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)(2 * K);  // bytes: the kernel walks K in 128-byte steps
  cudaError_t e = cudaSuccess;
  const int r = h3b::launch_gemm(A, B, g, h3b::kEpiAddF32, st(stream), &e);
  if (r == 1) return fail(H3B_ERR_CUDA, "bf16_gemm_accumulate: cuTensorMapEncodeTiled failed");
  return cuda_status(e, "bf16_gemm_accumulate");
}

int64_t h3b_key_mean_workspace_bytes(int64_t L, int64_t H) { return h3b::key_mean_workspace(L, H); }

int h3b_key_mean(const void* k, int64_t L, int64_t H, int64_t k_row_stride, void* mean, void* workspace,
                 int64_t workspace_bytes, void* stream) {
  if (L <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "L and H must be positive");
  if (!k || !mean || !workspace) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (workspace_bytes < h3b::key_mean_workspace(L, H)) return fail(H3B_ERR_INVALID_ARGUMENT, "workspace too small");
  if (k_row_stride < H * 128) return fail(H3B_ERR_INVALID_ARGUMENT, "k_row_stride < H*128");
  return cuda_status(h3b::launch_key_mean(k, L, H, k_row_stride, mean, workspace, st(stream)), "key_mean");
}

int h3b_key_mean_no_alloc(const void* k, int64_t L, int64_t H, int64_t k_row_stride, void* mean, void* stream) {
  if (L <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "L and H must be positive");
  if (!k || !mean) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (k_row_stride < H * 128) return fail(H3B_ERR_INVALID_ARGUMENT, "k_row_stride < H*128");
  const int64_t need = h3b::key_mean_workspace(L, H) / (int64_t)sizeof(double);
  if (need > h3b::key_mean_static_capacity())
    return fail(H3B_ERR_UNSUPPORTED, "key_mean_no_alloc: ceil(L/1024)*H*128 = " + std::to_string(need) +
                                         " partial sums exceed the fixed scratch of " +
                                         std::to_string(h3b::key_mean_static_capacity()) +
                                         "; use h3b_key_mean with a caller workspace");
  return cuda_status(h3b::launch_key_mean_static(k, L, H, k_row_stride, mean, st(stream)), "key_mean_no_alloc");
}

int h3b_pool_sim_quant(const void* x, int64_t L, int64_t H, int64_t x_row_stride, const void* mean, int block,
                       const void* thr, void* pooled, void* similar, void* qi8, void* scale, int64_t Lpad,
                       void* stream) {
  if (L <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "L and H must be positive");
  if (!x || !thr || !pooled || !similar || !qi8 || !scale) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (block != 32 && block != 64 && block != 128) return fail(H3B_ERR_UNSUPPORTED, "block must be 32, 64 or 128");
  const int64_t nb = (L + block - 1) / block;
  if (Lpad < nb * block) return fail(H3B_ERR_INVALID_ARGUMENT, "Lpad < ceil(L/block)*block");
  if (x_row_stride < H * 128 || x_row_stride % 4) return fail(H3B_ERR_INVALID_ARGUMENT, "bad x_row_stride");
  if (nb > INT_MAX || H > 65535) return fail(H3B_ERR_UNSUPPORTED, "too many blocks or heads");
  h3b::PoolArgs a{static_cast<const uint16_t*>(x), L, x_row_stride, Lpad, (int)H, block,
                  static_cast<const uint16_t*>(mean), static_cast<const float*>(thr), static_cast<uint16_t*>(pooled),
                  static_cast<uint8_t*>(similar), static_cast<int8_t*>(qi8), static_cast<float*>(scale), 0};
  return cuda_status(h3b::launch_pool_sim_quant(a, st(stream)), "pool_sim_quant");
}

int h3b_pool_sim_quant_slab(const void* x, int64_t rows, int64_t H, int64_t x_row_stride, const void* mean, int block,
                            const void* thr, void* pooled, void* similar, void* qi8, void* scale,
                            int64_t blocks_per_head, int64_t Lpad, void* stream) {
  if (rows <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "rows and H must be positive");
  if (!x || !thr || !pooled || !similar || !qi8 || !scale) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (block != 64 && block != 128) return fail(H3B_ERR_UNSUPPORTED, "block must be 64 or 128");
  const int64_t nb = (rows + block - 1) / block;
  if (blocks_per_head < nb) return fail(H3B_ERR_INVALID_ARGUMENT, "blocks_per_head < ceil(rows/block)");
  if (Lpad < nb * block) return fail(H3B_ERR_INVALID_ARGUMENT, "Lpad < ceil(rows/block)*block");
  if (x_row_stride < H * 128 || x_row_stride % 4) return fail(H3B_ERR_INVALID_ARGUMENT, "bad x_row_stride");
  if (nb > INT_MAX || H > 65535) return fail(H3B_ERR_UNSUPPORTED, "too many blocks or heads");
  h3b::PoolArgs a{static_cast<const uint16_t*>(x), rows, x_row_stride, Lpad, (int)H, block,
                  static_cast<const uint16_t*>(mean), static_cast<const float*>(thr), static_cast<uint16_t*>(pooled),
                  static_cast<uint8_t*>(similar), static_cast<int8_t*>(qi8), static_cast<float*>(scale),
                  blocks_per_head};
  return cuda_status(h3b::launch_pool_sim_quant(a, st(stream)), "pool_sim_quant_slab");
}

int h3b_quantize_per_thread_int8(const void* x, int64_t L, int64_t H, int64_t x_row_stride, const void* mean,
                                 int kind, void* qi8, void* scale, int64_t Lpad, void* stream) {
  if (L <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "L and H must be positive");
  if (!x || !qi8 || !scale) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (kind != 0 && kind != 1) return fail(H3B_ERR_INVALID_ARGUMENT, "kind must be 0 (Q) or 1 (K)");
  const int blk = kind == 0 ? 128 : 64, ng = kind == 0 ? 32 : 4;
  const int64_t nb = (L + blk - 1) / blk;
  if (Lpad < nb * blk) return fail(H3B_ERR_INVALID_ARGUMENT, "Lpad < ceil(L/block)*block");
  if (x_row_stride < H * 128 || x_row_stride % 4) return fail(H3B_ERR_INVALID_ARGUMENT, "bad x_row_stride");
  if (nb > INT_MAX || H > 65535) return fail(H3B_ERR_UNSUPPORTED, "too many blocks or heads");
  h3b::PoolArgs a{static_cast<const uint16_t*>(x), L, x_row_stride, Lpad, (int)H, blk,
                  static_cast<const uint16_t*>(mean), nullptr, nullptr, nullptr, static_cast<int8_t*>(qi8),
                  static_cast<float*>(scale), nb * ng};
  return cuda_status(h3b::launch_quant_per_thread(a, kind, st(stream)), "quantize_per_thread_int8");
}

int h3b_qk_rmsnorm_rope(void* qkv, int64_t L, int64_t H, int64_t row_stride, int64_t q_offset, int64_t k_offset,
                        const void* q_weight, const void* k_weight, const void* cos_table, const void* sin_table,
                        int rot_dim, float eps, void* stream) {
  if (L == 0) return ok();
  if (!qkv || !q_weight || !k_weight || !cos_table || !sin_table) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (L < 0 || H <= 0 || rot_dim < 8 || rot_dim > 128 || rot_dim % 8)
    return fail(H3B_ERR_UNSUPPORTED, "qk_rmsnorm_rope: rot_dim must be a multiple of 8 in [8, 128]");
  if (row_stride % 4 || q_offset % 4 || k_offset % 4 || q_offset + H * 128 > row_stride ||
      k_offset + H * 128 > row_stride)
    return fail(H3B_ERR_INVALID_ARGUMENT, "qk_rmsnorm_rope: bad offsets or stride");
  h3b::QkRopeArgs a{static_cast<uint16_t*>(qkv), L, row_stride, q_offset, k_offset, (int)H, rot_dim,
                    static_cast<const uint16_t*>(q_weight), static_cast<const uint16_t*>(k_weight),
                    static_cast<const uint16_t*>(cos_table), static_cast<const uint16_t*>(sin_table), eps};
  return cuda_status(h3b::launch_qk_rmsnorm_rope(a, st(stream)), "qk_rmsnorm_rope");
}

int h3b_value_fp8(const void* v, int64_t L, int64_t H, int64_t v_row_stride, int64_t Lpad, void* vt, void* vscale,
                  void* stream) {
  if (L <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "L and H must be positive");
  if (!v || !vt || !vscale) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (Lpad < L || Lpad % 128) return fail(H3B_ERR_INVALID_ARGUMENT, "Lpad must be >= L and a multiple of 128");
  if (v_row_stride < H * 128 || v_row_stride % 8) return fail(H3B_ERR_INVALID_ARGUMENT, "bad v_row_stride");
  if (!aligned16(v) || !aligned16(vt)) return fail(H3B_ERR_UNSUPPORTED, "v and vt must be 16-byte aligned");
  return cuda_status(h3b::launch_value_fp8(v, L, H, v_row_stride, Lpad, vt, vscale, st(stream)), "value_fp8");
}

int h3b_value_fp8_given_absmax(const void* v, int64_t rows, int64_t H, int64_t v_row_stride, const void* absmax,
                               void* vt, int64_t vt_row_pitch, void* vscale, void* stream) {
  if (rows <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "rows and H must be positive");
  if (!v || !absmax || !vt) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (vt_row_pitch < (rows + 127) / 128 * 128 || vt_row_pitch % 16)
    return fail(H3B_ERR_INVALID_ARGUMENT, "vt_row_pitch must cover ceil(rows/128)*128 tokens, a multiple of 16");
  if (v_row_stride < H * 128 || v_row_stride % 8) return fail(H3B_ERR_INVALID_ARGUMENT, "bad v_row_stride");
  if (!aligned16(v) || !aligned16(vt)) return fail(H3B_ERR_UNSUPPORTED, "v and vt must be 16-byte aligned");
  return cuda_status(h3b::launch_value_fp8_given_absmax(v, rows, H, v_row_stride, vt_row_pitch,
                                                        static_cast<const float*>(absmax), vt,
                                                        static_cast<float*>(vscale), st(stream)),
                     "value_fp8_given_absmax");
}

static int check_heads_args(int64_t rows, int64_t H, int64_t P, const void* a, const void* b) {
  if (!a || !b) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (rows < 0 || H <= 0 || P <= 0 || H % P) return fail(H3B_ERR_INVALID_ARGUMENT, "H must be a multiple of P");
  if (!aligned16(a) || !aligned16(b)) return fail(H3B_ERR_UNSUPPORTED, "buffers must be 16-byte aligned");
  if (rows * H * 16 > (int64_t)INT_MAX * 256) return fail(H3B_ERR_UNSUPPORTED, "too many rows");
  return H3B_OK;
}

int h3b_ulysses_pack(const void* src, int64_t rows, int64_t H, int64_t src_row_stride, const int64_t* head_order,
                     int64_t P, void* dst, void* stream) {
  if (rows == 0) return ok();
  const int r = check_heads_args(rows, H, P, src, dst);
  if (r != H3B_OK) return r;
  if (src_row_stride < H * 128 || src_row_stride % 8) return fail(H3B_ERR_INVALID_ARGUMENT, "bad src_row_stride");
  return cuda_status(h3b::launch_gather_heads(src, rows, H, src_row_stride, head_order, P, dst, st(stream)),
                     "ulysses_pack");
}

int h3b_ulysses_unpack(const void* src, int64_t rows, int64_t H, const int64_t* head_order, int64_t P, void* dst,
                       int64_t dst_row_stride, void* stream) {
  if (rows == 0) return ok();
  const int r = check_heads_args(rows, H, P, src, dst);
  if (r != H3B_OK) return r;
  if (dst_row_stride < H * 128 || dst_row_stride % 8) return fail(H3B_ERR_INVALID_ARGUMENT, "bad dst_row_stride");
  return cuda_status(h3b::launch_scatter_heads(src, rows, H, head_order, P, dst, dst_row_stride, st(stream)),
                     "ulysses_unpack");
}

int h3b_block_mask(const void* pooled_q, const void* similar_q, int64_t Qb, const void* pooled_k,
                   const void* similar_k, int64_t Kb, int64_t H, const h3b_mask_params* p, void* bitmap,
                   void* stream) {
  if (Qb <= 0 || Kb <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "Qb, Kb and H must be positive");
  if (!pooled_q || !similar_q || !pooled_k || !similar_k || !p || !bitmap || !p->budget)
    return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (Kb > 16384) return fail(H3B_ERR_UNSUPPORTED, "at most 16384 key blocks");
  if (p->mode != 0 && p->mode != 1) return fail(H3B_ERR_INVALID_ARGUMENT, "mode must be 0 or 1");
  h3b::MaskArgs a{static_cast<const uint16_t*>(pooled_q), static_cast<const uint8_t*>(similar_q),
                  static_cast<const uint16_t*>(pooled_k), static_cast<const uint8_t*>(similar_k), Qb, Kb, p->mode,
                  p->budget, p->protected_key_blocks, p->keep_first_column, p->keep_diagonal, p->temporal_radius,
                  p->temporal_spatial_radius, p->frames, p->frame_tokens, p->protected_tokens, p->query_tokens,
                  static_cast<uint32_t*>(bitmap), p->query_indices, p->protected_query_blocks};
  if (p->temporal_radius >= 0 && p->frame_tokens > 0 && p->query_tokens < 1)
    return fail(H3B_ERR_INVALID_ARGUMENT, "the temporal rail needs query_tokens >= 1");
  if (p->protected_query_blocks < 0 || p->protected_key_blocks < 0)
    return fail(H3B_ERR_INVALID_ARGUMENT, "protected block counts must be non-negative");
  return cuda_status(h3b::launch_block_mask(a, H, st(stream)), "block_mask");
}

int h3b_bitmap_to_lut(const void* bitmap, int64_t rows, int64_t Kb, void* lut, void* valid, void* stream) {
  if (rows == 0) return ok();
  if (!bitmap || !lut || !valid) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (rows < 0 || Kb <= 0 || Kb > INT_MAX) return fail(H3B_ERR_INVALID_ARGUMENT, "bad sizes");
  return cuda_status(h3b::launch_bitmap_to_lut(bitmap, rows, Kb, lut, valid, st(stream)), "bitmap_to_lut");
}

int h3b_attention(const void* q, const void* q_scale, int q_gran, int q_block, int64_t Lq, int64_t Lqpad,
                  const void* k, const void* k_scale, int k_gran, int64_t Lk, int64_t Lkpad, const void* vt,
                  const void* v_scale, int64_t H, const void* bitmap, float sm_scale, void* out,
                  int64_t out_row_stride, void* stream) {
  if (Lq == 0) return ok();
  if (!q || !q_scale || !k || !k_scale || !vt || !v_scale || !out) return fail(H3B_ERR_INVALID_ARGUMENT, "null pointer");
  if (Lq < 0 || Lk <= 0 || H <= 0) return fail(H3B_ERR_INVALID_ARGUMENT, "bad sizes");
  if (q_gran != 0 && q_gran != 1) return fail(H3B_ERR_INVALID_ARGUMENT, "q_gran must be 0 or 1");
  if (k_gran != 0 && k_gran != 1) return fail(H3B_ERR_INVALID_ARGUMENT, "k_gran must be 0 or 1");
  if (q_gran == 1) q_block = 128;
  if (q_block != 32 && q_block != 64 && q_block != 128)
    return fail(H3B_ERR_UNSUPPORTED, "q_block must be 32, 64 or 128");
  if (k_gran == 1 && (reinterpret_cast<uintptr_t>(k_scale) & 15u))
    return fail(H3B_ERR_UNSUPPORTED, "per_thread k_scale must be 16-byte aligned");
  if (Lqpad % 128 || Lqpad < Lq || Lkpad % 128 || Lkpad < Lk)
    return fail(H3B_ERR_INVALID_ARGUMENT, "Lqpad / Lkpad must be multiples of 128 covering Lq / Lk");
  if (out_row_stride < H * 128 || out_row_stride % 8) return fail(H3B_ERR_INVALID_ARGUMENT, "bad out_row_stride");
  if (H * Lqpad > INT_MAX || H * Lkpad > INT_MAX || (Lq + 127) / 128 > INT_MAX || H > 65535)
    return fail(H3B_ERR_UNSUPPORTED, "sizes exceed 32-bit TMA coordinates");
  if (!aligned16(q) || !aligned16(k) || !aligned16(vt) || !aligned16(out))
    return fail(H3B_ERR_UNSUPPORTED, "q, k, vt and out must be 16-byte aligned");
  h3b::AttnArgs a{};
  a.H = (int)H;
  a.Lq = Lq;
  a.Lqpad = Lqpad;
  a.Lk = Lk;
  a.Lkpad = Lkpad;
  a.Kb = (int)((Lk + 63) / 64);
  a.words = (a.Kb + 31) / 32;
  a.q_block = q_block;
  a.q_gran = q_gran;
  a.k_gran = k_gran;
  a.nqs = q_gran ? (int)((Lq + 127) / 128 * 32) : (int)((Lq + q_block - 1) / q_block);
  a.q_scale = static_cast<const float*>(q_scale);
  a.k_scale = static_cast<const float*>(k_scale);
  a.v_scale = static_cast<const float*>(v_scale);
  a.bitmap = static_cast<const uint32_t*>(bitmap);
  a.scale_log2 = sm_scale * 1.4426950408889634f;
  a.out = static_cast<uint16_t*>(out);
  a.out_stride = out_row_stride;
  cudaError_t e = cudaSuccess;
  const int r = h3b::launch_attention(q, k, vt, a, st(stream), &e);
  if (r == 1) return fail(H3B_ERR_CUDA, "attention: cuTensorMapEncodeTiled failed");
  if (r == 3) return fail(H3B_ERR_UNSUPPORTED, "attention: kernel register count differs from the planned split");
  return cuda_status(e, "attention");
}

}  // extern "C"
