// attn_mask.cu -- Sparge block-sparse mask: pooled scores, softmax, block
// selection, mandatory rails, and the conversion to the reference LUT ABI.
//
// Selector of SplitModalityProtectedSpargeAttentionBackend.long_sequence_video_queries
// (model/kernels.py:3668-3941): scores = bf16(pooled_q . pooled_k) * 128^-0.5,
// non-similar K blocks -> -inf, softmax, keep the `count` most probable K blocks
// (fixed Top-K, kernels.py:3206-3253) or the top-CDF prefix (SpargeAttn rule),
// then keep every non-similar K column and Q row, the protected prefix (key
// columns, and optionally whole query rows), and the optional first-column /
// diagonal / temporal-correspondence rails (kernels.py:5206-5294; for a chunk of
// selected video queries the rail takes each query block's centre from the
// chunk's token indices, kernels.py:5247-5254).
//
// Per CTA: one head, up to 8 query blocks (one warp each).  All threads first
// compute the 8 x Kb score matrix into shared memory (each thread one K block,
// reading its pooled vector once for all 8 rows); then each warp turns its row
// into probabilities and selects by a two-level radix select on the 16-bit
// bf16 probability keys (ties broken toward the lower block index), writing
// the row's bitmap words directly.  Output: uint32 bitmap [H, Qb, ceil(Kb/32)].
#include "h3b_kernels.cuh"

namespace h3b {

// Query-block rows per CTA: 8, or 4 above 8192 key blocks (the rows' bf16
// scores are staged in shared memory: rows x Kb x 2 bytes).
constexpr int kMaskMaxKb = 16384;
constexpr int kMaskThreads = 256;


__device__ __forceinline__ uint64_t fixed56(float p) {
  return __float2ull_rz(__fmul_rn(p, 72057594037927936.0f));
}

// Bins are scanned from the top (bin 255) down by the whole warp: lane l holds
// bins 255 - 8l .. 248 - 8l.  The lanes' totals are prefix-summed across the warp
// (lane 0 = top); the first lane whose running total crosses the bound then walks
// its own 8 bins in order, which gives exactly what one thread walking all 256 bins
// from the top would find.

// First bin b (from the top) at which count(bins above b) + hist[b] >= need;
// returns b and count(bins above b) in *above.  need <= the histogram's total.
__device__ __forceinline__ int warp_find_count(const uint32_t* hist, uint32_t base, uint32_t need, int lane,
                                               uint32_t* above) {
  const int hi = 255 - 8 * lane;
  uint32_t h[8], tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[i] = hist[hi - i];
    tot += h[i];
  }
  uint32_t pre = tot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, pre, off);
    if (lane >= off) pre += v;
  }
  const unsigned hit = __ballot_sync(0xffffffffu, base + pre >= need);
  const int L = hit ? __ffs(hit) - 1 : 31;
  int b = 0;
  uint32_t cum = base + pre - tot;
  if (lane == L) {
    b = hi - 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (cum + h[i] >= need) { b = hi - i; break; }
      cum += h[i];
    }
  }
  b = __shfl_sync(0xffffffffu, b, L);
  *above = __shfl_sync(0xffffffffu, cum, L);
  return b;
}

// First-level count + mass histogram update for one warp step (one key per lane;
// lanes past the end pass valid = false).  The probabilities of a row mostly share
// a few high bytes, so per-key 64-bit atomics would collide 32 ways.  Instead each
// distinct bin of the step is added once: the lowest pending lane's bin, its lanes
// by ballot, the count by popc and the lanes' fixed-point masses (each < 2^57) as
// three exact 24 / 24 / 9-bit warp sums.  Integer sums, so the totals equal the
// per-key atomics' in any order.  (The count-only histogram of select_threshold
// keeps per-key 32-bit atomics: measured faster there.)
template <bool MASS>
__device__ __forceinline__ void hist_add_by_bin(uint32_t* hist, unsigned long long* mass, int bin, bool valid,
                                                uint64_t m, int lane) {
  uint32_t pending = __ballot_sync(0xffffffffu, valid);
  while (pending) {
    const int leader = __ffs(pending) - 1;
    const int lb = __shfl_sync(0xffffffffu, bin, leader);
    const bool mine = valid && bin == lb;
    const uint32_t peers = __ballot_sync(0xffffffffu, mine);
    if constexpr (MASS) {
      const uint32_t lo = __reduce_add_sync(0xffffffffu, mine ? (uint32_t)(m & 0xffffffu) : 0u);
      const uint32_t mid = __reduce_add_sync(0xffffffffu, mine ? (uint32_t)((m >> 24) & 0xffffffu) : 0u);
      const uint32_t hi = __reduce_add_sync(0xffffffffu, mine ? (uint32_t)(m >> 48) : 0u);
      if (lane == leader)
        atomicAdd(&mass[lb], (unsigned long long)lo + ((unsigned long long)mid << 24) + ((unsigned long long)hi << 48));
    }
    if (lane == leader) atomicAdd(&hist[lb], (uint32_t)__popc(peers));
    pending &= ~peers;
  }
}

// Threshold key T and how many of the keys equal to T to keep, so that exactly
// `need` keys are kept (keys > T all kept).  hist: per-warp shared counters.
__device__ void select_threshold(const uint16_t* keys, int Kb, int need, uint32_t* hist, int lane, int* T_out,
                                 int* take_eq) {
  // level 1: high byte
  for (int i = lane; i < 256; i += 32) hist[i] = 0;
  __syncwarp();
  for (int j = lane; j < Kb; j += 32) atomicAdd(&hist[keys[j] >> 8], 1u);
  __syncwarp();
  uint32_t above = 0;
  const int b1 = warp_find_count(hist, 0u, (uint32_t)need, lane, &above);
  __syncwarp();
  // level 2: low byte among keys with high byte b1
  for (int i = lane; i < 256; i += 32) hist[i] = 0;
  __syncwarp();
  for (int j = lane; j < Kb; j += 32)
    if ((keys[j] >> 8) == b1) atomicAdd(&hist[keys[j] & 0xff], 1u);
  __syncwarp();
  uint32_t above2 = 0;
  const int b2 = warp_find_count(hist, above, (uint32_t)need, lane, &above2);
  __syncwarp();
  *T_out = (b1 << 8) | b2;
  *take_eq = need - (int)above2;
}

// Walk the bins from the top while the running mass stays <= thr: returns the
// first bin where it would exceed thr (-1: none), with the mass and count of the
// bins above it in *cm, *count (base_* added).
__device__ __forceinline__ int warp_find_mass(const uint32_t* hist, const unsigned long long* mass,
                                              unsigned long long base_m, int base_c, uint64_t thr, int lane,
                                              unsigned long long* cm_out, int* count_out) {
  const int hi = 255 - 8 * lane;
  unsigned long long mv[8], mtot = 0;
  uint32_t hv[8], ctot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mv[i] = mass[hi - i];
    hv[i] = hist[hi - i];
    mtot += mv[i];
    ctot += hv[i];
  }
  unsigned long long mpre = mtot;
  uint32_t cpre = ctot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const unsigned long long v = __shfl_up_sync(0xffffffffu, mpre, off);
    const uint32_t c = __shfl_up_sync(0xffffffffu, cpre, off);
    if (lane >= off) {
      mpre += v;
      cpre += c;
    }
  }
  const unsigned over = __ballot_sync(0xffffffffu, base_m + mpre > thr);
  if (!over) {
    *cm_out = __shfl_sync(0xffffffffu, base_m + mpre, 31);
    *count_out = base_c + (int)__shfl_sync(0xffffffffu, cpre, 31);
    return -1;
  }
  const int L = __ffs(over) - 1;
  unsigned long long cm = base_m + mpre - mtot;
  int count = base_c + (int)(cpre - ctot);
  int b = hi - 7;
  if (lane == L) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (cm + mv[i] <= thr) {
        cm += mv[i];
        count += (int)hv[i];
      } else {
        b = hi - i;
        break;
      }
    }
  }
  b = __shfl_sync(0xffffffffu, b, L);
  *cm_out = __shfl_sync(0xffffffffu, cm, L);
  *count_out = __shfl_sync(0xffffffffu, count, L);
  return b;
}

// Number of ranks whose cumulative probability (2^-56 fixed point, exact) stays <= thr.
__device__ int cdf_count(const uint16_t* keys, int Kb, uint64_t thr, uint32_t* hist, unsigned long long* mass,
                         int lane) {
  for (int i = lane; i < 256; i += 32) { hist[i] = 0; mass[i] = 0ull; }
  __syncwarp();
  for (int j0 = 0; j0 < Kb; j0 += 32) {
    const int j = j0 + lane;
    const bool valid = j < Kb;
    const uint16_t k = valid ? keys[j] : (uint16_t)0;
    hist_add_by_bin<true>(hist, mass, k >> 8, valid, valid ? fixed56(bf16_bits_to_f32(k)) : 0ull, lane);
  }
  __syncwarp();
  unsigned long long cm = 0;
  int count = 0;
  const int b1 = warp_find_mass(hist, mass, 0ull, 0, thr, lane, &cm, &count);
  __syncwarp();
  if (b1 < 0) return Kb;
  for (int i = lane; i < 256; i += 32) { hist[i] = 0; mass[i] = 0ull; }
  __syncwarp();
  for (int j = lane; j < Kb; j += 32) {
    const uint16_t k = keys[j];
    if ((k >> 8) == b1) {
      atomicAdd(&hist[k & 0xff], 1u);
      atomicAdd(&mass[k & 0xff], (unsigned long long)fixed56(bf16_bits_to_f32(k)));
    }
  }
  __syncwarp();
  unsigned long long cm2 = 0;
  int count2 = 0;
  const int b = warp_find_mass(hist, mass, cm, count, thr, lane, &cm2, &count2);
  if (b >= 0) {
    // the bin where the mass crosses thr: as many of its (equal) keys as still fit
    const uint64_t v = fixed56(bf16_bits_to_f32((uint16_t)((b1 << 8) | b)));
    const uint64_t extra = (thr - cm2) / v;   // v > 0: this bin's mass exceeds thr - cm2 >= 0
    const uint32_t hb = hist[b];
    count2 += (int)(extra < hb ? extra : hb);
  }
  return count2;
}

template <int kMaskRows>
__global__ void __launch_bounds__(kMaskThreads) block_mask_kernel(MaskArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  float* pq_s = reinterpret_cast<float*>(smem);                               // [8][128]
  uint32_t* hist_all = reinterpret_cast<uint32_t*>(pq_s + kMaskRows * 128);   // [8][256]
  unsigned long long* mass_all = reinterpret_cast<unsigned long long*>(hist_all + kMaskRows * 256);  // [8][256]
  uint16_t* xs = reinterpret_cast<uint16_t*>(mass_all + kMaskRows * 256);    // [8][Kb]
  __shared__ int any_sim_s;

  const int h = blockIdx.y;
  const int64_t i0 = (int64_t)blockIdx.x * kMaskRows;
  const int nrows = (int)((a.Qb - i0) < kMaskRows ? (a.Qb - i0) : kMaskRows);
  const int Kb = (int)a.Kb;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint8_t* simk = a.simk + (int64_t)h * Kb;

  if (tid == 0) any_sim_s = 0;
  for (int i = tid; i < kMaskRows * 128; i += kMaskThreads) {
    const int r = i >> 7, d = i & 127;
    pq_s[i] = r < nrows ? bf16_bits_to_f32(a.pq[((int64_t)h * a.Qb + i0 + r) * 128 + d]) : 0.f;
  }
  __syncthreads();
  int local_any = 0;
  const float kScale = 0.08838834764831845f;
  for (int j = tid; j < Kb; j += kMaskThreads) {
    const uint16_t* pkj = a.pk + ((int64_t)h * Kb + j) * 128;
    float acc[kMaskRows];
#pragma unroll
    for (int r = 0; r < kMaskRows; ++r) acc[r] = 0.f;
    for (int d0 = 0; d0 < 128; d0 += 8) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(pkj + d0));
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float kv = __uint_as_float(e & 1 ? (w[e >> 1] & 0xffff0000u) : (w[e >> 1] << 16));
#pragma unroll
        for (int r = 0; r < kMaskRows; ++r) acc[r] = fmaf(pq_s[r * 128 + d0 + e], kv, acc[r]);
      }
    }
    const bool sim = simk[j] != 0;
    local_any |= sim;
#pragma unroll
    for (int r = 0; r < kMaskRows; ++r) {
      const float sc = bf16r(__fmul_rn(bf16r(acc[r]), kScale));
      xs[r * Kb + j] = sim ? f32_to_bf16_bits(sc) : (uint16_t)0xff80u;  // -inf
    }
  }
  if (local_any) atomicOr(&any_sim_s, 1);
  __syncthreads();

  const int words = (Kb + 31) / 32;
  if (warp < nrows) {
    const int64_t qi = i0 + warp;
    uint16_t* x = xs + warp * Kb;
    uint32_t* hist = hist_all + warp * 256;
    unsigned long long* mass = mass_all + warp * 256;
    const bool simq = a.simq[(int64_t)h * a.Qb + qi] != 0;
    uint32_t* out = a.bitmap + ((int64_t)h * a.Qb + qi) * words;
    int T = 0x10000, take_eq = 0;  // nothing selected by default
    if (simq && any_sim_s) {
      float mx = -__int_as_float(0x7f800000);
      for (int j = lane; j < Kb; j += 32) mx = fmaxf(mx, bf16_bits_to_f32(x[j]));
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      float part = 0.f;
      for (int j = lane; j < Kb; j += 32) part = __fadd_rn(part, h3b_expf(__fsub_rn(bf16_bits_to_f32(x[j]), mx)));
      const float sum = warp_butterfly_sum(part);
      for (int j = lane; j < Kb; j += 32)
        x[j] = f32_to_bf16_bits(__fdiv_rn(h3b_expf(__fsub_rn(bf16_bits_to_f32(x[j]), mx)), sum));
      __syncwarp();
      int need;
      if (a.mode == 0) {
        long long c = (long long)__fmul_rn(a.budget[h], (float)Kb);
        need = (int)(c > Kb ? Kb : (c < 0 ? 0 : c));
      } else {
        const uint64_t thr = __float2ull_rz(__fmul_rn(a.budget[h], 72057594037927936.0f));
        need = cdf_count(x, Kb, thr, hist, mass, lane);
      }
      if (need > 0) select_threshold(x, Kb, need, hist, lane, &T, &take_eq);
    }
    // mark: keys > T, the first take_eq keys == T, plus the rails
    int eq_seen = 0;
    const int64_t video = a.frames * a.frame_tokens;
    for (int w = 0; w < words; ++w) {
      const int j = w * 32 + lane;
      bool on = false;
      bool is_eq = false;
      if (j < Kb) {
        const int key = x[j];
        // probabilities are non-negative: bf16 bit patterns order like the values
        on = key > T;
        is_eq = key == T;
        on |= !simk[j] || !simq || j < a.protected_kb || qi < a.protected_qb;
        on |= a.first_col && j == 0;
        on |= a.diag && (j == 2 * qi || j == 2 * qi + 1);
        if (a.temporal_radius >= 0 && a.frame_tokens > 0) {
          int64_t qc = qi * 128 + 64;
          if (qc > a.query_tokens - 1) qc = a.query_tokens - 1;
          // selected queries: the block centre's position in the video
          if (a.q_index) qc = a.q_index[qc];
          const int64_t qf = qc / a.frame_tokens, qs = qc % a.frame_tokens;
          const int64_t kc = (int64_t)j * 64 + 32 - a.protected_tokens;
          const bool valid = kc >= 0 && kc < video;
          const int64_t kcc = kc < 0 ? 0 : (kc > video - 1 ? video - 1 : kc);
          const int64_t kf = kcc / a.frame_tokens, ks = kcc % a.frame_tokens;
          const int64_t dist = 96 + (int64_t)a.temporal_spatial_radius * 64;
          const int64_t df = qf > kf ? qf - kf : kf - qf, ds = qs > ks ? qs - ks : ks - qs;
          on |= valid && df <= a.temporal_radius && ds <= dist;
        }
      }
      const uint32_t eqm = __ballot_sync(0xffffffffu, is_eq);
      const int rank = eq_seen + __popc(eqm & ((1u << lane) - 1u));
      on |= is_eq && rank < take_eq;
      eq_seen += __popc(eqm);
      const uint32_t word = __ballot_sync(0xffffffffu, on);
      if (lane == 0) out[w] = word;
    }
  }
}

// ------------------------------------------------------------------ LUT

__global__ void __launch_bounds__(128) bitmap_to_lut_kernel(const uint32_t* __restrict__ bm, int64_t rows, int Kb,
                                                            int32_t* __restrict__ lut, int32_t* __restrict__ valid) {
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int words = (Kb + 31) / 32;
  const uint32_t* b = bm + row * words;
  int32_t* out = lut + row * Kb;
  int n = 0, prev = 0;
  for (int w = 0; w < words; ++w) {
    const uint32_t word = b[w];
    const bool on = (word >> lane) & 1u;
    const uint32_t below = word & ((1u << lane) - 1u);
    const int pos = n + __popc(below);
    const int j = w * 32 + lane;
    const int pj = below ? w * 32 + 31 - __clz(below) : prev;
    if (on) out[pos] = j - pj;
    n += __popc(word);
    if (word) prev = w * 32 + 31 - __clz(word);
  }
  for (int t = n + lane; t < Kb; t += 32) out[t] = 0;
  if (lane == 0) valid[row] = n;
}

static size_t mask_smem_bytes(int64_t Kb, int rows) {
  return rows * 128 * sizeof(float) + rows * 256 * sizeof(uint32_t) + rows * 256 * sizeof(unsigned long long) +
         rows * (size_t)Kb * sizeof(uint16_t);
}

template <int ROWS>
static cudaError_t launch_block_mask_rows(const MaskArgs& a, int64_t H, cudaStream_t s) {
  const size_t smem = mask_smem_bytes(a.Kb, ROWS);
  cudaError_t e =
      cudaFuncSetAttribute(block_mask_kernel<ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((a.Qb + ROWS - 1) / ROWS), (unsigned)H);
  block_mask_kernel<ROWS><<<grid, kMaskThreads, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_block_mask(const MaskArgs& a, int64_t H, cudaStream_t s) {
  return a.Kb <= 8192 ? launch_block_mask_rows<8>(a, H, s) : launch_block_mask_rows<4>(a, H, s);
}

cudaError_t launch_bitmap_to_lut(const void* bm, int64_t rows, int64_t Kb, void* lut, void* valid, cudaStream_t s) {
  bitmap_to_lut_kernel<<<(unsigned)((rows + 3) / 4), 128, 0, s>>>(static_cast<const uint32_t*>(bm), rows, (int)Kb,
                                                                   static_cast<int32_t*>(lut),
                                                                   static_cast<int32_t*>(valid));
  return cudaGetLastError();
}

}  // namespace h3b
