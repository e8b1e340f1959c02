// attn.cu -- SageAttention-style quantized attention for sm_100a, dense or
// driven by a Sparge block bitmap.
//
//   S = Q_i8 . K_i8^T   tcgen05.mma kind::i8 accumulating onto tensor memory
//       that a bf16 MMA (kind::f16, K = 16, constant operands) has just set to
//       the float 1.5*2^23 (bits 0x4B400000): the accumulator then holds the
//       bits of the float 1.5*2^23 + S (|S| < 2^22), so S needs no integer->
//       float conversion and the block maximum is an integer maximum of the raw
//       bits; the bias is written by the tensor pipe, in order with the S MMAs,
//       instead of by the softmax threads
//   P = exp2(S * qs * ks * scale * log2 e - m) * 112 -> E4M3 (tensor memory,
//       over the S columns the softmax has already read into registers);
//       qs per query row group (q_block rows, or Sage per_thread: rows of equal
//       r % 8 in each 32), ks per 64-key block or per_thread group (keys of equal
//       (j % 8) / 2 in each 64-key block: KG = 4);
//       m is a lazily updated running max: it moves (to the tile max) only when
//       a tile's scores exceed it by more than kTau = 2, so P <= 2^kTau * 112 =
//       448, the E4M3 maximum, and the O rescale in tensor memory is rare.
//       Seven columns in eight take ex2.approx (MUFU), the eighth a polynomial
//       on the FMA pipe (packed fp32 pairs), which balances the two pipes
//       (kPolyMask16 selects the polynomial columns).
//   O += P . V          tcgen05.mma kind::f8f6f4, A = P from tensor memory, B = V^T
//                       from shared memory (E4M3 x E4M3 -> fp32, tensor memory)
//   out = O / l * v_scale[d] -> bf16, l the fp32 row sum of P
//
// One CTA per (two 128-query tiles A and B, head), 384 threads:
//   warp 0      TMA producer (the warp runs the schedule, one elected lane
//               issues the copies): both Q tiles once, then one step per PAIR of
//               selected 64-key blocks (K: 2 x [64 x 128 B], 128-byte swizzle;
//               V^T: 2 x [128 x 64 B], 64-byte swizzle) into a 6-stage ring; no
//               multicast.  The steps interleave the two tiles' own block
//               lists (A, B, A, B, ...); a step whose pair both tiles selected
//               next (every step of dense attention) serves both tiles
//   warp 1      TMEM allocator
//   warps 2, 3  MMA issuers of tiles A and B (warp-wide loop over the step
//               schedule, descriptors in uniform registers, one elected lane
//               issues): at each of its tile's steps, once the previous P is
//               written, PV(previous step), then the bias MMA and S(step); the
//               MMAs of one thread run in issue order, so the PV has read P
//               before the next S overwrites its columns
//               (P needs no shared memory, which leaves room for six K/V stages)
//   warps 4..7  softmax of tile A, warps 8..11 of tile B: one query row per
//               thread (its TMEM lane): S row from TMEM, per-block dequant
//               scales, online max / sum, P row to tensor memory (S columns
//               96..127 of its lane: the A operand of the P.V MMA), O rescaled
//               when the max moves, final normalisation.
// Every SM sub-partition thus runs two independent softmax warps (one per
// tile), and in dense attention each K/V pair is loaded once for 256 queries.
// TMEM: S_A 0..127, S_B 128..255, O_A 256..383, O_B 384..511; P_A and P_B in
// columns 96..127 of S_A and S_B.
#include "h3b_kernels.cuh"

namespace h3b {

constexpr int kAttnThreads = 384;  // three warpgroups
// Register split (setmaxnreg): the launch gives every thread kLaunchRegs (the
// __launch_bounds__ cap for 384 threads); the producer / MMA warpgroup drops to
// kCtrlRegs and each softmax warpgroup rises to kSoftmaxRegs.  The split must
// not exceed the launch total, or the increase would wait forever; the host
// checks the compiled register count against kLaunchRegs before launching.
constexpr int kLaunchRegs = 168;
constexpr int kCtrlRegs = 72;
constexpr int kSoftmaxRegs = 216;
static_assert(128 * (kCtrlRegs + 2 * kSoftmaxRegs) <= kAttnThreads * kLaunchRegs, "register split too large");
constexpr int kTileThreads = 128;
constexpr int kKVStages = 6;
constexpr int kQBytes = 128 * 128;
constexpr int kKVBytes = 32768;  // K pair 16 KB + V^T pair 2 x 8 KB
constexpr int kOffQ = 0;                          // 2 tiles
constexpr int kOffKV = kOffQ + 2 * kQBytes;
constexpr int kOffBar = kOffKV + kKVStages * kKVBytes;
constexpr int kOffBias = kOffBar + 256;          // 8 x 16-byte rows each: A and B of the bias MMA
constexpr int kAttnSmem = kOffBias + 256 + 1024;
constexpr float kLog2_112 = 6.807354922057604f;
constexpr float kTau = 2.0f;
constexpr float kMagicF = 12582912.0f;

// One query tile's selected K blocks, ascending, taken two at a time.
struct TileStream {
  const uint32_t* row;
  int words, w, Kb, dense_next;
  bool dense;
  uint32_t u;
  __device__ void init(const AttnArgs& a, int h, int qt, bool active) {
    Kb = active ? a.Kb : 0;
    dense_next = 0;
    dense = a.bitmap == nullptr || !active;
    u = 0;
    w = 0;
    words = 0;
    if (!dense) {
      const int64_t qb = (a.Lq + 127) / 128;
      row = a.bitmap + ((int64_t)h * qb + qt) * a.words;
      words = a.words;
      u = words > 0 ? row[0] : 0u;
    }
  }
  __device__ int next_block() {
    if (dense) return dense_next < Kb ? dense_next++ : -1;
    while (u == 0) {
      if (++w >= words) return -1;
      u = row[w];
    }
    const int b = __ffs(u) - 1;
    u &= u - 1;
    return w * 32 + b;
  }
  // blocks j0 < j1 (j1 = -1 when the tile selected an odd number of blocks)
  __device__ bool next_pair(int& j0, int& j1) {
    j0 = next_block();
    if (j0 < 0) return false;
    j1 = next_block();
    return true;
  }
};

// The K/V load schedule of a CTA: the two tiles' pair streams interleaved
// (A, B, A, B, ...); when both tiles' next pairs are the same blocks (always so
// for dense attention) one step serves both.  who: bit 0 tile A, bit 1 tile B.
struct StepIter {
  TileStream ta, tb;
  int a0, a1, b0, b1;
  bool pa, pb, turn_b;
  __device__ void init(const AttnArgs& a, int h, int qta, bool has_b) {
    ta.init(a, h, qta, true);
    tb.init(a, h, qta + 1, has_b);
    pa = ta.next_pair(a0, a1);
    pb = tb.next_pair(b0, b1);
    turn_b = false;
  }
  __device__ bool pending(int t) const { return t ? pb : pa; }
  __device__ bool next(int& j0, int& j1, int& who) {
    if (!pa && !pb) return false;
    if (pa && pb && a0 == b0 && a1 == b1)
      who = 3;
    else if (pa && (!pb || !turn_b))
      who = 1;
    else
      who = 2;
    j0 = who == 2 ? b0 : a0;
    j1 = who == 2 ? b1 : a1;
    if (who & 1) pa = ta.next_pair(a0, a1);
    if (who & 2) pb = tb.next_pair(b0, b1);
    if (who != 3) turn_b = who == 1;
    return true;
  }
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// A global load the compiler keeps at this point of the program (it would
// otherwise sink a read-only load to its first use, behind a barrier wait).
__device__ __forceinline__ float ld_early(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
// KG consecutive scales (KG = 1 or 4; 16-byte aligned for 4), loaded early
template <int KG>
__device__ __forceinline__ void ld_early_kg(const float* p, float (&v)[KG]) {
  if constexpr (KG == 1) {
    v[0] = ld_early(p);
  } else {
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]) : "l"(p));
  }
}
// K-major operand without swizzle whose every 8-row group and both 8-element K halves
// read the same 8 x 16-byte core matrix (leading and stride byte offsets 0)
__device__ __forceinline__ uint64_t sdesc_core_repeat(uint32_t smem_addr) {
  return (uint64_t)((smem_addr & 0x3FFFF) >> 4) | ((uint64_t)1 << 46);
}

// ---------------------------------------------------------------- softmax pieces
// All loops are fully unrolled over compile-time column ranges (NC = 64: one
// key block, 128: a pair), so the per-column work has no branches and the
// compiler can interleave the independent columns.
#define H3B_S32(arr, off) (*reinterpret_cast<uint32_t(*)[32]>(&(arr)[off]))

// 2^f on [-0.5, 0.5]: degree-3 polynomial fitted for this kernel (weighted least
// squares on Chebyshev nodes, relative error < 7.5e-5)
constexpr float kP0 = 0.9999280571937561f, kP1 = 0.6932609677314758f, kP2 = 0.2426111251115799f,
                kP3 = 0.05517164617776871f;
// four floats -> four E4M3 bytes (satfinite, round to nearest even), a lowest
__device__ __forceinline__ uint32_t e4m3x4_f32(float a, float b, float c, float d) {
  uint32_t r;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n\t"
      "mov.b32 %0, {lo, hi};\n\t}"
      : "=r"(r) : "f"(a), "f"(b), "f"(c), "f"(d));
  return r;
}
// maximum of the 64 raw columns [CB, CB + 64); the biased accumulator bits are
// positive floats, so integer order is score order
template <int CB>
__device__ __forceinline__ int raw_max64(const uint32_t (&s)[128]) {
  int m0 = (int)s[CB], m1 = (int)s[CB + 1], m2 = (int)s[CB + 2], m3 = (int)s[CB + 3];
#pragma unroll
  for (int c = 4; c < 64; c += 4) {
    m0 = max(m0, (int)s[CB + c]);
    m1 = max(m1, (int)s[CB + c + 1]);
    m2 = max(m2, (int)s[CB + c + 2]);
    m3 = max(m3, (int)s[CB + c + 3]);
  }
  return max(max(m0, m1), max(m2, m3));
}
// the same over the first n (1..63) columns of a ragged last block; the other
// columns become -inf, which the exponential maps to 0
template <int CB>
__device__ __forceinline__ int raw_max_ragged(uint32_t (&s)[128], int n) {
  int m0 = (int)s[CB];
#pragma unroll
  for (int c = 1; c < 64; ++c) {
    if (c < n)
      m0 = max(m0, (int)s[CB + c]);
    else
      s[CB + c] = 0xff800000u;
  }
  return m0;
}
// Sage per_thread K scales: four scale groups per 64-key block, column c in group
// (c % 8) / 2 -- the column pairs (2g, 2g + 1) of every 8-column chunk, which are
// exactly the packed pairs the exponential below works on.  Maxima per group.
template <int CB>
__device__ __forceinline__ void raw_max64_g(const uint32_t (&s)[128], int (&m)[4]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) m[g] = max((int)s[CB + 2 * g], (int)s[CB + 2 * g + 1]);
#pragma unroll
  for (int c = 8; c < 64; c += 8) {
#pragma unroll
    for (int g = 0; g < 4; ++g) m[g] = max(m[g], max((int)s[CB + c + 2 * g], (int)s[CB + c + 2 * g + 1]));
  }
}
// the same over the first n (1..63) columns; a group with no valid column keeps the
// bits of -inf (a negative integer, below every biased score)
template <int CB>
__device__ __forceinline__ void raw_max_ragged_g(uint32_t (&s)[128], int n, int (&m)[4]) {
  m[0] = (int)s[CB];
  m[1] = m[2] = m[3] = (int)0xff800000u;
#pragma unroll
  for (int c = 1; c < 64; ++c) {
    if (c < n)
      m[(c & 7) >> 1] = max(m[(c & 7) >> 1], (int)s[CB + c]);
    else
      s[CB + c] = 0xff800000u;
  }
}

// Columns whose exponential runs as the polynomial on the FMA pipe (the others take
// ex2.approx on the MUFU pipe): bit i of kPolyMask16 selects the column pair
// (2i, 2i + 1) of every 16 columns.  0x08: columns 6, 7 of every 16.
constexpr uint32_t kPolyMask16 = 0x08u;
__host__ __device__ constexpr bool poly_pair(int col) { return (kPolyMask16 >> ((col & 15) >> 1)) & 1u; }
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  // 2^x = 2^j * 2^f, j = rint(x) (low bits of t), f = x - j (exact); x clamped at -125
  const float2 kM = make_float2(kMagicF, kMagicF), kNM = make_float2(-kMagicF, -kMagicF);
  const float2 kN1 = make_float2(-1.f, -1.f);
  const float2 q0 = make_float2(kP0, kP0), q1 = make_float2(kP1, kP1), q2 = make_float2(kP2, kP2),
               q3 = make_float2(kP3, kP3);
  const float2 xp = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
  const float2 t = __fadd2_rn(xp, kM);
  const float2 f = __ffma2_rn(__fadd2_rn(t, kNM), kN1, xp);
  const float2 q = __ffma2_rn(__ffma2_rn(__ffma2_rn(q3, f, q2), f, q1), f, q0);
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

// P = 2^(S * cc + oo) over columns [CB, CB + 64), written back as floats, on
// packed fp32 pairs (FFMA2 / FADD2); the column pairs poly_pair() selects take the
// polynomial, the others ex2.approx; returns the sum.
// KG = 4 (per_thread K scales): pair k of each 8-column chunk is scale group k.
template <int CB, int KG>
__device__ __forceinline__ float exp_block(uint32_t (&s)[128], const float (&cc)[KG], const float (&oo)[KG]) {
  float2 c2[KG], o2[KG];
#pragma unroll
  for (int g = 0; g < KG; ++g) {
    c2[g] = make_float2(cc[g], cc[g]);
    o2[g] = make_float2(oo[g], oo[g]);
  }
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 64; c += 8) {
    float2 x[4], p[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      x[k] = __ffma2_rn(make_float2(__uint_as_float(s[CB + c + 2 * k]), __uint_as_float(s[CB + c + 2 * k + 1])),
                        c2[KG == 1 ? 0 : k], o2[KG == 1 ? 0 : k]);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      p[k] = poly_pair(c + 2 * k) ? exp2_poly2(x[k]) : make_float2(ex2(x[k].x), ex2(x[k].y));
    acc0 = __fadd2_rn(acc0, p[0]);
    acc1 = __fadd2_rn(acc1, p[1]);
    acc0 = __fadd2_rn(acc0, p[2]);
    acc1 = __fadd2_rn(acc1, p[3]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s[CB + c + 2 * k] = __float_as_uint(p[k].x);
      s[CB + c + 2 * k + 1] = __float_as_uint(p[k].y);
    }
  }
  const float2 t = __fadd2_rn(acc0, acc1);
  return t.x + t.y;
}
// P row -> tensor memory: the thread's lane, keys 4c..4c+3 in column c (E4M3, the
// lowest key in bits 0..7), the A-operand layout of the P.V MMA
template <int NC>
__device__ __forceinline__ void store_p(const uint32_t (&s)[128], uint32_t p_addr) {
  uint32_t w[32];
#pragma unroll
  for (int c = 0; c < NC / 4; ++c)
    w[c] = e4m3x4_f32(__uint_as_float(s[4 * c]), __uint_as_float(s[4 * c + 1]), __uint_as_float(s[4 * c + 2]),
                      __uint_as_float(s[4 * c + 3]));
  if constexpr (NC == 128)
    tmem_st32(p_addr, w);
  else
    tmem_st16(p_addr, *reinterpret_cast<uint32_t(*)[16]>(&w[0]));
}
// One key pair (or a single trailing block, NC = 64) for one query row of one
// tile.  The second block's scores load from TMEM while the first block's
// maximum is taken.  The running max m moves (to the tile max) only when the
// tile max exceeds it by more than kTau; then O is rescaled.  cnt = steps this
// tile already processed.  The MMA warp issued the PV of step cnt - 1 before
// this step's S, so that PV (the last reader of the P columns and the last
// writer of O) completed before S did: no MMA of this tile runs while the step
// rescales O or writes P.
template <int NC, int KG>
__device__ __forceinline__ bool softmax_step(uint32_t s_addr, uint32_t o_addr, uint32_t p_addr,
                                             const float (&c0)[KG], const float (&c1)[KG], int n0, int n1, int cnt,
                                             float& m, float& l) {
  uint32_t s[128];
  __syncwarp();
  tmem_ld32(s_addr, H3B_S32(s, 0));
  tmem_ld32(s_addr + 32, H3B_S32(s, 32));
  tmem_wait_ld_dep(H3B_S32(s, 0));
  reg_barrier32(H3B_S32(s, 32));
  if constexpr (NC == 128) {
    tmem_ld32(s_addr + 64, H3B_S32(s, 64));
    tmem_ld32(s_addr + 96, H3B_S32(s, 96));
  }
  float tmax;
  if constexpr (KG == 1) {
    const int mx0 = n0 == 64 ? raw_max64<0>(s) : raw_max_ragged<0>(s, n0);
    tmax = (__int_as_float(mx0) - kMagicF) * c0[0];
  } else {
    int mg[4];
    if (n0 == 64)
      raw_max64_g<0>(s, mg);
    else
      raw_max_ragged_g<0>(s, n0, mg);
    tmax = fmaxf(fmaxf((__int_as_float(mg[0]) - kMagicF) * c0[0], (__int_as_float(mg[1]) - kMagicF) * c0[1]),
                 fmaxf((__int_as_float(mg[2]) - kMagicF) * c0[2], (__int_as_float(mg[3]) - kMagicF) * c0[3]));
  }
  if constexpr (NC == 128) {
    tmem_wait_ld_dep(H3B_S32(s, 64));
    reg_barrier32(H3B_S32(s, 96));
    if constexpr (KG == 1) {
      const int mx1 = n1 == 64 ? raw_max64<64>(s) : raw_max_ragged<64>(s, n1);
      tmax = fmaxf(tmax, (__int_as_float(mx1) - kMagicF) * c1[0]);
    } else {
      int mg[4];
      if (n1 == 64)
        raw_max64_g<64>(s, mg);
      else
        raw_max_ragged_g<64>(s, n1, mg);
      tmax = fmaxf(tmax, fmaxf(fmaxf((__int_as_float(mg[0]) - kMagicF) * c1[0],
                                     (__int_as_float(mg[1]) - kMagicF) * c1[1]),
                               fmaxf((__int_as_float(mg[2]) - kMagicF) * c1[2],
                                     (__int_as_float(mg[3]) - kMagicF) * c1[3])));
    }
  }
  const float m_new = tmax > m + kTau ? tmax : m;
  float alpha = 1.f;
  if (__any_sync(0xffffffffu, m_new != m)) {
    alpha = ex2(m - m_new);
    m = m_new;
    if (cnt > 0) {
      // the PV of the previous step completed before this step's S (issued after it)
      __syncwarp();
#pragma unroll 1
      for (int c = 0; c < 128; c += 16) {
        uint32_t o[16];
        tmem_ld16(o_addr + c, o);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
        tmem_st16(o_addr + c, o);
      }
    }
  }
  const float off = kLog2_112 - m;
  float o0[KG];
#pragma unroll
  for (int g = 0; g < KG; ++g) o0[g] = off - kMagicF * c0[g];
  float psum = exp_block<0, KG>(s, c0, o0);
  if constexpr (NC == 128) {
    float o1[KG];
#pragma unroll
    for (int g = 0; g < KG; ++g) o1[g] = off - kMagicF * c1[g];
    psum += exp_block<64, KG>(s, c1, o1);
  }
  store_p<NC>(s, p_addr);
  tmem_wait_st();
  tc_fence_before();
  l = l * alpha + psum;
  return true;
}

// KG: K scales per 64-key block (1: per block; 4: Sage per_thread groups)
template <int KG>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, AttnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;                   // 1
  uint64_t* kv_full = bars + 1;              // kKVStages
  uint64_t* kv_empty = kv_full + kKVStages;  // kKVStages
  uint64_t* s_full = kv_empty + kKVStages;   // 2 (per tile): S MMA done
  uint64_t* p_full = s_full + 2;             // 2 (per tile, 128 arrivals): P written, S read
  uint64_t* o_full = p_full + 2;             // 2 (per tile)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int qta = 2 * blockIdx.x;
  const int num_qt = (int)((a.Lq + 127) / 128);
  const bool has_b = qta + 1 < num_qt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kKVStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);  // one release per tile
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], kTileThreads);
    }
    mbar_init(&o_full[0], 1);
    mbar_init(&o_full[1], 1);
    *abort_flag = 0;
    // bias operands: A = 1.0 and B = 0.75 * 2^23 in element 0 of each core row (bf16),
    // so A . B^T over K = 16 (two copies of the core row) is 1.5 * 2^23 everywhere
    uint32_t* bias = reinterpret_cast<uint32_t*>(smem + kOffBias);
    for (int i = 0; i < 64; ++i) bias[i] = (i & 3) == 0 ? ((i < 32) ? 0x3F80u : 0x4AC0u) : 0u;
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp < 4) {
    // each register change sits inside its role's branch, so the compiler
    // budgets every role's code by that role's own limit
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
  }
  if (warp == 0) {
    // TMA producer: the whole warp walks the schedule (warp-uniform control
    // flow), one elected lane issues the copies
    StepIter it;
    it.init(a, h, qta, has_b);
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, 2 * kQBytes);
      tma_load_2d(smem + kOffQ, &tmQ, q_full, 0, (int)(h * a.Lqpad + (int64_t)qta * 128));
      tma_load_2d(smem + kOffQ + kQBytes, &tmQ, q_full, 0, (int)(h * a.Lqpad + (int64_t)(qta + 1) * 128));
    }
    __syncwarp();
    int stage = 0;
    uint32_t phase = 0;
    int j0, j1, who;
    while (it.next(j0, j1, who)) {
      if (!mbar_wait_warp(&kv_empty[stage], phase ^ 1, abort_flag, H3B_STATUS_ATTN_TIMEOUT)) break;
      if (elect_one()) {
        uint8_t* kst = smem + kOffKV + stage * kKVBytes;
        uint8_t* vst = kst + 16384;
        mbar_arrive_expect_tx(&kv_full[stage], j1 >= 0 ? 32768u : 16384u);
        tma_load_2d(kst, &tmK, &kv_full[stage], 0, (int)(h * a.Lkpad + (int64_t)j0 * 64));
        tma_load_2d(vst, &tmV, &kv_full[stage], j0 * 64, h * 128);
        if (j1 >= 0) {
          tma_load_2d(kst + 8192, &tmK, &kv_full[stage], 0, (int)(h * a.Lkpad + (int64_t)j1 * 64));
          tma_load_2d(vst + 8192, &tmV, &kv_full[stage], j1 * 64, h * 128);
        }
      }
      __syncwarp();
      if (++stage == kKVStages) { stage = 0; phase ^= 1; }
    }
  } else if (warp == 2 || warp == 3) {
    // MMA issuer of tile t = warp - 2: the whole warp runs the CTA's step
    // schedule (so the descriptors live in uniform registers), one elected lane
    // issues tcgen05.mma / commit.  At each step of its tile: [wait P of the
    // tile's previous step] PV(previous step), S(this step).  Every stage takes
    // one release per tile per fill (kv_empty counts 2): a commit after the
    // tile's PV on it, or a plain arrive at the steps the tile skips.
    const int t = warp - 2;
    StepIter it;
    it.init(a, h, qta, has_b);
    bool ok = mbar_wait_warp(q_full, 0, abort_flag, H3B_STATUS_ATTN_TIMEOUT);
    constexpr uint32_t idesc_pv = idesc_e4m3(128, 128);
    const uint64_t qdesc = sdesc_kmajor_sw128(smem_u32(smem + kOffQ + t * kQBytes));
    const uint32_t kv_addr = smem_u32(smem + kOffKV);
    const uint64_t bias_a = sdesc_core_repeat(smem_u32(smem + kOffBias));
    const uint64_t bias_b = sdesc_core_repeat(smem_u32(smem + kOffBias + 128));
    const uint32_t s_tmem = tmem + (uint32_t)(t * 128);
    const uint32_t o_tmem = tmem + 256 + (uint32_t)(t * 128);
    const uint32_t p_tmem = s_tmem + 96;  // P over S columns 96..127 (the S row is in registers by then)
    int stage = 0;
    uint32_t phase = 0;
    int pst = -1;          // stage of the pending PV (-1: none)
    bool ptwo = false, first = true;
    uint32_t ppar = 0;     // parity of the next p_full phase
    auto wait_p = [&]() -> bool {
      if (!mbar_wait_warp(&p_full[t], ppar, abort_flag, H3B_STATUS_ATTN_TIMEOUT)) return false;
      ppar ^= 1u;
      tc_fence_after();
      return true;
    };
    // PV of the pending step, A = P from tensor memory (32 keys = 8 columns per MMA)
    auto issue_pv = [&]() {
      const uint32_t vbase = kv_addr + (uint32_t)(pst * kKVBytes + 16384);
      if (elect_one()) {
        mma_f8_ts(o_tmem, p_tmem, sdesc_kmajor_sw64(vbase), idesc_pv, first ? 0u : 1u);
        mma_f8_ts(o_tmem, p_tmem + 8, sdesc_kmajor_sw64(vbase + 32), idesc_pv, 1u);
        if (ptwo) {
          mma_f8_ts(o_tmem, p_tmem + 16, sdesc_kmajor_sw64(vbase + 8192), idesc_pv, 1u);
          mma_f8_ts(o_tmem, p_tmem + 24, sdesc_kmajor_sw64(vbase + 8192 + 32), idesc_pv, 1u);
        }
        mma_commit(&kv_empty[pst]);
      }
      __syncwarp();
      first = false;
      pst = -1;
    };
    int j0, j1, who;
    while (ok && it.next(j0, j1, who)) {
      if (!mbar_wait_warp(&kv_full[stage], phase, abort_flag, H3B_STATUS_ATTN_TIMEOUT)) { ok = false; break; }
      tc_fence_after();
      if ((who >> t) & 1) {
        const bool two = j1 >= 0;
        // the previous step's PV first: its P lies in the S columns this step's S
        // overwrites (MMAs of one thread run in issue order)
        if (pst >= 0) {
          if (!wait_p()) { ok = false; break; }
          issue_pv();
        }
        const uint64_t kdesc = sdesc_kmajor_sw128(kv_addr + (uint32_t)(stage * kKVBytes));
        const uint32_t idesc_s = two ? idesc_i8(128, 128) : idesc_i8(128, 64);
        if (elect_one()) {
          mma_bf16_ss(s_tmem, bias_a, bias_b, two ? idesc_bf16(128, 128) : idesc_bf16(128, 64), 0u);
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_i8_ss(s_tmem, qdesc + (uint64_t)(2 * k), kdesc + (uint64_t)(2 * k), idesc_s, 1u);
          mma_commit(&s_full[t]);
        }
        __syncwarp();
        pst = stage;
        ptwo = two;
        if (!it.pending(t)) {
          // the tile's last step: its PV releases the stage now
          if (!wait_p()) { ok = false; break; }
          issue_pv();
        }
      } else {
        if (elect_one()) mbar_arrive(&kv_empty[stage]);
        __syncwarp();
      }
      if (++stage == kKVStages) { stage = 0; phase ^= 1; }
    }
    if (ok) {
      if (elect_one()) mma_commit(&o_full[t]);
      __syncwarp();
    }
  } else if (warp >= 4) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // softmax: tile t, TMEM lane quadrant warp % 4, one query row per thread
    const int t = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int64_t qrow = (int64_t)(qta + t) * 128 + r;
    const bool row_ok = qrow < a.Lq;
    // Q scale group: q_block rows, or Sage per_thread (rows of equal r % 8 in each 32)
    const int64_t qsi = a.q_gran ? (qrow >> 5) * 8 + (qrow & 7) : qrow / a.q_block;
    const float qs = row_ok ? __ldg(a.q_scale + (int64_t)h * a.nqs + qsi) : 0.f;
    const float qsl = qs * a.scale_log2;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + (uint32_t)(t * 128);
    const uint32_t o_addr = tmem + lane_off + 256 + (uint32_t)(t * 128);
    const uint32_t p_addr = s_addr + 96;
    const float* ksc = a.k_scale + (int64_t)h * a.Kb * KG;
    TileStream ts;
    ts.init(a, h, qta + t, t == 0 || has_b);
    float m = -__int_as_float(0x7f800000), l = 0.f;
    int cnt = 0;
    bool ok = true;
    // the next pair's blocks and scales are fetched one step ahead, so their
    // latency hides behind the current step (a zero scale, for an all-zero
    // query row or key block, is floored so that masked -inf columns stay -inf)
    int j0, j1;
    bool have = ts.next_pair(j0, j1);
    float c0[KG], c1[KG];
#pragma unroll
    for (int g = 0; g < KG; ++g) {
      c0[g] = have ? fmaxf(qsl * __ldg(ksc + (int64_t)j0 * KG + g), 1e-30f) : 0.f;
      c1[g] = have && j1 >= 0 ? fmaxf(qsl * __ldg(ksc + (int64_t)j1 * KG + g), 1e-30f) : 0.f;
    }
    while (have) {
      const bool two = j1 >= 0;
      const int n0 = (int)min((int64_t)64, a.Lk - (int64_t)j0 * 64);
      const int n1 = two ? (int)min((int64_t)64, a.Lk - (int64_t)j1 * 64) : 64;
      int nj0, nj1;
      const bool nhave = ts.next_pair(nj0, nj1);
      float nc0[KG], nc1[KG];
#pragma unroll
      for (int g = 0; g < KG; ++g) nc0[g] = nc1[g] = 0.f;
      if (nhave) {
        ld_early_kg<KG>(ksc + (int64_t)nj0 * KG, nc0);
        ld_early_kg<KG>(ksc + (int64_t)(nj1 >= 0 ? nj1 : nj0) * KG, nc1);
      }
      if (!mbar_wait_warp(&s_full[t], (uint32_t)(cnt & 1), abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
        ok = false;
        break;
      }
      tc_fence_after();
      ok = two ? softmax_step<128, KG>(s_addr, o_addr, p_addr, c0, c1, n0, n1, cnt, m, l)
               : softmax_step<64, KG>(s_addr, o_addr, p_addr, c0, c1, n0, n1, cnt, m, l);
      if (!ok) break;
      mbar_arrive(&p_full[t]);
      ++cnt;
      have = nhave;
      j0 = nj0;
      j1 = nj1;
#pragma unroll
      for (int g = 0; g < KG; ++g) {
        c0[g] = fmaxf(qsl * nc0[g], 1e-30f);
        c1[g] = fmaxf(qsl * nc1[g], 1e-30f);
      }
    }
    // epilogue: O / l * v_scale
    uint16_t* dst = a.out + (row_ok ? qrow : 0) * a.out_stride + (int64_t)h * 128;
    if (ok && cnt > 0) {
      if (mbar_wait_warp(&o_full[t], 0u, abort_flag, H3B_STATUS_ATTN_TIMEOUT)) {
        tc_fence_after();
        __syncwarp();
        const float inv_l = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll 1
        for (int c = 0; c < 128; c += 16) {
          uint32_t o[16];
          tmem_ld16(o_addr + c, o);
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
    } else if (row_ok && cnt == 0) {
      for (int c = 0; c < 128; c += 8) *reinterpret_cast<uint4*>(dst + c) = make_uint4(0, 0, 0, 0);
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
  auto kern = a.k_gran ? attn_kernel<4> : attn_kernel<1>;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e == cudaSuccess && fa.numRegs != kLaunchRegs) {
    *err = cudaSuccess;
    return 3;  // the register split was planned for a different launch register count
  }
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  if (e == cudaSuccess) {
    dim3 grid((unsigned)(((a.Lq + 127) / 128 + 1) / 2), (unsigned)a.H);
    kern<<<grid, kAttnThreads, kAttnSmem, s>>>(tq, tk, tv, a);
    e = cudaGetLastError();
  }
  *err = e;
  return e == cudaSuccess ? 0 : 2;
}

}  // namespace h3b
