// h3b_packed.cuh -- packed fp32-pair arithmetic shared by the activation
// quantizers and the GEMM's GELU + ConvRot epilogue: the int8 code of a scaled
// value, IEEE-exact packed add / mul / fma, the radix-4 regular-Hadamard
// butterfly in the reference's operation order, and tanh-GELU.  Both users must
// give the same bits, so the arithmetic lives in one place.
#pragma once

#include "h3b_common.cuh"

namespace h3b {

// int8 code of a scaled value s: clamp to [-128, 127], round half to even by
// adding 1.5 * 2^23, and take the low byte of the sum's bits -- the code of
// rintf + clamp + (int) (clamping first cannot change the rounded result).
__device__ __forceinline__ uint32_t code_byte(float s) {
  const float c = fminf(127.0f, fmaxf(-128.0f, s));
  return __float_as_uint(__fadd_rn(c, 12582912.0f)) & 0xffu;
}

// ---------------------------------------------------------------- packed pairs
// Two values that take the same place in two independent computations (two
// 256-column groups, or two 64-column blocks of one group) ride as the lanes of a
// float2, so the per-element arithmetic runs as packed FFMA2 / FADD2 / FMUL2 --
// IEEE round-to-nearest per lane, the same bits as the scalar operations.
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 splat2(float v) { return make_float2(v, v); }
// a - b with one rounding: b * -1 is exact, so the fused product-add rounds a - b
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a); }
// both lanes rounded to bf16 (cvt.rn.bf16x2.f32) and widened back
__device__ __forceinline__ float2 bf16r2(float2 v) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(v.y), "f"(v.x));
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
}
// both lanes rounded to bf16 and packed (lane x in bits 0..15, lane y in 16..31)
__device__ __forceinline__ uint32_t pack_bf16x2(float2 v) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(v.y), "f"(v.x));
  return p;
}
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t p) {
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xffff0000u));
}
// packed bf16 sum, correctly rounded (add.rn.bf16x2)
__device__ __forceinline__ uint32_t hadd2_bf16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float2 div2_rn_by(float2 a, float2 b, float2 rb) {
  const float2 q = mul2(a, rb);
  const float2 r = fma2(q, make_float2(-b.x, -b.y), a);
  return fma2(r, rb, q);
}

// One radix-4 butterfly of the regular H4 matrix on both lanes, outputs in the
// reference's operation order (int8_linear.cu:217-250): y0 = ((x0+x1)+x2)-x3,
// y1 = ((x0+x1)-x2)+x3, y2 = ((x0-x1)+x2)+x3, y3 = ((-x0+x1)+x2)+x3, times 1/2.
// x0+x1 and x0-x1 are shared; (-x0+x1)+x2 == x2-(x0-x1) exactly.
__device__ __forceinline__ void h4_stage2(const float2* x, int s, float2* y, int base) {
  const float2 h = splat2(0.5f);
  const float2 x0 = x[base], x1 = x[base + s], x2 = x[base + 2 * s], x3 = x[base + 3 * s];
  const float2 s01 = add2(x0, x1), d01 = sub2(x0, x1);
  y[base] = mul2(h, sub2(add2(s01, x2), x3));
  y[base + s] = mul2(h, add2(sub2(s01, x2), x3));
  y[base + 2 * s] = mul2(h, add2(add2(d01, x2), x3));
  y[base + 3 * s] = mul2(h, add2(sub2(x2, d01), x3));
}
// Two radix-4 stages (stride 1 then 4) over the 16 values of each lane.
__device__ __forceinline__ void fht16x2(float2 (&v)[16]) {
  float2 t[16];
#pragma unroll
  for (int b0 = 0; b0 < 16; b0 += 4) h4_stage2(v, 1, t, b0);
#pragma unroll
  for (int b0 = 0; b0 < 4; ++b0) h4_stage2(t, 4, v, b0);
}

// exp(x) for x in [-20, 0], the argument range of the GELU's tanh, on both
// lanes: the IEEE operations of h3b_expf on that range without its range
// branches.  rint(x log2 e) is taken by adding and subtracting 1.5 * 2^23 (round
// half to even, as rintf), the integer exponent comes from that sum's low bits,
// and one power-of-two scaling replaces the two half scalings (equal, since every
// product stays normal for n >= -29).  Matches h3b_expf bit for bit on every
// float of [-20, 0].
__device__ __forceinline__ float2 expf_neg20x2(float2 x) {
  const float kLog2e = 1.44269502162933349609375f;
  const float kLn2Hi = 0.693145751953125f;
  const float kLn2Lo = 1.428606765330187045e-06f;
  const float2 t = add2(mul2(x, splat2(kLog2e)), splat2(12582912.0f));
  const float2 n = sub2(t, splat2(12582912.0f));
  float2 r = fma2(n, splat2(-kLn2Hi), x);
  r = fma2(n, splat2(-kLn2Lo), r);
  float2 p = splat2(1.0f / 5040.0f);
  p = fma2(p, r, splat2(1.0f / 720.0f));
  p = fma2(p, r, splat2(1.0f / 120.0f));
  p = fma2(p, r, splat2(1.0f / 24.0f));
  p = fma2(p, r, splat2(1.0f / 6.0f));
  p = fma2(p, r, splat2(0.5f));
  p = fma2(p, r, splat2(1.0f));
  p = fma2(p, r, splat2(1.0f));
  // p * 2^n as one integer add of n << 23 to p's bits (p in [0.7, 1.42], n >= -29: the
  // product is normal, so this is the exact power-of-two scaling); the magic sum's
  // bits shifted left by 23 are n << 23 in two's complement
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}
// RN(1 / d) for d in [1, 2]: the approximate reciprocal refined by one Newton
// step, y + y (1 - d y).  Checked against the IEEE reciprocal (__frcp_rn) on
// every float of [1, 2] on B200: identical bits.
__device__ __forceinline__ float2 rcp2_1to2(float2 d) {
  float yx, yy;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(yx) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(yy) : "f"(d.y));
  const float2 y = make_float2(yx, yy);
  return fma2(fma2(make_float2(-d.x, -d.y), y, splat2(1.0f)), y, y);
}
// GELU (tanh form) on both lanes.  tanh(x) = sign(x) (1 - e) / (1 + e), e =
// exp(-2|x|): the quotient is correctly rounded by Markstein's final step from
// RN(1 / (1 + e)) (equal to IEEE division for every e in [2e-9, 1], the range
// exp(-2|x|) takes for |x| < 10).  The exponent is clamped at -20, so |x| >= 10
// gives e = exp(-20), 1 - e and 1 + e both round to 1 and tanh = +-1 exactly; the
// sign is the sign bit of x (t >= 0; a -0 only ever reaches 1 + t).
__device__ __forceinline__ float2 gelu_tanh2(float2 v) {
  const float kBeta = 0.7978845608028654f;
  const float kKappa = 0.044715f;
  const float2 cube = mul2(mul2(mul2(splat2(kKappa), v), v), v);
  const float2 x = mul2(splat2(kBeta), add2(v, cube));
  const float2 m2a = mul2(splat2(-2.0f), make_float2(fabsf(x.x), fabsf(x.y)));
  const float2 e = expf_neg20x2(make_float2(fmaxf(m2a.x, -20.0f), fmaxf(m2a.y, -20.0f)));
  const float2 num = sub2(splat2(1.0f), e), den = add2(splat2(1.0f), e);
  float2 t = div2_rn_by(num, den, rcp2_1to2(den));
  t.x = __uint_as_float(__float_as_uint(t.x) | (__float_as_uint(x.x) & 0x80000000u));
  t.y = __uint_as_float(__float_as_uint(t.y) | (__float_as_uint(x.y) & 0x80000000u));
  return mul2(mul2(splat2(0.5f), v), add2(splat2(1.0f), t));
}

// int8 codes of a pair of values that are already bf16 (bf16(v) = v): code_byte(bf16(v / st))
// on both lanes, the two code bytes in bits 0..7 (lane x) and 8..15 (lane y); the bits
// above are not zero (the caller combines two pairs with byte_perm)
__device__ __forceinline__ uint32_t codes2_bf16(float2 v, float2 st2, float2 rst2) {
  const float2 d = bf16r2(div2_rn_by(v, st2, rst2));
  const float2 c = make_float2(fminf(127.0f, fmaxf(-128.0f, d.x)), fminf(127.0f, fmaxf(-128.0f, d.y)));
  const float2 r = add2(c, splat2(12582912.0f));
  return __byte_perm(__float_as_uint(r.x), __float_as_uint(r.y), 0x0040u);
}
// int8 codes of both lanes: the scalar code_byte(bf16(bf16(v) / st)) lane by lane
__device__ __forceinline__ void codes2(float2 v, float2 st2, float2 rst2, uint32_t& bx, uint32_t& by) {
  const float2 d = bf16r2(div2_rn_by(bf16r2(v), st2, rst2));
  bx = code_byte(d.x);
  by = code_byte(d.y);
}

}  // namespace h3b
