// Device float helpers whose operation order is part of the parity contract with the reference's scalar path
// (crates/voxrt/src/tensor.rs). Every operation is an explicit IEEE round-to-nearest intrinsic; the library is also
// compiled with -fmad=false so that no a*b+c is contracted behind our back.
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace vxg {

// tensor.rs:829-831
__device__ __constant__ static const float kExpPoly[6] = {1.0f / 120.0f, 1.0f / 24.0f, 1.0f / 6.0f, 0.5f, 1.0f, 1.0f};

// Round to nearest, ties to even, for |y| < 2^22 without a conversion instruction: adding 1.5 * 2^23 leaves a float
// whose unit in the last place is 1, so the addition itself rounds y (ties to even, because 1.5 * 2^23 is even);
// subtracting it back is exact. The integer is the difference of the bit patterns. This is the classic "magic
// number" rounding trick; it keeps the rounding on the FMA pipe instead of the slow conversion unit.
__device__ __forceinline__ float rint_shift(float y, int* ni) {
  const float t = __fadd_rn(y, 12582912.0f);
  *ni = __float_as_int(t) - 0x4B400000;
  return __fsub_rn(t, 12582912.0f);
}

// exp by range reduction x = n ln2 + r (hi/lo split) and a degree-6 Horner polynomial, inputs clamped to
// [-87, 88] (tensor.rs:838-848). NaN passes through the clamp as in Rust's f32::clamp. |x * log2(e)| <= 127 after
// the clamp, well inside rint_shift's range.
__device__ __forceinline__ float exp_poly(float x) {
  x = x < -87.0f ? -87.0f : x;
  x = x > 88.0f ? 88.0f : x;
  int ni;
  const float n = rint_shift(__fmul_rn(x, 1.44269504088896340736f), &ni);
  float r = __fmaf_rn(-n, 0.69314575f, x);
  r = __fmaf_rn(-n, 1.4286068e-6f, r);
  float p = 1.0f / 720.0f;
#pragma unroll
  for (int i = 0; i < 6; i++) p = __fmaf_rn(p, r, kExpPoly[i]);
  const int e = (ni + 127) << 23;
  return __fmul_rn(p, __int_as_float(e));
}

__device__ __forceinline__ float rcp_approx(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}

// Correctly rounded x / d for 1 <= d < 3e37 and 1e-30 < |x| < 1e30, after P. Markstein ("Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): one Newton step on an approximate
// reciprocal, then the quotient's residual r = x - d*q0 (exact with an FMA) corrects q0 to the rounded quotient.
// Callers route everything outside that range to the IEEE division; over the two inputs it is used with here (the
// SiLU and sigmoid below) it has been checked bit for bit against __fdiv_rn on all 2^32 f32 arguments.
__device__ __forceinline__ float div_markstein(float x, float d) {
  const float y0 = rcp_approx(d);
  const float e = __fmaf_rn(-d, y0, 1.0f);
  const float y1 = __fmaf_rn(y0, e, y0);
  const float q0 = __fmul_rn(x, y1);
  const float r = __fmaf_rn(-d, q0, x);
  return __fmaf_rn(r, y1, q0);
}

__device__ __forceinline__ float silu_fast(float x) {  // tensor.rs:852-854: x / (1 + exp_poly(-x))
  const float d = __fadd_rn(1.0f, exp_poly(-x));
  if (fabsf(x) < 1e30f && d < 3.0e37f && fabsf(x) > 1e-30f) return div_markstein(x, d);
  return __fdiv_rn(x, d);
}

// silu_fast for arguments with 1e-30 < |x| < 1e30 and x > -85 (the caller checks): there exp_poly's upper clamp
// cannot act (-x < 85), its lower clamp is a plain max (x is not NaN), 1 + exp_poly(-x) < 3e37, so the division
// is always the Markstein one. Same operations in the same order as silu_fast, without the branches.
__device__ __forceinline__ float silu_inrange(float x) {
  const float y = fmaxf(-x, -87.0f);
  int ni;
  const float n = rint_shift(__fmul_rn(y, 1.44269504088896340736f), &ni);
  float r = __fmaf_rn(-n, 0.69314575f, y);
  r = __fmaf_rn(-n, 1.4286068e-6f, r);
  float p = 1.0f / 720.0f;
#pragma unroll
  for (int i = 0; i < 6; i++) p = __fmaf_rn(p, r, kExpPoly[i]);
  const float d = __fadd_rn(1.0f, __fmul_rn(p, __int_as_float((ni + 127) << 23)));
  return div_markstein(x, d);
}

// silu_inrange on two arguments. The steps that are fused multiply-adds, or a lone multiply or
// subtraction, run as packed f32x2 instructions (each half rounded exactly like the scalar step: fma(-n, c, y) is
// computed as fma(n, -c, y), fma(-d, a, b) as fma(nd, a, b) with nd = -d, both exact sign moves). The two places
// where a product feeds an addition (the shifter rounding of y * log2(e), and 1 + p * 2^n) stay scalar: ptxas fuses
// a packed multiply that feeds a packed add into one FMA, which would skip the product's rounding.
__device__ __forceinline__ void silu2_inrange(float& x0, float& x1) {
  const float y0 = fmaxf(-x0, -87.0f), y1 = fmaxf(-x1, -87.0f);
  const float t0 = __fadd_rn(__fmul_rn(y0, 1.44269504088896340736f), 12582912.0f);
  const float t1 = __fadd_rn(__fmul_rn(y1, 1.44269504088896340736f), 12582912.0f);
  const uint64_t n = fadd2(pk2(t0, t1), pk2(-12582912.0f, -12582912.0f));  // exact
  uint64_t r = ffma2(n, pk2(-0.69314575f, -0.69314575f), pk2(y0, y1));
  r = ffma2(n, pk2(-1.4286068e-6f, -1.4286068e-6f), r);
  uint64_t q = pk2(1.0f / 720.0f, 1.0f / 720.0f);
  q = ffma2(q, r, pk2(1.0f / 120.0f, 1.0f / 120.0f));
  q = ffma2(q, r, pk2(1.0f / 24.0f, 1.0f / 24.0f));
  q = ffma2(q, r, pk2(1.0f / 6.0f, 1.0f / 6.0f));
  q = ffma2(q, r, pk2(0.5f, 0.5f));
  q = ffma2(q, r, pk2(1.0f, 1.0f));
  q = ffma2(q, r, pk2(1.0f, 1.0f));
  float q0, q1;
  upk2(q, q0, q1);
  const float d0 = __fadd_rn(1.0f, __fmul_rn(q0, __int_as_float((__float_as_int(t0) - 0x4B400000 + 127) << 23)));
  const float d1 = __fadd_rn(1.0f, __fmul_rn(q1, __int_as_float((__float_as_int(t1) - 0x4B400000 + 127) << 23)));
  // div_markstein(x, d)
  const uint64_t nd = pk2(-d0, -d1), xx = pk2(x0, x1);
  const uint64_t a0 = pk2(rcp_approx(d0), rcp_approx(d1));
  const uint64_t e = ffma2(nd, a0, pk2(1.0f, 1.0f));
  const uint64_t a1 = ffma2(a0, e, a0);
  const uint64_t qq = fmul2(xx, a1);
  const uint64_t rr = ffma2(nd, qq, xx);
  upk2(ffma2(rr, a1, qq), x0, x1);
}

// sigmoid_fast for x > -85 (so not NaN): exp_poly's clamps reduce to a max and 1 + exp_poly(-x) < 3e37, so the
// division is always the Markstein one. Same operations in the same order as sigmoid_fast, without branches.
__device__ __forceinline__ float sigmoid_inrange(float x) {
  const float y = fmaxf(-x, -87.0f);
  int ni;
  const float n = rint_shift(__fmul_rn(y, 1.44269504088896340736f), &ni);
  float r = __fmaf_rn(-n, 0.69314575f, y);
  r = __fmaf_rn(-n, 1.4286068e-6f, r);
  float p = 1.0f / 720.0f;
#pragma unroll
  for (int i = 0; i < 6; i++) p = __fmaf_rn(p, r, kExpPoly[i]);
  const float d = __fadd_rn(1.0f, __fmul_rn(p, __int_as_float((ni + 127) << 23)));
  return div_markstein(1.0f, d);
}

// quantize_group's code for |v * inv| <= 127 (1 + 2^-23), v * inv not NaN (inv finite): the rounding shifter's
// low byte is the code in two's complement, no clamp needed.
__device__ __forceinline__ uint32_t quant_byte_fast(float v, float inv) {
  return __float_as_uint(__fadd_rn(__fmul_rn(v, inv), 12582912.0f)) & 0xFFu;
}

__device__ __forceinline__ float max_nan(float a, float b) {  // NaN if either input is NaN
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

__device__ __forceinline__ float sigmoid_fast(float x) {  // tensor.rs:858-860: 1 / (1 + exp_poly(-x))
  const float d = __fadd_rn(1.0f, exp_poly(-x));
  if (d < 3.0e37f) return div_markstein(1.0f, d);
  return __fdiv_rn(1.0f, d);
}

// quantize_group's per-element step (packed.rs:527-535): clamp(round_ties_even(v * inv), -127, 127) as i8, NaN -> 0
// (Rust's saturating cast). |v * inv| <= 127 (1 + 2^-23) for finite v, so rint_shift applies; the code is read
// from the bit pattern of the clamped value plus the shifter.
__device__ __forceinline__ int quant_code(float v, float inv) {
  int ni;
  float q = rint_shift(__fmul_rn(v, inv), &ni);
  q = q < -127.0f ? -127.0f : q;
  q = q > 127.0f ? 127.0f : q;
  return q != q ? 0 : __float_as_int(__fadd_rn(q, 12582912.0f)) - 0x4B400000;
}

// scale = absmax / 127 (1 for an all-zero group) and its reciprocal, as quantize_group computes them.
__device__ __forceinline__ float quant_scale(float amax) { return amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f); }

}  // namespace vxg
