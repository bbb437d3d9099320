// Device float helpers whose operation order is part of the parity contract with the reference's scalar path
// (crates/voxrt/src/tensor.rs). Every operation is an explicit IEEE round-to-nearest intrinsic; the library is also
// compiled with -fmad=false so that no a*b+c is contracted behind our back.
#pragma once
#include <cstdint>

namespace vxg {

// tensor.rs:829-831
__device__ __constant__ static const float kExpPoly[6] = {1.0f / 120.0f, 1.0f / 24.0f, 1.0f / 6.0f, 0.5f, 1.0f, 1.0f};

// exp by range reduction x = n ln2 + r (hi/lo split) and a degree-6 Horner polynomial, inputs clamped to
// [-87, 88] (tensor.rs:838-848). NaN passes through the clamp as in Rust's f32::clamp.
__device__ __forceinline__ float exp_poly(float x) {
  x = x < -87.0f ? -87.0f : x;
  x = x > 88.0f ? 88.0f : x;
  const float n = rintf(__fmul_rn(x, 1.44269504088896340736f));
  float r = __fmaf_rn(-n, 0.69314575f, x);
  r = __fmaf_rn(-n, 1.4286068e-6f, r);
  float p = 1.0f / 720.0f;
#pragma unroll
  for (int i = 0; i < 6; i++) p = __fmaf_rn(p, r, kExpPoly[i]);
  const int e = ((int)n + 127) << 23;
  return __fmul_rn(p, __int_as_float(e));
}

__device__ __forceinline__ float silu_fast(float x) {  // tensor.rs:852-854
  return __fdiv_rn(x, __fadd_rn(1.0f, exp_poly(-x)));
}

__device__ __forceinline__ float sigmoid_fast(float x) {  // tensor.rs:858-860
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_poly(-x)));
}

// quantize_group's per-element step (packed.rs:527-535): clamp(round_ties_even(v * inv), -127, 127) as i8.
__device__ __forceinline__ int quant_code(float v, float inv) {
  float q = rintf(__fmul_rn(v, inv));
  q = q < -127.0f ? -127.0f : q;
  q = q > 127.0f ? 127.0f : q;
  return q != q ? 0 : (int)q;  // NaN -> 0 as Rust's saturating cast
}

// scale = absmax / 127 (1 for an all-zero group) and its reciprocal, as quantize_group computes them.
__device__ __forceinline__ float quant_scale(float amax) { return amax == 0.0f ? 1.0f : __fdiv_rn(amax, 127.0f); }

}  // namespace vxg
