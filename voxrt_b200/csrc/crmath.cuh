// Correctly rounded single-precision exp and tanh, bit-identical on the host and the device.
//
// The decoder's LSTM cell (sigmoid = 1 / (1 + exp(-x)), tanh) and the VAD head's sigmoid call exp / tanh on f32
// values; the reference takes them from a libm. Here they are defined as the correctly rounded values (round to
// nearest even of the exact mathematical result), which fixes every bit independently of any library, so the host
// decoder, the GPU decoder and the checker agree exactly.
//
// Method: evaluate in IEEE double with only correctly rounded operations (fma, +, *, /, rint), which give the same
// bits on the CPU and on the GPU, then round to f32. exp uses Cody-Waite reduction x = k ln2 + r (ln2 split into two
// doubles) and the degree-13 Taylor polynomial of exp(r) on |r| <= ln2 / 2 (truncation below 2^-57 relative); tanh uses
// its Taylor series to degree 23 for |x| < 1/4 and (e - 1) / (e + 1) with e = exp(2|x|) above. Both stay within
// 2^-50 of the exact value. Rounding that result to f32 can only go wrong when the exact value lies within 2^-48 of a
// point halfway between two floats; those inputs are found exhaustively over all 2^32 floats (crmath_gen.cpp, with
// the exact values from decimal arithmetic, crmath_gen.py) and their correctly rounded results stored in
// crmath_tables.h, which the functions consult whenever the double result falls that close to a halfway point.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#ifdef __CUDACC__
#define VX_HD __host__ __device__ __forceinline__
#else
#define VX_HD inline
#endif

#include "crmath_tables.h"

namespace vxg {
namespace crm {

VX_HD uint32_t fbits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
VX_HD float ffrom(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
VX_HD double dfrom(uint64_t u) {
  double d;
  memcpy(&d, &u, 8);
  return d;
}

VX_HD double dfma(double a, double b, double c) { return fma(a, b, c); }

// exp(x) in double for |x| <= 250.
VX_HD double exp_d(double x) {
  const double k = rint(x * 0x1.71547652b82fep+0);  // x / ln2, rounded
  double r = dfma(-k, 0x1.62e42fefa39efp-1, x);     // x - k ln2_hi (exact in one rounding)
  r = dfma(-k, 0x1.abc9e3b39803fp-56, r);            // - k ln2_lo
  double p = 0x1.6124613a86d09p-33;                   // 1/13!
  p = dfma(p, r, 0x1.1eed8eff8d898p-29);
  p = dfma(p, r, 0x1.ae64567f544e4p-26);
  p = dfma(p, r, 0x1.27e4fb7789f5cp-22);
  p = dfma(p, r, 0x1.71de3a556c734p-19);
  p = dfma(p, r, 0x1.a01a01a01a01ap-16);
  p = dfma(p, r, 0x1.a01a01a01a01ap-13);
  p = dfma(p, r, 0x1.6c16c16c16c17p-10);
  p = dfma(p, r, 0x1.1111111111111p-7);
  p = dfma(p, r, 0x1.5555555555555p-5);
  p = dfma(p, r, 0x1.5555555555555p-3);
  p = dfma(p, r, 0x1.0000000000000p-1);
  p = dfma(p, r, 1.0);
  p = dfma(p, r, 1.0);
  const int ki = (int)k;  // |k| <= 361: 2^k is a normal double
  return p * dfrom((uint64_t)(ki + 1023) << 52);
}

// tanh(x) in double for 0 <= x <= 20.
VX_HD double tanh_d(double x) {
  if (x < 0.25) {
    const double x2 = x * x;
    double p = -0x1.497d8eea25259p-15;  // coefficient of x^23
    p = dfma(p, x2, 0x1.967e18afcafadp-14);
    p = dfma(p, x2, -0x1.f57d7734d1664p-13);
    p = dfma(p, x2, 0x1.3558248036744p-11);
    p = dfma(p, x2, -0x1.7da36452b75e3p-10);
    p = dfma(p, x2, 0x1.d6d3d0e157de0p-9);
    p = dfma(p, x2, -0x1.226e355e6c23dp-7);
    p = dfma(p, x2, 0x1.664f4882c10fap-6);
    p = dfma(p, x2, -0x1.ba1ba1ba1ba1cp-5);
    p = dfma(p, x2, 0x1.1111111111111p-3);
    p = dfma(p, x2, -0x1.5555555555555p-2);
    return dfma(p * x2, x, x);  // x + x^3 * (...)
  }
  const double e = exp_d(2.0 * x);
  return (e - 1.0) / (e + 1.0);
}

// Is the double y so close to a point halfway between the two floats around it that rounding y could differ from
// rounding the exact value (|exact - y| < 2^-50 |y|)? Tested with margin: within 2^-48 |y|.
VX_HD bool near_half(double y) {
  const double ay = fabs(y);
  float f = (float)ay;  // nearest float
  double fd = (double)f;
  // the halfway point between f and its neighbour on the side of ay
  const uint32_t fb = fbits(f);
  if (fb >= 0x7F800000u) return false;  // rounds to infinity: the exp overflow threshold is far from a tie
  const double g = (double)ffrom(ay >= fd ? fb + 1u : (fb == 0 ? 0u : fb - 1u));
  const double half = 0.5 * (fd + g);
  return fabs(ay - half) <= 0x1p-48 * ay;
}

// Binary search of a table of (input bits, result bits) pairs sorted by input bits.
VX_HD bool lookup(const uint32_t* tab, int n, uint32_t key, uint32_t* out) {
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const uint32_t k = tab[2 * mid];
    if (k == key) {
      *out = tab[2 * mid + 1];
      return true;
    }
    if (k < key) lo = mid + 1;
    else hi = mid - 1;
  }
  return false;
}

VX_HD float expf_cr(float x) {
  if (x != x) return x;
  if (x > 89.0f) return ffrom(0x7F800000u);
  if (x < -104.0f) return 0.0f;
  const double y = exp_d((double)x);
  if (near_half(y)) {
    uint32_t r;
#ifdef __CUDA_ARCH__
    if (lookup(kExpTieTableDev, kExpTies, fbits(x), &r)) return ffrom(r);
#else
    if (lookup(kExpTieTable, kExpTies, fbits(x), &r)) return ffrom(r);
#endif
  }
  return (float)y;
}

VX_HD float tanhf_cr(float x) {
  if (x != x) return x;
  const float ax = fabsf(x);
  if (ax == 0.0f) return x;  // keeps the sign of zero
  if (ax >= 20.0f) return x > 0.0f ? 1.0f : -1.0f;
  const double y = tanh_d((double)ax);
  float r = (float)y;
  if (near_half(y)) {
    uint32_t t;
#ifdef __CUDA_ARCH__
    if (lookup(kTanhTieTableDev, kTanhTies, fbits(ax), &t)) r = ffrom(t);
#else
    if (lookup(kTanhTieTable, kTanhTies, fbits(ax), &t)) r = ffrom(t);
#endif
  }
  return x < 0.0f ? -r : r;
}

}  // namespace crm
}  // namespace vxg
