/*
 * Timed CPU baseline: C++ restatement of the reference's x86 kernels on the Quad16 layout
 * (crates/voxrt/src/kernels/x86.rs) and of gemm_ep's row-block thread split (kernels/mod.rs:324-362).
 * Test infrastructure (see oracle.h): bit-identical to the scalar oracle, which the CPU test suite checks.
 *
 * AVX-512 VNNI (x86.rs:46-154): a 512-bit lane owns one output row of a 16-row block; weights are offset to
 * unsigned by xor 0x80 (= w + 128) for vpdpbusd, and 128 * (Σ x over the group) is subtracted afterwards. The float
 * step per group is fma(float(sum), sx * sw, acc), as in the scalar kernel.
 * AVX2 (x86.rs:163-290): ternary weights as u = w + 1 in {0,1,2} through vpmaddubsw (i16, group <= 256), corrected
 * by Σ x; arbitrary int8 weights through |w| * sign(x, w), widened to i32 every step.
 */
#include "oracle.h"
#include "oracle_internal.h"

#include <immintrin.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <vector>

namespace vxo {

static bool cpu_vnni() {
  static int v = -1;
  if (v < 0) {
    __builtin_cpu_init();
    v = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
        __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("fma");
  }
  return v;
}
static bool cpu_avx2() {
  static int v = -1;
  if (v < 0) {
    __builtin_cpu_init();
    v = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  }
  return v;
}

static int force_kernel = -1; /* -1 auto, 0 scalar, 1 avx2, 2 vnni (tests pick each) */

Q16* q16_prepare(const int8_t* w_rows, const float* scales, int out, int inp, int group, bool ternary) {
  Q16* q = new Q16;
  q->out = out;
  q->inp = inp;
  q->group = group;
  q->ternary = ternary;
  const int ng = inp / group, out_pad = (out + 15) / 16 * 16;
  q->w = (int8_t*)aligned_alloc(64, std::max<size_t>(64, ((size_t)out_pad * inp + 63) / 64 * 64));
  std::memset(q->w, 0, (size_t)out_pad * inp);
  for (int r = 0; r < out; r++)
    for (int c4 = 0; c4 < inp / 4; c4++) { /* put_quad16 (packed.rs:276-282) */
      size_t o = ((size_t)(r / 16) * (inp / 4) + c4) * 64 + (r % 16) * 4;
      std::memcpy(q->w + o, w_rows + (size_t)r * inp + c4 * 4, 4);
    }
  q->scales_q = (float*)aligned_alloc(64, std::max<size_t>(64, ((size_t)out_pad * ng * 4 + 63) / 64 * 64));
  std::memset(q->scales_q, 0, (size_t)out_pad * ng * 4);
  q->scales = new float[(size_t)out * ng];
  std::memcpy(q->scales, scales, (size_t)out * ng * 4);
  for (int r = 0; r < out; r++) /* finish (packed.rs:143-150) */
    for (int g = 0; g < ng; g++) q->scales_q[((size_t)(r / 16) * ng + g) * 16 + r % 16] = scales[(size_t)r * ng + g];
  return q;
}

void q16_free(Q16* q) {
  if (!q) return;
  free(q->w);
  free(q->scales_q);
  delete[] q->scales;
  delete q;
}

static inline float ep_apply(int ep, float s, float old, float v) {
  switch (ep) {
    case VXO_EP_SILU: return silu_fast(v);
    case VXO_EP_ADD_SCALED: return std::fmaf(s, v, old);
    default: return v;
  }
}

/* store_block (x86.rs:20-38): only rows in [r0, r1) */
static inline void store_block(const float* vals, float* y, int out, int rbase, int r0, int r1, int t, int ep,
                               float s) {
  int lo = std::max(r0, rbase), hi = std::min(r1, rbase + 16);
  for (int o = lo; o < hi; o++) y[(size_t)t * out + o] = ep_apply(ep, s, y[(size_t)t * out + o], vals[o - rbase]);
}

template <int T>
__attribute__((target("avx512f,avx512bw,avx512vnni,fma"))) static void vnni_tile(const Q16* W, const int8_t* xp,
                                                                                 const float* sx,
                                                                                 const int32_t* gsum, float* y,
                                                                                 int rb, int r0, int r1, int t,
                                                                                 int ep, float es) {
  const int inp = W->inp, g = W->group, ng = inp / g, qpg = g / 4;
  const int8_t* wb = W->w + (size_t)rb * (inp / 4) * 64;
  const float* sq = W->scales_q + (size_t)rb * ng * 16;
  const __m512i flip = _mm512_set1_epi8((char)0x80);
  __m512 accf[T];
  #pragma GCC unroll 16
  for (int j = 0; j < T; j++) accf[j] = _mm512_setzero_ps();
  for (int gi = 0; gi < ng; gi++) {
    __m512i acc[T];
    #pragma GCC unroll 16
    for (int j = 0; j < T; j++) acc[j] = _mm512_setzero_si512();
    for (int q = gi * qpg; q < (gi + 1) * qpg; q++) {
      __m512i wv = _mm512_xor_si512(_mm512_loadu_si512((const void*)(wb + (size_t)q * 64)), flip);
      #pragma GCC unroll 16
      for (int j = 0; j < T; j++) {
        int32_t xb;
        std::memcpy(&xb, xp + (size_t)(t + j) * inp + q * 4, 4);
        acc[j] = _mm512_dpbusd_epi32(acc[j], wv, _mm512_set1_epi32(xb));
      }
    }
    __m512 sw = _mm512_loadu_ps(sq + gi * 16);
    #pragma GCC unroll 16
    for (int j = 0; j < T; j++) {
      int tok = t + j;
      __m512i corr = _mm512_set1_epi32(128 * gsum[(size_t)tok * ng + gi]);
      __m512 s = _mm512_cvtepi32_ps(_mm512_sub_epi32(acc[j], corr));
      __m512 p = _mm512_mul_ps(_mm512_set1_ps(sx[(size_t)tok * ng + gi]), sw);
      accf[j] = _mm512_fmadd_ps(s, p, accf[j]);
    }
  }
  bool full = rb * 16 >= r0 && rb * 16 + 16 <= r1;
  alignas(64) float vals[16];
  #pragma GCC unroll 16
  for (int j = 0; j < T; j++) {
    float* dst = y + (size_t)(t + j) * W->out + rb * 16;
    if (full && ep == VXO_EP_STORE) {
      _mm512_storeu_ps(dst, accf[j]);
    } else if (full && ep == VXO_EP_ADD_SCALED) {
      _mm512_storeu_ps(dst, _mm512_fmadd_ps(_mm512_set1_ps(es), accf[j], _mm512_loadu_ps(dst)));
    } else {
      _mm512_storeu_ps(vals, accf[j]);
      store_block(vals, y, W->out, rb * 16, r0, r1, t + j, ep, es);
    }
  }
}

__attribute__((target("avx512f,avx512bw,avx512vnni,fma"))) static void gemm_vnni_range(
    const Q16* W, const int8_t* x, const float* sx, const int32_t* gsum, float* y, int r0, int r1, int t0, int t1,
    int ep, float es) {
  for (int rb = r0 / 16; rb < (r1 + 15) / 16; rb++) {
    int t = t0;
    while (t < t1) {
      int left = t1 - t;
      if (left >= 8) {
        vnni_tile<8>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
        t += 8;
      } else if (left >= 4) {
        vnni_tile<4>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
        t += 4;
      } else if (left >= 2) {
        vnni_tile<2>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
        t += 2;
      } else {
        vnni_tile<1>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
        t += 1;
      }
    }
  }
}

template <int T, bool TERN>
__attribute__((target("avx2,fma"))) static void avx2_tile(const Q16* W, const int8_t* xp, const float* sx,
                                                          const int32_t* gsum, float* y, int rb, int r0, int r1,
                                                          int t, int ep, float es) {
  const int inp = W->inp, g = W->group, ng = inp / g, qpg = g / 4;
  const int8_t* wb = W->w + (size_t)rb * (inp / 4) * 64;
  const float* sq = W->scales_q + (size_t)rb * ng * 16;
  const __m256i ones8 = _mm256_set1_epi8(1), ones16 = _mm256_set1_epi16(1);
  __m256 accf[T][2];
  #pragma GCC unroll 16
  for (int j = 0; j < T; j++) accf[j][0] = accf[j][1] = _mm256_setzero_ps();
  for (int gi = 0; gi < ng; gi++) {
    __m256i acc[T][2];
    #pragma GCC unroll 16
    for (int j = 0; j < T; j++) acc[j][0] = acc[j][1] = _mm256_setzero_si256();
    for (int q = gi * qpg; q < (gi + 1) * qpg; q++) {
      __m256i w0 = _mm256_loadu_si256((const __m256i*)(wb + (size_t)q * 64));
      __m256i w1 = _mm256_loadu_si256((const __m256i*)(wb + (size_t)q * 64 + 32));
      #pragma GCC unroll 16
      for (int j = 0; j < T; j++) {
        int32_t xv;
        std::memcpy(&xv, xp + (size_t)(t + j) * inp + q * 4, 4);
        __m256i xb = _mm256_set1_epi32(xv);
        if (TERN) {
          __m256i u0 = _mm256_add_epi8(w0, ones8), u1 = _mm256_add_epi8(w1, ones8);
          acc[j][0] = _mm256_add_epi16(acc[j][0], _mm256_maddubs_epi16(u0, xb));
          acc[j][1] = _mm256_add_epi16(acc[j][1], _mm256_maddubs_epi16(u1, xb));
        } else {
          __m256i u0 = _mm256_abs_epi8(w0), u1 = _mm256_abs_epi8(w1);
          __m256i p0 = _mm256_maddubs_epi16(u0, _mm256_sign_epi8(xb, w0));
          __m256i p1 = _mm256_maddubs_epi16(u1, _mm256_sign_epi8(xb, w1));
          acc[j][0] = _mm256_add_epi32(acc[j][0], _mm256_madd_epi16(p0, ones16));
          acc[j][1] = _mm256_add_epi32(acc[j][1], _mm256_madd_epi16(p1, ones16));
        }
      }
    }
    __m256 sw[2] = {_mm256_loadu_ps(sq + gi * 16), _mm256_loadu_ps(sq + gi * 16 + 8)};
    #pragma GCC unroll 16
    for (int j = 0; j < T; j++) {
      int tok = t + j;
      __m256 sxv = _mm256_set1_ps(sx[(size_t)tok * ng + gi]);
      __m256i corr = _mm256_set1_epi32(gsum[(size_t)tok * ng + gi]);
      #pragma GCC unroll 16
      for (int hh = 0; hh < 2; hh++) {
        __m256i sum = TERN ? _mm256_sub_epi32(_mm256_madd_epi16(acc[j][hh], ones16), corr) : acc[j][hh];
        __m256 p = _mm256_mul_ps(sxv, sw[hh]);
        accf[j][hh] = _mm256_fmadd_ps(_mm256_cvtepi32_ps(sum), p, accf[j][hh]);
      }
    }
  }
  bool full = rb * 16 >= r0 && rb * 16 + 16 <= r1;
  alignas(32) float vals[16];
  #pragma GCC unroll 16
  for (int j = 0; j < T; j++) {
    float* dst = y + (size_t)(t + j) * W->out + rb * 16;
    if (full && ep == VXO_EP_STORE) {
      _mm256_storeu_ps(dst, accf[j][0]);
      _mm256_storeu_ps(dst + 8, accf[j][1]);
    } else if (full && ep == VXO_EP_ADD_SCALED) {
      __m256 s = _mm256_set1_ps(es);
      _mm256_storeu_ps(dst, _mm256_fmadd_ps(s, accf[j][0], _mm256_loadu_ps(dst)));
      _mm256_storeu_ps(dst + 8, _mm256_fmadd_ps(s, accf[j][1], _mm256_loadu_ps(dst + 8)));
    } else {
      _mm256_storeu_ps(vals, accf[j][0]);
      _mm256_storeu_ps(vals + 8, accf[j][1]);
      store_block(vals, y, W->out, rb * 16, r0, r1, t + j, ep, es);
    }
  }
}

template <bool TERN>
__attribute__((target("avx2,fma"))) static void gemm_avx2_range(const Q16* W, const int8_t* x, const float* sx,
                                                                const int32_t* gsum, float* y, int r0, int r1,
                                                                int t0, int t1, int ep, float es) {
  for (int rb = r0 / 16; rb < (r1 + 15) / 16; rb++) {
    int t = t0;
    while (t < t1) {
      int left = t1 - t;
      int step = left >= 4 ? 4 : left >= 2 ? 2 : 1;
      if (step == 4) avx2_tile<4, TERN>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
      else if (step == 2) avx2_tile<2, TERN>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
      else avx2_tile<1, TERN>(W, x, sx, gsum, y, rb, r0, r1, t, ep, es);
      t += step;
    }
  }
}

/* gemm_scalar_range on the Quad16 plane (kernels/mod.rs:195-209, element access via quad16_offset) */
static void gemm_scalar_q16(const Q16* W, const int8_t* x, const float* sx, float* y, int r0, int r1, int t0,
                            int t1, int ep, float es) {
  const int inp = W->inp, g = W->group, ng = inp / g;
  for (int o = r0; o < r1; o++)
    for (int t = t0; t < t1; t++) {
      float acc = 0.0f;
      for (int gi = 0; gi < ng; gi++) {
        int32_t s = 0;
        for (int c = gi * g; c < (gi + 1) * g; c++) {
          size_t off = ((size_t)(o / 16) * (inp / 4) + c / 4) * 64 + (o % 16) * 4 + c % 4;
          s += (int32_t)W->w[off] * (int32_t)x[(size_t)t * inp + c];
        }
        acc = std::fmaf((float)s, sx[(size_t)t * ng + gi] * W->scales[(size_t)o * ng + gi], acc);
      }
      float* slot = y + (size_t)t * W->out + o;
      *slot = ep_apply(ep, es, *slot, acc);
    }
}

static int pick_kernel(const Q16* W) {
  if (force_kernel == 2 && cpu_vnni()) return 2;
  if (force_kernel == 1 && cpu_avx2() && (!W->ternary || W->group <= 256)) return 1;
  if (force_kernel == 0) return 0;
  if (force_kernel < 0) {
    if (cpu_vnni()) return 2;
    if (cpu_avx2() && (!W->ternary || W->group <= 256)) return 1;
  }
  return 0;
}

void q16_gemm_range(const Q16* W, const int8_t* x, const float* sx, const int32_t* gsum, int n, int ep,
                    float ep_scale, float* y, int r0, int r1, int t0, int t1) {
  (void)n;
  switch (pick_kernel(W)) {
    case 2: gemm_vnni_range(W, x, sx, gsum, y, r0, r1, t0, t1, ep, ep_scale); break;
    case 1:
      if (W->ternary) gemm_avx2_range<true>(W, x, sx, gsum, y, r0, r1, t0, t1, ep, ep_scale);
      else gemm_avx2_range<false>(W, x, sx, gsum, y, r0, r1, t0, t1, ep, ep_scale);
      break;
    default: gemm_scalar_q16(W, x, sx, y, r0, r1, t0, t1, ep, ep_scale); break;
  }
}

void q16_gemm_ep(const Q16* W, const int8_t* x, const float* sx, int n, int ep, float ep_scale, const float* bias,
                 float* y) {
  std::vector<int32_t> gsum((size_t)n * (W->inp / W->group));
  group_sums(x, n, W->inp, W->group, gsum.data());
  /* kernels/mod.rs:333-347: threads * 8 blocks (VOXRT_GEMM_BLOCKS default), at most out/8, whole 16-row tiles */
  int th = threads();
  int blocks = std::max(1, std::min(th * 8, W->out / 8));
  int chunk = ((W->out + blocks - 1) / blocks + 15) / 16 * 16;
  int n_blocks = (W->out + chunk - 1) / chunk;
  parallel_for(n_blocks, [&](int bi) {
    int r0 = bi * chunk, r1 = std::min(r0 + chunk, W->out);
    q16_gemm_range(W, x, sx, gsum.data(), n, ep, ep_scale, y, r0, r1, 0, n);
  });
  if (bias)
    for (int t = 0; t < n; t++)
      for (int o = 0; o < W->out; o++) y[(size_t)t * W->out + o] += bias[o];
}

} // namespace vxo

using namespace vxo;

extern "C" {

/* Prepared-weight handle for the timed CPU baseline (the reference repacks at load time, transcriber load path). */
void* vxo_q16_prepare(const int8_t* w_rows, const float* scales, int out, int inp, int group, int ternary) {
  return q16_prepare(w_rows, scales, out, inp, group, ternary != 0);
}
void vxo_q16_free(void* h) { q16_free((Q16*)h); }

/* gemm_ep with the selected x86 kernel; gsum is computed here (QuantAct::from_rows does it while quantising). */
void vxo_q16_gemm(void* h, const int8_t* x, const float* sx, int n, int ep, float ep_scale, const float* bias,
                  float* y) {
  q16_gemm_ep((const Q16*)h, x, sx, n, ep, ep_scale, bias, y);
}

/* Single-threaded range form (x86_kernels.rs `check`): rows [r0, r1) x tokens [t0, t1). */
void vxo_q16_gemm_range(void* h, const int8_t* x, const float* sx, int n, int ep, float ep_scale, float* y, int r0,
                        int r1, int t0, int t1) {
  const Q16* W = (const Q16*)h;
  std::vector<int32_t> gsum((size_t)n * (W->inp / W->group));
  group_sums(x, n, W->inp, W->group, gsum.data());
  q16_gemm_range(W, x, sx, gsum.data(), n, ep, ep_scale, y, r0, r1, t0, t1);
}

/* Single-thread throughput probe after x86_bench.rs:31-71: the selected kernel on weight rows [0, rows) x all n
 * tokens, Store epilogue, group sums computed beforehand (the reference computes them while quantising); returns the
 * best of `reps` wall-clock seconds. */
double vxo_q16_bench_range(void* h, const int8_t* x, const float* sx, int n, float* y, int rows, int reps) {
  const Q16* W = (const Q16*)h;
  std::vector<int32_t> gsum((size_t)n * (W->inp / W->group));
  group_sums(x, n, W->inp, W->group, gsum.data());
  double best = 1e30;
  for (int i = 0; i < reps; i++) {
    const auto t0 = std::chrono::steady_clock::now();
    q16_gemm_range(W, x, sx, gsum.data(), n, 0, 0.0f, y, 0, rows, 0, n);
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    best = std::min(best, dt);
  }
  return best;
}

/* -1 auto, 0 scalar, 1 AVX2, 2 AVX-512 VNNI; returns the kernel that will run for a ternary group-128 matrix. */
int vxo_force_kernel(int k) {
  force_kernel = k;
  Q16 probe;
  probe.ternary = true;
  probe.group = 128;
  return pick_kernel(&probe);
}
int vxo_cpu_has_vnni(void) { return cpu_vnni() ? 1 : 0; }
int vxo_cpu_has_avx2(void) { return cpu_avx2() ? 1 : 0; }

} // extern "C"
