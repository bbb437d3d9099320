/* Internal helpers shared by oracle.cpp and vnni.cpp (test infrastructure, see oracle.h). */
#ifndef VXG_ORACLE_INTERNAL_H
#define VXG_ORACLE_INTERNAL_H

#include <cstdint>
#include <functional>

namespace vxo {

/* Run f(i) for i in [0, n) on the oracle's thread pool (inline when the pool has one thread). The reference uses
 * rayon the same way; every task writes disjoint outputs, so results do not depend on the thread count. */
void parallel_for(int n, const std::function<void(int)>& f);
int threads();

/* Quad16 weight plane (packed.rs:22-33, put_quad16 :276-282) with per-row-block scales (finish :132-161). */
struct Q16 {
  int out = 0, inp = 0, group = 0;
  bool ternary = false;
  int8_t* w = nullptr;      /* out_pad * inp bytes */
  float* scales_q = nullptr; /* [out_pad/16][ng][16] */
  float* scales = nullptr;   /* [out, ng] */
};
Q16* q16_prepare(const int8_t* w_rows, const float* scales, int out, int inp, int group, bool ternary);
void q16_free(Q16* q);

/* y[t, o] for o in [r0, r1), t in [t0, t1) with the fastest bit-exact kernel this CPU has (AVX-512 VNNI, else AVX2
 * for ternary groups <= 256, else the scalar reference). Single-threaded. */
void q16_gemm_range(const Q16* W, const int8_t* x, const float* sx, const int32_t* gsum, int n, int ep,
                    float ep_scale, float* y, int r0, int r1, int t0, int t1);
/* gemm_ep (kernels/mod.rs:324-362): row-block parallel over the pool, then the optional bias add. */
void q16_gemm_ep(const Q16* W, const int8_t* x, const float* sx, int n, int ep, float ep_scale, const float* bias,
                 float* y);
/* Σ of int8 codes per (token, group) (packed.rs:349-360). */
void group_sums(const int8_t* x, int n, int inp, int group, int32_t* gsum);

float quantize_group(const float* src, int n, int8_t* dst);
float exp_poly(float x);
float silu_fast(float x);
float sigmoid_fast(float x);

} // namespace vxo

#endif
