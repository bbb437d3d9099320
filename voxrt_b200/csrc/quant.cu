// Per-(token, group) int8 quantisation and the fused LayerNorm -> quantise pass.
//
// quantize_group (crates/voxrt/src/packed.rs:527-535): s = absmax/127 (1 for an all-zero group), inv = 1/s,
// q = clamp(round_ties_even(v * inv), -127, 127). absmax is order-free, so a warp-shuffle max is exact.
//
// LayerNorm (tensor.rs:333-362 row_mean_var_portable, :712-719 layer_norm_row): the row sum and the sum of squared
// deviations are eight sequential chains (element 8m + c feeds chain c), combined as
// hsum4(chain[0..4] + chain[4..8]) = ((c0+c4) + (c1+c5)) + ((c2+c6) + (c3+c7)); the tail (d % 8) is added in
// order. Here lanes 0..7 of a warp each run one chain over the row staged in shared memory, so the float order is
// the reference's exactly; normalisation and quantisation then use all 32 lanes (float4 per lane).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.h"
#include "internal.h"
#include "math.cuh"

namespace vxg {
namespace quant {

constexpr int WARPS = 4;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Quantise `n` values at `src` (shared or global) with stride-1 access, group = n, all 32 lanes.
// Writes codes to dst and returns the scale (valid in every lane).
__device__ __forceinline__ float quantize_group_warp(const float* src, int n, int8_t* dst, int lane) {
  float amax = 0.0f;
  for (int i = lane; i < n; i += 32) amax = fmaxf(amax, fabsf(src[i]));
  amax = warp_max(amax);
  const float s = quant_scale(amax);
  const float inv = __fdiv_rn(1.0f, s);
  for (int i = lane; i < n; i += 32) dst[i] = (int8_t)quant_code(src[i], inv);
  return s;
}

// Mean and biased variance of row[0..d) in the reference order; result valid in all lanes.
__device__ __forceinline__ void row_mean_var(const float* row, int d, int lane, float& mean, float& var) {
  const int n8 = d / 8 * 8;
  float chain = 0.0f;
  if (lane < 8)
    for (int c = lane; c < n8; c += 8) chain = __fadd_rn(chain, row[c]);
  // t4[l] = s0[l] + s1[l] with s0 = chains 0..3, s1 = chains 4..7; hsum4 = (t0 + t1) + (t2 + t3)
  float partner = __shfl_down_sync(0xffffffffu, chain, 4);
  float t = __fadd_rn(chain, partner);                       // lanes 0..3: t4[lane]
  float t1 = __shfl_down_sync(0xffffffffu, t, 1);            // lane 0: t4[1], lane 2: t4[3]
  float pair = __fadd_rn(t, t1);                             // lane 0: t0+t1, lane 2: t2+t3
  float pair2 = __shfl_down_sync(0xffffffffu, pair, 2);      // lane 0: t2+t3
  float sum = __fadd_rn(pair, pair2);                        // lane 0
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int c = n8; c < d; c++) sum = __fadd_rn(sum, row[c]);
  mean = __fdiv_rn(sum, (float)d);
  chain = 0.0f;
  if (lane < 8)
    for (int c = lane; c < n8; c += 8) {
      const float a = __fsub_rn(row[c], mean);
      chain = __fmaf_rn(a, a, chain);
    }
  partner = __shfl_down_sync(0xffffffffu, chain, 4);
  t = __fadd_rn(chain, partner);
  t1 = __shfl_down_sync(0xffffffffu, t, 1);
  pair = __fadd_rn(t, t1);
  pair2 = __shfl_down_sync(0xffffffffu, pair, 2);
  float sq = __fadd_rn(pair, pair2);
  sq = __shfl_sync(0xffffffffu, sq, 0);
  for (int c = n8; c < d; c++) {
    const float a = __fsub_rn(row[c], mean);
    sq = __fadd_rn(sq, __fmul_rn(a, a));
  }
  var = __fdiv_rn(sq, (float)d);
}

// y = (x - mean) * inv * g + b in place (left to right, no fusion), inv = 1 / sqrt(var + 1e-5).
__device__ __forceinline__ void layer_norm_inplace(float* row, int d, const float* g, const float* b, int lane) {
  float mean, var;
  row_mean_var(row, d, lane, mean, var);
  __syncwarp();
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
  for (int k = lane; k < d; k += 32)
    row[k] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(row[k], mean), inv), __ldg(g + k)), __ldg(b + k));
  __syncwarp();
}

// One warp per row. Optional residual add first: x = fma(vs, v, x), the reference's AddScaled epilogue
// (kernels/mod.rs:42-48) applied to the GEMM output v, stored to x_res when given. Then an optional LayerNorm
// (g0, b0) whose f32 output is written to x_out (the encoder's norm_out, which produces the next layer's residual
// stream), then LayerNorm (g1, b1) -> quantise per group. With g1 == nullptr the row is quantised without a second
// LayerNorm.
__global__ void __launch_bounds__(WARPS * 32) ln_quant_kernel(const float* x, const float* v, float vs, float* x_res,
                                                               int n, int d, const float* g0, const float* b0,
                                                               float* x_out, const float* g1,
                                                               const float* b1, int group, int8_t* __restrict__ q,
                                                               float* __restrict__ scales, int vec) {
  extern __shared__ float srow[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* row = srow + (size_t)warp * d;
  const int ng = d / group;
  for (int t = blockIdx.x * WARPS + warp; t < n; t += gridDim.x * WARPS) {
    const float* xr = x + (size_t)t * d;
    if (vec) {
      for (int k = lane * 4; k < d; k += 128) *reinterpret_cast<float4*>(row + k) = *reinterpret_cast<const float4*>(xr + k);
    } else {
      for (int k = lane; k < d; k += 32) row[k] = xr[k];
    }
    if (v) {
      const float* vr = v + (size_t)t * d;
      for (int k = lane; k < d; k += 32) row[k] = __fmaf_rn(vs, vr[k], row[k]);
      if (x_res)
        for (int k = lane; k < d; k += 32) x_res[(size_t)t * d + k] = row[k];
    }
    __syncwarp();
    if (g0) {
      layer_norm_inplace(row, d, g0, b0, lane);
      if (x_out)
        for (int k = lane; k < d; k += 32) x_out[(size_t)t * d + k] = row[k];
    }
    if (g1) layer_norm_inplace(row, d, g1, b1, lane);
    if (q) {
      for (int gi = 0; gi < ng; gi++) {
        const float s = quantize_group_warp(row + gi * group, group, q + (size_t)t * d + gi * group, lane);
        if (lane == 0) scales[(size_t)t * ng + gi] = s;
      }
    }
    __syncwarp();
  }
}

// d = 128 NV, group 128: four rows per warp. The warp stages its four rows in shared memory (after the optional
// residual add), then every lane runs one of the reference's eight sum chains of one row (lane L: row L >> 3,
// chain L & 7; element 8m + c feeds chain c, in increasing m), so all 32 lanes carry chains and the four rows'
// chains run side by side; the eight chains of a row are combined inside their 8-lane segment in the reference's
// order, hsum4(chain[0..4] + chain[4..8]). Normalisation and quantisation then run row by row on all 32 lanes (a
// float4 per lane per 128 columns).
constexpr int LN4_WARPS = 4, LN4_ROWS = 4;

// Shared layout of a staged row r: logical float4 slot 32 j + l is stored at slot 32 j + (l ^ 2 r), i.e. element e at
// e ^ 8 r. A chain step of the four rows (lane L reads element 8 m + (L & 7) of row L >> 3) then lands in banks
// 8 ((m ^ r) mod 4) + c, all 32 distinct, while every float4 access of a row stays a permutation within its 128-float
// group (conflict-free) and the row pitch stays d floats.
template <int NV>
__device__ __forceinline__ float ln4_chain_sum(const float* row, int r, int c, bool var, float mean) {
  float chain = 0.0f;
#pragma unroll
  for (int b = 0; b < 16 * NV; b += 16) {
    float a[16];
#pragma unroll
    for (int k = 0; k < 16; k++) {
      const float xv = row[(((b + k) ^ r) << 3) + c];
      a[k] = var ? __fsub_rn(xv, mean) : xv;
    }
#pragma unroll
    for (int k = 0; k < 16; k++) chain = var ? __fmaf_rn(a[k], a[k], chain) : __fadd_rn(chain, a[k]);
  }
  // within the 8-lane segment (c = lane & 7): t4[c] = chain[c] + chain[c + 4]; (t0 + t1) + (t2 + t3) in c = 0
  const float t = __fadd_rn(chain, __shfl_down_sync(0xffffffffu, chain, 4));
  const float pair = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 1));
  const float sum = __fadd_rn(pair, __shfl_down_sync(0xffffffffu, pair, 2));
  return __shfl_sync(0xffffffffu, sum, (threadIdx.x & 31) & ~7);  // segment's lane 0
}

template <int NV>
__global__ void __launch_bounds__(LN4_WARPS * 32, 3) ln_quant_rows4_kernel(
    const float* x, const float* v, float vs, float* x_res, int n, const float* g0, const float* b0, float* x_out,
    const float* g1, const float* b1, int8_t* __restrict__ q, float* __restrict__ scales) {
  constexpr int D = 128 * NV;
  extern __shared__ __align__(16) float sm4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* rows = sm4 + (size_t)warp * LN4_ROWS * D;  // [4][D]
  const int my_r = lane >> 3, my_c = lane & 7;
  for (int t0 = (blockIdx.x * LN4_WARPS + warp) * LN4_ROWS; t0 < n; t0 += gridDim.x * LN4_WARPS * LN4_ROWS) {
    const int nr = ::min(LN4_ROWS, n - t0);
    // stage (residual add first), four rows, two at a time so their loads overlap
#pragma unroll 2
    for (int r = 0; r < nr; r++) {
      const size_t t = (size_t)(t0 + r);
      float4 xv[NV];
      const float4* xr = reinterpret_cast<const float4*>(x + t * D);
#pragma unroll
      for (int j = 0; j < NV; j++) xv[j] = xr[32 * j + lane];
      if (v) {
        const float4* vr = reinterpret_cast<const float4*>(v + t * D);
#pragma unroll
        for (int j = 0; j < NV; j++) {
          const float4 a = __ldg(vr + 32 * j + lane);
          xv[j] = make_float4(__fmaf_rn(vs, a.x, xv[j].x), __fmaf_rn(vs, a.y, xv[j].y), __fmaf_rn(vs, a.z, xv[j].z),
                              __fmaf_rn(vs, a.w, xv[j].w));
        }
        if (x_res)
#pragma unroll
          for (int j = 0; j < NV; j++) reinterpret_cast<float4*>(x_res + t * D)[32 * j + lane] = xv[j];
      }
#pragma unroll
      for (int j = 0; j < NV; j++) reinterpret_cast<float4*>(rows + r * D)[32 * j + (lane ^ (2 * r))] = xv[j];
    }
    __syncwarp();
    // one LayerNorm over the staged rows, in place; f32 result also to `out` when given
    auto norm = [&](const float* g, const float* b, float* out) {
      // every lane runs its chain (the shuffles need the whole warp); rows r >= nr of a tail group hold stale data
      // whose statistics are never used
      const float* row = rows + my_r * D;
      const float mean = __fdiv_rn(ln4_chain_sum<NV>(row, my_r, my_c, false, 0.0f), (float)D);
      const float var = __fdiv_rn(ln4_chain_sum<NV>(row, my_r, my_c, true, mean), (float)D);
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
      __syncwarp();
#pragma unroll 1
      for (int r = 0; r < nr; r++) {
        const float mr = __shfl_sync(0xffffffffu, mean, r * 8), ir = __shfl_sync(0xffffffffu, inv, r * 8);
        float4* rw = reinterpret_cast<float4*>(rows + r * D);
#pragma unroll
        for (int j = 0; j < NV; j++) {
          const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + 32 * j + lane);
          const float4 bb = __ldg(reinterpret_cast<const float4*>(b) + 32 * j + lane);
          float4 y = rw[32 * j + (lane ^ (2 * r))];
          y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.x, mr), ir), gg.x), bb.x);
          y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.y, mr), ir), gg.y), bb.y);
          y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.z, mr), ir), gg.z), bb.z);
          y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.w, mr), ir), gg.w), bb.w);
          rw[32 * j + (lane ^ (2 * r))] = y;
          if (out) reinterpret_cast<float4*>(out + (size_t)(t0 + r) * D)[32 * j + lane] = y;
        }
      }
      __syncwarp();
    };
    if (g0) norm(g0, b0, x_out);
    if (g1) norm(g1, b1, nullptr);
    if (q) {
      static_assert(NV == 8, "the reduce-scatter below assumes 8 groups per row");
#pragma unroll 1
      for (int r = 0; r < nr; r++) {
        const size_t t = (size_t)(t0 + r);
        const float4* rw = reinterpret_cast<const float4*>(rows + r * D);
        float4 y[NV];
        float m[NV];
#pragma unroll
        for (int j = 0; j < NV; j++) {
          y[j] = rw[32 * j + (lane ^ (2 * r))];
          m[j] = fmaxf(fmaxf(fabsf(y[j].x), fabsf(y[j].y)), fmaxf(fabsf(y[j].z), fabsf(y[j].w)));
        }
        // All eight group maxima at once (max is order-free, so exact): halve the groups held per lane at the
        // xor-16, 8 and 4 exchanges, then finish over xor 2 and 1; lane L ends with the maximum of group
        // 4 b4 + 2 b3 + b2 (bits of L), computes that group's scale and reciprocal, and the others fetch them.
        const int b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1;
        float m4[4], m2[2];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float send = b4 ? m[k] : m[k + 4];
          m4[k] = fmaxf(b4 ? m[k + 4] : m[k], __shfl_xor_sync(0xffffffffu, send, 16));
        }
#pragma unroll
        for (int k = 0; k < 2; k++) {
          const float send = b3 ? m4[k] : m4[k + 2];
          m2[k] = fmaxf(b3 ? m4[k + 2] : m4[k], __shfl_xor_sync(0xffffffffu, send, 8));
        }
        float g1v = fmaxf(b2 ? m2[1] : m2[0], __shfl_xor_sync(0xffffffffu, b2 ? m2[0] : m2[1], 4));
        g1v = fmaxf(g1v, __shfl_xor_sync(0xffffffffu, g1v, 2));
        g1v = fmaxf(g1v, __shfl_xor_sync(0xffffffffu, g1v, 1));
        const float my_sc = quant_scale(g1v);
        const float my_inv = __fdiv_rn(1.0f, my_sc);
        if ((lane & 3) == 0) scales[t * NV + 4 * b4 + 2 * b3 + b2] = my_sc;
#pragma unroll
        for (int j = 0; j < NV; j++) {
          const float inv = __shfl_sync(0xffffffffu, my_inv, 4 * j);  // lane 4 j holds group j
          const uint32_t w = ((uint32_t)quant_code(y[j].x, inv) & 0xFFu) |
                             (((uint32_t)quant_code(y[j].y, inv) & 0xFFu) << 8) |
                             (((uint32_t)quant_code(y[j].z, inv) & 0xFFu) << 16) |
                             (((uint32_t)quant_code(y[j].w, inv) & 0xFFu) << 24);
          reinterpret_cast<uint32_t*>(q + t * D)[32 * j + lane] = w;
        }
      }
    }
    __syncwarp();  // the rows are restaged by the next group
  }
}

}  // namespace quant
}  // namespace vxg

namespace vxg {

vxg_status ln_quant_run(const float* x, const float* v, float vs, float* x_res, int n, int d, const float* g0,
                        const float* b0, float* x_out, const float* g1, const float* b1, int group, int8_t* q,
                        float* scales, cudaStream_t stream) {
  VXG_ARG(x && n >= 0 && d > 0, "bad input");
  VXG_ARG(!q || (group > 0 && d % group == 0 && scales), "group must divide d and scales must be given");
  VXG_ARG((g0 == nullptr) == (b0 == nullptr) && (g1 == nullptr) == (b1 == nullptr), "gamma/beta pairs");
  VXG_ARG(!x_out || g0, "x_out needs the first LayerNorm");
  VXG_ARG(!x_res || v, "x_res needs the residual input");
  VXG_ARG(d <= 8192, "row width %d exceeds 8192", d);
  if (n == 0) return VXG_OK;
  const size_t smem = (size_t)quant::WARPS * d * sizeof(float);
  const int vec = (d % 4 == 0) && (((uintptr_t)x & 15) == 0);
  {
    const vxg_status sa = smem_attr((const void*)quant::ln_quant_kernel, quant::WARPS * 8192 * (int)sizeof(float));
    if (sa != VXG_OK) return sa;
  }
  const bool aligned = (((uintptr_t)x | (uintptr_t)v | (uintptr_t)x_res | (uintptr_t)x_out | (uintptr_t)q |
                         (uintptr_t)g0 | (uintptr_t)b0 | (uintptr_t)g1 | (uintptr_t)b1) & 15) == 0;
  if (d == 1024 && (!q || group == 128) && aligned) {
    constexpr int smem4 = quant::LN4_WARPS * quant::LN4_ROWS * 1024 * (int)sizeof(float);  // 64 KB
    const vxg_status sa = smem_attr((const void*)quant::ln_quant_rows4_kernel<8>, smem4);
    if (sa != VXG_OK) return sa;
    const int per_block = quant::LN4_WARPS * quant::LN4_ROWS;
    const int blocks = std::min((n + per_block - 1) / per_block, sm_count() * 3);  // three resident blocks per SM
    quant::ln_quant_rows4_kernel<8><<<blocks, quant::LN4_WARPS * 32, smem4, stream>>>(x, v, vs, x_res, n, g0, b0,
                                                                                       x_out, g1, b1, q, scales);
    note_launch();
    VXG_CUDA(cudaGetLastError());
    return VXG_OK;
  }
  const int blocks = std::min((n + quant::WARPS - 1) / quant::WARPS, sm_count() * 16);
  quant::ln_quant_kernel<<<blocks, quant::WARPS * 32, smem, stream>>>(x, v, vs, x_res, n, d, g0, b0, x_out, g1, b1,
                                                                      group, q, scales, vec);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

}  // namespace vxg

using namespace vxg;

extern "C" {

vxg_status vxg_ln_quant(const float* x, int n, int d, const float* g0, const float* b0, float* x_out,
                        const float* g1, const float* b1, int group, int8_t* q, float* scales, void* stream) {
  clear_error();
  return ln_quant_run(x, nullptr, 0.0f, nullptr, n, d, g0, b0, x_out, g1, b1, group, q, scales,
                      (cudaStream_t)stream);
}

vxg_status vxg_quantize_rows(const float* x, int n, int inp, int group, int8_t* q, float* scales, void* stream) {
  clear_error();
  VXG_ARG(q && scales, "NULL output");
  return vxg_ln_quant(x, n, inp, nullptr, nullptr, nullptr, nullptr, nullptr, group, q, scales, stream);
}

}  // extern "C"
