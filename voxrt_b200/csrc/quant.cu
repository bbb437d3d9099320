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

// Vectorised form for rows of 128 * NV floats quantised in groups of 128 (the encoder's d = 1024): lane l holds
// columns 128 j + 4 l .. + 3 as float4 j, so every load and store moves 512 contiguous bytes per warp and each
// 128-column quantisation group is one float4 per lane. The reference's 8-chain mean / variance order still runs on
// the row staged in shared memory; everything else (residual add, normalisation, quantisation) stays in registers
// with the same per-element operations as ln_quant_kernel.
template <int NV>
__global__ void __launch_bounds__(256, 2) ln_quant_vec_kernel(const float* x, const float* v, float vs, float* x_res,
                                                              int n, const float* g0, const float* b0, float* x_out,
                                                              const float* g1, const float* b1,
                                                              int8_t* __restrict__ q, float* __restrict__ scales) {
  constexpr int D = 128 * NV;
  __shared__ __align__(16) float srow[8][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* row = srow[warp];
  // Each warp walks rows t, t + stride, ...; the next row's x (and v) loads are issued before the current row's
  // sequential sum chains run, so the memory system stays busy while the warp computes. Rows are disjoint, so the
  // early load never reads a row this warp (or any other) is about to write.
  const int stride = gridDim.x * 8;
  float4 xn[NV], vn[NV];
  auto fetch = [&](int r) {
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)r * D);
#pragma unroll
    for (int j = 0; j < NV; j++) xn[j] = xr[32 * j + lane];
    if (v) {
      const float4* vr = reinterpret_cast<const float4*>(v + (size_t)r * D);
#pragma unroll
      for (int j = 0; j < NV; j++) vn[j] = __ldg(vr + 32 * j + lane);
    }
  };
  int t = blockIdx.x * 8 + warp;
  if (t < n) fetch(t);
  for (; t < n; t += stride) {
    float4 xv[NV];
#pragma unroll
    for (int j = 0; j < NV; j++) xv[j] = xn[j];
    if (v) {
#pragma unroll
      for (int j = 0; j < NV; j++) {
        const float4 a = vn[j];
        xv[j] = make_float4(__fmaf_rn(vs, a.x, xv[j].x), __fmaf_rn(vs, a.y, xv[j].y), __fmaf_rn(vs, a.z, xv[j].z),
                            __fmaf_rn(vs, a.w, xv[j].w));
      }
    }
    if (t + stride < n) fetch(t + stride);
    if (v) {
      if (x_res)
#pragma unroll
        for (int j = 0; j < NV; j++) reinterpret_cast<float4*>(x_res + (size_t)t * D)[32 * j + lane] = xv[j];
    }
    auto norm = [&](const float* g, const float* b) {
#pragma unroll
      for (int j = 0; j < NV; j++) reinterpret_cast<float4*>(row)[32 * j + lane] = xv[j];
      __syncwarp();
      float mean, var;
      row_mean_var(row, D, lane, mean, var);
      __syncwarp();
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
#pragma unroll
      for (int j = 0; j < NV; j++) {
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g) + 32 * j + lane);
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b) + 32 * j + lane);
        xv[j].x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[j].x, mean), inv), gg.x), bb.x);
        xv[j].y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[j].y, mean), inv), gg.y), bb.y);
        xv[j].z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[j].z, mean), inv), gg.z), bb.z);
        xv[j].w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv[j].w, mean), inv), gg.w), bb.w);
      }
    };
    if (g0) {
      norm(g0, b0);
      if (x_out)
#pragma unroll
        for (int j = 0; j < NV; j++) reinterpret_cast<float4*>(x_out + (size_t)t * D)[32 * j + lane] = xv[j];
    }
    if (g1) norm(g1, b1);
    if (q) {
#pragma unroll
      for (int j = 0; j < NV; j++) {
        float amax = fmaxf(fmaxf(fabsf(xv[j].x), fabsf(xv[j].y)), fmaxf(fabsf(xv[j].z), fabsf(xv[j].w)));
        amax = warp_max(amax);
        const float sc = quant_scale(amax);
        const float inv = __fdiv_rn(1.0f, sc);
        const uint32_t w = ((uint32_t)quant_code(xv[j].x, inv) & 0xFFu) |
                           (((uint32_t)quant_code(xv[j].y, inv) & 0xFFu) << 8) |
                           (((uint32_t)quant_code(xv[j].z, inv) & 0xFFu) << 16) |
                           (((uint32_t)quant_code(xv[j].w, inv) & 0xFFu) << 24);
        reinterpret_cast<uint32_t*>(q + (size_t)t * D)[32 * j + lane] = w;
        if (lane == 0) scales[(size_t)t * NV + j] = sc;
      }
    }
    __syncwarp();
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
    const int blocks = std::min((n + 7) / 8, sm_count() * 2);  // two resident blocks per SM, rows strided over them
    quant::ln_quant_vec_kernel<8><<<blocks, 256, 0, stream>>>(x, v, vs, x_res, n, g0, b0, x_out, g1, b1, q, scales);
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
