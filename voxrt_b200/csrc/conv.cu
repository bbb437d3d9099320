// Conformer conv module middle: GLU -> depthwise conv over time (BatchNorm folded) -> SiLU -> int8 for pw2.
//
// Reference: ConvModule::forward_fused (crates/voxrt/src/encoder.rs:582-629) with glu_row_portable
// (tensor.rs:917-924: a * sigmoid_fast(b)), the tap loop (encoder.rs:608-623: r = dw_bias; for kk in 0..k:
// j = i + kk; if pad <= j < t + pad: r += w[kk] * a[j - pad], a plain multiply then add), silu_row_portable
// (tensor.rs:966-972) and quantize_group per 128 channels. BN fold: ConvModule::load (encoder.rs:546-579).
//
// One block per (utterance, 64-row tile, 128-channel slice): the GLU output of the tile plus its halo is staged
// in shared memory (coalesced float4 loads of both GLU halves), each thread owns one channel for the conv, and
// each warp then quantises whole 128-channel rows of the tile.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.h"
#include "internal.h"
#include "math.cuh"

namespace vxg {
namespace conv {

constexpr int TR = kConvTR;  // output rows per block
constexpr int TC = 128;   // channels per block (= quantisation group)
constexpr int MAXK = 15;  // largest supported kernel
constexpr int THREADS = 128;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// PRE: g already holds the GLU outputs (rows of d floats at stride ldg), computed by the pointwise_conv1 GEMM.
template <bool PRE>
__global__ void __launch_bounds__(THREADS) glu_dw_silu_quant_kernel(
    const float* __restrict__ g, int ldg, int d, const int* __restrict__ tile_utt, const int* __restrict__ tile_r0,
    const int* __restrict__ off, const int* __restrict__ len, const float* __restrict__ dw_w,
    const float* __restrict__ dw_b, int k, float* hb, int8_t* q, float* scales) {
  extern __shared__ float sm[];
  const int pad = (k - 1) / 2;
  const int halo = TR + k - 1;
  float* a_s = sm;                 // [halo][TC]  GLU outputs, rows r0 - pad ..
  float* h_s = sm + halo * TC;     // [TR][TC]    conv + SiLU outputs
  const int u = tile_utt[blockIdx.x], r0 = tile_r0[blockIdx.x], c0 = blockIdx.y * TC;
  const int t = len[u], base = off[u];
  const int rows = min(TR, t - r0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // GLU for rows j in [r0 - pad, r0 + rows + pad) inside the utterance (others are never read)
  for (int idx = tid; idx < halo * (TC / 4); idx += THREADS) {
    const int hr = idx / (TC / 4), c4 = (idx % (TC / 4)) * 4;
    const int j = r0 - pad + hr;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (j >= 0 && j < t && hr < rows + k - 1) {
      const float* gr = g + (size_t)(base + j) * ldg;
      const float4 ga = *reinterpret_cast<const float4*>(gr + c0 + c4);
      if constexpr (PRE) {
        v = ga;
      } else {
        const float4 gb = *reinterpret_cast<const float4*>(gr + d + c0 + c4);
        v.x = __fmul_rn(ga.x, sigmoid_fast(gb.x));
        v.y = __fmul_rn(ga.y, sigmoid_fast(gb.y));
        v.z = __fmul_rn(ga.z, sigmoid_fast(gb.z));
        v.w = __fmul_rn(ga.w, sigmoid_fast(gb.w));
      }
    }
    *reinterpret_cast<float4*>(a_s + hr * TC + c4) = v;
  }
  __syncthreads();
  {
    const int c = tid;  // one channel per thread
    float w[MAXK];
#pragma unroll
    for (int kk = 0; kk < MAXK; kk++) w[kk] = kk < k ? __ldg(dw_w + (size_t)kk * d + c0 + c) : 0.0f;
    const float bias = __ldg(dw_b + c0 + c);
    for (int r = 0; r < rows; r++) {
      const int i = r0 + r;
      float acc = bias;
#pragma unroll
      for (int kk = 0; kk < MAXK; kk++) {
        if (kk < k) {
          const int j = i + kk;  // padded index; input row j - pad
          if (j >= pad && j - pad < t) acc = __fadd_rn(acc, __fmul_rn(w[kk], a_s[(r + kk) * TC + c]));
        }
      }
      h_s[r * TC + c] = silu_fast(acc);
    }
  }
  __syncthreads();
  const int ng = d / TC;
  for (int r = warp; r < rows; r += THREADS / 32) {
    const float4 v = *reinterpret_cast<const float4*>(h_s + r * TC + lane * 4);
    const size_t row = (size_t)(base + r0 + r);
    if (hb) *reinterpret_cast<float4*>(hb + row * d + c0 + lane * 4) = v;
    if (q) {
      float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      amax = warp_max(amax);
      const float s = quant_scale(amax);
      const float inv = __fdiv_rn(1.0f, s);
      const uint32_t wq = ((uint32_t)quant_code(v.x, inv) & 0xFFu) | (((uint32_t)quant_code(v.y, inv) & 0xFFu) << 8) |
                          (((uint32_t)quant_code(v.z, inv) & 0xFFu) << 16) |
                          (((uint32_t)quant_code(v.w, inv) & 0xFFu) << 24);
      *reinterpret_cast<uint32_t*>(q + row * d + c0 + lane * 4) = wq;
      if (lane == 0) scales[row * ng + blockIdx.y] = s;
    }
  }
}

// Kernel size 9 (the model's): same arithmetic as above, reorganised.
//   * GLU: when every gate of a warp's four-channel chunk is > -85 the branch-free sigmoid runs (identical result),
//     otherwise sigmoid_fast.
//   * conv: 256 threads, two per channel: thread (c, half) slides a 9-value register window down rows
//     32 half .. 32 half + 31 of its channel, one shared load per output; interior tiles (every tap in range) skip
//     the per-tap range test.
//   * SiLU writes back over the GLU row it no longer needs, so the block holds one (64 + 8) x 128 tile (36 KB),
//     except rows 32 .. 39, whose GLU values the lower half still reads: those outputs go to an 8-row side
//     buffer (4 KB).
//   * quantisation: the shifter's low byte when the row maximum is 0 or normal, else quant_code.
constexpr int K9 = 9, P9 = 4, H9 = TR + K9 - 1;
constexpr int THREADS9 = 256, HALF9 = TR / 2;
constexpr int SMEM9 = (H9 + K9 - 1) * TC * 4;  // tile + halo, then the side rows HALF9 .. HALF9 + 7

template <bool PRE>
__global__ void __launch_bounds__(THREADS9) glu_dw9_silu_quant_kernel(
    const float* __restrict__ g, int ldg, int d, const int* __restrict__ tile_utt, const int* __restrict__ tile_r0,
    const int* __restrict__ off, const int* __restrict__ len, const float* __restrict__ dw_w,
    const float* __restrict__ dw_b, float* hb, int8_t* q, float* scales) {
  extern __shared__ float a_s[];  // [H9][TC]: GLU rows r0 - 4 .., then SiLU outputs in rows 0 .. rows - 1
  float* side = a_s + H9 * TC;    // [8][TC]: SiLU outputs of rows HALF9 .. HALF9 + 7
  const int u = tile_utt[blockIdx.x], r0 = tile_r0[blockIdx.x], c0 = blockIdx.y * TC;
  const int t = len[u], base = off[u];
  const int rows = min(TR, t - r0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if constexpr (PRE) {  // the GLU outputs themselves (zero outside the utterance), every load of the tile in flight
    constexpr int ITER = H9 * (TC / 4) / THREADS9;
    static_assert(H9 * (TC / 4) % THREADS9 == 0, "tile + halo must split evenly over the block");
    float4 gv[ITER];
#pragma unroll
    for (int it = 0; it < ITER; it++) {
      const int idx = tid + it * THREADS9, hr = idx / (TC / 4), c4 = (idx % (TC / 4)) * 4;
      const int j = r0 - P9 + hr;
      const bool in = j >= 0 && j < t && hr < rows + K9 - 1;
      gv[it] = in ? __ldg(reinterpret_cast<const float4*>(g + (size_t)(base + j) * ldg + c0 + c4))
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int it = 0; it < ITER; it++) {
      const int idx = tid + it * THREADS9;
      *reinterpret_cast<float4*>(a_s + (idx / (TC / 4)) * TC + (idx % (TC / 4)) * 4) = gv[it];
    }
  }
  for (int idx = tid; !PRE && idx < H9 * (TC / 4); idx += THREADS9) {
    const int hr = idx / (TC / 4), c4 = (idx % (TC / 4)) * 4;
    const int j = r0 - P9 + hr;
    const bool in = j >= 0 && j < t && hr < rows + K9 - 1;
    float4 ga = make_float4(0.f, 0.f, 0.f, 0.f), gb = ga;
    if (in) {
      const float* gr = g + (size_t)(base + j) * ldg;
      ga = *reinterpret_cast<const float4*>(gr + c0 + c4);
      gb = *reinterpret_cast<const float4*>(gr + d + c0 + c4);
    }
    const bool fast = !in || (gb.x > -85.0f && gb.y > -85.0f && gb.z > -85.0f && gb.w > -85.0f);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (__all_sync(0xffffffffu, fast)) {
      if (in) {
        v.x = __fmul_rn(ga.x, sigmoid_inrange(gb.x));
        v.y = __fmul_rn(ga.y, sigmoid_inrange(gb.y));
        v.z = __fmul_rn(ga.z, sigmoid_inrange(gb.z));
        v.w = __fmul_rn(ga.w, sigmoid_inrange(gb.w));
      }
    } else if (in) {
      v.x = __fmul_rn(ga.x, sigmoid_fast(gb.x));
      v.y = __fmul_rn(ga.y, sigmoid_fast(gb.y));
      v.z = __fmul_rn(ga.z, sigmoid_fast(gb.z));
      v.w = __fmul_rn(ga.w, sigmoid_fast(gb.w));
    }
    *reinterpret_cast<float4*>(a_s + hr * TC + c4) = v;
  }
  __syncthreads();
  {
    const int c = tid & (TC - 1), half = tid / TC;  // channel; rows HALF9 * half .. of the tile
    const int rb = half * HALF9, re = min(rb + HALF9, rows);
    float w[K9];
#pragma unroll
    for (int kk = 0; kk < K9; kk++) w[kk] = __ldg(dw_w + (size_t)kk * d + c0 + c);
    const float bias = __ldg(dw_b + c0 + c);
    const bool interior = r0 >= P9 && r0 + rows + P9 <= t;
    // taps of output row r (tile-relative) over the GLU rows win[o .. o + 8]
    auto conv_row = [&](const float (&win)[K9 + 1], int o, int r) -> float {
      float acc = bias;  // encoder.rs:608-623: r = bias; r += w[kk] * a[j - pad] for taps inside the utterance
      if (interior) {
#pragma unroll
        for (int kk = 0; kk < K9; kk++) acc = __fadd_rn(acc, __fmul_rn(w[kk], win[o + kk]));
      } else {
        const int i = r0 + r;
#pragma unroll
        for (int kk = 0; kk < K9; kk++)
          if (i + kk >= P9 && i + kk - P9 < t) acc = __fadd_rn(acc, __fmul_rn(w[kk], win[o + kk]));
      }
      return acc;
    };
    auto in_range = [](float a) { return fabsf(a) > 1e-30f && fabsf(a) < 1e30f && a > -85.0f; };
    // Two output rows per step (GLU rows r .. r + 9 in a register window), so SiLU runs on packed pairs; each
    // row's SiLU output overwrites its own GLU row, which no later row of its half reads (rows HALF9 .. + 7, which
    // the lower half reads, go to the side buffer).
    auto out_row = [&](int r) -> float* {
      return (half == 1 && r < HALF9 + K9 - 1) ? side + (r - HALF9) * TC + c : a_s + r * TC + c;
    };
    float win[K9 + 1];
#pragma unroll
    for (int kk = 0; kk < K9 - 1; kk++) win[kk + 2] = rb < rows ? a_s[(rb + kk) * TC + c] : 0.0f;
    int r = rb;
#pragma unroll 2
    for (; r + 1 < re; r += 2) {
#pragma unroll
      for (int kk = 0; kk < K9 - 1; kk++) win[kk] = win[kk + 2];
      win[K9 - 1] = a_s[(r + K9 - 1) * TC + c];
      win[K9] = a_s[(r + K9) * TC + c];
      float a0 = conv_row(win, 0, r), a1 = conv_row(win, 1, r + 1);
      if (__all_sync(0xffffffffu, in_range(a0) && in_range(a1))) {
        silu2_inrange(a0, a1);
      } else {
        a0 = silu_fast(a0);
        a1 = silu_fast(a1);
      }
      *out_row(r) = a0;
      *out_row(r + 1) = a1;
    }
    if (r < re) {  // odd row count: the last row alone
#pragma unroll
      for (int kk = 0; kk < K9 - 1; kk++) win[kk] = win[kk + 2];
      win[K9 - 1] = a_s[(r + K9 - 1) * TC + c];
      const float a0 = conv_row(win, 0, r);
      *out_row(r) = __all_sync(0xffffffffu, in_range(a0)) ? silu_inrange(a0) : silu_fast(a0);
    }
  }
  __syncthreads();
  const int ng = d / TC;
  for (int r = warp; r < rows; r += THREADS9 / 32) {
    const float* src = (r >= HALF9 && r < HALF9 + K9 - 1) ? side + (r - HALF9) * TC : a_s + r * TC;
    const float4 v = *reinterpret_cast<const float4*>(src + lane * 4);
    const size_t row = (size_t)(base + r0 + r);
    if (hb) *reinterpret_cast<float4*>(hb + row * d + c0 + lane * 4) = v;
    if (q) {
      const float amax = warp_max(fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      const float s = quant_scale(amax);
      const float inv = __fdiv_rn(1.0f, s);
      uint32_t wq;
      if (amax == 0.0f || amax >= 2e-36f) {  // uniform across the warp (one row)
        wq = quant_byte_fast(v.x, inv) | (quant_byte_fast(v.y, inv) << 8) | (quant_byte_fast(v.z, inv) << 16) |
             (quant_byte_fast(v.w, inv) << 24);
      } else {
        wq = ((uint32_t)quant_code(v.x, inv) & 0xFFu) | (((uint32_t)quant_code(v.y, inv) & 0xFFu) << 8) |
             (((uint32_t)quant_code(v.z, inv) & 0xFFu) << 16) | (((uint32_t)quant_code(v.w, inv) & 0xFFu) << 24);
      }
      *reinterpret_cast<uint32_t*>(q + row * d + c0 + lane * 4) = wq;
      if (lane == 0) scales[row * ng + blockIdx.y] = s;
    }
  }
}

}  // namespace conv
}  // namespace vxg

using namespace vxg;

namespace vxg {

vxg_status conv_run(const BatchPlan& b, const int* dtab, const float* g, int ld_g, const float* dw_t,
                    const float* dw_bias, int d, int k, float* hb, int8_t* q, float* scales, cudaStream_t st,
                    bool glu_done) {
  VXG_ARG(d % conv::TC == 0 && k >= 1 && k <= conv::MAXK && k % 2 == 1, "d %% 128 == 0 and odd k <= 15 required");
  VXG_ARG(ld_g >= (glu_done ? d : 2 * d) && ld_g % 4 == 0 && ((uintptr_t)g & 15) == 0,
          "g rows must hold %d floats, 16B aligned", glu_done ? d : 2 * d);
  VXG_ARG(hb || (q && scales), "no output requested");
  if (k == conv::K9) {
    const void* kfn = glu_done ? (const void*)conv::glu_dw9_silu_quant_kernel<true>
                               : (const void*)conv::glu_dw9_silu_quant_kernel<false>;
    vxg_status sa = smem_attr(kfn, conv::SMEM9);
    if (sa != VXG_OK) return sa;
    const dim3 grid(b.conv_tiles, d / conv::TC);
    if (glu_done)
      conv::glu_dw9_silu_quant_kernel<true><<<grid, conv::THREADS9, conv::SMEM9, st>>>(
          g, ld_g, d, dtab + b.o_conv_u, dtab + b.o_conv_r, dtab + b.o_off, dtab + b.o_len, dw_t, dw_bias, hb, q,
          scales);
    else
      conv::glu_dw9_silu_quant_kernel<false><<<grid, conv::THREADS9, conv::SMEM9, st>>>(
          g, ld_g, d, dtab + b.o_conv_u, dtab + b.o_conv_r, dtab + b.o_off, dtab + b.o_len, dw_t, dw_bias, hb, q,
          scales);
    note_launch();
    VXG_CUDA(cudaGetLastError());
    return VXG_OK;
  }
  const size_t smem = (size_t)((conv::TR + k - 1) + conv::TR) * conv::TC * sizeof(float);
  const void* kfn = glu_done ? (const void*)conv::glu_dw_silu_quant_kernel<true>
                             : (const void*)conv::glu_dw_silu_quant_kernel<false>;
  vxg_status sa = smem_attr(kfn, (int)(((conv::TR + conv::MAXK - 1) + conv::TR) * conv::TC * sizeof(float)));
  if (sa != VXG_OK) return sa;
  const dim3 grid(b.conv_tiles, d / conv::TC);
  if (glu_done)
    conv::glu_dw_silu_quant_kernel<true><<<grid, conv::THREADS, smem, st>>>(
        g, ld_g, d, dtab + b.o_conv_u, dtab + b.o_conv_r, dtab + b.o_off, dtab + b.o_len, dw_t, dw_bias, k, hb, q,
        scales);
  else
    conv::glu_dw_silu_quant_kernel<false><<<grid, conv::THREADS, smem, st>>>(
        g, ld_g, d, dtab + b.o_conv_u, dtab + b.o_conv_r, dtab + b.o_off, dtab + b.o_len, dw_t, dw_bias, k, hb, q,
        scales);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return VXG_OK;
}

}  // namespace vxg

extern "C" {

vxg_status vxg_fold_bn(const float* dw, const float* gamma, const float* beta, const float* mean, const float* var,
                       int d, int k, float* dw_t, float* dw_bias) {
  clear_error();
  VXG_ARG(dw && gamma && beta && mean && var && dw_t && dw_bias && d > 0 && k > 0, "bad arguments");
  for (int c = 0; c < d; c++) {  // encoder.rs:555-570, f32 arithmetic in the reference's order
    volatile float vs = var[c] + 1e-5f;
    const float s = gamma[c] / std::sqrt((float)vs);
    for (int kk = 0; kk < k; kk++) dw_t[(size_t)kk * d + c] = dw[(size_t)c * k + kk] * s;
    volatile float ms = mean[c] * s;
    dw_bias[c] = beta[c] - (float)ms;
  }
  return VXG_OK;
}

size_t vxg_conv_workspace_bytes(int rows, int n_utt) {
  if (rows <= 0 || n_utt <= 0) return 0;
  return (size_t)(3 * n_utt + 2 * (rows / kAttnBQ + n_utt) + 2 * (rows / conv::TR + n_utt)) * sizeof(int);
}

vxg_status vxg_conv_glu_dw_silu_quant(const float* g, int ld_g, const int* off, const int* len, int n_utt,
                                      const float* dw_t, const float* dw_bias, int d, int k, float* hb, int8_t* q,
                                      float* scales, void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  VXG_ARG(g && off && len && dw_t && dw_bias && workspace && n_utt > 0, "NULL pointer or empty batch");
  int expect = 0, tmax = 1;
  for (int u = 0; u < n_utt; u++) {
    VXG_ARG(len[u] > 0 && off[u] == expect, "utterances must be stacked in order (utterance %d)", u);
    expect += len[u];
    tmax = std::max(tmax, len[u]);
  }
  BatchPlan b;
  batch_plan(b, len, n_utt, tmax);
  if (ws_bytes < b.tab.size() * sizeof(int)) {
    set_error("workspace too small: %zu < %zu bytes", ws_bytes, b.tab.size() * sizeof(int));
    return VXG_ERR_ARG;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int* dtab = static_cast<int*>(workspace);
  VXG_CUDA(cudaMemcpyAsync(dtab, b.tab.data(), b.tab.size() * sizeof(int), cudaMemcpyHostToDevice, st));
  return conv_run(b, dtab, g, ld_g, dw_t, dw_bias, d, k, hb, q, scales, st);
}

// ------------------------------------------------------------------------------------------ allocation-free form
// Some callers cannot allocate device memory when they run the conv module: a serving process that sizes every
// buffer at start-up and runs under a hard device-memory budget shared with other tenants, and a streaming engine
// on a latency deadline, where cudaMalloc/cudaFree would synchronise with work in flight. They also may not own an
// allocator to hand us a workspace. This form keeps its index tables in a fixed static device array instead of a
// caller workspace; the batch must fit that array.
//
// The tables are built on the device: the utterance lengths travel by value in the build kernel's parameters, and
// that kernel writes the array. No host-side staging buffer is involved, so nothing the call leaves behind on the
// host is read later by the GPU.
constexpr int kStaticTabInts = 16384;  // 64 KB: off, len and two ints per 64-row tile
constexpr int kStaticMaxUtt = 1000;    // utterance lengths passed by value: 4 KB of kernel parameters

static __device__ __align__(256) int g_conv_static_tab[kStaticTabInts];

struct StaticLens {
  int n;
  int len[kStaticMaxUtt];
};

// [off n][len n][tile utterance tiles][tile first row tiles], the layout conv_run reads from a BatchPlan. Every
// entry the conv kernel reads is written here, so nothing in the array has to start at zero.
__global__ void __launch_bounds__(1024) build_static_tab_kernel(const StaticLens a, int tiles) {
  __shared__ int s_off[kStaticMaxUtt], s_tile[kStaticMaxUtt];
  const int n = a.n;
  if (threadIdx.x == 0) {
    int off = 0, t = 0;
    for (int u = 0; u < n; u++) {
      s_off[u] = off;
      s_tile[u] = t;
      off += a.len[u];
      t += (a.len[u] + conv::TR - 1) / conv::TR;
    }
  }
  __syncthreads();
  int* tab = g_conv_static_tab;
  for (int u = threadIdx.x; u < n; u += blockDim.x) {
    const int l = a.len[u];
    tab[u] = s_off[u];
    tab[n + u] = l;
    for (int r = 0, t = s_tile[u]; r < l; r += conv::TR, t++) {
      tab[2 * n + t] = u;
      tab[2 * n + tiles + t] = r;
    }
  }
}

static std::mutex g_static_mu;  // guards the per-device set-up below
static int* g_static_dev[64];   // device address of g_conv_static_tab, per device, found at set-up

}  // extern "C"

extern "C" vxg_status vxg_conv_glu_dw_silu_quant_static(const float* g, int ld_g, const int* off, const int* len,
                                                         int n_utt, const float* dw_t, const float* dw_bias, int d,
                                                         int k, float* hb, int8_t* q, float* scales, void* stream) {
  clear_error();
  VXG_ARG(g && off && len && dw_t && dw_bias && n_utt > 0, "NULL pointer or empty batch");
  if (n_utt > kStaticMaxUtt) {
    set_error("batch of %d utterances; the allocation-free conv entry takes at most %d", n_utt, kStaticMaxUtt);
    return VXG_ERR_ARG;
  }
  long need = 2L * n_utt;
  int expect = 0, tiles = 0;
  for (int u = 0; u < n_utt; u++) {
    VXG_ARG(len[u] > 0 && off[u] == expect, "utterances must be stacked in order (utterance %d)", u);
    expect += len[u];
    tiles += (len[u] + conv::TR - 1) / conv::TR;
  }
  need += 2L * tiles;
  if (need > kStaticTabInts) {
    set_error("batch needs %ld index entries (2 per utterance + 2 per %d-row tile); the static table holds %d",
              need, conv::TR, kStaticTabInts);
    return VXG_ERR_ARG;
  }
  int dev = 0;
  VXG_CUDA(cudaGetDevice(&dev));
  VXG_ARG(dev >= 0 && dev < 64, "device ordinal %d out of range", dev);
  int* dtab = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_dev[dev]) {  // set-up, once per device, with that device current
      void* p = nullptr;
      VXG_CUDA(cudaGetSymbolAddress(&p, g_conv_static_tab));
      g_static_dev[dev] = static_cast<int*>(p);
    }
    dtab = g_static_dev[dev];
  }
  BatchPlan b;
  b.n_utt = n_utt;
  b.rows = expect;
  b.conv_tiles = tiles;
  b.o_off = 0;
  b.o_len = n_utt;
  b.o_conv_u = 2 * n_utt;
  b.o_conv_r = 2 * n_utt + tiles;
  StaticLens a;
  a.n = n_utt;
  std::memcpy(a.len, len, (size_t)n_utt * sizeof(int));
  cudaStream_t st = (cudaStream_t)stream;
  build_static_tab_kernel<<<1, 1024, 0, st>>>(a, tiles);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  return conv_run(b, dtab, g, ld_g, dw_t, dw_bias, d, k, hb, q, scales, st);
}
