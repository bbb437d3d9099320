// Internal launchers shared by the C ABI wrappers and the encoder. A batch of utterances is stacked along the
// token axis; its index tables are built once on the host (batch_plan) and uploaded once per forward, so the
// per-layer launches take device pointers only.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "common.h"

namespace vxg {

struct BatchPlan {
  int n_utt = 0, rows = 0, tmax = 0;
  int Mv = 0;  // columns of the transposed V: sum of 16-padded lengths
  int att_tiles = 0, conv_tiles = 0;
  std::vector<int> tab;  // [off U][len U][voff U][att_u T][att_q T][conv_u C][conv_r C]
  // int offsets of each table inside `tab` (and inside its device copy)
  int o_off = 0, o_len = 0, o_voff = 0, o_att_u = 0, o_att_q = 0, o_conv_u = 0, o_conv_r = 0;
};

// q|k|v projection with the attention's per-head int8 operands produced in the epilogue: for the q heads
// Qu = quant(q + bias_u) and Qv = quant(q + bias_v), for the k heads K = quant(k), one group per (row, head), laid
// out [head][row][128] with scales [head][row]; the v heads are stored as f32 into y as usual.
constexpr int kGemmQKQuant = 17;
struct QkQuant {
  const float* bu = nullptr;  // bias_u, bias_v [heads][128]
  const float* bv = nullptr;
  int8_t *qu = nullptr, *qv = nullptr, *kh = nullptr;
  float *squ = nullptr, *sqv = nullptr, *sk = nullptr;
  int heads = 0;
};

constexpr int kAttnBQ = 128;  // attention query rows per CTA
constexpr int kConvTR = 64;   // conv-module rows per block

// Tables for utterances of the given lengths stacked in order; tmax >= max(len).
void batch_plan(BatchPlan& b, const int* len, int n, int tmax);

// Attention: workspace layout for a plan, and the launch (prep kernels + core) with device tables `dtab`.
size_t attention_ws_bytes(int rows, int tmax, int n_utt, int heads, int Mv);
// qk_ready: the per-head int8 Q / K (and their scales) are already in the workspace at attention_qk_buffers(),
// produced by the q|k|v GEMM's kGemmQKQuant epilogue; the Q / K preparation pass is then skipped.
vxg_status attention_run(const BatchPlan& b, const int* dtab, const float* qkv, int ld_qkv, const float* rel_k,
                         const float* bias_u, const float* bias_v, int heads, float scaling, float* ctx,
                         int8_t* ctx_q, float* ctx_s, void* workspace, size_t ws_bytes, cudaStream_t st,
                         bool qk_ready = false);
QkQuant attention_qk_buffers(const BatchPlan& b, int heads, void* workspace);

// Conv module middle with device tables.
// glu_done: g already holds the GLU outputs [rows][d] (the pointwise_conv1 GEMM's kGemmGlu epilogue), so the
// kernel reads them instead of computing a * sigmoid(b) from the [rows][2d] projection.
vxg_status conv_run(const BatchPlan& b, const int* dtab, const float* g, int ld_g, const float* dw_t,
                    const float* dw_bias, int d, int k, float* hb, int8_t* q, float* scales, cudaStream_t st,
                    bool glu_done = false);

// Ternary GEMM (2-bit codes or int8-resident weights). `ep` is a vxg_epilogue or kGemmSiluQuant, the fused
// SiLU -> per-(row, 128 columns) int8 epilogue that writes q [M, N] and q_scales [M, N/128] instead of y.
constexpr int kGemmSiluQuant = 16;
// pointwise_conv1 with the GLU fused: the weight rows are interleaved by glu_interleave_row (each 128-row tile holds
// 64 value channels and their 64 gates, 16 + 16 per 32-row slice), and the epilogue writes glu(a, b) = a *
// sigmoid_fast(b) as y [M, N/2] instead of the N columns.
constexpr int kGemmGlu = 18;
// Source row (in the reference's order: N/2 value channels, then N/2 gates) of interleaved row r.
inline int glu_interleave_row(int r, int n_half) {
  const int j = r / 128, cs = (r / 32) % 4, h = (r / 16) % 2, i = r % 16;
  return h * n_half + 64 * j + 16 * cs + i;
}

// Largest K for which the GEMM keeps a tile's weight slab resident in shared memory (2-bit codes are unpacked once
// per slab); larger K streams int8 weight chunks.
constexpr int kGemmResidentK = 1024;
vxg_status gemm_launch(bool packed, const int8_t* x, const float* sx, const void* w, const float* scales_t, int M,
                       int N, int K, int G, int ep, float ep_scale, const float* bias, float* y, int8_t* q,
                       float* q_scales, int32_t* group_sums, cudaStream_t st, const QkQuant* qk = nullptr);

// Residual add (x = fma(vs, v, x), stored to x_res when given) -> optional LayerNorm (g0, b0) stored to x_out ->
// optional LayerNorm (g1, b1) -> per-group int8. v == nullptr skips the add.
vxg_status ln_quant_run(const float* x, const float* v, float vs, float* x_res, int n, int d, const float* g0,
                        const float* b0, float* x_out, const float* g1, const float* b1, int group, int8_t* q,
                        float* scales, cudaStream_t stream);

// f32 linear in the reference's lane order (M >= 2).
vxg_status linear_lanes(const float* x, const float* w, const float* bias, float* y, int M, int N, int K, int relu,
                        cudaStream_t st);

}  // namespace vxg
