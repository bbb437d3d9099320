/*
 * CPU oracle for the ternary FastConformer encoder hot path of lmaksym/voxrt 0.2.1.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is compared against. Only the test
 * suite, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the product library (libvxg) never
 * links, loads or calls it, and has no CPU fallback.
 *
 * Every function restates the reference's own scalar ("portable") arithmetic in plain C++ with the same operation
 * order: Rust never contracts a*b+c, and every `mul_add` in the reference is an explicit fmaf() here. Build with
 * -ffp-contract=off -fno-fast-math. Citations are crates/voxrt/src/<file>:<line> of the reference.
 *
 * Pinning: the trit codec is pinned by the reference's real-weight fixtures and the LSD-first known answer; the
 * quantiser by the reference's tie cases; exp_poly by its f64 error bound; the GEMM by the overflow known answer and
 * by the AVX-512 VNNI restatement agreeing bit for bit (the reference's own kernel tests are SIMD == scalar tests and
 * store no GEMM outputs). The encoder-level composition (attention, conv module, subsampling) follows the reference
 * source but has no stored reference outputs here: its golden tensors and the model weights are absent, and the
 * reference (Rust) cannot be built in this image, so encoder-level parity is "unpinned" beyond these component pins.
 */
#ifndef VXG_ORACLE_H
#define VXG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- codec (trits.rs) ---- */
void vxo_unpack_row(const uint8_t* packed, int in_features, int8_t* out);
void vxo_pack_row(const int8_t* trits, int n, uint8_t* out);
float vxo_f16_to_f32(uint16_t h);
/* qweight [out, ceil(in/5)] + f16 scales [out, in/group] -> int8 rows [out, in] + f32 scales [out, in/group] */
void vxo_unpack_matrix(const uint8_t* qweight, const uint16_t* scales_f16, int out, int in, int group, int8_t* w,
                       float* scales);

/* ---- quantisation (packed.rs) ---- */
float vxo_quantize_group(const float* src, int n, int8_t* dst);
void vxo_quantize_rows(const float* x, int n, int inp, int group, int8_t* q, float* scales);
void vxo_layer_norm_row(const float* x, const float* g, const float* b, int d, float* y);
void vxo_ln_quant_rows(const float* x, int n, int d, const float* g, const float* b, int group, int8_t* q,
                       float* scales);

/* ---- GEMM (kernels/mod.rs) ---- */
enum { VXO_EP_STORE = 0, VXO_EP_SILU = 1, VXO_EP_ADD_SCALED = 2 };
/* y[t, o] (row stride N) for rows o in [r0, r1) and tokens t in [t0, t1); w int8 rows [N, K], sw [N, K/G],
 * x int8 [M, K], sx [M, K/G]. sums (optional) receives the int32 group sums [M, N, K/G]. bias (optional) is added
 * after the epilogue, as gemm_ep does. */
void vxo_gemm(const int8_t* w, const float* sw, const int8_t* x, const float* sx, int M, int N, int K, int G,
              int ep, float ep_scale, const float* bias, float* y, int32_t* sums, int r0, int r1, int t0, int t1);

/* ---- f32 helpers (tensor.rs) ---- */
float vxo_exp_poly(float x);
float vxo_silu_fast(float x);
float vxo_sigmoid_fast(float x);
void vxo_glu_rows(const float* g, int n, int d, float* a);
void vxo_vad_probs(const float* sub, int t, int d, int h, int k, const float* proj_w, const float* proj_b,
                   const float* ctx_w, const float* ctx_b, const float* out_w, float out_b, float* p);
int vxo_segment(const float* p, int t, float thr, int min_pause, int max_frames, int min_frames, int pad, int* out,
                int cap);
void vxo_math_cr(int fn, const float* x, size_t n, float* y);
float vxo_exp_row_scaled(float* row, int n, float scale);
void vxo_linear(const float* x, int n, int in_f, const float* w, const float* b, int out_f, float* y);

/* ---- encoder (encoder.rs) ---- */
typedef struct vxo_tern {
  const int8_t* w;    /* int8 rows [out, in] */
  const float* s;     /* f32 scales [out, in/group] */
  int out, in, group;
} vxo_tern;

typedef struct vxo_layer {
  vxo_tern ff1_1, ff1_2, qkv, o, relk, pw1, pw2, ff2_1, ff2_2;
  const float* ln_g[5]; /* norm_feed_forward1, norm_self_att, norm_conv, norm_feed_forward2, norm_out */
  const float* ln_b[5];
  const float* bias_u;  /* [h, dh] */
  const float* bias_v;
  const float* dw_w;    /* [k, d] tap-major, BatchNorm folded */
  const float* dw_b;    /* [d] folded shift */
} vxo_layer;

void vxo_rel_pos_table(int t, int d, float* out);
/* BatchNorm(eval) fold into the depthwise conv: dw [d, 1, k] -> tap-major [k, d] + shift [d] (encoder.rs:555-579) */
void vxo_fold_bn(const float* dw, const float* gamma, const float* beta, const float* mean, const float* var, int d,
                 int k, float* dw_t, float* dw_bias);
void vxo_attn_core_int8(const float* qkv, const float* rel_k, int t, int d, int h, int dh, const float* bias_u,
                        const float* bias_v, float scaling, float* ctx);
/* The same for the listed 8-row query blocks only (long-form parity on sampled rows); other ctx rows untouched. */
void vxo_attn_core_int8_rows(const float* qkv, const float* rel_k, int t, int d, int h, int dh, const float* bias_u,
                             const float* bias_v, float scaling, float* ctx, const int* blocks, int n_blocks);
/* Conv module middle: g [t, 2d] (pw1 output) -> hb [t, d] = SiLU(dwconv(GLU(g))) with folded BN weights. */
void vxo_conv_middle(const float* g, int t, int d, int k, const float* dw_w, const float* dw_b, float* hb);
/* One ConformerLayer::forward_profiled on x [t, d] in place (int8 path, int8 attention core, int8 context). */
void vxo_layer_forward(const vxo_layer* L, int d, int heads, int k, float* x, int t, const float* pos_emb);
/* The same with the weights repacked once up front (the reference repacks at load time). */
void* vxo_layer_prepare(const vxo_layer* L);
void vxo_layer_free(void* prep);
void vxo_layer_forward_prepared(void* prep, const vxo_layer* L, int d, int heads, int k, float* x, int t,
                                const float* pos_emb);

/* ---- subsampling (subsampling.rs) ---- */
typedef struct vxo_sub {
  int channels, kernel, stride, n_mels, d_model;
  const float* conv0_w; /* [k*k, C] tap-major */
  const float* conv0_b;
  const float* dw_w[2]; /* [k*k, C] */
  const float* dw_b[2];
  const float* pw_w[2]; /* [C, C] */
  const float* pw_b[2];
  const float* lin_w;   /* [d_model, F3*C], columns channels-last (f*C + c) */
  const float* lin_b;
} vxo_sub;
int vxo_sub_out_frames(int t, int k, int s);
void vxo_subsampling_forward(const vxo_sub* S, const float* feats, int t, float* out);

/* ---- TDT decoder, int8 mode (decoder.rs) ---- */
typedef struct vxo_tdt {
  int hidden, vocab, n_dur, blank, max_symbols, d_model, n_layers;
  const int* durations;      /* [n_dur] */
  const float* embedding;    /* [vocab, hidden] */
  const int8_t* w_ih[4];     /* int8 rows [4 hidden, hidden] (vxo_tdt_int8_rows) */
  const float* s_ih[4];      /* [4 hidden, hidden/128] */
  const int8_t* w_hh[4];
  const float* s_hh[4];
  const float* b[4];         /* b_ih + b_hh [4 hidden] */
  const uint16_t* proj_w;    /* decoder_projector f16 bits [hidden, hidden] */
  const float* proj_b;
  const int8_t* head_w;      /* joint head int8 rows [vocab + n_dur, hidden] */
  const float* head_s;
  const float* head_b;
  const float* enc_w;        /* encoder_projector f32 [hidden, d_model] */
  const float* enc_b;
} vxo_tdt;
void vxo_tdt_int8_rows(const uint16_t* w_f16, int out, int inp, int8_t* rows, float* scales);
void vxo_tdt_pred_step(const vxo_tdt* D, int token, const float* h_in, const float* c_in, float* g_out, float* h_out,
                       float* c_out);
void vxo_tdt_joint(const vxo_tdt* D, const float* enc_t, const float* g, float* logits);
void vxo_tdt_project(const vxo_tdt* D, const float* enc, int t, float* proj);
int vxo_tdt_greedy(const vxo_tdt* D, const float* proj, int t, int* tokens, int* frames, int* durs, int cap);

/* ---- threading for the timed CPU baseline: 0 = all hardware threads ---- */
void vxo_set_threads(int n);
int vxo_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
