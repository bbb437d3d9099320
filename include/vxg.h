/*
 * vxg: B200 (sm_100a) kernels for the ternary FastConformer encoder of lmaksym/voxrt 0.2.1, behind a C ABI.
 *
 * Conventions (mirroring the reference FFI, crates/voxrt-ffi/src/lib.rs:61-110):
 *   - every entry point returns a vxg_status; on failure a message is kept per thread in vxg_last_error();
 *   - nothing aborts or traps: device-side waits are bounded and report VXG_ERR_TIMEOUT through vxg_device_status;
 *   - no torch or CUDA types in the signatures: device buffers are plain pointers, a stream is a `void*`
 *     (a cudaStream_t, NULL for the legacy default stream);
 *   - "device" pointers must be CUDA device memory on the current device; "host" pointers are host memory.
 */
#ifndef VXG_H
#define VXG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum vxg_status {
  VXG_OK = 0,
  VXG_ERR_ARG = 1,         /* invalid argument (shape, alignment, NULL) */
  VXG_ERR_CUDA = 2,        /* CUDA runtime / driver error */
  VXG_ERR_TIMEOUT = 3,     /* a kernel's bounded wait expired (see vxg_device_status) */
  VXG_ERR_OOM = 4,         /* device allocation failed */
  VXG_ERR_UNSUPPORTED = 5, /* shape or device the kernels do not cover */
} vxg_status;

/* Epilogue applied at every output store: kernels/mod.rs:14-49 `enum Epilogue`. */
typedef enum vxg_epilogue {
  VXG_EP_STORE = 0,      /* y = v */
  VXG_EP_SILU = 1,       /* y = silu_fast(v) */
  VXG_EP_ADD_SCALED = 2, /* y = fma(scale, v, y): residual add into a pre-filled y */
} vxg_epilogue;

/* Last error message on this thread ("" if none); replaces voxrt_last_error (crates/voxrt-ffi/src/lib.rs:70). */
const char* vxg_last_error(void);

/* Library version; replaces voxrt_version (crates/voxrt-ffi/src/lib.rs:76). */
const char* vxg_version(void);

/* Synchronise the current device, return its device status word in *code (0 = no kernel reported a problem;
 * nonzero = a bounded wait expired, code identifies the role) and clear it. No reference counterpart: the
 * reference's CPU kernels cannot time out. */
vxg_status vxg_device_status(int* code);

/* ---------------------------------------------------------------------------------------- ternary weights
 * Load-time repack of one thrush-ternary-v2 module (5 base-3 digits per byte, LSD first, code = trit + 1;
 * f16 scale per (row, group)) into the device format the GEMM reads: 2-bit codes tiled per 128 output rows and
 * 128 input columns, and f32 scales tile-major [out_pad/128][in/group][128]. Host to host; upload with cudaMemcpy.
 * Replaces TernaryMatrix::from_packed_layout (crates/voxrt/src/packed.rs:73-130) + finish (:132-161). */
size_t vxg_ternary_codes_bytes(int out, int in);             /* bytes of `codes` */
size_t vxg_ternary_scales_count(int out, int in, int group); /* floats of `scales_t` */
int vxg_ternary_out_pad(int out);                           /* out rounded up to the 128-row tile */
vxg_status vxg_ternary_repack(const uint8_t* qweight, const uint16_t* scales_f16, int out, int in, int group,
                              uint8_t* codes, float* scales_t);

/* ------------------------------------------------------------------------------------------ ternary GEMM
 * y[t, o] = ep(Σ_g fma(float(S_g[t, o]), sx[t, g] * sw[o, g], acc)) (+ bias[o]) for t < M, o < N, where
 * S_g = Σ_{c in group g} w[o, c] x[t, c] exactly in int32: tcgen05.mma kind::i8 with per-group TMEM accumulators.
 * Bit-identical to gemm_scalar_range / the x86 kernels. Replaces kernels::gemm_ep (crates/voxrt/src/kernels/
 * mod.rs:324-362) and gemm_rows_range's full-range form (:257-282).
 *   x [M, K] int8 (device, 16-byte aligned, row stride K), sx [M, K/G] f32 (device),
 *   codes / scales_t from vxg_ternary_repack (device), bias [N] or NULL, y [M, N] f32 (device; read first for
 *   ADD_SCALED), group_sums [M, N, K/G] int32 or NULL (device; the exact integer sums, for parity checks).
 *   K and G multiples of 128, K a multiple of G, K/G <= 32, K <= 32768 (else VXG_ERR_UNSUPPORTED). */
vxg_status vxg_gemm_ternary_i8(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t, int M,
                               int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias, float* y,
                               int32_t* group_sums, void* stream);

/* The same GEMM with int8-resident weights (no in-SM unpack; 4x the weight bytes): w_rows [out_pad, in] int8 and
 * scales_t (tile-major, as above) from vxg_ternary_repack_i8. Bit-identical to vxg_gemm_ternary_i8. Replaces the
 * same reference interfaces (kernels/mod.rs:324-362) for a CPU layout choice the reference also makes
 * (Layout::Rows vs Layout::Packed2, packed.rs:8-27). */
size_t vxg_ternary_i8_bytes(int out, int in); /* bytes of `w_rows` = out_pad * in */
vxg_status vxg_ternary_repack_i8(const uint8_t* qweight, const uint16_t* scales_f16, int out, int in, int group,
                                 int8_t* w_rows, float* scales_t);
vxg_status vxg_gemm_ternary_i8w(const int8_t* x, const float* sx, const int8_t* w_rows, const float* scales_t,
                                int M, int N, int K, int G, vxg_epilogue ep, float ep_scale, const float* bias,
                                float* y, int32_t* group_sums, void* stream);

/* Feed-forward linear1 with its consumers fused: y = silu_fast(GEMM) is quantised per (row, 128 columns) for
 * linear2 straight from the accumulators, so only q [M, N] int8 and q_scales [M, N/128] f32 reach memory.
 * Bit-identical to vxg_gemm_ternary_i8 with VXG_EP_SILU followed by vxg_quantize_rows(group 128). N % 128 == 0,
 * q 16-byte aligned. Replaces the Silu GEMM + QuantAct::quantize pair in FeedForward::forward_fused
 * (crates/voxrt/src/encoder.rs:79-94). The _w form takes int8-resident weights. */
vxg_status vxg_gemm_ternary_silu_q(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t,
                                   int M, int N, int K, int G, int8_t* q, float* q_scales, void* stream);
vxg_status vxg_gemm_ternary_silu_q_w(const int8_t* x, const float* sx, const int8_t* w_rows, const float* scales_t,
                                     int M, int N, int K, int G, int8_t* q, float* q_scales, void* stream);

/* Stacked q|k|v projection (N = 3 * heads * 128, 2-bit codes) with the attention's per-head int8 operands made in
 * the epilogue: Qu = quant(q + bias_u), Qv = quant(q + bias_v), K = quant(k), one 128-wide group per (row, head),
 * codes [heads][M][128] (16-byte aligned) and scales [heads][M]; the v columns are stored as f32 into y [M, N]
 * (columns 2 * heads * 128 .. N; the q and k columns of y are not written). Bit-identical to the Store GEMM followed
 * by the reference's per-head quantisation. Replaces the qkv gemm + quant_rows / from_f32_rows steps of
 * Attention::forward_fused and attn_core_int8 (crates/voxrt/src/encoder.rs:138-187, :349-377). */
vxg_status vxg_gemm_ternary_qkv_quant(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t,
                                      int M, int heads, int K, int G, const float* bias_u, const float* bias_v,
                                      int8_t* qu, int8_t* qv, int8_t* kh, float* squ, float* sqv, float* sk, float* y,
                                      void* stream);

/* pointwise_conv1 with the GLU in the epilogue: y [M, N/2] = a * sigmoid_fast(b) (glu_row, crates/voxrt/src/
 * tensor.rs:936-940) of the projection's value half a and gate half b. The weights must be repacked with their
 * rows permuted: row r of the repacked module is row vxg_glu_source_row(r, N) of the reference's [value; gate]
 * order (every 128-row tile then holds 64 channels and their 64 gates). N % 128 == 0, y 32-byte aligned.
 * Replaces the pw1 gemm + glu_row pair of ConvModule::forward_fused (encoder.rs:594-596). */
int vxg_glu_source_row(int r, int n);
vxg_status vxg_gemm_ternary_glu(const int8_t* x, const float* sx, const uint8_t* codes, const float* scales_t, int M,
                                int N, int K, int G, float* y, void* stream);

/* ------------------------------------------------------------------------------------------- quantisation
 * Per-(token, group) symmetric int8: scale = absmax/127 (1 for an all-zero group), code = clamp(round_ties_even(
 * v / scale as v * (1/scale)), +-127). x [n, inp] f32 -> q [n, inp] int8 + scales [n, inp/group] (all device).
 * Replaces QuantAct::quantize / quantize_layout (crates/voxrt/src/packed.rs:302-312, quantize_group :527-535). */
vxg_status vxg_quantize_rows(const float* x, int n, int inp, int group, int8_t* q, float* scales, void* stream);

/* Fused LayerNorm -> int8 (eps 1e-5, biased variance, the reference's 8-chain reduction order). Optional first
 * LayerNorm (g0, b0) whose f32 output is stored to x_out (may equal x) -- the encoder's norm_out feeding the next
 * layer -- then LayerNorm (g1, b1) and quantisation per `group`. g1 == NULL skips the second LayerNorm; q == NULL
 * skips quantisation. d <= 8192. Replaces TernaryLinear::prepare_normed (crates/voxrt/src/ternary_linear.rs:
 * 132-158) with layer_norm_row (tensor.rs:712-719), and LayerNormP::forward for norm_out (encoder.rs:60-62). */
vxg_status vxg_ln_quant(const float* x, int n, int d, const float* g0, const float* b0, float* x_out,
                        const float* g1, const float* b1, int group, int8_t* q, float* scales, void* stream);

/* --------------------------------------------------------------------------------------- int8 attention
 * Relative-position MHSA core on int8 scores for a batch of utterances stacked along the token axis: utterance u
 * occupies rows [off[u], off[u] + len[u]) of qkv (row stride ld_qkv floats, q | k | v of heads * 128 each) and
 * uses rows [tmax - len[u], tmax + len[u] - 1) of the shared relative table rel_k [2 * tmax - 1, heads * 128]
 * (positions tmax-1 .. -(tmax-1), the relative_k_proj output). Outputs, per token and head: the f32 context
 * ctx [rows, heads * 128] and/or its per-head int8 quantisation ctx_q + ctx_s [rows, heads] (the output
 * projection's input). off/len are host arrays; workspace is caller-owned device memory of at least
 * vxg_attention_workspace_bytes(). Bit-identical to attn_core_int8 (crates/voxrt/src/encoder.rs:317-534), which
 * it replaces together with the per-head operand quantisation of Attention::forward_fused (encoder.rs:138-187).
 * head_dim must be 128. */
size_t vxg_attention_workspace_bytes(int rows, int tmax, int n_utt, int heads);
vxg_status vxg_attention_i8(const float* qkv, int ld_qkv, const float* rel_k, int tmax, const int* off,
                            const int* len, int n_utt, const float* bias_u, const float* bias_v, int heads,
                            int head_dim, float scaling, float* ctx, int8_t* ctx_q, float* ctx_s, void* workspace,
                            size_t ws_bytes, void* stream);

/* ------------------------------------------------------------------------------------------- conv module
 * BatchNorm(eval) folded into the bias-free depthwise conv, host to host: dw [d, 1, k] -> tap-major dw_t [k, d]
 * and dw_bias [d] (f32, the reference's arithmetic order). Replaces ConvModule::load (encoder.rs:546-579). */
vxg_status vxg_fold_bn(const float* dw, const float* gamma, const float* beta, const float* mean, const float* var,
                       int d, int k, float* dw_t, float* dw_bias);

/* GLU -> depthwise conv over time (zero padding at each utterance's edges) -> SiLU, then per-128-channel int8
 * for pointwise_conv2. g [rows, 2d] (row stride ld_g) is pointwise_conv1's output; utterance u occupies rows
 * [off[u], off[u] + len[u]) (host arrays). Outputs hb [rows, d] f32 (or NULL) and/or q [rows, d] int8 +
 * scales [rows, d/128]. workspace >= vxg_conv_workspace_bytes(). d % 128 == 0, odd k <= 15. Replaces the middle
 * of ConvModule::forward_fused (encoder.rs:596-626). */
size_t vxg_conv_workspace_bytes(int rows, int n_utt);
vxg_status vxg_conv_glu_dw_silu_quant(const float* g, int ld_g, const int* off, const int* len, int n_utt,
                                      const float* dw_t, const float* dw_bias, int d, int k, float* hb, int8_t* q,
                                      float* scales, void* workspace, size_t ws_bytes, void* stream);

/* Allocation-free form of vxg_conv_glu_dw_silu_quant (no counterpart in the reference): same arguments and
 * results, but the index tables live in a static 64 KB device array inside the library instead of a caller
 * workspace, for callers that may not allocate device memory at run time (a server that sizes every buffer at
 * start-up under a fixed device-memory budget, or a streaming engine that cannot afford the synchronisation of
 * cudaMalloc / cudaFree). It allocates no device memory and calls no allocating CUDA routine; a small kernel on
 * `stream` writes the tables from the lengths, which it receives by value. Limits: n_utt <= 1000 and
 * 2 * n_utt + 2 * sum(ceil(len[u] / 64)) <= 16384, else VXG_ERR_ARG with a message. The first call on each device
 * does the set-up (looks up the array's device address); make it before any stream capture. The address stays valid
 * for the life of the device context: after cudaDeviceReset the library's device state is gone, this entry
 * included. The array is shared: calls that overlap on the GPU (other streams, other host threads) race on it, so
 * serialise them on one stream. */
vxg_status vxg_conv_glu_dw_silu_quant_static(const float* g, int ld_g, const int* off, const int* len, int n_utt,
                                             const float* dw_t, const float* dw_bias, int d, int k, float* hb,
                                             int8_t* q, float* scales, void* stream);

/* ------------------------------------------------------------------------------------------- subsampling
 * f32 dw-striding Conv2d x8 front end, bit-identical to Subsampling::forward (crates/voxrt/src/subsampling.rs:
 * 109-204), for a batch of log-mel inputs stacked along time: utterance u has t_in[u] frames (host array) of
 * n_mels bins; outputs are stacked the same way, vxg_sub_out_frames(t_in[u]) rows of d_model each. Weights in the
 * layouts Subsampling::load prepares (subsampling.rs:31-96): conv [9][256] tap-major, pointwise [256][256],
 * linear [d_model][F3*256] with channels-last columns. Utterances must give >= 2 output frames (a single output
 * row would take the reference's gemv order). Replaces Subsampling::forward / GpuEncoder::subsample
 * (metal/mod.rs:623). */
int vxg_sub_out_frames(int t_in);
size_t vxg_subsampling_workspace_bytes(const int* t_in, int n_utt, int n_mels);
vxg_status vxg_subsampling(const float* feats, const int* t_in, int n_utt, int n_mels, const float* conv0_w,
                           const float* conv0_b, const float* dw1_w, const float* dw1_b, const float* pw1_w,
                           const float* pw1_b, const float* dw2_w, const float* dw2_b, const float* pw2_w,
                           const float* pw2_b, const float* lin_w, const float* lin_b, int d_model, float* out,
                           void* workspace, size_t ws_bytes, void* stream);

/* f32 y[M, N] = x[M, K] w[N, K]^T (+ bias) (+ ReLU) in the reference's `linear` order for M >= 2
 * (tile_rows_portable, crates/voxrt/src/tensor.rs:233-260): four fused lanes over 4-column steps, hsum4, bias.
 * K % 16 == 0. */
vxg_status vxg_linear_f32(const float* x, int M, int K, const float* w, const float* bias, int N, int relu, float* y,
                          void* stream);

/* ---------------------------------------------------------------------------------------------- encoder
 * The whole quantised FastConformer encoder (subsampling + layers) resident on one GPU. Weights are given in the
 * model file's layouts (host pointers, read during vxg_encoder_create only): ternary modules as thrush-ternary-v2
 * qweight + f16 scale bits, dense tensors as f32 (HF layouts; f16 tensors converted by the caller). */
typedef struct vxg_ternary_tensor {
  const uint8_t* qweight;  /* [out, ceil(in/5)] base-3, 5 trits per byte, LSD first */
  const uint16_t* scales;  /* [out, in/group] f16 bits */
  int out, in, group;
} vxg_ternary_tensor;

typedef struct vxg_layer_weights { /* encoder.layers.{i}.* (reference/ternary.json names) */
  vxg_ternary_tensor ff1_linear1, ff1_linear2, q_proj, k_proj, v_proj, o_proj, relative_k_proj, pointwise_conv1,
      pointwise_conv2, ff2_linear1, ff2_linear2;
  const float *norm_ff1_w, *norm_ff1_b, *norm_attn_w, *norm_attn_b, *norm_conv_w, *norm_conv_b, *norm_ff2_w,
      *norm_ff2_b, *norm_out_w, *norm_out_b; /* [d] */
  const float *bias_u, *bias_v;                               /* [heads, head_dim] */
  const float* dw_weight;                                     /* depthwise_conv.weight [d, 1, k] */
  const float *bn_weight, *bn_bias, *bn_mean, *bn_var;        /* conv.norm (BatchNorm, eval) [d] */
} vxg_layer_weights;

typedef struct vxg_subsampling_weights { /* encoder.subsampling.* in HF layouts */
  const float *conv0_w, *conv0_b; /* [C,1,3,3], [C] */
  const float *dw1_w, *dw1_b;     /* layers.2 */
  const float *pw1_w, *pw1_b;     /* layers.3 [C,C,1,1] */
  const float *dw2_w, *dw2_b;     /* layers.5 */
  const float *pw2_w, *pw2_b;     /* layers.6 */
  const float *lin_w, *lin_b;     /* linear [d, C*n_mels/8] (HF flatten order c*F3 + f), [d] */
} vxg_subsampling_weights;

enum { VXG_WEIGHTS_2BIT = 0, VXG_WEIGHTS_INT8 = 1 };

typedef struct vxg_encoder_desc {
  int d_model, ff, heads, conv_kernel, n_layers, n_mels, sub_channels;
  int weight_format; /* VXG_WEIGHTS_2BIT: in-SM unpack of 2-bit codes; VXG_WEIGHTS_INT8: int8-resident */
  const vxg_layer_weights* layers; /* [n_layers] */
  const vxg_subsampling_weights* sub;
} vxg_encoder_desc;

typedef struct vxg_encoder vxg_encoder; /* one GPU, one stream, internally serialised (like GpuEncoder's Mutex) */

/* Upload and repack all weights on `device`. Replaces GpuEncoder::load (crates/voxrt/src/metal/mod.rs:463) and
 * Encoder::load_with (encoder.rs:791). */
vxg_status vxg_encoder_create(const vxg_encoder_desc* desc, int device, vxg_encoder** out);
void vxg_encoder_destroy(vxg_encoder* e);
int vxg_encoder_out_frames(int t_in); /* Subsampling::out_frames (subsampling.rs:99-106) */

/* Log-mel feats [t_in, n_mels] (host) -> encoder output [t_e, d_model] (host, out_cap floats). Replaces
 * GpuEncoder::forward_feats (metal/mod.rs:592) / Transcriber::encode (transcriber.rs:194-225). */
vxg_status vxg_encoder_forward_feats(vxg_encoder* e, const float* feats, int t_in, float* out, size_t out_cap,
                                     int* t_e);

/* A batch of utterances in one token-stacked forward: host feats[u] [t_in[u], n_mels] -> host outs[u]
 * [t_e[u], d_model]. One pinned host->device copy in, one device->host copy out. */
vxg_status vxg_encoder_forward_batch(vxg_encoder* e, const float* const* feats, const int* t_in, int n,
                                     float* const* outs, int* t_e);

/* Device-resident form: feats stacked [sum t_in, n_mels] and out stacked [sum t_e, d_model] in device memory,
 * ordered on the caller's `stream` (NULL = the legacy default stream, as in every CUDA call): the forward runs
 * after the work already queued there, and work queued there afterwards waits for it. Returns before completion. */
vxg_status vxg_encoder_forward_device(vxg_encoder* e, const float* feats, const int* t_in, int n, float* out,
                                      int* t_e, void* stream);

/* The subsampling front end alone on the encoder's resident weights: feats stacked [sum t_in, n_mels] (device) ->
 * out stacked [sum t_e, d_model] (device), ordered on `stream` like vxg_encoder_forward_device. The VAD head's input.
 * Replaces Transcriber::subsample (crates/voxrt/src/transcriber.rs:182-192). */
vxg_status vxg_encoder_subsample_device(vxg_encoder* e, const float* feats, const int* t_in, int n, float* out,
                                        int* t_e, void* stream);

/* Layers only on subsampled input (device, stacked [sum t, d_model]) -> out (device). Replaces
 * GpuEncoder::forward (metal/mod.rs:586). Synchronous. */
vxg_status vxg_encoder_forward_layers_device(vxg_encoder* e, const float* x, const int* t, int n, float* out,
                                             void* stream);

/* Per-kernel-class device time: with profiling on, each step of a forward is bracketed by CUDA events on the
 * encoder's stream; vxg_encoder_profile synchronises, returns the milliseconds and step counts accumulated since
 * the last call per class (VXG_PROF_*) plus the algorithmic int8 ops of the ternary GEMMs, and resets them.
 * Counterpart of the reference's VOXRT_PROFILE counters (ternary_linear.rs:12-13, encoder.rs:297, :647-653). */
enum {
  VXG_PROF_SUB = 0,   /* subsampling front end */
  VXG_PROF_LNQ = 1,   /* LayerNorm -> int8 (and norm_out) */
  VXG_PROF_GEMM = 2,  /* ternary GEMMs */
  VXG_PROF_ATTN = 3,  /* attention (prep + core) */
  VXG_PROF_CONV = 4,  /* conv module middle */
  VXG_PROF_QUANT = 5, /* plain quantisation */
  VXG_PROF_CLASSES = 6
};
vxg_status vxg_encoder_set_profiling(vxg_encoder* e, int on);
vxg_status vxg_encoder_profile(vxg_encoder* e, double* ms, int* launches, double* gemm_ops);

/* Kernels this library has launched in this process (all devices). No reference counterpart. */
unsigned long long vxg_kernel_launches(void);

/* ---------------------------------------------------------------------------------------------- TDT decoder
 * The token-and-duration transducer decoder run after the encoder: prediction network (embedding + LSTM stack +
 * decoder projector), joint head and NeMo GreedyTDTInfer, in the reference's default int8 mode (per-row int8 LSTM
 * and head weights, decoder.rs:95-107). The greedy loop runs either on host threads, as the reference's does, or
 * batched on the GPU (vxg_tdt_greedy_device), with identical emissions; the encoder projection runs on the GPU.
 * Weights are host pointers in the model file's layouts, read during create only. */
typedef struct vxg_tdt_desc {
  int hidden, vocab, n_durations, blank, max_symbols, d_model, n_layers; /* n_layers <= 4, hidden % 128 == 0 */
  const int* durations;                     /* [n_durations] frame advances, e.g. {0, 1, 2, 3, 4} */
  const float* embedding;                   /* decoder.embedding.weight [vocab, hidden] */
  const uint16_t* w_ih[4];                  /* decoder.lstm.weight_ih_l{l} f16 bits [4 hidden, hidden] */
  const uint16_t* w_hh[4];                  /* decoder.lstm.weight_hh_l{l} f16 bits [4 hidden, hidden] */
  const float* b_ih[4];                     /* [4 hidden] */
  const float* b_hh[4];                     /* [4 hidden] */
  const uint16_t* proj_w;                   /* decoder.decoder_projector.weight f16 bits [hidden, hidden] */
  const float* proj_b;                      /* [hidden] */
  const uint16_t* head_w;                   /* joint.head.weight f16 bits [vocab + n_durations, hidden] */
  const float* head_b;                      /* [vocab + n_durations] */
  const float* enc_w;                       /* encoder_projector.weight f32 [hidden, d_model] */
  const float* enc_b;                       /* [hidden] */
  int device; /* GPU for vxg_tdt_project_device and the *_device decode entries, or -1 for none */
} vxg_tdt_desc;

typedef struct vxg_tdt vxg_tdt; /* immutable after create: every call below may run concurrently */

typedef struct vxg_emission { /* decoder::Emission (decoder.rs:7-12) */
  int32_t token, frame, duration;
} vxg_emission;

/* Quantise and lay out the weights. Replaces Decoder::load (decoder.rs:61-110). */
vxg_status vxg_tdt_create(const vxg_tdt_desc* desc, vxg_tdt** out);
void vxg_tdt_destroy(vxg_tdt* d);

/* Decoder::project_encoder (decoder.rs:123-134): enc [t, d_model] -> proj [t, hidden], f32 linear in the
 * reference's lane order (t >= 2: tile_rows order; t == 1: gemv order). Device pointers, ordered on `stream`. */
vxg_status vxg_tdt_project_device(const vxg_tdt* d, const float* enc, int t, float* proj, void* stream);

/* Decoder::greedy (decoder.rs:204-266) over projected frames proj [t, hidden] (host). Writes at most `cap`
 * emissions and the full count to *n (so *n > cap means the output was truncated). */
vxg_status vxg_tdt_greedy(const vxg_tdt* d, const float* proj, int t, vxg_emission* out, size_t cap, size_t* n);

/* n utterances decoded on up to `threads` host threads (0 = all hardware threads); utterance u reads proj[u]
 * [t[u], hidden] and writes out[u] (cap[u] entries) and n_out[u]. Same results as n calls of vxg_tdt_greedy. */
vxg_status vxg_tdt_greedy_batch(const vxg_tdt* d, int n, const float* const* proj, const int* t,
                                vxg_emission* const* out, const size_t* cap, size_t* n_out, int threads);

/* One prediction-network step (decoder.rs:136-175) and one joint evaluation (decoder.rs:178-192), exposed for
 * parity checks. States are [n_layers, hidden]; logits [vocab + n_durations]. Host pointers. */
vxg_status vxg_tdt_pred_step(const vxg_tdt* d, int token, const float* h, const float* c, float* g, float* h_out,
                             float* c_out);
vxg_status vxg_tdt_joint(const vxg_tdt* d, const float* enc_t, const float* g, float* logits);

/* Decoder::greedy (decoder.rs:204-266) for n utterances on the decoder's GPU (desc.device; must be current), all in
 * lockstep rounds whose weight products serve every unfinished utterance at once. proj: device [sum t, hidden], the
 * projected frames of utterance u at rows sum_{v<u} t[v] .. (vxg_tdt_project_device of the stacked encoder output);
 * t: host [n] frame counts; cap: host [n] capacities; out: device [sum cap] emissions, utterance u's at
 * out + sum_{v<u} cap[v]; n_out: device [n] emission counts (n_out[u] > cap[u]: utterance u was truncated; at most
 * t[u] * max_symbols emissions exist). Work is ordered on `stream`; the call blocks
 * the calling thread until every utterance is finished (it polls a device count) and returns with the results
 * queued on `stream`. Emissions are identical to vxg_tdt_greedy's. hidden <= 1024 (else VXG_ERR_UNSUPPORTED).
 * Scratch is allocated on `stream` per call (about n * (4 n_layers + 8) * hidden * 4 bytes). */
vxg_status vxg_tdt_greedy_device(const vxg_tdt* d, int n, const float* proj, const int* t, vxg_emission* out,
                                 const size_t* cap, int* n_out, void* stream);

/* The GPU decode's prediction-network step and joint evaluation for n independent inputs, for parity checks
 * against vxg_tdt_pred_step / vxg_tdt_joint. Device pointers: tokens [n]; h, c, h_out, c_out [n, n_layers,
 * hidden]; g [n, hidden]; enc [n, hidden]; logits [n, vocab + n_durations]. Ordered on `stream`. */
vxg_status vxg_tdt_pred_step_device(const vxg_tdt* d, int n, const int* tokens, const float* h, const float* c,
                                    float* g, float* h_out, float* c_out, void* stream);
vxg_status vxg_tdt_joint_device(const vxg_tdt* d, int n, const float* enc, const float* g, float* logits,
                                void* stream);

/* ------------------------------------------------------------------------------------------------ math
 * The correctly rounded f32 exp (fn 0) and tanh (fn 1) that the decoder's LSTM cell and the VAD head use in place of
 * the reference's libm calls (libm::expf / libm::tanhf, crates/voxrt/src/tensor.rs:784-786, decoder.rs:165-168,
 * vad.rs:79): y[i] = the exact value rounded to nearest even, the same bits on the host and the device. */
vxg_status vxg_math_host(int fn, const float* x, size_t n, float* y);
vxg_status vxg_math_device(int fn, const float* x, size_t n, float* y, void* stream);

/* -------------------------------------------------------------------------------------------- frontend
 * NeMo log-mel features on the GPU (16 kHz, n_fft 512, Hann window 400, hop 160, Slaney mel, pre-emphasis 0.97,
 * log with a 2^-24 guard, then per-utterance per-feature normalisation with unbiased std + 1e-5). Replaces
 * Frontend::compute / log_mel / normalize (crates/voxrt/src/frontend.rs:112-200). The FFT is this library's own, so
 * features agree with the reference's realfft-based ones to f32 rounding, not bit for bit. */
typedef struct vxg_frontend vxg_frontend;
/* slaney_mel_filterbank (frontend.rs:74-90): fb [n_mels, n_fft/2 + 1], host. */
vxg_status vxg_mel_filterbank(int sample_rate, int n_fft, int n_mels, float* fb);
int vxg_frontend_frames(long long n_samples); /* Frontend::n_frames: n_samples / 160 */
vxg_status vxg_frontend_create(int sample_rate, int n_mels, int device, vxg_frontend** out);
void vxg_frontend_destroy(vxg_frontend* f);
vxg_status vxg_frontend_info(const vxg_frontend* f, int* sample_rate, int* n_mels);
/* samples: the utterances' 16 kHz f32 samples stacked (device); n_samples [n] (host); feats: stacked
 * [sum frames, n_mels] (device); n_frames [n] (host, optional) receives the frame counts. normalize = 0 gives the
 * log-mel before normalisation (log_mel). Ordered on `stream`; returns once the work is queued and its index tables
 * are no longer needed (the call waits for the stream). */
vxg_status vxg_frontend_device(vxg_frontend* f, const float* samples, const long long* n_samples, int n,
                               int normalize, float* feats, int* n_frames, void* stream);

/* ------------------------------------------------------------------------------------------ model directory
 * A thrush-ternary-v2 model directory (config.json, ternary.json, model.safetensors), memory-mapped read-only.
 * Replaces ModelFile (crates/voxrt/src/format.rs:76-309): open checks the format ("thrush-ternary-v2") and tensor
 * naming ("hf") and parses the safetensors header; validate lists every tensor the loaders read that is missing or
 * has the wrong dtype / shape, one per line (format.rs:153-309). */
typedef struct vxg_model vxg_model;

typedef struct vxg_model_cfg { /* config.json / ternary.json fields the loaders use */
  int d_model, ff, n_layers, heads, n_mels, conv_kernel, sub_channels, group;
  int dec_hidden, dec_layers, vocab, blank, max_symbols, n_durations;
  int vad_hidden, vad_kernel;
  double vad_frame_seconds;
} vxg_model_cfg;

vxg_status vxg_model_open(const char* dir, vxg_model** out); /* ModelFile::open (format.rs:88-118) */
void vxg_model_close(vxg_model* m);
/* Number of problems (0 = valid) and, in buf, the problems separated by newlines. ModelFile::validate. */
int vxg_model_validate(const vxg_model* m, char* buf, size_t cap);
vxg_status vxg_model_config(const vxg_model* m, vxg_model_cfg* cfg);
/* One tensor of the safetensors file: dtype (0 F16, 1 BF16, 2 F32, 3 U8, 4 I8, 5 other), shape (up to 8 dims),
 * and a pointer to its bytes inside the mapping (valid until vxg_model_close). ModelFile::tensor (format.rs:136). */
vxg_status vxg_model_tensor(const vxg_model* m, const char* name, int* dtype, int64_t* shape, int* ndim,
                            const void** data, size_t* bytes);
/* A float tensor (F32, or F16 / BF16 widened exactly) copied into out[count]; count must be its element count.
 * load_f32 (tensor.rs:20-37). */
vxg_status vxg_model_tensor_f32(vxg_model* m, const char* name, float* out, size_t count);
/* The encoder / decoder from a model directory (validated first; f16 dense tensors widened to f32 exactly).
 * Replace Encoder::load_with (encoder.rs:791) / GpuEncoder::load (metal/mod.rs:463) and Decoder::load
 * (decoder.rs:57-110). The model may be closed once these return. */
vxg_status vxg_encoder_create_from_model(vxg_model* m, int weight_format, int device, vxg_encoder** out);
vxg_status vxg_tdt_create_from_model(vxg_model* m, int device, vxg_tdt** out);

/* ----------------------------------------------------------------------------------------------- VAD head
 * Speech probability per encoder frame from the subsampler output: sigmoid(out(relu(ctx(relu(proj(x)))))), with
 * the reference's summation orders (VadHead::probs, crates/voxrt/src/vad.rs:39-82) and the correctly rounded exp of
 * vxg_math_*. Runs on a GPU; weights are host pointers in the model file's layouts, read during create only. */
typedef struct vxg_vad vxg_vad;
typedef struct vxg_vad_desc {
  int d_model, hidden, kernel; /* kernel odd (same padding) */
  const float* proj_w;         /* vad_head.proj.weight [hidden, d_model, 1] */
  const float* proj_b;         /* [hidden] */
  const float* ctx_w;          /* vad_head.ctx.weight [hidden, hidden, kernel] */
  const float* ctx_b;          /* [hidden] */
  const float* out_w;          /* vad_head.out.weight [1, hidden, 1] */
  float out_b;
  double frame_seconds;        /* 0.08 */
  int device;
} vxg_vad_desc;
vxg_status vxg_vad_create(const vxg_vad_desc* desc, vxg_vad** out);
vxg_status vxg_vad_create_from_model(vxg_model* m, int device, vxg_vad** out); /* VadHead::load (vad.rs:21-36) */
void vxg_vad_destroy(vxg_vad* v);
vxg_status vxg_vad_info(const vxg_vad* v, int* d_model, int* hidden, int* kernel, double* frame_seconds);
/* sub: stacked [sum t, d_model] (device), utterance u's t[u] frames (host) convolved within the utterance only;
 * probs: [sum t] (device). Synchronous on `stream`. */
vxg_status vxg_vad_probs_device(const vxg_vad* v, const float* sub, const int* t, int n, float* probs, void* stream);

/* Segmentation of a probability track into speech segments [start, end) in encoder frames (segment, vad.rs:140-240):
 * speech runs with pauses shorter than min_pause_frames tolerated, short runs merged while within max_frames, runs
 * above max_frames split at the weakest frame of the last 63 frames (~5 s) of each window, then pad_frames of
 * context on each side, never past the midpoint of the gap to a neighbour. Host computation. */
typedef struct vxg_segment_cfg { /* SegmentConfig (vad.rs:86-103) */
  float threshold;      /* 0.5 */
  int min_pause_frames; /* 8 */
  int max_frames;       /* 750 (60 s) */
  int min_frames;       /* 125 (10 s) */
  int pad_frames;       /* 2 */
} vxg_segment_cfg;
typedef struct vxg_vad_segment {
  int start, end;
} vxg_vad_segment;
void vxg_segment_cfg_default(vxg_segment_cfg* cfg);
/* Writes at most cap segments; *n = their full count. */
vxg_status vxg_segment(const float* probs, int t, const vxg_segment_cfg* cfg, vxg_vad_segment* out, size_t cap,
                       size_t* n);

/* ------------------------------------------------------------------------------------------------ long form
 * Streaming / long-form transcription (LongForm, crates/voxrt/src/longform.rs): VAD on fixed absolute-time blocks
 * (with context on each side), a segment automaton that closes only segments whose extent no future audio can
 * change, and per-segment transcription (frontend -> encoder -> projection -> TDT greedy on the GPU). Text is out of
 * scope: a segment is its absolute sample range, its transcription the emissions (frames in absolute encoder frames).
 * A vxg_longform is used by one thread at a time. */
typedef struct vxg_longform vxg_longform;
typedef struct vxg_longform_cfg {
  vxg_segment_cfg seg;
  long long block_samples;      /* VAD block, 160000 (10 s) */
  long long ctx_samples;        /* VAD context on each side of a block, 20480 (16 frames) */
  int samples_per_frame;        /* hop x subsampling factor = 1280 (80 ms) */
  int sample_rate;              /* 16000 */
  double long_form_threshold_s; /* audio up to this length is transcribed whole: 30 */
  int collect_only;             /* record closed segments' ranges without transcribing them */
} vxg_longform_cfg;
void vxg_longform_cfg_default(vxg_longform_cfg* cfg);
/* VAD probabilities of `want` frames starting `skip` frames into the audio block samples[0 .. n) (an external VAD in
 * place of the GPU head). Returns the number written (<= want), or a negative value on failure. */
typedef long long (*vxg_vad_block_fn)(void* user, const float* samples, long long n, long long skip, long long want,
                                      float* probs);
/* LongForm::new (longform.rs:29-49). The components must live as long as the vxg_longform; they run on the encoder's
 * device. vxg_longform_create_with_vad takes the probabilities from `fn` and only collects ranges. */
vxg_status vxg_longform_create(vxg_frontend* fe, vxg_encoder* enc, vxg_vad* vad, vxg_tdt* dec,
                               const vxg_longform_cfg* cfg, vxg_longform** out);
vxg_status vxg_longform_create_with_vad(vxg_vad_block_fn fn, void* user, const vxg_longform_cfg* cfg,
                                        vxg_longform** out);
void vxg_longform_destroy(vxg_longform* lf);
/* Feed audio (LongForm::push, longform.rs:55-66) / end the stream (LongForm::flush, :69-97). The segments closed by
 * this call are written as absolute sample pairs ranges[2 i], ranges[2 i + 1] (at most cap pairs; *n_closed = their
 * count). */
vxg_status vxg_longform_push(vxg_longform* lf, const float* samples, long long n, long long* ranges, size_t cap,
                             size_t* n_closed);
vxg_status vxg_longform_flush(vxg_longform* lf, long long* ranges, size_t cap, size_t* n_closed);
/* Every segment closed so far, as absolute sample pairs (LongForm::ranges); *n = their count. */
vxg_status vxg_longform_ranges(const vxg_longform* lf, long long* ranges, size_t cap, size_t* n);
/* All emissions so far (absolute encoder frames); *n = their count. */
vxg_status vxg_longform_emissions(const vxg_longform* lf, vxg_emission* out, size_t cap, size_t* n);
/* Diagnostics: high-water mark of the audio buffer (samples), absolute sample of the buffer's start, and the
 * number of VAD probabilities held. */
vxg_status vxg_longform_stats(const vxg_longform* lf, long long* max_pending, long long* base_sample,
                              long long* n_probs);
/* Transcriber::transcribe_long (transcriber.rs:356-420): audio up to long_form_threshold_s whole; longer audio cut
 * by a collect-only LongForm fed in 10 s chunks, then every segment encoded in token-stacked forwards and decoded in
 * one lockstep GPU batch. Emissions in absolute encoder frames (at most cap; *n_out = count); ranges (optional)
 * receives the segments' sample pairs (at most rcap pairs; *n_ranges = count). */
vxg_status vxg_transcribe_long(vxg_frontend* fe, vxg_encoder* enc, vxg_vad* vad, vxg_tdt* dec, const float* samples,
                               long long n, const vxg_longform_cfg* cfg, vxg_emission* out, size_t cap,
                               size_t* n_out, long long* ranges, size_t rcap, size_t* n_ranges);

#ifdef __cplusplus
}
#endif
#endif /* VXG_H */
