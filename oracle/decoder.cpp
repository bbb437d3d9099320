/*
 * CPU oracle for the TDT decoder of lmaksym/voxrt 0.2.1 (crates/voxrt/src/decoder.rs), in its default int8 mode
 * (VOXRT_DECODER unset -> "int8", decoder.rs:95-107): per-row int8 LSTM and joint-head weights, f16 decoder
 * projector, f32 encoder projector.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): the checker the product decoder is compared against. Scalar C++ in the
 * reference's operation order. The reference's libm calls (libm::expf in sigmoid, libm::tanhf) are taken as the
 * correctly rounded functions, evaluated here in x87 extended precision and rounded to f32 (the library implements the
 * same definition independently); the reference's `libm` crate itself is not reproduced, so that boundary is not
 * pinned to the reference.
 */
#include <cmath>
#include <cstring>
#include <vector>

#include "oracle.h"
#include "oracle_internal.h"

namespace {

float hsum4(const float* a) { return (a[0] + a[1]) + (a[2] + a[3]); }

/* gemv_f16 (tensor.rs:529-559): gemv_f16_avx2 (:561-600) and gemv_f16_portable (:308-326) agree: rows below
 * out/4*4 take dot_lanes8 (:267-281, lanes c+l and c+4+l fused, hsum4 of the lane pairs), the remaining rows a plain
 * in-order sum; then + bias. */
void gemv_f16(const float* x, int in_f, const uint16_t* w, const float* b, int out_f, float* y) {
  const int o4 = out_f / 4 * 4;
  for (int o = 0; o < out_f; o++) {
    const uint16_t* wr = w + (size_t)o * in_f;
    float r;
    if (o < o4) {
      const int n8 = in_f / 8 * 8;
      float a[4] = {0, 0, 0, 0}, bb[4] = {0, 0, 0, 0};
      for (int c = 0; c < n8; c += 8)
        for (int l = 0; l < 4; l++) {
          a[l] = std::fmaf(x[c + l], vxo_f16_to_f32(wr[c + l]), a[l]);
          bb[l] = std::fmaf(x[c + 4 + l], vxo_f16_to_f32(wr[c + 4 + l]), bb[l]);
        }
      float t4[4];
      for (int l = 0; l < 4; l++) t4[l] = a[l] + bb[l];
      r = hsum4(t4);
      for (int c = n8; c < in_f; c++) r += x[c] * vxo_f16_to_f32(wr[c]);
    } else {
      r = 0.0f;
      for (int c = 0; c < in_f; c++) r = r + x[c] * vxo_f16_to_f32(wr[c]);
    }
    y[o] = r + (b ? b[o] : 0.0f);
  }
}

/* gemm_single (kernels/mod.rs:285-315) for one token: QuantAct::quantize_layout (packed.rs:307-312, group 128), the
 * scalar group-sum / FMA chain (kernels/mod.rs:166-210, Store), then y += bias. */
void gemm_single(const int8_t* w, const float* s, int out, int inp, const float* x, const float* bias, float* y) {
  std::vector<int8_t> q(inp);
  std::vector<float> sq(inp / 128);
  vxo_quantize_rows(x, 1, inp, 128, q.data(), sq.data());
  vxo_gemm(w, s, q.data(), sq.data(), 1, out, inp, 128, VXO_EP_STORE, 0.0f, nullptr, y, nullptr, 0, out, 0, 1);
  if (bias)
    for (int o = 0; o < out; o++) y[o] += bias[o];
}

/* sigmoid (tensor.rs:784-786), exp correctly rounded */
static float expf_cr(float x) { return (float)expl((long double)x); }
static float tanhf_cr(float x) { return (float)tanhl((long double)x); }
float sigmoid(float v) { return 1.0f / (1.0f + expf_cr(-v)); }

/* Decoder::argmax (decoder.rs:194-202): first index of the maximum under a strict '>' */
int argmax(const float* v, int n) {
  int best = 0;
  for (int i = 0; i < n; i++)
    if (v[i] > v[best]) best = i;
  return best;
}

}  // namespace

/* int8_rows (decoder.rs:270-303): one symmetric scale per row s = amax/127 (1 for an all-zero row), codes
 * round_ties_even(v * (1/s)) clamped to +-127; the scale is replicated for every 128-wide group. */
extern "C" void vxo_tdt_int8_rows(const uint16_t* w_f16, int out, int inp, int8_t* rows, float* scales) {
  const int ng = inp / 128;
  std::vector<float> row(inp);
  for (int r = 0; r < out; r++) {
    float amax = 0.0f;
    for (int k = 0; k < inp; k++) {
      row[k] = vxo_f16_to_f32(w_f16[(size_t)r * inp + k]);
      amax = std::fmax(amax, std::fabs(row[k]));
    }
    const float s = amax == 0.0f ? 1.0f : amax / 127.0f;
    const float inv = 1.0f / s;
    for (int k = 0; k < inp; k++) {
      float v = std::nearbyintf(row[k] * inv);
      v = std::fmin(std::fmax(v, -127.0f), 127.0f);
      rows[(size_t)r * inp + k] = (int8_t)v;
    }
    for (int g = 0; g < ng; g++) scales[(size_t)r * ng + g] = s;
  }
}

/* Decoder::pred_step (decoder.rs:136-175), int8 LSTM branch: gates = gemm_single(w_ih, x) + b, gh = gemm_single(
 * w_hh, h_prev), gates += gh, then i, f, g, o and c' = f*c + i*g, h' = o*tanh(c'); the decoder projector is a
 * gemv_f16 of the last layer's h. States are [layers][hidden]. */
extern "C" void vxo_tdt_pred_step(const vxo_tdt* D, int token, const float* h_in, const float* c_in, float* g_out,
                                  float* h_out, float* c_out) {
  const int h = D->hidden;
  std::vector<float> x(D->embedding + (size_t)token * h, D->embedding + (size_t)(token + 1) * h);
  std::vector<float> gates(4 * h), gh(4 * h);
  for (int l = 0; l < D->n_layers; l++) {
    const float* hp = h_in + (size_t)l * h;
    const float* cp = c_in + (size_t)l * h;
    gemm_single(D->w_ih[l], D->s_ih[l], 4 * h, h, x.data(), D->b[l], gates.data());
    gemm_single(D->w_hh[l], D->s_hh[l], 4 * h, h, hp, nullptr, gh.data());
    for (int k = 0; k < 4 * h; k++) gates[k] += gh[k];
    float* hn = h_out + (size_t)l * h;
    float* cn = c_out + (size_t)l * h;
    for (int k = 0; k < h; k++) {
      const float i = sigmoid(gates[k]);
      const float f = sigmoid(gates[h + k]);
      const float g = tanhf_cr(gates[2 * h + k]);
      const float o = sigmoid(gates[3 * h + k]);
      cn[k] = f * cp[k] + i * g;
      hn[k] = o * tanhf_cr(cn[k]);
    }
    std::memcpy(x.data(), hn, sizeof(float) * h);
  }
  gemv_f16(x.data(), h, D->proj_w, D->proj_b, h, g_out);
}

/* Decoder::joint (decoder.rs:178-192), int8 head: z = max(enc_t + g, 0), quantised per 128-group, head GEMM + bias. */
extern "C" void vxo_tdt_joint(const vxo_tdt* D, const float* enc_t, const float* g, float* logits) {
  const int h = D->hidden;
  std::vector<float> z(h);
  for (int k = 0; k < h; k++) z[k] = std::fmax(enc_t[k] + g[k], 0.0f);
  gemm_single(D->head_w, D->head_s, D->vocab + D->n_dur, h, z.data(), D->head_b, logits);
}

/* Decoder::project_encoder (decoder.rs:123-134): linear (tensor.rs:98-127) of enc [t, d] to [t, hidden]. */
extern "C" void vxo_tdt_project(const vxo_tdt* D, const float* enc, int t, float* proj) {
  vxo_linear(enc, t, D->d_model, D->enc_w, D->enc_b, D->hidden, proj);
}

/* Decoder::greedy (decoder.rs:204-266): NeMo GreedyTDTInfer. The prediction network output is reused after a
 * blank (it depends only on the last token and the state). Returns the number of emissions written (at most cap;
 * the count is exact even when cap truncates). */
extern "C" int vxo_tdt_greedy(const vxo_tdt* D, const float* proj, int t, int* tokens, int* frames, int* durs,
                              int cap) {
  const int h = D->hidden, L = D->n_layers, nout = D->vocab + D->n_dur;
  std::vector<float> hs(L * h, 0.0f), cs(L * h, 0.0f), hn(L * h), cn(L * h), g(h), logits(nout);
  int last = D->blank, tf = 0, n = 0;
  bool have_pred = false;
  while (tf < t) {
    int symbols = 0, dur = 0;
    for (;;) {
      if (!have_pred) {
        vxo_tdt_pred_step(D, last, hs.data(), cs.data(), g.data(), hn.data(), cn.data());
        have_pred = true;
      }
      vxo_tdt_joint(D, proj + (size_t)tf * h, g.data(), logits.data());
      const int k = argmax(logits.data(), D->vocab);
      const int di = argmax(logits.data() + D->vocab, D->n_dur);
      dur = D->durations[di];
      if (k != D->blank) {
        if (n < cap) {
          tokens[n] = k;
          frames[n] = tf;
          durs[n] = dur;
        }
        n++;
        hs.swap(hn);
        cs.swap(cn);
        have_pred = false;
        last = k;
      }
      symbols++;
      tf += dur;
      if (dur != 0 || symbols >= D->max_symbols) break;
      if (k == D->blank) break;
    }
    if (dur == 0) tf += 1;
  }
  return n;
}
