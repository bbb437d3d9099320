// TDT decoder on the host: NeMo GreedyTDTInfer over projected encoder frames, in the reference's default int8 mode
// (crates/voxrt/src/decoder.rs). The reference runs this loop on the CPU after the encoder, one utterance per
// thread; so does this file. The per-step products (joint head [vocab + durations, hidden], LSTM gates) are
// one-token int8 GEMVs with the ternary kernels' exact arithmetic (int32 group sums, then the reference's FMA chain
// over groups), run 16 rows at a time with AVX-512 VNNI when the CPU has it; the decoder projector is an f32 GEMV
// in dot_lanes8 order. Every float step keeps the reference's operation order (compiled with -ffp-contract=off).
#include "tdt.h"

#include <cuda_runtime.h>
#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>

#include "common.h"
#include "crmath.cuh"

namespace vxg {
namespace tdt {
namespace {

float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {  // subnormal: normalise
    int e = -1;
    do {
      man <<= 1;
      e++;
    } while ((man & 0x400u) == 0);
    bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// int8_rows (decoder.rs:270-303): one symmetric scale per row, s = amax/127 (1 for an all-zero row), codes
// round_ties_even(v * (1/s)) clamped to +-127, the scale replicated for every 128-wide group.
void i8rows_from_f16(I8Rows& W, const uint16_t* w, int out, int inp) {
  W.out = out, W.inp = inp, W.ng = inp / 128, W.blocks = (out + 15) / 16;
  W.rows.assign((size_t)out * inp, 0);
  W.scale.assign((size_t)W.blocks * 16, 0.0f);
  std::vector<float> row(inp);
  for (int r = 0; r < out; r++) {
    float amax = 0.0f;
    for (int k = 0; k < inp; k++) {
      row[k] = f16_to_f32(w[(size_t)r * inp + k]);
      amax = std::fmax(amax, std::fabs(row[k]));
    }
    const float s = amax == 0.0f ? 1.0f : amax / 127.0f;
    const float inv = 1.0f / s;
    for (int k = 0; k < inp; k++)
      W.rows[(size_t)r * inp + k] = (int8_t)std::fmin(std::fmax(std::nearbyintf(row[k] * inv), -127.0f), 127.0f);
    W.scale[r] = s;
  }
  W.q16.assign((size_t)W.blocks * inp * 16, 0);
  W.wsum.assign((size_t)W.blocks * W.ng * 16, 0);
  for (int blk = 0; blk < W.blocks; blk++)
    for (int r = 0; r < 16; r++) {
      const int o = blk * 16 + r;
      if (o >= out) continue;
      for (int c = 0; c < inp; c++) {
        const int8_t v = W.rows[(size_t)o * inp + c];
        W.q16[(((size_t)blk * (inp / 4) + c / 4) * 16 + r) * 4 + (c & 3)] = v;
        W.wsum[((size_t)blk * W.ng + c / 128) * 16 + r] += v;
      }
    }
}

void f16rows_from(F16Rows& P, const uint16_t* w, const float* b, int out, int inp) {
  P.out = out, P.inp = inp, P.blocks = (out + 15) / 16;
  P.rows.resize((size_t)out * inp);
  for (size_t i = 0; i < P.rows.size(); i++) P.rows[i] = f16_to_f32(w[i]);
  P.t16.assign((size_t)P.blocks * inp * 16, 0.0f);
  for (int o = 0; o < out; o++)
    for (int c = 0; c < inp; c++) P.t16[((size_t)(o / 16) * inp + c) * 16 + (o % 16)] = P.rows[(size_t)o * inp + c];
  P.bias.assign(b, b + out);
}

// QuantAct::quantize_layout for one token (packed.rs:307-312 -> quantize_group_portable :527-535), group 128.
void quantize(const float* x, int inp, int8_t* q, float* sq) {
  for (int g = 0; g < inp / 128; g++) {
    const float* v = x + g * 128;
    float amax = 0.0f;
    for (int k = 0; k < 128; k++) amax = std::fmax(amax, std::fabs(v[k]));
    const float s = amax == 0.0f ? 1.0f : amax / 127.0f;
    const float inv = 1.0f / s;
    for (int k = 0; k < 128; k++)
      q[g * 128 + k] = (int8_t)std::fmin(std::fmax(std::nearbyintf(v[k] * inv), -127.0f), 127.0f);
    sq[g] = s;
  }
}

// gemm_single (kernels/mod.rs:285-315) of one token on int8 rows: per row, S_g exact in int32, acc = fma(float(S_g),
// sq[g] * s_row, acc) over the groups in order (the scalar kernel, :166-210), y = acc, then y += bias.
void gemv_i8_scalar(const I8Rows& W, const int8_t* q, const float* sq, const float* bias, float* y) {
  for (int o = 0; o < W.out; o++) {
    const int8_t* wr = W.rows.data() + (size_t)o * W.inp;
    float acc = 0.0f;
    for (int g = 0; g < W.ng; g++) {
      int32_t s = 0;
      for (int k = g * 128; k < g * 128 + 128; k++) s += (int32_t)wr[k] * (int32_t)q[k];
      acc = std::fmaf((float)s, sq[g] * W.scale[o], acc);
    }
    y[o] = bias ? acc + bias[o] : acc;
  }
}

// The same 16 rows at a time: activations offset to unsigned (q + 128) so vpdpbusd forms the products, and the
// group's 128 * (sum of codes) removed again, which leaves the exact signed sums; the float chain then runs on the 16
// lanes (every lane the scalar fma / mul).
__attribute__((target("avx512f,avx512bw,avx512vnni"))) void gemv_i8_vnni(const I8Rows& W, const int8_t* q,
                                                                           const float* sq, const float* bias,
                                                                           float* y) {
  alignas(64) uint8_t xu[4096];
  for (int k = 0; k < W.inp; k++) xu[k] = (uint8_t)(q[k] + 128);
  const int steps = W.inp / 4;
  for (int blk = 0; blk < W.blocks; blk++) {
    const int8_t* wb = W.q16.data() + (size_t)blk * steps * 64;
    const __m512 sv = _mm512_loadu_ps(W.scale.data() + blk * 16);
    __m512 acc = _mm512_setzero_ps();
    for (int g = 0; g < W.ng; g++) {
      __m512i s = _mm512_setzero_si512();
      for (int c4 = g * 32; c4 < g * 32 + 32; c4++) {
        int32_t xw;
        std::memcpy(&xw, xu + 4 * c4, 4);
        s = _mm512_dpbusd_epi32(s, _mm512_set1_epi32(xw), _mm512_loadu_si512(wb + (size_t)c4 * 64));
      }
      const __m512i ws = _mm512_loadu_si512(W.wsum.data() + ((size_t)blk * W.ng + g) * 16);
      s = _mm512_sub_epi32(s, _mm512_slli_epi32(ws, 7));
      acc = _mm512_fmadd_ps(_mm512_cvtepi32_ps(s), _mm512_mul_ps(_mm512_set1_ps(sq[g]), sv), acc);
    }
    alignas(64) float out[16];
    _mm512_store_ps(out, acc);
    const int n = std::min(16, W.out - blk * 16);
    for (int r = 0; r < n; r++) y[blk * 16 + r] = bias ? out[r] + bias[blk * 16 + r] : out[r];
  }
}

// The same product for `nu` tokens at once (nu <= kMaxTok): for each 16-row block, every 64-byte weight load feeds
// eight tokens' accumulators, and the block (inp * 16 bytes) stays in L1 while all tokens pass over it, so a decoding
// round streams the weights once instead of once per utterance. Token j reads q + j*inp, sq + j*ng and writes
// y + j*ldy; per token and row the arithmetic is gemv_i8_scalar's.
constexpr int kMaxTok = 64;
__attribute__((target("avx512f,avx512bw,avx512vnni"))) void gemv_i8_vnni_multi(const I8Rows& W, int nu,
                                                                                 const int8_t* q, const float* sq,
                                                                                 const float* bias, float* y,
                                                                                 size_t ldy) {
  static thread_local std::vector<uint8_t> xbuf;
  xbuf.resize((size_t)kMaxTok * W.inp);
  for (int j = 0; j < nu; j++)
    for (int k = 0; k < W.inp; k++) xbuf[(size_t)j * W.inp + k] = (uint8_t)(q[(size_t)j * W.inp + k] + 128);
  const int steps = W.inp / 4;
  for (int blk = 0; blk < W.blocks; blk++) {
    const int8_t* wb = W.q16.data() + (size_t)blk * steps * 64;
    const __m512 sv = _mm512_loadu_ps(W.scale.data() + blk * 16);
    const int n = std::min(16, W.out - blk * 16);
    for (int j0 = 0; j0 < nu; j0 += 8) {
      const int m = std::min(8, nu - j0);
      const uint8_t* xu = xbuf.data() + (size_t)j0 * W.inp;
      __m512 acc[8];
      for (int j = 0; j < 8; j++) acc[j] = _mm512_setzero_ps();
      for (int g = 0; g < W.ng; g++) {
        __m512i s[8];
        for (int j = 0; j < 8; j++) s[j] = _mm512_setzero_si512();
        for (int c4 = g * 32; c4 < g * 32 + 32; c4++) {
          const __m512i wv = _mm512_loadu_si512(wb + (size_t)c4 * 64);
          for (int j = 0; j < m; j++) {
            int32_t xw;
            std::memcpy(&xw, xu + (size_t)j * W.inp + 4 * c4, 4);
            s[j] = _mm512_dpbusd_epi32(s[j], _mm512_set1_epi32(xw), wv);
          }
        }
        const __m512i ws = _mm512_slli_epi32(_mm512_loadu_si512(W.wsum.data() + ((size_t)blk * W.ng + g) * 16), 7);
        for (int j = 0; j < m; j++)
          acc[j] = _mm512_fmadd_ps(_mm512_cvtepi32_ps(_mm512_sub_epi32(s[j], ws)),
                                   _mm512_mul_ps(_mm512_set1_ps(sq[(size_t)(j0 + j) * W.ng + g]), sv), acc[j]);
      }
      for (int j = 0; j < m; j++) {
        alignas(64) float out[16];
        _mm512_store_ps(out, acc[j]);
        float* yj = y + (size_t)(j0 + j) * ldy + blk * 16;
        for (int r = 0; r < n; r++) yj[r] = bias ? out[r] + bias[blk * 16 + r] : out[r];
      }
    }
  }
}

// Products for `nu` tokens (any count): the VNNI kernel in runs of kMaxTok tokens, else one token at a time.
void gemv_i8_multi(const Decoder& D, const I8Rows& W, int nu, const int8_t* q, const float* sq, const float* bias,
                   float* y, size_t ldy) {
  for (int j0 = 0; j0 < nu; j0 += kMaxTok) {
    const int m = std::min(kMaxTok, nu - j0);
    if (D.vnni && W.inp <= 4096)
      gemv_i8_vnni_multi(W, m, q + (size_t)j0 * W.inp, sq + (size_t)j0 * W.ng, bias, y + (size_t)j0 * ldy, ldy);
    else
      for (int j = j0; j < j0 + m; j++)
        gemv_i8_scalar(W, q + (size_t)j * W.inp, sq + (size_t)j * W.ng, bias, y + (size_t)j * ldy);
  }
}

void gemv_i8(const Decoder& D, const I8Rows& W, const int8_t* q, const float* sq, const float* bias, float* y) {
  if (D.vnni && W.inp <= 4096)
    gemv_i8_vnni(W, q, sq, bias, y);
  else
    gemv_i8_scalar(W, q, sq, bias, y);
}

float hsum4(float a0, float a1, float a2, float a3) { return (a0 + a1) + (a2 + a3); }

// gemv_f16 (tensor.rs:529-600 / gemv_f16_portable :308-326): rows below out/4*4 in dot_lanes8 order (:267-281:
// lanes c+l and c+4+l fused over 8-column steps, hsum4 of the lane pairs), the rest a plain in-order sum; + bias.
void gemv_f16_scalar(const F16Rows& P, const float* x, float* y, int o0, int o1) {
  const int o4 = P.out / 4 * 4, n8 = P.inp / 8 * 8;
  for (int o = o0; o < o1; o++) {
    const float* wr = P.rows.data() + (size_t)o * P.inp;
    float r;
    if (o < o4) {
      float a[4] = {0, 0, 0, 0}, bb[4] = {0, 0, 0, 0};
      for (int c = 0; c < n8; c += 8)
        for (int l = 0; l < 4; l++) {
          a[l] = std::fmaf(x[c + l], wr[c + l], a[l]);
          bb[l] = std::fmaf(x[c + 4 + l], wr[c + 4 + l], bb[l]);
        }
      r = hsum4(a[0] + bb[0], a[1] + bb[1], a[2] + bb[2], a[3] + bb[3]);
      for (int c = n8; c < P.inp; c++) r += x[c] * wr[c];
    } else {
      r = 0.0f;
      for (int c = 0; c < P.inp; c++) r = r + x[c] * wr[c];
    }
    y[o] = r + P.bias[o];
  }
}

__attribute__((target("avx512f"))) void gemv_f16_avx512(const F16Rows& P, const float* x, float* y) {
  const int full = (P.out / 4 * 4) / 16;  // 16-row blocks made only of dot_lanes8 rows
  for (int blk = 0; blk < full; blk++) {
    const float* wb = P.t16.data() + (size_t)blk * P.inp * 16;
    __m512 a[4], b[4];
    for (int l = 0; l < 4; l++) a[l] = b[l] = _mm512_setzero_ps();
    for (int c = 0; c < P.inp; c += 8)
      for (int l = 0; l < 4; l++) {
        a[l] = _mm512_fmadd_ps(_mm512_set1_ps(x[c + l]), _mm512_loadu_ps(wb + (size_t)(c + l) * 16), a[l]);
        b[l] = _mm512_fmadd_ps(_mm512_set1_ps(x[c + 4 + l]), _mm512_loadu_ps(wb + (size_t)(c + 4 + l) * 16), b[l]);
      }
    const __m512 r = _mm512_add_ps(_mm512_add_ps(_mm512_add_ps(a[0], b[0]), _mm512_add_ps(a[1], b[1])),
                                   _mm512_add_ps(_mm512_add_ps(a[2], b[2]), _mm512_add_ps(a[3], b[3])));
    _mm512_storeu_ps(y + blk * 16, _mm512_add_ps(r, _mm512_loadu_ps(P.bias.data() + blk * 16)));
  }
  gemv_f16_scalar(P, x, y, full * 16, P.out);
}

// gemv_f16 for `nu` tokens: each 16-row block (inp * 64 bytes) is reused from cache by every token before the next
// block is read. Token j reads x + j*ldx and writes y + j*ldy; per token the arithmetic is gemv_f16_avx512's.
__attribute__((target("avx512f"))) void gemv_f16_avx512_multi(const F16Rows& P, int nu, const float* x, size_t ldx,
                                                              float* y, size_t ldy) {
  const int full = (P.out / 4 * 4) / 16;
  for (int blk = 0; blk < full; blk++) {
    const float* wb = P.t16.data() + (size_t)blk * P.inp * 16;
    const __m512 bias = _mm512_loadu_ps(P.bias.data() + blk * 16);
    for (int j = 0; j < nu; j++) {
      const float* xj = x + (size_t)j * ldx;
      __m512 a[4], b[4];
      for (int l = 0; l < 4; l++) a[l] = b[l] = _mm512_setzero_ps();
      for (int c = 0; c < P.inp; c += 8)
        for (int l = 0; l < 4; l++) {
          a[l] = _mm512_fmadd_ps(_mm512_set1_ps(xj[c + l]), _mm512_loadu_ps(wb + (size_t)(c + l) * 16), a[l]);
          b[l] = _mm512_fmadd_ps(_mm512_set1_ps(xj[c + 4 + l]), _mm512_loadu_ps(wb + (size_t)(c + 4 + l) * 16), b[l]);
        }
      const __m512 r = _mm512_add_ps(_mm512_add_ps(_mm512_add_ps(a[0], b[0]), _mm512_add_ps(a[1], b[1])),
                                     _mm512_add_ps(_mm512_add_ps(a[2], b[2]), _mm512_add_ps(a[3], b[3])));
      _mm512_storeu_ps(y + (size_t)j * ldy + blk * 16, _mm512_add_ps(r, bias));
    }
  }
  for (int j = 0; j < nu; j++) gemv_f16_scalar(P, x + (size_t)j * ldx, y + (size_t)j * ldy, full * 16, P.out);
}

void gemv_f16_multi(const Decoder& D, const F16Rows& P, int nu, const float* x, size_t ldx, float* y, size_t ldy) {
  if (D.vnni && P.inp % 8 == 0)
    gemv_f16_avx512_multi(P, nu, x, ldx, y, ldy);
  else
    for (int j = 0; j < nu; j++) gemv_f16_scalar(P, x + (size_t)j * ldx, y + (size_t)j * ldy, 0, P.out);
}

void gemv_f16(const Decoder& D, const F16Rows& P, const float* x, float* y) {
  if (D.vnni && P.inp % 8 == 0)
    gemv_f16_avx512(P, x, y);
  else
    gemv_f16_scalar(P, x, y, 0, P.out);
}

// sigmoid (tensor.rs:784-786) and the LSTM cell's tanh with the correctly rounded exp / tanh of crmath.cuh in place of
// the reference's libm calls, so the host and GPU decoders produce the same bits
float sigmoid(float v) { return 1.0f / (1.0f + crm::expf_cr(-v)); }
static inline float tanh_cr(float v) { return crm::tanhf_cr(v); }

int argmax(const float* v, int n) {  // decoder.rs:194-202: first maximum under a strict '>'
  int best = 0;
  for (int i = 0; i < n; i++)
    if (v[i] > v[best]) best = i;
  return best;
}

// Per-thread scratch of one greedy decode.
struct Scratch {
  std::vector<float> x, gates, gh, z, g, logits, h, c, hn, cn;
  std::vector<int8_t> q;
  std::vector<float> sq;
  explicit Scratch(const Decoder& D)
      : x(D.hidden), gates(4 * D.hidden), gh(4 * D.hidden), z(D.hidden), g(D.hidden),
        logits(D.vocab + D.n_dur), h((size_t)D.n_layers * D.hidden), c(h.size()), hn(h.size()), cn(h.size()),
        q(D.hidden), sq(D.hidden / 128) {}
};

// Decoder::pred_step (decoder.rs:136-175), int8 LSTM branch.
void pred_step(const Decoder& D, Scratch& S, int token, const float* hp_all, const float* cp_all, float* g,
               float* hn_all, float* cn_all) {
  const int h = D.hidden;
  std::memcpy(S.x.data(), D.embedding.data() + (size_t)token * h, sizeof(float) * h);
  for (int l = 0; l < D.n_layers; l++) {
    const float* hp = hp_all + (size_t)l * h;
    const float* cp = cp_all + (size_t)l * h;
    quantize(S.x.data(), h, S.q.data(), S.sq.data());
    gemv_i8(D, D.w_ih[l], S.q.data(), S.sq.data(), D.b[l].data(), S.gates.data());
    quantize(hp, h, S.q.data(), S.sq.data());
    gemv_i8(D, D.w_hh[l], S.q.data(), S.sq.data(), nullptr, S.gh.data());
    for (int k = 0; k < 4 * h; k++) S.gates[k] += S.gh[k];
    float* hn = hn_all + (size_t)l * h;
    float* cn = cn_all + (size_t)l * h;
    for (int k = 0; k < h; k++) {
      const float i = sigmoid(S.gates[k]);
      const float f = sigmoid(S.gates[h + k]);
      const float gg = tanh_cr(S.gates[2 * h + k]);
      const float o = sigmoid(S.gates[3 * h + k]);
      cn[k] = f * cp[k] + i * gg;
      hn[k] = o * tanh_cr(cn[k]);
    }
    std::memcpy(S.x.data(), hn, sizeof(float) * h);
  }
  gemv_f16(D, D.proj, S.x.data(), g);
}

// Decoder::joint (decoder.rs:178-192): head(relu(enc_t + g)) with the int8 head.
void joint(const Decoder& D, Scratch& S, const float* enc_t, const float* g, float* logits) {
  for (int k = 0; k < D.hidden; k++) S.z[k] = std::fmax(enc_t[k] + g[k], 0.0f);
  quantize(S.z.data(), D.hidden, S.q.data(), S.sq.data());
  gemv_i8(D, D.head, S.q.data(), S.sq.data(), D.head_b.data(), logits);
}

// Decoder::greedy (decoder.rs:204-266). The prediction network output is kept across blanks (it depends only on
// the last token and the state).
size_t greedy(const Decoder& D, Scratch& S, const float* proj, int t, vxg_emission* out, size_t cap) {
  const int h = D.hidden;
  std::fill(S.h.begin(), S.h.end(), 0.0f);
  std::fill(S.c.begin(), S.c.end(), 0.0f);
  int last = D.blank, tf = 0;
  size_t n = 0;
  bool have_pred = false;
  while (tf < t) {
    int symbols = 0, dur = 0;
    for (;;) {
      if (!have_pred) {
        pred_step(D, S, last, S.h.data(), S.c.data(), S.g.data(), S.hn.data(), S.cn.data());
        have_pred = true;
      }
      joint(D, S, proj + (size_t)tf * h, S.g.data(), S.logits.data());
      const int k = argmax(S.logits.data(), D.vocab);
      dur = D.durations[argmax(S.logits.data() + D.vocab, D.n_dur)];
      if (k != D.blank) {
        if (n < cap) out[n] = vxg_emission{k, tf, dur};
        n++;
        S.h.swap(S.hn);
        S.c.swap(S.cn);
        have_pred = false;
        last = k;
      }
      symbols++;
      tf += dur;
      if (dur != 0 || symbols >= D.max_symbols) break;
      if (k == D.blank) break;
    }
    if (dur == 0) tf += 1;
  }
  return n;
}

// Decoder::greedy for several utterances in lockstep. Each round every unfinished utterance takes exactly the next
// step of the reference's loop (a prediction-network step first when its cached output is stale, then one joint
// evaluation and the loop's bookkeeping), so its emissions are those of greedy(); the rounds only let the weight
// products of all utterances share one pass over the weights.
struct Lane {
  const float* proj = nullptr;
  int t = 0, tf = 0, symbols = 0, last = 0, dur = 0;
  bool have_pred = false, done = false;
  vxg_emission* out = nullptr;
  size_t cap = 0, n = 0;
};

void greedy_lockstep(const Decoder& D, std::vector<Lane>& lanes) {
  const int h = D.hidden, nl = D.n_layers, U = (int)lanes.size(), nout = D.vocab + D.n_dur, ng = h / 128;
  std::vector<float> H((size_t)U * nl * h, 0.0f), Cs(H.size(), 0.0f), Hn(H.size()), Cn(H.size());
  std::vector<float> G((size_t)U * h), X((size_t)U * h), Z((size_t)U * h), gates((size_t)U * 4 * h),
      gh((size_t)U * 4 * h), hl((size_t)U * h), logits((size_t)U * nout);
  std::vector<int8_t> q((size_t)U * h);
  std::vector<float> sq((size_t)U * ng);
  std::vector<int> idx;
  for (int i = 0; i < U; i++) {
    lanes[i].last = D.blank;
    lanes[i].done = lanes[i].t <= 0;
  }
  for (;;) {
    // prediction-network steps of the lanes whose cached output is stale
    idx.clear();
    for (int i = 0; i < U; i++)
      if (!lanes[i].done && !lanes[i].have_pred) idx.push_back(i);
    const int np = (int)idx.size();
    if (np) {
      for (int j = 0; j < np; j++)
        std::memcpy(&X[(size_t)j * h], D.embedding.data() + (size_t)lanes[idx[j]].last * h, sizeof(float) * h);
      for (int l = 0; l < nl; l++) {
        for (int j = 0; j < np; j++) quantize(&X[(size_t)j * h], h, &q[(size_t)j * h], &sq[(size_t)j * ng]);
        gemv_i8_multi(D, D.w_ih[l], np, q.data(), sq.data(), D.b[l].data(), gates.data(), (size_t)4 * h);
        for (int j = 0; j < np; j++)
          quantize(&H[((size_t)idx[j] * nl + l) * h], h, &q[(size_t)j * h], &sq[(size_t)j * ng]);
        gemv_i8_multi(D, D.w_hh[l], np, q.data(), sq.data(), nullptr, gh.data(), (size_t)4 * h);
        for (int j = 0; j < np; j++) {
          float* gt = &gates[(size_t)j * 4 * h];
          const float* ghj = &gh[(size_t)j * 4 * h];
          for (int k = 0; k < 4 * h; k++) gt[k] += ghj[k];
          const float* cp = &Cs[((size_t)idx[j] * nl + l) * h];
          float* hn = &Hn[((size_t)idx[j] * nl + l) * h];
          float* cn = &Cn[((size_t)idx[j] * nl + l) * h];
          for (int k = 0; k < h; k++) {
            const float i = sigmoid(gt[k]);
            const float f = sigmoid(gt[h + k]);
            const float gg = tanh_cr(gt[2 * h + k]);
            const float o = sigmoid(gt[3 * h + k]);
            cn[k] = f * cp[k] + i * gg;
            hn[k] = o * tanh_cr(cn[k]);
          }
          std::memcpy(&X[(size_t)j * h], hn, sizeof(float) * h);
        }
      }
      gemv_f16_multi(D, D.proj, np, X.data(), (size_t)h, Z.data(), (size_t)h);
      for (int j = 0; j < np; j++) {
        std::memcpy(&G[(size_t)idx[j] * h], &Z[(size_t)j * h], sizeof(float) * h);
        lanes[idx[j]].have_pred = true;
      }
    }
    // one joint evaluation per unfinished lane
    idx.clear();
    for (int i = 0; i < U; i++)
      if (!lanes[i].done) idx.push_back(i);
    const int na = (int)idx.size();
    if (!na) break;
    for (int j = 0; j < na; j++) {
      const Lane& L = lanes[idx[j]];
      const float* e = L.proj + (size_t)L.tf * h;
      const float* g = &G[(size_t)idx[j] * h];
      float* z = &Z[(size_t)j * h];
      for (int k = 0; k < h; k++) z[k] = std::fmax(e[k] + g[k], 0.0f);
      quantize(z, h, &q[(size_t)j * h], &sq[(size_t)j * ng]);
    }
    gemv_i8_multi(D, D.head, na, q.data(), sq.data(), D.head_b.data(), logits.data(), (size_t)nout);
    for (int j = 0; j < na; j++) {
      Lane& L = lanes[idx[j]];
      const float* lg = &logits[(size_t)j * nout];
      const int k = argmax(lg, D.vocab);
      L.dur = D.durations[argmax(lg + D.vocab, D.n_dur)];
      if (k != D.blank) {
        if (L.n < L.cap) L.out[L.n] = vxg_emission{k, L.tf, L.dur};
        L.n++;
        const size_t o = (size_t)idx[j] * nl * h;
        std::memcpy(&H[o], &Hn[o], sizeof(float) * nl * h);
        std::memcpy(&Cs[o], &Cn[o], sizeof(float) * nl * h);
        L.have_pred = false;
        L.last = k;
      }
      L.symbols++;
      L.tf += L.dur;
      if (L.dur != 0 || L.symbols >= D.max_symbols || k == D.blank) {  // the reference's inner loop ends
        if (L.dur == 0) L.tf += 1;
        L.symbols = 0;
        if (L.tf >= L.t) L.done = true;
      }
    }
  }
}

bool cpu_vnni() {
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
         __builtin_cpu_supports("avx512vnni");
}

}  // namespace
}  // namespace tdt
}  // namespace vxg

using namespace vxg;

extern "C" {

vxg_status vxg_tdt_create(const vxg_tdt_desc* desc, vxg_tdt** out) {
  clear_error();
  VXG_ARG(desc && out, "NULL argument");
  *out = nullptr;
  const vxg_tdt_desc& s = *desc;
  VXG_ARG(s.hidden > 0 && s.hidden % 128 == 0 && s.hidden <= 4096, "hidden %d must be a multiple of 128, <= 4096",
          s.hidden);
  VXG_ARG(s.vocab > 0 && s.n_durations > 0 && s.blank >= 0 && s.blank < s.vocab && s.max_symbols > 0 &&
              s.d_model > 0 && s.n_layers >= 1 && s.n_layers <= 4,
          "bad decoder sizes");
  VXG_ARG(s.durations && s.embedding && s.proj_w && s.proj_b && s.head_w && s.head_b && s.enc_w && s.enc_b,
          "NULL weight");
  for (int i = 0; i < s.n_durations; i++) VXG_ARG(s.durations[i] >= 0, "negative duration %d", s.durations[i]);
  for (int l = 0; l < s.n_layers; l++)
    VXG_ARG(s.w_ih[l] && s.w_hh[l] && s.b_ih[l] && s.b_hh[l], "NULL LSTM weight in layer %d", l);
  auto* t = new vxg_tdt();
  tdt::Decoder& D = t->d;
  D.hidden = s.hidden, D.vocab = s.vocab, D.n_dur = s.n_durations, D.blank = s.blank;
  D.max_symbols = s.max_symbols, D.d_model = s.d_model, D.n_layers = s.n_layers;
  D.durations.assign(s.durations, s.durations + s.n_durations);
  const int h = s.hidden;
  D.embedding.assign(s.embedding, s.embedding + (size_t)s.vocab * h);
  D.w_ih.resize(s.n_layers);
  D.w_hh.resize(s.n_layers);
  D.b.resize(s.n_layers);
  for (int l = 0; l < s.n_layers; l++) {
    tdt::i8rows_from_f16(D.w_ih[l], s.w_ih[l], 4 * h, h);
    tdt::i8rows_from_f16(D.w_hh[l], s.w_hh[l], 4 * h, h);
    D.b[l].resize(4 * h);
    for (int k = 0; k < 4 * h; k++) D.b[l][k] = s.b_ih[l][k] + s.b_hh[l][k];  // decoder.rs:74
  }
  tdt::f16rows_from(D.proj, s.proj_w, s.proj_b, h, h);
  tdt::i8rows_from_f16(D.head, s.head_w, s.vocab + s.n_durations, h);
  D.head_b.assign(s.head_b, s.head_b + s.vocab + s.n_durations);
  D.enc_w.assign(s.enc_w, s.enc_w + (size_t)h * s.d_model);
  D.enc_b.assign(s.enc_b, s.enc_b + h);
  D.vnni = tdt::cpu_vnni();
  D.device = s.device;
  if (s.device >= 0) {
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess) e = cudaSetDevice(s.device);
    if (e == cudaSuccess) e = cudaMalloc(&D.enc_w_dev, sizeof(float) * D.enc_w.size());
    if (e == cudaSuccess) e = cudaMalloc(&D.enc_b_dev, sizeof(float) * h);
    if (e == cudaSuccess)
      e = cudaMemcpy(D.enc_w_dev, D.enc_w.data(), sizeof(float) * D.enc_w.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(D.enc_b_dev, D.enc_b.data(), sizeof(float) * h, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaSetDevice(prev);
      vxg_tdt_destroy(t);
      return cuda_fail(e, "vxg_tdt_create: encoder projector upload");
    }
    const vxg_status st = tdt::upload_device_model(D);  // prediction network and joint for vxg_tdt_greedy_device
    cudaSetDevice(prev);
    if (st != VXG_OK) {
      vxg_tdt_destroy(t);
      return st;
    }
  }
  *out = t;
  return VXG_OK;
}

void vxg_tdt_destroy(vxg_tdt* t) {
  if (!t) return;
  if (t->d.enc_w_dev) cudaFree(t->d.enc_w_dev);
  if (t->d.enc_b_dev) cudaFree(t->d.enc_b_dev);
  tdt::free_device_model(t->d);
  delete t;
}

vxg_status vxg_tdt_greedy(const vxg_tdt* t, const float* proj, int frames, vxg_emission* out, size_t cap, size_t* n) {
  clear_error();
  VXG_ARG(t && n && frames >= 0 && (proj || frames == 0) && (out || cap == 0), "bad arguments");
  tdt::Scratch S(t->d);
  *n = tdt::greedy(t->d, S, proj, frames, out, cap);
  return VXG_OK;
}

vxg_status vxg_tdt_greedy_batch(const vxg_tdt* t, int n, const float* const* proj, const int* frames,
                                vxg_emission* const* out, const size_t* cap, size_t* n_out, int threads) {
  clear_error();
  VXG_ARG(t && n >= 0 && (n == 0 || (proj && frames && out && cap && n_out)), "bad arguments");
  for (int u = 0; u < n; u++)
    VXG_ARG(frames[u] >= 0 && (proj[u] || frames[u] == 0) && (out[u] || cap[u] == 0), "utterance %d: bad arguments",
            u);
  int nt = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
  nt = std::max(1, std::min(nt, n));
  // longest utterances first, so the last ones to start are the short ones
  std::vector<int> order(n);
  for (int u = 0; u < n; u++) order[u] = u;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return frames[a] > frames[b]; });
  // each worker decodes groups of utterances of similar length in lockstep: as many as keep every thread busy, at
  // least 8 (one VNNI pass feeds eight) and at most 64
  const int kLockstep = std::max(8, std::min(64, (n + nt - 1) / nt));
  const int groups = (n + kLockstep - 1) / kLockstep;
  std::atomic<int> next{0};
  auto work = [&]() {
    std::vector<tdt::Lane> lanes;
    for (int gi = next.fetch_add(1); gi < groups; gi = next.fetch_add(1)) {
      lanes.assign(std::min(kLockstep, n - gi * kLockstep), tdt::Lane{});
      for (size_t j = 0; j < lanes.size(); j++) {
        const int u = order[gi * kLockstep + (int)j];
        lanes[j].proj = proj[u];
        lanes[j].t = frames[u];
        lanes[j].out = out[u];
        lanes[j].cap = cap[u];
      }
      tdt::greedy_lockstep(t->d, lanes);
      for (size_t j = 0; j < lanes.size(); j++) n_out[order[gi * kLockstep + (int)j]] = lanes[j].n;
    }
  };
  std::vector<std::thread> pool;
  for (int i = 1; i < nt; i++) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
  return VXG_OK;
}

vxg_status vxg_tdt_pred_step(const vxg_tdt* t, int token, const float* h, const float* c, float* g, float* h_out,
                             float* c_out) {
  clear_error();
  VXG_ARG(t && h && c && g && h_out && c_out, "NULL argument");
  VXG_ARG(token >= 0 && token < t->d.vocab, "token %d out of range", token);
  tdt::Scratch S(t->d);
  tdt::pred_step(t->d, S, token, h, c, g, h_out, c_out);
  return VXG_OK;
}

vxg_status vxg_tdt_joint(const vxg_tdt* t, const float* enc_t, const float* g, float* logits) {
  clear_error();
  VXG_ARG(t && enc_t && g && logits, "NULL argument");
  tdt::Scratch S(t->d);
  tdt::joint(t->d, S, enc_t, g, logits);
  return VXG_OK;
}

}  // extern "C"
