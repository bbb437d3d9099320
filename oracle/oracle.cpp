/*
 * CPU oracle: scalar restatement of the reference's int8 encoder path (test infrastructure; see oracle.h).
 * Build: -O2 -ffp-contract=off -fno-fast-math. Every `mul_add` of the reference is fmaf() here; every other float
 * expression keeps the reference's left-to-right association.
 */
#include "oracle.h"
#include "oracle_internal.h"

#include <algorithm>
#include <cfloat>
#include <atomic>
#include <cfenv>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace vxo {

/* ------------------------------------------------------------------------------------------------ thread pool */

namespace {
struct Pool {
  std::mutex mu;
  std::condition_variable cv, done_cv;
  std::vector<std::thread> workers;
  const std::function<void(int)>* job = nullptr;
  std::atomic<int> next{0};
  int n = 0, active = 0;
  uint64_t gen = 0;
  bool stop = false;
  int want = 0; /* 0 = hardware threads */

  int size() const {
    int w = want > 0 ? want : (int)std::thread::hardware_concurrency();
    return w < 1 ? 1 : w;
  }
  void resize() {
    shutdown();
    stop = false;
    int w = size();
    for (int i = 1; i < w; i++) workers.emplace_back([this] { loop(); });
  }
  void shutdown() {
    {
      std::lock_guard<std::mutex> g(mu);
      stop = true;
    }
    cv.notify_all();
    for (auto& t : workers) t.join();
    workers.clear();
  }
  void work() {
    for (;;) {
      int i = next.fetch_add(1);
      if (i >= n) break;
      (*job)(i);
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> l(mu);
      cv.wait(l, [&] { return stop || gen != seen; });
      if (stop) return;
      seen = gen;
      active++;
      l.unlock();
      work();
      l.lock();
      if (--active == 0) done_cv.notify_all();
    }
  }
  void run(int count, const std::function<void(int)>& f) {
    if (count <= 0) return;
    if (workers.empty() || count == 1) {
      for (int i = 0; i < count; i++) f(i);
      return;
    }
    {
      std::lock_guard<std::mutex> g(mu);
      job = &f;
      n = count;
      next = 0;
      gen++;
    }
    cv.notify_all();
    work();
    std::unique_lock<std::mutex> l(mu);
    done_cv.wait(l, [&] { return active == 0 && next.load() >= n; });
    job = nullptr;
  }
  ~Pool() { shutdown(); }
};

Pool& pool() {
  static Pool p;
  static bool init = [] {
    p.resize();
    return true;
  }();
  (void)init;
  return p;
}
std::mutex pool_run_mu; /* one parallel region at a time (no nesting) */
thread_local bool in_region = false;
} // namespace

void parallel_for(int n, const std::function<void(int)>& f) {
  if (in_region) { /* nested: run inline */
    for (int i = 0; i < n; i++) f(i);
    return;
  }
  std::lock_guard<std::mutex> g(pool_run_mu);
  in_region = true;
  std::function<void(int)> wrapped = [&](int i) {
    bool prev = in_region;
    in_region = true;
    f(i);
    in_region = prev;
  };
  pool().run(n, wrapped);
  in_region = false;
}

int threads() { return pool().size(); }

/* ---------------------------------------------------------------------------------------------- scalar math */

static inline float hsum4(const float a[4]) { return (a[0] + a[1]) + (a[2] + a[3]); } /* tensor.rs:227-229 */

static inline float rte(float v) { return std::nearbyintf(v); } /* round_ties_even under FE_TONEAREST */

static inline float fclamp(float x, float lo, float hi) { /* Rust f32::clamp: NaN passes through */
  if (x < lo) x = lo;
  if (x > hi) x = hi;
  return x;
}

/* packed.rs:527-535 quantize_group_portable (bit-equal to the AVX2/NEON paths, packed.rs:453-522) */
float quantize_group(const float* src, int n, int8_t* dst) {
  float amax = 0.0f;
  for (int i = 0; i < n; i++) amax = std::fmax(amax, std::fabs(src[i]));
  float s = amax == 0.0f ? 1.0f : amax / 127.0f;
  float inv = 1.0f / s;
  for (int i = 0; i < n; i++) {
    float q = fclamp(rte(src[i] * inv), -127.0f, 127.0f);
    dst[i] = std::isnan(q) ? (int8_t)0 : (int8_t)q; /* Rust `as i8` saturates, NaN -> 0 */
  }
  return s;
}

/* tensor.rs:829-831 */
static const float EXP_LN2_HI = 0.69314575f;
static const float EXP_LN2_LO = 1.4286068e-6f;
static const float EXP_POLY[6] = {1.0f / 120.0f, 1.0f / 24.0f, 1.0f / 6.0f, 0.5f, 1.0f, 1.0f};
static const float LOG2_E = 1.44269504088896340736f;

/* tensor.rs:838-848 exp_poly */
float exp_poly(float x) {
  x = fclamp(x, -87.0f, 88.0f);
  float n = rte(x * LOG2_E);
  float r = std::fmaf(-n, EXP_LN2_HI, x);
  r = std::fmaf(-n, EXP_LN2_LO, r);
  float p = 1.0f / 720.0f;
  for (int i = 0; i < 6; i++) p = std::fmaf(p, r, EXP_POLY[i]);
  uint32_t bits = (uint32_t)(((int32_t)n + 127) << 23);
  float e;
  std::memcpy(&e, &bits, 4);
  return p * e;
}

float silu_fast(float x) { return x / (1.0f + exp_poly(-x)); }    /* tensor.rs:852-854 */
float sigmoid_fast(float x) { return 1.0f / (1.0f + exp_poly(-x)); } /* tensor.rs:858-860 */

/* tensor.rs:333-362 row_mean_var_portable */
static void row_mean_var(const float* xi, int d, float* mean_out, float* var_out) {
  int n8 = d / 8 * 8;
  float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
  for (int c = 0; c < n8; c += 8)
    for (int l = 0; l < 4; l++) {
      s0[l] += xi[c + l];
      s1[l] += xi[c + 4 + l];
    }
  float t4[4];
  for (int l = 0; l < 4; l++) t4[l] = s0[l] + s1[l];
  float sum = hsum4(t4);
  for (int c = n8; c < d; c++) sum += xi[c];
  float mean = sum / (float)d;
  float q0[4] = {0, 0, 0, 0}, q1[4] = {0, 0, 0, 0};
  for (int c = 0; c < n8; c += 8)
    for (int l = 0; l < 4; l++) {
      float a = xi[c + l] - mean, e = xi[c + 4 + l] - mean;
      q0[l] = std::fmaf(a, a, q0[l]);
      q1[l] = std::fmaf(e, e, q1[l]);
    }
  for (int l = 0; l < 4; l++) t4[l] = q0[l] + q1[l];
  float sq = hsum4(t4);
  for (int c = n8; c < d; c++) {
    float a = xi[c] - mean;
    sq += a * a;
  }
  *mean_out = mean;
  *var_out = sq / (float)d;
}

/* tensor.rs:712-719 layer_norm_row (eps 1e-5, biased variance) */
static void layer_norm_row(const float* xi, const float* g, const float* b, int d, float* y) {
  float mean, var;
  row_mean_var(xi, d, &mean, &var);
  float inv = 1.0f / std::sqrt(var + 1e-5f);
  for (int k = 0; k < d; k++) y[k] = (xi[k] - mean) * inv * g[k] + b[k];
}

static float apply_ep(int ep, float s, float old, float v) { /* kernels/mod.rs:42-48 */
  switch (ep) {
    case VXO_EP_SILU: return silu_fast(v);
    case VXO_EP_ADD_SCALED: return std::fmaf(s, v, old);
    default: return v;
  }
}

void group_sums(const int8_t* x, int n, int inp, int group, int32_t* gsum) {
  int ng = inp / group;
  for (int t = 0; t < n; t++)
    for (int g = 0; g < ng; g++) {
      int32_t s = 0;
      for (int c = g * group; c < (g + 1) * group; c++) s += x[(size_t)t * inp + c];
      gsum[(size_t)t * ng + g] = s;
    }
}

} // namespace vxo

using namespace vxo;

/* ------------------------------------------------------------------------------------------------- C API */

extern "C" {

void vxo_set_threads(int n) {
  Pool& p = pool();
  p.want = n;
  p.resize();
}
int vxo_get_threads(void) { return vxo::threads(); }

/* trits.rs:7-27 */
void vxo_unpack_row(const uint8_t* packed, int in_features, int8_t* out) {
  int full = in_features / 5;
  for (int i = 0; i < full; i++) {
    unsigned v = packed[i];
    for (int s = 0; s < 5; s++) {
      out[i * 5 + s] = (int8_t)((int)(v % 3) - 1);
      v /= 3;
    }
  }
  int rem = in_features - full * 5;
  if (rem > 0) {
    unsigned v = packed[full];
    for (int s = 0; s < rem; s++) {
      out[full * 5 + s] = (int8_t)((int)(v % 3) - 1);
      v /= 3;
    }
  }
}

/* trits.rs:30-41 (pad digits 0) */
void vxo_pack_row(const int8_t* trits, int n, uint8_t* out) {
  int nb = (n + 4) / 5;
  for (int i = 0; i < nb; i++) {
    unsigned v = 0, p = 1;
    for (int s = 0; s < 5 && i * 5 + s < n; s++) {
      v += (unsigned)(trits[i * 5 + s] + 1) * p;
      p *= 3;
    }
    out[i] = (uint8_t)v;
  }
}

/* IEEE binary16 -> binary32, exact (half 2.7.1 `to_f32`) */
float vxo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400));
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

/* TernaryMatrix::from_packed_layout, Rows layout (packed.rs:73-130) */
void vxo_unpack_matrix(const uint8_t* qweight, const uint16_t* scales_f16, int out, int in, int group, int8_t* w,
                       float* scales) {
  int rb = (in + 4) / 5, ng = in / group;
  for (int r = 0; r < out; r++) vxo_unpack_row(qweight + (size_t)r * rb, in, w + (size_t)r * in);
  for (size_t i = 0; i < (size_t)out * ng; i++) scales[i] = vxo_f16_to_f32(scales_f16[i]);
}

float vxo_quantize_group(const float* src, int n, int8_t* dst) { return quantize_group(src, n, dst); }

/* QuantAct::quantize (packed.rs:302-312 -> from_rows :317-436): per (token, group) */
void vxo_quantize_rows(const float* x, int n, int inp, int group, int8_t* q, float* scales) {
  int ng = inp / group;
  parallel_for(n, [&](int t) {
    for (int g = 0; g < ng; g++)
      scales[(size_t)t * ng + g] =
          quantize_group(x + (size_t)t * inp + g * group, group, q + (size_t)t * inp + g * group);
  });
}

void vxo_layer_norm_row(const float* x, const float* g, const float* b, int d, float* y) {
  layer_norm_row(x, g, b, d, y);
}

/* TernaryLinear::prepare_normed (ternary_linear.rs:132-158): LayerNorm row -> quantise, no f32 intermediate kept */
void vxo_ln_quant_rows(const float* x, int n, int d, const float* g, const float* b, int group, int8_t* q,
                       float* scales) {
  int ng = d / group;
  parallel_for(n, [&](int t) {
    std::vector<float> row(d);
    layer_norm_row(x + (size_t)t * d, g, b, d, row.data());
    for (int gi = 0; gi < ng; gi++)
      scales[(size_t)t * ng + gi] =
          quantize_group(row.data() + gi * group, group, q + (size_t)t * d + gi * group);
  });
}

/* gemm_scalar_range (kernels/mod.rs:166-210) + Epilogue::apply (:42-48) + gemm_ep's bias add (:355-361) */
void vxo_gemm(const int8_t* w, const float* sw, const int8_t* x, const float* sx, int M, int N, int K, int G,
              int ep, float ep_scale, const float* bias, float* y, int32_t* sums, int r0, int r1, int t0, int t1) {
  (void)M;
  int ng = K / G;
  parallel_for(r1 - r0, [&](int oi) {
    int o = r0 + oi;
    const int8_t* wr = w + (size_t)o * K;
    for (int t = t0; t < t1; t++) {
      const int8_t* xr = x + (size_t)t * K;
      float acc = 0.0f;
      for (int gi = 0; gi < ng; gi++) {
        int32_t s = 0;
        for (int c = gi * G; c < (gi + 1) * G; c++) s += (int32_t)wr[c] * (int32_t)xr[c];
        if (sums) sums[((size_t)t * N + o) * ng + gi] = s;
        acc = std::fmaf((float)s, sx[(size_t)t * ng + gi] * sw[(size_t)o * ng + gi], acc);
      }
      float* slot = &y[(size_t)t * N + o];
      float v = apply_ep(ep, ep_scale, *slot, acc);
      if (bias) v += bias[o];
      *slot = v;
    }
  });
}

float vxo_exp_poly(float x) { return exp_poly(x); }
float vxo_silu_fast(float x) { return silu_fast(x); }
float vxo_sigmoid_fast(float x) { return sigmoid_fast(x); }

/* Correctly rounded f32 exp and tanh, the definition the library's decoder and VAD use for the reference's libm
 * calls: evaluated in x87 extended precision (64-bit significand) and rounded to f32. Exact except where the
 * extended result lies within its own error (~2^-63) of a halfway point, which the exhaustive checks would show. */
static float expf_cr(float x) { return (float)expl((long double)x); }
static float tanhf_cr(float x) { return (float)tanhl((long double)x); }
void vxo_math_cr(int fn, const float* x, size_t n, float* y) {
  parallel_for((int)((n + 65535) / 65536), [&](int b) {
    const size_t a = (size_t)b * 65536, e = std::min(n, a + 65536);
    for (size_t i = a; i < e; i++) y[i] = fn == 0 ? expf_cr(x[i]) : tanhf_cr(x[i]);
  });
}

/* VadHead::probs (vad.rs:39-82) for one utterance: sub [t, d] -> p [t]. proj + relu with acc = b, acc += w * x in
 * column order; ctx conv (k taps, same padding, out-of-range taps skipped) ci-outer kk-inner + relu; out: z = b,
 * z += w * h in order; p = 1 / (1 + expf(-z)) with the correctly rounded expf above. */
void vxo_vad_probs(const float* sub, int t, int d, int h, int k, const float* proj_w, const float* proj_b,
                   const float* ctx_w, const float* ctx_b, const float* out_w, float out_b, float* p) {
  const int pad = (k - 1) / 2;
  std::vector<float> a((size_t)t * h), hb(h);
  for (int i = 0; i < t; i++)
    for (int j = 0; j < h; j++) {
      float acc = proj_b[j];
      for (int c = 0; c < d; c++) acc += proj_w[(size_t)j * d + c] * sub[(size_t)i * d + c];
      a[(size_t)i * h + j] = std::fmax(acc, 0.0f);
    }
  for (int i = 0; i < t; i++) {
    for (int o = 0; o < h; o++) {
      float acc = ctx_b[o];
      for (int ci = 0; ci < h; ci++)
        for (int kk = 0; kk < k; kk++) {
          const int j = i + kk - pad;
          if (j >= 0 && j < t) acc += ctx_w[((size_t)o * h + ci) * k + kk] * a[(size_t)j * h + ci];
        }
      hb[o] = std::fmax(acc, 0.0f);
    }
    float z = out_b;
    for (int o = 0; o < h; o++) z += out_w[o] * hb[o];
    p[i] = 1.0f / (1.0f + expf_cr(-z));
  }
}

/* segment (vad.rs:140-240): speech runs [start, end) in frames written as pairs to out (at most cap); returns the
 * count. Steps: runs with short pauses tolerated; short runs merged into the previous one within max_frames; runs
 * above max_frames cut at the first minimum of the window's last min(63, max/2) frames; padding bounded by the
 * midpoints of the gaps. */
int vxo_segment(const float* p, int t, float thr, int min_pause, int max_frames, int min_frames, int pad, int* out,
                int cap) {
  if (t <= 0) return 0;
  std::vector<std::pair<int, int>> runs, merged, segs;
  int i = 0;
  while (i < t) {
    if (p[i] >= thr) {
      const int s = i;
      int last = i;
      while (i < t) {
        if (p[i] >= thr) {
          last = i++;
          continue;
        }
        int j = i;
        while (j < t && p[j] < thr) j++;
        const bool stop = j - i >= min_pause || j == t;
        i = j;
        if (stop) break;
      }
      runs.push_back({s, last + 1});
    } else {
      i++;
    }
  }
  if (runs.empty()) segs.push_back({0, t});
  for (auto r : runs) {
    if (!merged.empty() &&
        (r.second - r.first < min_frames || merged.back().second - merged.back().first < min_frames) &&
        r.second - merged.back().first <= max_frames)
      merged.back().second = r.second;
    else
      merged.push_back(r);
  }
  for (auto r : merged) {
    int s = r.first;
    while (r.second - s > max_frames) {
      const int win_end = s + max_frames, look = std::min(63, max_frames / 2);
      int best = win_end;
      float best_p = FLT_MAX;
      for (int f = win_end - look; f < win_end; f++)
        if (p[f] < best_p) best_p = p[f], best = f;
      segs.push_back({s, std::max(best, s + 1)});
      s = std::max(best, s + 1);
    }
    segs.push_back({s, r.second});
  }
  if (!runs.empty()) {
    const int n = (int)segs.size();
    std::vector<std::pair<int, int>> b(n);
    for (int q = 0; q < n; q++) {
      b[q].first = q == 0 ? 0 : segs[q - 1].second + (segs[q].first - segs[q - 1].second + 1) / 2;
      b[q].second = q + 1 == n ? t : segs[q].second + (segs[q + 1].first - segs[q].second) / 2;
    }
    for (int q = 0; q < n; q++) {
      segs[q].first = std::max(std::max(segs[q].first - pad, 0), b[q].first);
      segs[q].second = std::min(segs[q].second + pad, b[q].second);
    }
  }
  for (int q = 0; q < std::min(cap, (int)segs.size()); q++) out[2 * q] = segs[q].first, out[2 * q + 1] = segs[q].second;
  return (int)segs.size();
}

/* glu_row_portable (tensor.rs:917-924) over n rows of g [n, 2d]: a[i, c] = g[i, c] * sigmoid_fast(g[i, d + c]) */
void vxo_glu_rows(const float* g, int n, int d, float* a) {
  for (int i = 0; i < n; i++)
    for (int c = 0; c < d; c++) a[(size_t)i * d + c] = g[(size_t)i * 2 * d + c] * sigmoid_fast(g[(size_t)i * 2 * d + d + c]);
}

/* exp_row_scaled_portable (tensor.rs:810-826) */
float vxo_exp_row_scaled(float* row, int n, float scale) {
  float mx = -INFINITY;
  for (int j = 0; j < n; j++) mx = std::fmax(mx, row[j] * scale);
  float lanes[4] = {0, 0, 0, 0};
  int n4 = n / 4 * 4;
  for (int j = 0; j < n4; j += 4)
    for (int l = 0; l < 4; l++) {
      row[j + l] = exp_poly(row[j + l] * scale - mx);
      lanes[l] += row[j + l];
    }
  float sum = hsum4(lanes);
  for (int j = n4; j < n; j++) {
    row[j] = exp_poly(row[j] * scale - mx);
    sum += row[j];
  }
  return sum;
}

/* linear (tensor.rs:98-127): n == 1 -> gemv_portable (:285-303, dot_lanes8 :266-281 / dot :79-95); otherwise
 * tile_rows_portable (:233-260): per (row, token) four fused lanes over 4-column steps, hsum4, tail, bias */
void vxo_linear(const float* x, int n, int in_f, const float* w, const float* b, int out_f, float* y) {
  if (n == 1) {
    int o4 = out_f / 4 * 4;
    for (int o = 0; o < out_f; o++) {
      const float* wr = w + (size_t)o * in_f;
      float r;
      if (o < o4) {
        int n8 = in_f / 8 * 8;
        float a[4] = {0, 0, 0, 0}, bb[4] = {0, 0, 0, 0};
        for (int c = 0; c < n8; c += 8)
          for (int l = 0; l < 4; l++) {
            a[l] = std::fmaf(x[c + l], wr[c + l], a[l]);
            bb[l] = std::fmaf(x[c + 4 + l], wr[c + 4 + l], bb[l]);
          }
        float t4[4];
        for (int l = 0; l < 4; l++) t4[l] = a[l] + bb[l];
        r = hsum4(t4);
        for (int c = n8; c < in_f; c++) r += x[c] * wr[c];
      } else {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int n8 = in_f / 8 * 8;
        for (int c = 0; c < n8; c += 8)
          for (int k = 0; k < 8; k++) acc[k] += x[c + k] * wr[c + k];
        float s = -0.0f;
        for (int k = 0; k < 8; k++) s = s + acc[k];
        for (int c = n8; c < in_f; c++) s += x[c] * wr[c];
        r = s;
      }
      y[o] = r + (b ? b[o] : 0.0f);
    }
    return;
  }
  int c4 = in_f / 4 * 4;
  parallel_for(n, [&](int tk) {
    const float* xr = x + (size_t)tk * in_f;
    for (int o = 0; o < out_f; o++) {
      const float* wr = w + (size_t)o * in_f;
      float acc[4] = {0, 0, 0, 0};
      for (int c = 0; c < c4; c += 4)
        for (int l = 0; l < 4; l++) acc[l] = std::fmaf(wr[c + l], xr[c + l], acc[l]);
      float tail = 0.0f;
      for (int c = c4; c < in_f; c++) tail += wr[c] * xr[c];
      y[(size_t)tk * out_f + o] = hsum4(acc) + tail + (b ? b[o] : 0.0f);
    }
  });
}

/* rel_pos_table (encoder.rs:760-776). The reference calls Rust libm 0.2.16 (a musl port); this uses the host C
 * library's powf/sinf/cosf, so the table is pinned only up to libm's last-ulp differences. Both the oracle and the
 * CUDA path consume the table this function makes. */
void vxo_rel_pos_table(int t, int d, float* out) {
  int np = 2 * t - 1, half = d / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; i++) inv[i] = 1.0f / powf(10000.0f, 2.0f * (float)i / (float)d);
  for (int r = 0; r < np; r++) {
    float pos = (float)((int64_t)t - 1 - r);
    for (int i = 0; i < half; i++) {
      float f = inv[i] * pos;
      out[(size_t)r * d + 2 * i] = sinf(f);
      out[(size_t)r * d + 2 * i + 1] = cosf(f);
    }
  }
}

/* ConvModule::load BN fold (encoder.rs:555-570) and tap-major transpose (:571-577) */
void vxo_fold_bn(const float* dw, const float* gamma, const float* beta, const float* mean, const float* var, int d,
                 int k, float* dw_t, float* dw_bias) {
  for (int c = 0; c < d; c++) {
    float s = gamma[c] / std::sqrt(var[c] + 1e-5f);
    for (int kk = 0; kk < k; kk++) dw_t[kk * d + c] = dw[c * k + kk] * s;
    dw_bias[c] = beta[c] - mean[c] * s;
  }
}

} // extern "C"

/* --------------------------------------------------------------------------------------- attention core */

namespace {

/* gemm_rows_range of the attention core (kernels/mod.rs:257-282): int8 "weight" rows (from_f32_rows) x int8 acts
 * with one group per row, Store epilogue. Writes y[(t - t0) * W.out + o] for t in [t0, t1), o in [r0, r1): the
 * token range is taken relative to the activation pointers, so callers keep only their own rows. */
void rows_gemm(const Q16* W, const int8_t* x, const float* sx, const int32_t* gsum, float* y, int r0, int r1, int t0,
               int t1) {
  const int ng = W->inp / W->group;
  q16_gemm_range(W, x + (size_t)t0 * W->inp, sx + (size_t)t0 * ng, gsum + (size_t)t0 * ng, t1 - t0, VXO_EP_STORE,
                 0.0f, y, r0, r1, 0, t1 - t0);
}

} // namespace

/* attn_core_int8 restricted to the 8-row query blocks listed in `blocks` (all blocks when blocks == NULL): query rows
 * are independent once the per-head operands (Qu, Qv, K, R, V^T and their scales) are quantised over all frames, so a
 * subset of blocks gives exactly the full computation's rows; the other rows of ctx are left untouched. */
static void attn_core_blocks(const float* qkv, const float* rel_k, int t, int d, int h, int dh, const float* bias_u,
                             const float* bias_v, float scaling, float* ctx, const int* blocks, int n_blocks);

extern "C" void vxo_attn_core_int8(const float* qkv, const float* rel_k, int t, int d, int h, int dh,
                                   const float* bias_u, const float* bias_v, float scaling, float* ctx) {
  attn_core_blocks(qkv, rel_k, t, d, h, dh, bias_u, bias_v, scaling, ctx, nullptr, 0);
}

extern "C" void vxo_attn_core_int8_rows(const float* qkv, const float* rel_k, int t, int d, int h, int dh,
                                        const float* bias_u, const float* bias_v, float scaling, float* ctx,
                                        const int* blocks, int n_blocks) {
  attn_core_blocks(qkv, rel_k, t, d, h, dh, bias_u, bias_v, scaling, ctx, blocks, n_blocks);
}

static void attn_core_blocks(const float* qkv, const float* rel_k, int t, int d, int h, int dh, const float* bias_u,
                             const float* bias_v, float scaling, float* ctx, const int* blocks, int n_blocks) {
  /* encoder.rs:317-534 (int8 context: VOXRT_ATTN_CTX default) */
  const int np = 2 * t - 1;
  const int t2 = (t + 1) / 2 * 2, np2 = (np + 1) / 2 * 2, t16 = (t + 15) / 16 * 16;
  const int d3 = 3 * d;
  struct HeadOps {
    std::vector<int8_t> qu, qv, k, rel, v;
    std::vector<float> squ, sqv, sk, srel, sv;
    std::vector<int32_t> gqu, gqv;
    Q16 *k16 = nullptr, *rel16 = nullptr, *v16 = nullptr;
  };
  std::vector<HeadOps> ops(h);
  /* per (head, operand) tasks (encoder.rs:349-417) */
  parallel_for(h * 5, [&](int item) {
    int head = item / 5, kind = item % 5;
    HeadOps& op = ops[head];
    std::vector<float> row(std::max(dh, t16));
    if (kind == 0 || kind == 1) { /* QuantAct::from_rows(t, dh, dh): q + bias */
      const float* bias = (kind == 0 ? bias_u : bias_v) + head * dh;
      std::vector<int8_t>& q = kind == 0 ? op.qu : op.qv;
      std::vector<float>& s = kind == 0 ? op.squ : op.sqv;
      std::vector<int32_t>& gs = kind == 0 ? op.gqu : op.gqv;
      q.assign((size_t)t * dh, 0);
      s.assign(t, 0.0f);
      gs.assign(t, 0);
      for (int i = 0; i < t; i++) {
        const float* qi = qkv + (size_t)i * d3 + head * dh;
        for (int c = 0; c < dh; c++) row[c] = qi[c] + bias[c];
        s[i] = quantize_group(row.data(), dh, q.data() + (size_t)i * dh);
      }
      group_sums(q.data(), t, dh, dh, gs.data());
    } else if (kind == 2) { /* from_f32_rows(t2, dh, dh): keys, zero rows past t */
      op.k.assign((size_t)t2 * dh, 0);
      op.sk.assign(t2, 0.0f);
      for (int j = 0; j < t2; j++) {
        if (j < t)
          for (int c = 0; c < dh; c++) row[c] = qkv[(size_t)j * d3 + d + head * dh + c];
        else
          std::fill(row.begin(), row.begin() + dh, 0.0f);
        op.sk[j] = quantize_group(row.data(), dh, op.k.data() + (size_t)j * dh);
      }
      op.k16 = q16_prepare(op.k.data(), op.sk.data(), t2, dh, dh, false);
    } else if (kind == 3) { /* from_f32_rows(np2, dh, dh): relative positions */
      op.rel.assign((size_t)np2 * dh, 0);
      op.srel.assign(np2, 0.0f);
      for (int p = 0; p < np2; p++) {
        if (p < np)
          for (int c = 0; c < dh; c++) row[c] = rel_k[(size_t)p * d + head * dh + c];
        else
          std::fill(row.begin(), row.begin() + dh, 0.0f);
        op.srel[p] = quantize_group(row.data(), dh, op.rel.data() + (size_t)p * dh);
      }
      op.rel16 = q16_prepare(op.rel.data(), op.srel.data(), np2, dh, dh, false);
    } else { /* from_f32_rows(dh, t16, t16): vᵀ per channel over time, one group */
      op.v.assign((size_t)dh * t16, 0);
      op.sv.assign(dh, 0.0f);
      for (int c = 0; c < dh; c++) {
        for (int i = 0; i < t; i++) row[i] = qkv[(size_t)i * d3 + 2 * d + head * dh + c];
        for (int i = t; i < t16; i++) row[i] = 0.0f;
        op.sv[c] = quantize_group(row.data(), t16, op.v.data() + (size_t)c * t16);
      }
      op.v16 = q16_prepare(op.v.data(), op.sv.data(), dh, t16, t16, false);
    }
  });
  const int nb = blocks ? n_blocks : (t + 7) / 8;
  /* one task per (head, 8 query rows) (encoder.rs:440-532) */
  parallel_for(h * nb, [&](int item) {
    int head = item / nb, blk = blocks ? blocks[item % nb] : item % nb;
    int i0 = blk * 8, rows = std::min(8, t - i0);
    const HeadOps& op = ops[head];
    std::vector<float> s1((size_t)rows * t2), s2((size_t)rows * np2);
    rows_gemm(op.k16, op.qu.data(), op.squ.data(), op.gqu.data(), s1.data(), 0, t2, i0, i0 + rows);
    /* position band p = t-1-i+j for these rows, widened to even row pairs (encoder.rs:469-473) */
    int p0 = (t - i0 - rows) & ~1;
    int p1 = (2 * t - 1 - i0 + 1) / 2 * 2;
    rows_gemm(op.rel16, op.qv.data(), op.sqv.data(), op.gqv.data(), s2.data(), p0, p1, i0, i0 + rows);
    std::vector<float> probs((size_t)8 * t16, 0.0f);
    float inv_sum[8];
    for (int r = 0; r < rows; r++) {
      int i = i0 + r;
      float* prow = probs.data() + (size_t)r * t16;
      for (int j = 0; j < t; j++) prow[j] = s1[(size_t)r * t2 + j] + s2[(size_t)r * np2 + (t - 1 - i) + j];
      inv_sum[r] = 1.0f / vxo_exp_row_scaled(prow, t, scaling);
      for (int j = t; j < t16; j++) prow[j] = 0.0f;
    }
    /* int8 probabilities (per-row scale absmax/127, 1/Σ folded into the scale) x int8 vᵀ (encoder.rs:489-502) */
    std::vector<int8_t> qp((size_t)rows * t16);
    std::vector<float> sp(rows);
    std::vector<int32_t> gp(rows);
    for (int r = 0; r < rows; r++) {
      sp[r] = quantize_group(probs.data() + (size_t)r * t16, t16, qp.data() + (size_t)r * t16);
      sp[r] *= inv_sum[r];
    }
    group_sums(qp.data(), rows, t16, t16, gp.data());
    std::vector<float> out((size_t)rows * dh);
    rows_gemm(op.v16, qp.data(), sp.data(), gp.data(), out.data(), 0, dh, 0, rows);
    for (int r = 0; r < rows; r++)
      std::memcpy(ctx + (size_t)(i0 + r) * d + head * dh, out.data() + (size_t)r * dh, dh * sizeof(float));
  });
  for (auto& op : ops) {
    q16_free(op.k16);
    q16_free(op.rel16);
    q16_free(op.v16);
  }
}

/* ConvModule::forward_fused middle (encoder.rs:596-624): GLU (glu_row_portable, tensor.rs:917-924), depthwise conv
 * over time with folded BN (bias first, taps in order, multiply then add, zero padding), SiLU (tensor.rs:966-972). */
extern "C" void vxo_conv_middle(const float* g, int t, int d, int k, const float* dw_w, const float* dw_b, float* hb) {
  const int pad = (k - 1) / 2;
  std::vector<float> a((size_t)t * d);
  parallel_for(t, [&](int i) {
    const float* gi = g + (size_t)i * 2 * d;
    for (int c = 0; c < d; c++) a[(size_t)i * d + c] = gi[c] * sigmoid_fast(gi[d + c]);
  });
  parallel_for(t, [&](int i) {
    float* row = hb + (size_t)i * d;
    std::memcpy(row, dw_b, d * sizeof(float));
    for (int kk = 0; kk < k; kk++) {
      int j = i + kk;
      if (j >= pad && j - pad < t) {
        const float* w = dw_w + (size_t)kk * d;
        const float* aj = a.data() + (size_t)(j - pad) * d;
        for (int c = 0; c < d; c++) row[c] += w[c] * aj[c];
      }
    }
    for (int c = 0; c < d; c++) row[c] = silu_fast(row[c]);
  });
}

/* ---------------------------------------------------------------------------------------------- layer */

namespace {

struct Prep {
  Q16* m[9] = {};
};

void tern_gemm(const Q16* W, const int8_t* xq, const float* sx, int n, int ep, float s, float* y) {
  q16_gemm_ep(W, xq, sx, n, ep, s, nullptr, y);
}

} // namespace

/* Load-time repack of a layer's nine ternary modules (TernaryLinear::load_stacked -> Quad16, packed.rs:73-161). */
extern "C" void* vxo_layer_prepare(const vxo_layer* L) {
  const vxo_tern* mods[9] = {&L->ff1_1, &L->ff1_2, &L->qkv, &L->o, &L->relk, &L->pw1, &L->pw2, &L->ff2_1, &L->ff2_2};
  Prep* P = new Prep;
  for (int i = 0; i < 9; i++)
    P->m[i] = q16_prepare(mods[i]->w, mods[i]->s, mods[i]->out, mods[i]->in, mods[i]->group, true);
  return P;
}

extern "C" void vxo_layer_free(void* prep) {
  Prep* P = static_cast<Prep*>(prep);
  if (!P) return;
  for (int i = 0; i < 9; i++) q16_free(P->m[i]);
  delete P;
}

extern "C" void vxo_layer_forward_prepared(void* prep, const vxo_layer* L, int d, int heads, int k, float* x, int t,
                                           const float* pos_emb) {
  /* ConformerLayer::forward_profiled (encoder.rs:706-756) */
  Prep& P = *static_cast<Prep*>(prep);
  const int ff = L->ff1_1.out, G = L->ff1_1.group, dh = d / heads;
  std::vector<int8_t> aq((size_t)t * std::max(ff, 2 * d));
  std::vector<float> as((size_t)t * (std::max(ff, 2 * d) / G));
  std::vector<float> hbuf((size_t)t * std::max(ff, 3 * d));

  auto ffn = [&](const float* g, const float* b, const Q16* w1, const Q16* w2) { /* encoder.rs:79-94 */
    vxo_ln_quant_rows(x, t, d, g, b, G, aq.data(), as.data());
    std::fill(hbuf.begin(), hbuf.begin() + (size_t)t * ff, 0.0f);
    tern_gemm(w1, aq.data(), as.data(), t, VXO_EP_SILU, 0.0f, hbuf.data());
    vxo_quantize_rows(hbuf.data(), t, ff, G, aq.data(), as.data());
    tern_gemm(w2, aq.data(), as.data(), t, VXO_EP_ADD_SCALED, 0.5f, x);
  };
  ffn(L->ln_g[0], L->ln_b[0], P.m[0], P.m[1]);

  { /* Attention::forward_fused (encoder.rs:138-187), int8 core */
    vxo_ln_quant_rows(x, t, d, L->ln_g[1], L->ln_b[1], G, aq.data(), as.data());
    std::vector<float> qkv((size_t)t * 3 * d, 0.0f);
    tern_gemm(P.m[2], aq.data(), as.data(), t, VXO_EP_STORE, 0.0f, qkv.data());
    int np = 2 * t - 1;
    std::vector<int8_t> pq((size_t)np * d);
    std::vector<float> ps((size_t)np * (d / G)), rel_k((size_t)np * d, 0.0f);
    vxo_quantize_rows(pos_emb, np, d, G, pq.data(), ps.data()); /* wp.forward -> prepare (quantize_layout) */
    tern_gemm(P.m[4], pq.data(), ps.data(), np, VXO_EP_STORE, 0.0f, rel_k.data());
    std::vector<float> ctx((size_t)t * d, 0.0f);
    float scaling = 1.0f / std::sqrt((float)dh);
    vxo_attn_core_int8(qkv.data(), rel_k.data(), t, d, heads, dh, L->bias_u, L->bias_v, scaling, ctx.data());
    vxo_quantize_rows(ctx.data(), t, d, G, aq.data(), as.data());
    tern_gemm(P.m[3], aq.data(), as.data(), t, VXO_EP_ADD_SCALED, 1.0f, x);
  }

  { /* ConvModule::forward_fused (encoder.rs:582-629) */
    vxo_ln_quant_rows(x, t, d, L->ln_g[2], L->ln_b[2], G, aq.data(), as.data());
    std::vector<float> g((size_t)t * 2 * d, 0.0f), hb((size_t)t * d);
    tern_gemm(P.m[5], aq.data(), as.data(), t, VXO_EP_STORE, 0.0f, g.data());
    vxo_conv_middle(g.data(), t, d, k, L->dw_w, L->dw_b, hb.data());
    vxo_quantize_rows(hb.data(), t, d, G, aq.data(), as.data());
    tern_gemm(P.m[6], aq.data(), as.data(), t, VXO_EP_ADD_SCALED, 1.0f, x);
  }

  ffn(L->ln_g[3], L->ln_b[3], P.m[7], P.m[8]);

  { /* norm_out through a scratch copy (encoder.rs:752-754) */
    std::vector<float> s((size_t)t * d);
    parallel_for(t, [&](int i) { layer_norm_row(x + (size_t)i * d, L->ln_g[4], L->ln_b[4], d, s.data() + (size_t)i * d); });
    std::memcpy(x, s.data(), s.size() * sizeof(float));
  }
}

extern "C" void vxo_layer_forward(const vxo_layer* L, int d, int heads, int k, float* x, int t, const float* pos_emb) {
  void* P = vxo_layer_prepare(L);
  vxo_layer_forward_prepared(P, L, d, heads, k, x, t, pos_emb);
  vxo_layer_free(P);
}

/* --------------------------------------------------------------------------------------------- subsampling */

static int out_len(int n, int k, int s, int p) { return (n + 2 * p - k) / s + 1; } /* subsampling.rs:26-28 */

extern "C" int vxo_sub_out_frames(int t, int k, int s) { /* subsampling.rs:99-106 */
  int p = (k - 1) / 2, n = t;
  for (int i = 0; i < 3; i++) n = out_len(n, k, s, p);
  return n;
}

extern "C" void vxo_subsampling_forward(const vxo_sub* S, const float* feats, int t, float* out) {
  /* Subsampling::forward (subsampling.rs:109-204), channels-last [T, F, C] */
  const int c = S->channels, k = S->kernel, s = S->stride, p = (k - 1) / 2, nm = S->n_mels;
  const int t1 = out_len(t, k, s, p), f1 = out_len(nm, k, s, p);
  std::vector<float> x((size_t)t1 * f1 * c);
  parallel_for(t1, [&](int ot) { /* conv0: 1 -> C, ReLU */
    for (int of = 0; of < f1; of++) {
      float* o = x.data() + ((size_t)ot * f1 + of) * c;
      std::memcpy(o, S->conv0_b, c * sizeof(float));
      for (int kt = 0; kt < k; kt++) {
        int it = ot * s + kt - p;
        if (it < 0 || it >= t) continue;
        for (int kf = 0; kf < k; kf++) {
          int i_f = of * s + kf - p;
          if (i_f < 0 || i_f >= nm) continue;
          float v = feats[(size_t)it * nm + i_f];
          const float* wt = S->conv0_w + (size_t)(kt * k + kf) * c;
          for (int ch = 0; ch < c; ch++) o[ch] += wt[ch] * v;
        }
      }
      for (int ch = 0; ch < c; ch++) o[ch] = std::fmax(o[ch], 0.0f);
    }
  });
  int tc = t1, fc = f1;
  for (int stage = 0; stage < 2; stage++) {
    const int t2 = out_len(tc, k, s, p), f2 = out_len(fc, k, s, p);
    std::vector<float> y((size_t)t2 * f2 * c);
    parallel_for(t2, [&](int ot) { /* depthwise 3x3 stride 2, no activation */
      for (int of = 0; of < f2; of++) {
        float* o = y.data() + ((size_t)ot * f2 + of) * c;
        std::memcpy(o, S->dw_b[stage], c * sizeof(float));
        for (int kt = 0; kt < k; kt++) {
          int it = ot * s + kt - p;
          if (it < 0 || it >= tc) continue;
          for (int kf = 0; kf < k; kf++) {
            int i_f = of * s + kf - p;
            if (i_f < 0 || i_f >= fc) continue;
            const float* xi = x.data() + ((size_t)it * fc + i_f) * c;
            const float* wt = S->dw_w[stage] + (size_t)(kt * k + kf) * c;
            for (int ch = 0; ch < c; ch++) o[ch] += wt[ch] * xi[ch];
          }
        }
      }
    });
    const int n_pos = t2 * f2;
    std::vector<float> z((size_t)n_pos * c);
    vxo_linear(y.data(), n_pos, c, S->pw_w[stage], S->pw_b[stage], c, z.data()); /* pointwise 1x1 as a GEMM */
    for (auto& v : z) v = std::fmax(v, 0.0f);
    x.swap(z);
    tc = t2;
    fc = f2;
  }
  vxo_linear(x.data(), tc, fc * c, S->lin_w, S->lin_b, S->d_model, out);
}
