// NeMo log-mel frontend on the GPU: pre-emphasis, centre padding, symmetric Hann window, 512-point real FFT, power,
// Slaney mel filterbank, log, then per-utterance per-feature normalisation, for a batch of utterances stacked along
// the sample axis.
//
// Reference: Frontend (crates/voxrt/src/frontend.rs:36-200): MelConfig defaults (:13-33), hz_to_mel / mel_to_hz and
// slaney_mel_filterbank (:45-90, computed in f64 on the host here too), Frontend::new's window (:95-100), log_mel
// (:112-166), normalize (:169-191). Arithmetic per step follows the reference: pre-emphasis x[i] = s[i] - 0.97 *
// s[i-1] as a product then a subtraction; power re^2 + im^2 in f32; the mel sum in f64 over f32 weights and powers,
// cast to f32 before adding the 2^-24 guard; logf; mean and (unbiased) variance in f64, std cast to f32 + 1e-5, then
// (x - mean) / std in f32. The FFT itself is a radix-2 transform here, not realfft's, so the spectra agree with the
// reference to f32 rounding rather than bit for bit.
//
// Layout: one block of 256 threads per 8 frames. Each frame's 512 real samples are transformed as a 256-point complex
// FFT of the even / odd samples (z[n] = x[2n] + i x[2n+1]) followed by the split step that yields the 257 bins of the
// real transform; the twiddles are f64-accurate f32 values from the host. The filterbank is applied sparsely: each
// mel filter only touches its own bin range (zero weights add +0.0 to a sum of non-negative terms, so skipping them
// changes nothing).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "common.h"
#include "internal.h"

namespace vxg {
namespace fe {

constexpr int NFFT = 512, NH = 256, NBINS = NFFT / 2 + 1, WIN = 400, HOP = 160, NMEL_MAX = 256;
constexpr int FPB = 8;         // frames per block
constexpr int THREADS = 256;
constexpr float LOG_GUARD = 5.9604645e-8f;  // 2^-24, frontend.rs:10
constexpr float NORM_EPS = 1e-5f;           // frontend.rs:11

struct Params {
  const float* samples;  // stacked samples of all utterances
  const long long* s_off;  // [n] first sample of utterance u
  const int* s_len;        // [n] samples
  const long long* f_off;  // [n] first output frame of utterance u
  const int* fr_utt;       // [total frames] utterance of each output frame
  int total_frames;
  float* feats;            // [total frames, n_mels]
  const float* window;     // [WIN]
  const float2* tw;        // [NH] e^{-2 pi i k / NH}, then [NH] e^{-2 pi i k / NFFT} for the split step
  const float* fb;         // [n_mels, NBINS]
  const int* fb_lo;        // [n_mels] first nonzero bin
  const int* fb_hi;        // [n_mels] one past the last nonzero bin
  int n_mels;
  float preemph;
};

__device__ __forceinline__ unsigned brev8(unsigned k) { return __brev(k) >> 24; }

__global__ void __launch_bounds__(THREADS) logmel_kernel(const Params p) {
  __shared__ float2 z[FPB][NH];
  __shared__ float pw[FPB][NBINS + 3];
  const int tid = threadIdx.x;
  const int f0 = blockIdx.x * FPB;
  // load: frame t of utterance u covers padded samples [t*HOP, t*HOP + NFFT); the window occupies [56, 456)
  for (int idx = tid; idx < FPB * NFFT; idx += THREADS) {
    const int fl = idx / NFFT, j = idx % NFFT, f = f0 + fl;
    float v = 0.0f;
    if (f < p.total_frames) {
      const int u = p.fr_utt[f];
      const int t = (int)(f - p.f_off[u]);
      const int woff = (NFFT - WIN) / 2;
      if (j >= woff && j < woff + WIN) {
        const long long i = (long long)t * HOP + j - NFFT / 2;  // index into the unpadded, pre-emphasised signal
        if (i >= 0 && i < p.s_len[u]) {
          const float* s = p.samples + p.s_off[u];
          const float x = i == 0 ? s[0] : __fsub_rn(s[i], __fmul_rn(p.preemph, s[i - 1]));
          v = __fmul_rn(x, p.window[j - woff]);
        }
      }
    }
    // even / odd samples -> real / imaginary part, stored in bit-reversed order for the in-place transform
    const int n = j >> 1;
    float* zz = reinterpret_cast<float*>(&z[fl][brev8((unsigned)n)]);
    zz[j & 1] = v;
  }
  __syncthreads();
  // 256-point radix-2 decimation-in-time transform, 128 butterflies per frame per stage
  for (int len = 2; len <= NH; len <<= 1) {
    const int half = len >> 1, step = NH / len;
    for (int b = tid; b < FPB * (NH / 2); b += THREADS) {
      const int fl = b / (NH / 2), k = b % (NH / 2);
      const int grp = k / half, pos = k % half;
      const int i0 = grp * len + pos, i1 = i0 + half;
      const float2 w = p.tw[pos * step];
      const float2 a = z[fl][i0], c = z[fl][i1];
      const float tr = __fsub_rn(__fmul_rn(c.x, w.x), __fmul_rn(c.y, w.y));
      const float ti = __fadd_rn(__fmul_rn(c.x, w.y), __fmul_rn(c.y, w.x));
      z[fl][i0] = make_float2(__fadd_rn(a.x, tr), __fadd_rn(a.y, ti));
      z[fl][i1] = make_float2(__fsub_rn(a.x, tr), __fsub_rn(a.y, ti));
    }
    __syncthreads();
  }
  // split step: X[k] = (Z[k] + conj(Z[N/2 - k])) / 2 + e^{-2 pi i k / N} (Z[k] - conj(Z[N/2 - k])) / (2i)
  for (int idx = tid; idx < FPB * NBINS; idx += THREADS) {
    const int fl = idx / NBINS, k = idx % NBINS;
    float re, im;
    if (k == 0 || k == NH) {
      const float2 z0 = z[fl][0];
      re = k == 0 ? __fadd_rn(z0.x, z0.y) : __fsub_rn(z0.x, z0.y);
      im = 0.0f;
    } else {
      const float2 a = z[fl][k], b = z[fl][NH - k];
      const float er = __fmul_rn(0.5f, __fadd_rn(a.x, b.x)), ei = __fmul_rn(0.5f, __fsub_rn(a.y, b.y));
      const float orr = __fmul_rn(0.5f, __fadd_rn(a.y, b.y)), oi = __fmul_rn(-0.5f, __fsub_rn(a.x, b.x));
      const float2 w = p.tw[NH + k];
      re = __fadd_rn(er, __fsub_rn(__fmul_rn(orr, w.x), __fmul_rn(oi, w.y)));
      im = __fadd_rn(ei, __fadd_rn(__fmul_rn(orr, w.y), __fmul_rn(oi, w.x)));
    }
    pw[fl][k] = __fadd_rn(__fmul_rn(re, re), __fmul_rn(im, im));
  }
  __syncthreads();
  // mel: f64 sum over the filter's bins, cast, guard, log
  for (int idx = tid; idx < FPB * p.n_mels; idx += THREADS) {
    const int fl = idx / p.n_mels, m = idx % p.n_mels, f = f0 + fl;
    if (f >= p.total_frames) continue;
    const float* w = p.fb + (size_t)m * NBINS;
    double acc = 0.0;
    for (int k = p.fb_lo[m]; k < p.fb_hi[m]; k++) acc = __dadd_rn(acc, __dmul_rn((double)w[k], (double)pw[fl][k]));
    p.feats[(size_t)f * p.n_mels + m] = logf(__fadd_rn((float)acc, LOG_GUARD));
  }
}

// normalize (frontend.rs:169-191): per utterance and mel bin, f64 mean and unbiased variance over the frames; one
// block per (utterance, 32 mel bins), each warp-lane column of the block a mel bin, rows split over the 8 warps.
__global__ void __launch_bounds__(256) norm_kernel(float* feats, const long long* f_off, const int* n_fr, int n_mels) {
  __shared__ double red[8][32];
  __shared__ float stat[2][32];
  const int u = blockIdx.x, m = blockIdx.y * 32 + (threadIdx.x & 31), w = threadIdx.x >> 5;
  const int n = n_fr[u];
  if (n < 2) return;  // fewer than two frames: left as is
  float* base = feats + (size_t)f_off[u] * n_mels;
  const bool ok = m < n_mels;
  // mean: the sequential f64 sum of the reference is not reproduced by a tree sum bit for bit; both are within f64
  // rounding, far below the f32 features' resolution
  double s = 0.0;
  if (ok)
    for (int t = w; t < n; t += 8) s += (double)base[(size_t)t * n_mels + m];
  red[w][threadIdx.x & 31] = s;
  __syncthreads();
  if (w == 0) {  // each lane reduces its own column
    double a = 0.0;
    for (int k = 0; k < 8; k++) a += red[k][threadIdx.x & 31];
    red[0][threadIdx.x & 31] = a / (double)n;
  }
  __syncthreads();
  const double mean = red[0][threadIdx.x & 31];
  __syncthreads();
  double v = 0.0;
  if (ok)
    for (int t = w; t < n; t += 8) {
      const double d = (double)base[(size_t)t * n_mels + m] - mean;
      v += d * d;
    }
  red[w][threadIdx.x & 31] = v;
  __syncthreads();
  if (w == 0) {
    double a = 0.0;
    for (int k = 0; k < 8; k++) a += red[k][threadIdx.x & 31];
    stat[0][threadIdx.x & 31] = (float)mean;
    stat[1][threadIdx.x & 31] = __fadd_rn((float)sqrt(a / ((double)n - 1.0)), NORM_EPS);
  }
  __syncthreads();
  if (!ok) return;
  const float mf = stat[0][threadIdx.x & 31], sd = stat[1][threadIdx.x & 31];
  for (int t = w; t < n; t += 8) {
    float* q = base + (size_t)t * n_mels + m;
    *q = __fdiv_rn(__fsub_rn(*q, mf), sd);
  }
}

// librosa hz_to_mel / mel_to_hz (Slaney, htk=False), frontend.rs:45-71
double hz_to_mel(double f) {
  const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp, logstep = std::log(6.4) / 27.0;
  return f >= min_log_hz ? min_log_mel + std::log(f / min_log_hz) / logstep : f / f_sp;
}
double mel_to_hz(double m) {
  const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, min_log_mel = min_log_hz / f_sp, logstep = std::log(6.4) / 27.0;
  return m >= min_log_mel ? min_log_hz * std::exp(logstep * (m - min_log_mel)) : f_sp * m;
}

}  // namespace fe
}  // namespace vxg

using namespace vxg;

struct vxg_frontend {
  int device = 0, n_mels = 0, sample_rate = 0;
  float preemph = 0.97f;
  std::vector<float> fb;  // host copy [n_mels, NBINS]
  float* d_window = nullptr;
  float2* d_tw = nullptr;
  float* d_fb = nullptr;
  int* d_lo = nullptr;
  int* d_hi = nullptr;
  // per-batch tables, grown on demand
  void* d_tab = nullptr;
  size_t tab_cap = 0;
  ~vxg_frontend() {
    cudaSetDevice(device);
    cudaFree(d_window);
    cudaFree(d_tw);
    cudaFree(d_fb);
    cudaFree(d_lo);
    cudaFree(d_hi);
    cudaFree(d_tab);
  }
};

extern "C" {

// slaney_mel_filterbank (frontend.rs:74-90): f64 arithmetic, cast to f32
vxg_status vxg_mel_filterbank(int sample_rate, int n_fft, int n_mels, float* fb) {
  clear_error();
  VXG_ARG(fb && sample_rate > 0 && n_fft > 0 && n_mels > 0, "bad arguments");
  const int n_bins = n_fft / 2 + 1;
  const double sr = sample_rate;
  std::vector<double> fftf(n_bins), mel_f(n_mels + 2);
  for (int k = 0; k < n_bins; k++) fftf[k] = (double)k * sr / (double)n_fft;
  const double lo = fe::hz_to_mel(0.0), hi = fe::hz_to_mel(sr / 2.0);
  for (int i = 0; i < n_mels + 2; i++) mel_f[i] = fe::mel_to_hz(lo + (hi - lo) * (double)i / (double)(n_mels + 1));
  for (int i = 0; i < n_mels; i++) {
    const double enorm = 2.0 / (mel_f[i + 2] - mel_f[i]);
    for (int k = 0; k < n_bins; k++) {
      const double lower = (fftf[k] - mel_f[i]) / (mel_f[i + 1] - mel_f[i]);
      const double upper = (mel_f[i + 2] - fftf[k]) / (mel_f[i + 2] - mel_f[i + 1]);
      const double w = std::max(std::min(lower, upper), 0.0);
      fb[(size_t)i * n_bins + k] = (float)(w * enorm);
    }
  }
  return VXG_OK;
}

int vxg_frontend_frames(long long n_samples) { return (int)(n_samples / fe::HOP); }

vxg_status vxg_frontend_create(int sample_rate, int n_mels, int device, vxg_frontend** out) {
  clear_error();
  VXG_ARG(out, "NULL argument");
  VXG_ARG(sample_rate == 16000 && n_mels > 0 && n_mels <= fe::NMEL_MAX,
          "the frontend covers 16 kHz audio and at most %d mel bins", fe::NMEL_MAX);
  *out = nullptr;
  VXG_CUDA(cudaSetDevice(device));
  vxg_frontend* F = new vxg_frontend();
  F->device = device;
  F->n_mels = n_mels;
  F->sample_rate = sample_rate;
  F->fb.resize((size_t)n_mels * fe::NBINS);
  vxg_status s = vxg_mel_filterbank(sample_rate, fe::NFFT, n_mels, F->fb.data());
  if (s != VXG_OK) {
    delete F;
    return s;
  }
  std::vector<int> lo(n_mels), hi(n_mels);
  for (int m = 0; m < n_mels; m++) {
    int a = fe::NBINS, b = 0;
    for (int k = 0; k < fe::NBINS; k++)
      if (F->fb[(size_t)m * fe::NBINS + k] != 0.0f) {
        a = std::min(a, k);
        b = k + 1;
      }
    lo[m] = a < b ? a : 0;
    hi[m] = a < b ? b : 0;
  }
  std::vector<float> win(fe::WIN);  // torch.hann_window(400, periodic=False), frontend.rs:95-100
  for (int k = 0; k < fe::WIN; k++) win[k] = (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * (double)k / (double)(fe::WIN - 1)));
  std::vector<float2> tw(2 * fe::NH);
  for (int k = 0; k < fe::NH; k++) {
    const double a = -2.0 * M_PI * (double)k / (double)fe::NH, b = -2.0 * M_PI * (double)k / (double)fe::NFFT;
    tw[k] = make_float2((float)std::cos(a), (float)std::sin(a));
    tw[fe::NH + k] = make_float2((float)std::cos(b), (float)std::sin(b));
  }
  auto up = [&](void** dst, const void* src, size_t bytes) -> cudaError_t {
    cudaError_t e = cudaMalloc(dst, bytes);
    if (e != cudaSuccess) return e;
    return cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
  };
  cudaError_t e;
  if ((e = up((void**)&F->d_window, win.data(), win.size() * 4)) != cudaSuccess ||
      (e = up((void**)&F->d_tw, tw.data(), tw.size() * sizeof(float2))) != cudaSuccess ||
      (e = up((void**)&F->d_fb, F->fb.data(), F->fb.size() * 4)) != cudaSuccess ||
      (e = up((void**)&F->d_lo, lo.data(), lo.size() * 4)) != cudaSuccess ||
      (e = up((void**)&F->d_hi, hi.data(), hi.size() * 4)) != cudaSuccess) {
    delete F;
    return cuda_fail(e, "frontend upload");
  }
  *out = F;
  return VXG_OK;
}

void vxg_frontend_destroy(vxg_frontend* f) { delete f; }

vxg_status vxg_frontend_info(const vxg_frontend* f, int* sample_rate, int* n_mels) {
  clear_error();
  VXG_ARG(f, "NULL argument");
  if (sample_rate) *sample_rate = f->sample_rate;
  if (n_mels) *n_mels = f->n_mels;
  return VXG_OK;
}

vxg_status vxg_frontend_device(vxg_frontend* F, const float* samples, const long long* n_samples, int n, int normalize,
                               float* feats, int* n_frames, void* stream) {
  clear_error();
  VXG_ARG(F && samples && n_samples && n > 0 && feats, "NULL pointer or empty batch");
  VXG_CUDA(cudaSetDevice(F->device));
  // host tables: sample offsets, lengths, frame offsets, and the utterance of every frame
  std::vector<long long> s_off(n), f_off(n);
  std::vector<int> s_len(n), nfr(n);
  long long so = 0, fo = 0;
  for (int u = 0; u < n; u++) {
    VXG_ARG(n_samples[u] >= 0 && n_samples[u] < (1LL << 31), "utterance %d: %lld samples", u, n_samples[u]);
    s_off[u] = so;
    s_len[u] = (int)n_samples[u];
    f_off[u] = fo;
    nfr[u] = vxg_frontend_frames(n_samples[u]);
    if (n_frames) n_frames[u] = nfr[u];
    so += n_samples[u];
    fo += nfr[u];
  }
  VXG_ARG(fo < (1LL << 31), "batch too large: %lld frames", fo);
  const int total = (int)fo;
  if (total == 0) return VXG_OK;
  std::vector<int> fr_utt(total);
  for (int u = 0; u < n; u++)
    for (int t = 0; t < nfr[u]; t++) fr_utt[f_off[u] + t] = u;
  const size_t bytes = n * (2 * sizeof(long long) + 2 * sizeof(int)) + (size_t)total * sizeof(int);
  if (bytes > F->tab_cap) {
    cudaFree(F->d_tab);
    F->d_tab = nullptr;
    VXG_CUDA(cudaMalloc(&F->d_tab, bytes + bytes / 4));
    F->tab_cap = bytes + bytes / 4;
  }
  std::vector<uint8_t> h(bytes);
  uint8_t* q = h.data();
  auto put = [&](const void* src, size_t b) {
    memcpy(q, src, b);
    q += b;
  };
  put(s_off.data(), n * 8);
  put(f_off.data(), n * 8);
  put(s_len.data(), n * 4);
  put(nfr.data(), n * 4);
  put(fr_utt.data(), (size_t)total * 4);
  cudaStream_t st = (cudaStream_t)stream;
  VXG_CUDA(cudaMemcpyAsync(F->d_tab, h.data(), bytes, cudaMemcpyHostToDevice, st));
  uint8_t* d = static_cast<uint8_t*>(F->d_tab);
  fe::Params p;
  p.samples = samples;
  p.s_off = reinterpret_cast<const long long*>(d);
  p.f_off = reinterpret_cast<const long long*>(d + n * 8);
  p.s_len = reinterpret_cast<const int*>(d + n * 16);
  const int* d_nfr = reinterpret_cast<const int*>(d + n * 20);
  p.fr_utt = reinterpret_cast<const int*>(d + n * 24);
  p.total_frames = total;
  p.feats = feats;
  p.window = F->d_window;
  p.tw = F->d_tw;
  p.fb = F->d_fb;
  p.fb_lo = F->d_lo;
  p.fb_hi = F->d_hi;
  p.n_mels = F->n_mels;
  p.preemph = F->preemph;
  fe::logmel_kernel<<<(total + fe::FPB - 1) / fe::FPB, fe::THREADS, 0, st>>>(p);
  note_launch();
  VXG_CUDA(cudaGetLastError());
  if (normalize) {
    fe::norm_kernel<<<dim3(n, (F->n_mels + 31) / 32), 256, 0, st>>>(feats, p.f_off, d_nfr, F->n_mels);
    note_launch();
    VXG_CUDA(cudaGetLastError());
  }
  // the tables are read by the kernels above: keep them until they finish before the next call reuses the buffer
  VXG_CUDA(cudaStreamSynchronize(st));
  return VXG_OK;
}

}  // extern "C"
