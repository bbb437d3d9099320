// VAD head on the GPU and the segmenter on the host: VadHead::probs (crates/voxrt/src/vad.rs:39-82) and segment
// (vad.rs:140-240).
//
// probs = sigmoid(out(relu(ctx(relu(proj(x)))))) per encoder frame of the subsampler output x [t, d_model]:
//   proj  a[i][j] = max(b[j] + sum_c w[j][c] x[i][c], 0), the sum a running mul-then-add over c in order;
//   ctx   h[i][o] = max(b[o] + sum_ci sum_kk w[o][ci][kk] a[i + kk - pad][ci], 0) over taps inside the utterance
//         (same padding: missing taps are skipped, not added as zero), ci outer, kk inner;
//   out   z = b + sum_o w[o] h[i][o] in order; p = 1 / (1 + exp(-z)) with the correctly rounded exp of crmath.cuh.
// Every sum keeps the reference's order with separately rounded products and adds, so the probabilities are bit for
// bit those of the reference's loops (given its libm expf rounds correctly at these points).
// Weights are transposed at create so that the threads of a block (one output each) read consecutive addresses.
#include <algorithm>
#include <vector>

#include "common.h"
#include "crmath.cuh"

struct vxg_vad {
  int device = -1, d = 0, h = 0, k = 0;
  double frame_seconds = 0.0;
  float out_b = 0.0f;
  void* block = nullptr;
  float* proj_wt = nullptr;  // [d][h]
  float* proj_b = nullptr;   // [h]
  float* ctx_wt = nullptr;   // [h ci][k][h o]
  float* ctx_b = nullptr;    // [h]
  float* out_w = nullptr;    // [h]
};

namespace vxg {
namespace vad {
namespace {

constexpr int kProjRows = 4;

// relu(proj(x)) for kProjRows stacked rows per block; thread o computes outputs o, o + blockDim, ...
__global__ void proj_kernel(const float* __restrict__ x, int rows, int d, int h, const float* __restrict__ wt,
                            const float* __restrict__ b, float* __restrict__ a) {
  extern __shared__ float xs[];  // [kProjRows][d]
  const int r0 = blockIdx.x * kProjRows, nr = min(kProjRows, rows - r0);
  for (int i = threadIdx.x; i < kProjRows * d; i += blockDim.x)
    xs[i] = i / d < nr ? x[(size_t)(r0 + i / d) * d + i % d] : 0.0f;
  __syncthreads();
  for (int o = threadIdx.x; o < h; o += blockDim.x) {
    float acc[kProjRows];
#pragma unroll
    for (int r = 0; r < kProjRows; r++) acc[r] = b[o];
    // unrolled so that the weight loads of 16 columns are in flight ahead of the (sequential) sums
#pragma unroll 16
    for (int c = 0; c < d; c++) {
      const float w = wt[(size_t)c * h + o];
#pragma unroll
      for (int r = 0; r < kProjRows; r++) acc[r] = __fadd_rn(acc[r], __fmul_rn(w, xs[r * d + c]));
    }
    for (int r = 0; r < nr; r++) a[(size_t)(r0 + r) * h + o] = fmaxf(acc[r], 0.0f);
  }
}

// ctx conv + relu, out + sigmoid: one block per frame. offs [n + 1]: first row of each utterance.
__global__ void ctx_out_kernel(const float* __restrict__ a, const int* __restrict__ offs, int n, int h, int k,
                               const float* __restrict__ wt, const float* __restrict__ b,
                               const float* __restrict__ out_w, float out_b, float* __restrict__ probs) {
  extern __shared__ float sm[];  // taps [k][h], then hb [h]
  float* taps = sm;
  float* hb = sm + (size_t)k * h;
  const int i = blockIdx.x;
  int lo = 0, hi = n;  // utterance u with offs[u] <= i < offs[u + 1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] <= i) lo = mid;
    else hi = mid;
  }
  const int s = offs[lo], e = offs[lo + 1], pad = (k - 1) / 2;
  for (int q = threadIdx.x; q < k * h; q += blockDim.x) {
    const int j = i + q / h - pad;
    taps[q] = j >= s && j < e ? a[(size_t)j * h + q % h] : 0.0f;
  }
  __syncthreads();
  const bool interior5 = k == 5 && i - 2 >= s && i + 2 < e;  // the model's kernel, every tap inside the utterance
  for (int o = threadIdx.x; o < h; o += blockDim.x) {
    float acc = b[o];
    if (interior5) {
#pragma unroll 4
      for (int ci = 0; ci < h; ci++) {
        const float* wr = wt + (size_t)ci * 5 * h + o;
#pragma unroll
        for (int kk = 0; kk < 5; kk++) acc = __fadd_rn(acc, __fmul_rn(wr[(size_t)kk * h], taps[kk * h + ci]));
      }
    } else {
      for (int ci = 0; ci < h; ci++)
        for (int kk = 0; kk < k; kk++) {
          const int j = i + kk - pad;
          if (j >= s && j < e) acc = __fadd_rn(acc, __fmul_rn(wt[((size_t)ci * k + kk) * h + o], taps[kk * h + ci]));
        }
    }
    hb[o] = fmaxf(acc, 0.0f);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float z = out_b;
    for (int o = 0; o < h; o++) z = __fadd_rn(z, __fmul_rn(out_w[o], hb[o]));
    probs[i] = __fdiv_rn(1.0f, __fadd_rn(1.0f, crm::expf_cr(-z)));
  }
}

}  // namespace

// segment (vad.rs:140-240) on host probabilities.
size_t segment(const float* p, int t, const vxg_segment_cfg& cfg, std::vector<vxg_vad_segment>& out) {
  out.clear();
  if (t <= 0) return 0;
  // 1. speech runs, pauses shorter than min_pause_frames tolerated
  std::vector<vxg_vad_segment> runs;
  int i = 0;
  while (i < t) {
    if (p[i] >= cfg.threshold) {
      const int s = i;
      int last = i;
      while (i < t) {
        if (p[i] >= cfg.threshold) {
          last = i;
          i++;
        } else {
          int j = i;
          while (j < t && p[j] < cfg.threshold) j++;
          if (j - i >= cfg.min_pause_frames || j == t) {
            i = j;
            break;
          }
          i = j;
        }
      }
      runs.push_back({s, last + 1});
    } else {
      i++;
    }
  }
  if (runs.empty()) {
    out.push_back({0, t});
    return 1;
  }
  // 2. short runs merge into the previous one while the result stays within max_frames
  std::vector<vxg_vad_segment> merged;
  for (const auto& r : runs) {
    if (!merged.empty()) {
      auto& prev = merged.back();
      if ((r.end - r.start < cfg.min_frames || prev.end - prev.start < cfg.min_frames) &&
          r.end - prev.start <= cfg.max_frames) {
        prev.end = r.end;
        continue;
      }
    }
    merged.push_back(r);
  }
  // 3. the hard cap: split at the lowest-probability frame of the window's last ~5 s
  for (const auto& r : merged) {
    int s = r.start;
    while (r.end - s > cfg.max_frames) {
      const int win_end = s + cfg.max_frames;
      const int look = std::min(63, cfg.max_frames / 2);
      int best = win_end;
      float best_p = 3.4028234663852886e38f;
      for (int f = win_end - look; f < win_end; f++)
        if (p[f] < best_p) {
          best_p = p[f];
          best = f;
        }
      const int cut = std::max(best, s + 1);
      out.push_back({s, cut});
      s = cut;
    }
    out.push_back({s, r.end});
  }
  // 4. context padding, never past the midpoint of the gap to a neighbour
  const size_t n = out.size();
  std::vector<std::pair<int, int>> bounds(n);
  for (size_t q = 0; q < n; q++) {
    const int lo = q == 0 ? 0 : out[q - 1].end + (out[q].start - out[q - 1].end + 1) / 2;
    const int hi = q + 1 == n ? t : out[q].end + (out[q + 1].start - out[q].end) / 2;
    bounds[q] = {lo, hi};
  }
  for (size_t q = 0; q < n; q++) {
    out[q].start = std::max(std::max(out[q].start - cfg.pad_frames, 0), bounds[q].first);
    out[q].end = std::min(out[q].end + cfg.pad_frames, bounds[q].second);
  }
  return n;
}

}  // namespace vad
}  // namespace vxg

using namespace vxg;

extern "C" {

void vxg_segment_cfg_default(vxg_segment_cfg* c) {
  if (!c) return;
  c->threshold = 0.5f;
  c->min_pause_frames = 8;
  c->max_frames = 750;
  c->min_frames = 125;
  c->pad_frames = 2;
}

vxg_status vxg_segment(const float* probs, int t, const vxg_segment_cfg* cfg, vxg_vad_segment* out, size_t cap,
                       size_t* n) {
  clear_error();
  VXG_ARG(n && cfg && t >= 0 && (probs || t == 0) && (out || cap == 0), "bad arguments");
  VXG_ARG(cfg->max_frames >= 2 && cfg->min_pause_frames >= 0 && cfg->min_frames >= 0 && cfg->pad_frames >= 0,
          "bad segment config");
  std::vector<vxg_vad_segment> segs;
  *n = vad::segment(probs, t, *cfg, segs);
  for (size_t i = 0; i < std::min(cap, segs.size()); i++) out[i] = segs[i];
  return VXG_OK;
}

vxg_status vxg_vad_create(const vxg_vad_desc* desc, vxg_vad** out) {
  clear_error();
  VXG_ARG(desc && out, "NULL argument");
  *out = nullptr;
  const vxg_vad_desc& s = *desc;
  VXG_ARG(s.d_model > 0 && s.hidden > 0 && s.kernel > 0 && s.kernel % 2 == 1, "bad VAD sizes");
  VXG_ARG(s.proj_w && s.proj_b && s.ctx_w && s.ctx_b && s.out_w, "NULL weight");
  VXG_ARG(s.device >= 0, "the VAD head runs on a GPU (device >= 0)");
  const int d = s.d_model, h = s.hidden, k = s.kernel;
  std::vector<float> pwt((size_t)d * h), cwt((size_t)h * k * h);
  for (int j = 0; j < h; j++)
    for (int c = 0; c < d; c++) pwt[(size_t)c * h + j] = s.proj_w[(size_t)j * d + c];
  for (int o = 0; o < h; o++)
    for (int ci = 0; ci < h; ci++)
      for (int kk = 0; kk < k; kk++) cwt[((size_t)ci * k + kk) * h + o] = s.ctx_w[((size_t)o * h + ci) * k + kk];
  auto* v = new vxg_vad();
  v->device = s.device, v->d = d, v->h = h, v->k = k, v->frame_seconds = s.frame_seconds, v->out_b = s.out_b;
  const size_t nf = pwt.size() + 3 * (size_t)h + cwt.size();
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e == cudaSuccess) e = cudaSetDevice(s.device);
  if (e == cudaSuccess) e = cudaMalloc(&v->block, sizeof(float) * nf);
  if (e == cudaSuccess) {
    float* f = static_cast<float*>(v->block);
    v->proj_wt = f, f += pwt.size();
    v->proj_b = f, f += h;
    v->ctx_wt = f, f += cwt.size();
    v->ctx_b = f, f += h;
    v->out_w = f;
    e = cudaMemcpy(v->proj_wt, pwt.data(), sizeof(float) * pwt.size(), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaMemcpy(v->proj_b, s.proj_b, sizeof(float) * h, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(v->ctx_wt, cwt.data(), sizeof(float) * cwt.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(v->ctx_b, s.ctx_b, sizeof(float) * h, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(v->out_w, s.out_w, sizeof(float) * h, cudaMemcpyHostToDevice);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    vxg_vad_destroy(v);
    return cuda_fail(e, "vxg_vad_create");
  }
  *out = v;
  return VXG_OK;
}

void vxg_vad_destroy(vxg_vad* v) {
  if (!v) return;
  if (v->block) cudaFree(v->block);
  delete v;
}

vxg_status vxg_vad_info(const vxg_vad* v, int* d_model, int* hidden, int* kernel, double* frame_seconds) {
  clear_error();
  VXG_ARG(v, "NULL argument");
  if (d_model) *d_model = v->d;
  if (hidden) *hidden = v->h;
  if (kernel) *kernel = v->k;
  if (frame_seconds) *frame_seconds = v->frame_seconds;
  return VXG_OK;
}

vxg_status vxg_vad_probs_device(const vxg_vad* v, const float* sub, const int* t, int n, float* probs, void* stream) {
  clear_error();
  VXG_ARG(v && t && n >= 0 && (n == 0 || (sub && probs)), "bad arguments");
  int cur = -1;
  VXG_CUDA(cudaGetDevice(&cur));
  VXG_ARG(cur == v->device, "current device %d is not the VAD's device %d", cur, v->device);
  std::vector<int> offs(n + 1, 0);
  for (int u = 0; u < n; u++) {
    VXG_ARG(t[u] >= 0, "utterance %d: negative frame count", u);
    offs[u + 1] = offs[u] + t[u];
  }
  const int rows = offs[n];
  if (rows == 0) return VXG_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t proj_smem = sizeof(float) * vad::kProjRows * v->d, ctx_smem = sizeof(float) * ((size_t)v->k + 1) * v->h;
  VXG_ARG(proj_smem <= 200 * 1024 && ctx_smem <= 200 * 1024, "VAD sizes exceed shared memory");
  vxg_status s = smem_attr(reinterpret_cast<const void*>(vad::proj_kernel), 200 * 1024);
  if (s == VXG_OK) s = smem_attr(reinterpret_cast<const void*>(vad::ctx_out_kernel), 200 * 1024);
  if (s != VXG_OK) return s;
  void* ws = nullptr;
  const size_t a_bytes = ((sizeof(float) * (size_t)rows * v->h) + 255) / 256 * 256;
  cudaMemPool_t pool = scratch_pool();
  VXG_CUDA(pool ? cudaMallocFromPoolAsync(&ws, a_bytes + sizeof(int) * (n + 1), pool, st)
                : cudaMallocAsync(&ws, a_bytes + sizeof(int) * (n + 1), st));
  float* a = static_cast<float*>(ws);
  int* offs_dev = reinterpret_cast<int*>(static_cast<char*>(ws) + a_bytes);
  cudaError_t e = cudaMemcpyAsync(offs_dev, offs.data(), sizeof(int) * (n + 1), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    vad::proj_kernel<<<(rows + vad::kProjRows - 1) / vad::kProjRows, 128, proj_smem, st>>>(sub, rows, v->d, v->h,
                                                                                         v->proj_wt, v->proj_b, a);
    vad::ctx_out_kernel<<<rows, 128, ctx_smem, st>>>(a, offs_dev, n, v->h, v->k, v->ctx_wt, v->ctx_b, v->out_w,
                                                     v->out_b, probs);
    note_launch(2);
    e = cudaGetLastError();
  }
  // the host offsets must outlive the queued copy
  const cudaError_t e2 = cudaStreamSynchronize(st);
  cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "vxg_vad_probs_device");
  if (e2 != cudaSuccess) return cuda_fail(e2, "vxg_vad_probs_device");
  return VXG_OK;
}

}  // extern "C"
