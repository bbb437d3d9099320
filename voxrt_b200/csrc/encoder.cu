// The ternary FastConformer encoder on one B200: weights resident in HBM in the kernels' formats, one stream, a
// workspace grown on demand, and a forward over a batch of utterances stacked along the token axis.
//
// Reference: Encoder::forward (crates/voxrt/src/encoder.rs:816-856) -> Subsampling::forward, rel_pos_table,
// 24 x ConformerLayer::forward_profiled (encoder.rs:706-756). The GPU boundary mirrors GpuEncoder
// (crates/voxrt/src/metal/mod.rs:451-640): load / forward (layers on subsampled input) / forward_feats (log-mel in,
// encoder frames out), Send + Sync through an internal mutex, plus a token-stacked batch form.
//
// Per layer (token-stacked rows, all kernels bit-identical to the reference's int8 path):
//   ln_quant(norm_out of the previous layer, written back to x; norm_ff1)  -> ff1.linear1 (SiLU) -> quantise ->
//   ff1.linear2 (x += 0.5 v) -> ln_quant(norm_attn) -> qkv (Store) -> attention (int8 core, context quantised
//   per head) -> o_proj (x += v) -> ln_quant(norm_conv) -> pw1 (GLU epilogue) -> dwconv/SiLU/int8 -> pw2 (x += v) ->
//   ln_quant(norm_ff2) -> ff2 as ff1. The last layer's norm_out is a standalone LayerNorm into the output.
// relative_k_proj depends only on positions, so it runs once per layer on the batch's shared table (positions
// Tmax-1 .. -(Tmax-1)); each utterance reads its slice, which is bit-identical to its own table (rows are
// independent in both the quantisation and the GEMM).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "internal.h"

struct vxg_encoder;

namespace vxg {
namespace enc {

struct TernDev {
  bool packed = true;     // 2-bit codes (resident-slab GEMM, K <= 1024) or int8 rows
  void* w = nullptr;      // 2-bit codes or int8 rows
  float* s = nullptr;     // tile-major scales
  int out = 0, in = 0, group = 0;
};

struct LayerDev {
  TernDev ff1_1, ff1_2, qkv, o, relk, pw1, pw2, ff2_1, ff2_2;
  float* ln[5][2] = {};  // norm_ff1, norm_attn, norm_conv, norm_ff2, norm_out: gamma, beta
  float *bias_u = nullptr, *bias_v = nullptr, *dw_t = nullptr, *dw_b = nullptr;
};

// base-3 byte -> its five digits minus one (trits.rs:7-27)
struct TritTable {
  int8_t t[243][5];
  TritTable() {
    for (int b = 0; b < 243; b++) {
      int v = b;
      for (int k = 0; k < 5; k++) {
        t[b][k] = (int8_t)(v % 3 - 1);
        v /= 3;
      }
    }
  }
};
const TritTable& trit_table() {
  static TritTable tt;
  return tt;
}

void parallel_rows(int n, const std::function<void(int, int)>& f) {
  int nt = (int)std::min<unsigned>(std::max(1u, std::thread::hardware_concurrency()), 32u);
  nt = std::max(1, std::min(nt, n / 64));
  if (nt <= 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> th;
  const int chunk = (n + nt - 1) / nt;
  for (int i = 0; i < nt; i++) {
    const int a = i * chunk, b = std::min(n, a + chunk);
    if (a < b) th.emplace_back(f, a, b);
  }
  for (auto& t : th) t.join();
}

// Host threads that stay up for the encoder's lifetime and run the staging copies of host-buffer forwards, so a
// forward does not create and join threads for every chunk. run(n, f) calls f(0..n-1) on the workers and the
// calling thread and returns once every call has finished; one run at a time (the encoder's mutex is held).
class CopyPool {
 public:
  explicit CopyPool(int workers) {
    for (int i = 0; i < workers; i++) th_.emplace_back([this] { loop(); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : th_) t.join();
  }
  int workers() const { return (int)th_.size(); }
  void run(int n, const std::function<void(int)>& f) {
    std::unique_lock<std::mutex> lk(mu_);
    job_ = &f, n_ = n, next_ = 0, left_ = n;
    cv_.notify_all();
    while (next_ < n_) {  // the caller takes items too
      const int i = next_++;
      lk.unlock();
      f(i);
      lk.lock();
      --left_;
    }
    done_.wait(lk, [&] { return left_ == 0; });
    job_ = nullptr, n_ = 0, next_ = 0;  // no worker can take an item of this run any more
  }

 private:
  void loop() {
    std::unique_lock<std::mutex> lk(mu_);
    for (;;) {
      cv_.wait(lk, [&] { return stop_ || next_ < n_; });
      if (stop_) return;
      const int i = next_++;
      const std::function<void(int)>* f = job_;  // read under the lock, with the item it belongs to
      lk.unlock();
      (*f)(i);
      lk.lock();
      if (--left_ == 0) done_.notify_all();
    }
  }
  std::vector<std::thread> th_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  const std::function<void(int)>* job_ = nullptr;
  int n_ = 0, next_ = 0, left_ = 0;
  bool stop_ = false;
};

}  // namespace enc
}  // namespace vxg

using namespace vxg;
using namespace vxg::enc;

struct vxg_encoder {
  int device = 0;
  int d = 0, ff = 0, heads = 0, k = 0, n_layers = 0, n_mels = 0, sub_ch = 0, group = 128;
  bool packed = true;
  std::vector<LayerDev> layers;
  float* sub[12] = {};
  std::vector<void*> allocs;
  cudaStream_t stream = nullptr;
  cudaStream_t copy_stream = nullptr;  // input copies of host-buffer forwards from page-locked memory
  std::mutex mu;
  // workspace, grown on demand
  size_t cap_rows = 0, cap_np = 0, cap_tab = 0, cap_attn = 0, cap_subws = 0, cap_in = 0, cap_host = 0;
  float *x = nullptr, *v = nullptr, *qkv = nullptr, *g = nullptr, *relk = nullptr, *pos = nullptr;
  int8_t *aq = nullptr, *hq = nullptr, *ctxq = nullptr, *posq = nullptr;
  float *as = nullptr, *hs = nullptr, *ctxs = nullptr, *poss = nullptr;
  void* attn_ws = nullptr;
  void* sub_ws = nullptr;
  int* dtab = nullptr;
  float* feats = nullptr;  // device staging for host-buffer forwards
  float* host_pin = nullptr;
  std::unique_ptr<CopyPool> copy_pool;  // staging-copy threads, started by the first host-buffer forward
  std::map<int, std::vector<float>> pos_cache;
  // per-kernel-class CUDA-event timing (vxg_encoder_set_profiling): the counterpart of the reference's
  // VOXRT_PROFILE counters (ternary_linear.rs:12-13, encoder.rs:297, :647-653)
  bool profile = false;
  struct Ev {
    int cls;
    cudaEvent_t a, b;
    double ops;
  };
  std::vector<Ev> evs;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  double prof_ms[VXG_PROF_CLASSES] = {};
  int prof_n[VXG_PROF_CLASSES] = {};
  double prof_gemm_ops = 0.0;
  ~vxg_encoder();
};

namespace {

cudaEvent_t pool_event(vxg_encoder* E) {
  if (E->ev_used == E->ev_pool.size()) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    E->ev_pool.push_back(e);
  }
  return E->ev_pool[E->ev_used++];
}

// Bracket one kernel-class step with events on the encoder's stream (no-op unless profiling).
struct ProfScope {
  vxg_encoder* E;
  int cls;
  double ops;
  cudaEvent_t a = nullptr;
  ProfScope(vxg_encoder* e, int c, double o = 0.0) : E(e), cls(c), ops(o) {
    if (E->profile) {
      a = pool_event(E);
      cudaEventRecord(a, E->stream);
    }
  }
  ~ProfScope() {
    if (E->profile) {
      cudaEvent_t b = pool_event(E);
      cudaEventRecord(b, E->stream);
      E->evs.push_back({cls, a, b, ops});
    }
  }
};

template <typename T>
vxg_status dev_alloc(vxg_encoder* E, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, std::max<size_t>(bytes, 256));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  E->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return VXG_OK;
}

template <typename T>
vxg_status upload(vxg_encoder* E, T** p, const void* host, size_t bytes) {
  vxg_status s = dev_alloc(E, p, bytes);
  if (s != VXG_OK) return s;
  VXG_CUDA(cudaMemcpy(*p, host, bytes, cudaMemcpyHostToDevice));
  return VXG_OK;
}

// One thrush-ternary-v2 module (or several stacked along the output dimension) -> device format. glu: the rows are
// stored in glu_interleave_row order (pointwise_conv1, whose GEMM epilogue applies the GLU).
vxg_status load_tern(vxg_encoder* E, TernDev* T, const vxg_ternary_tensor* mods, int n_mods, bool glu = false) {
  int out = 0;
  const int in = mods[0].in, group = mods[0].group;
  for (int i = 0; i < n_mods; i++) {
    VXG_ARG(mods[i].qweight && mods[i].scales, "ternary module without data");
    VXG_ARG(mods[i].in == in && mods[i].group == group, "stacked modules differ in width or group");
    out += mods[i].out;
  }
  VXG_ARG(in % 128 == 0 && group % 128 == 0 && in % group == 0, "module width %d / group %d unsupported", in, group);
  const int rb = (in + 4) / 5, ng = in / group;
  std::vector<uint8_t> q((size_t)out * rb);
  std::vector<uint16_t> sc((size_t)out * ng);
  size_t r = 0;
  for (int i = 0; i < n_mods; i++) {  // TernaryLinear::load_stacked (ternary_linear.rs:59-99)
    std::memcpy(q.data() + r * rb, mods[i].qweight, (size_t)mods[i].out * rb);
    std::memcpy(sc.data() + r * ng, mods[i].scales, (size_t)mods[i].out * ng * 2);
    r += mods[i].out;
  }
  if (glu) {  // permute whole rows (codes and scales): each output row of the GEMM is independent of the others
    VXG_ARG(out % 128 == 0, "GLU projection width %d must be a multiple of 128", out);
    const std::vector<uint8_t> q0 = q;
    const std::vector<uint16_t> sc0 = sc;
    for (int o = 0; o < out; o++) {
      const int src = glu_interleave_row(o, out / 2);
      std::memcpy(q.data() + (size_t)o * rb, q0.data() + (size_t)src * rb, rb);
      std::memcpy(sc.data() + (size_t)o * ng, sc0.data() + (size_t)src * ng, (size_t)ng * 2);
    }
  }
  const size_t ns = vxg_ternary_scales_count(out, in, group);
  std::vector<float> st(ns);
  vxg_status s;
  // 2-bit codes where the GEMM keeps the weight slab resident and unpacks it once per slab; wider modules stream
  // int8 rows (unpacking 2-bit chunks for every tile would cost more than the tensor cores' time on them).
  T->packed = E->packed && in <= kGemmResidentK;
  if (T->packed) {
    std::vector<uint8_t> codes(vxg_ternary_codes_bytes(out, in));
    if ((s = vxg_ternary_repack(q.data(), sc.data(), out, in, group, codes.data(), st.data())) != VXG_OK) return s;
    if ((s = upload(E, &T->w, codes.data(), codes.size())) != VXG_OK) return s;
  } else {
    std::vector<int8_t> w(vxg_ternary_i8_bytes(out, in));
    if ((s = vxg_ternary_repack_i8(q.data(), sc.data(), out, in, group, w.data(), st.data())) != VXG_OK) return s;
    if ((s = upload(E, &T->w, w.data(), w.size())) != VXG_OK) return s;
  }
  if ((s = upload(E, &T->s, st.data(), ns * 4)) != VXG_OK) return s;
  T->out = out;
  T->in = in;
  T->group = group;
  return VXG_OK;
}

vxg_status load_vec(vxg_encoder* E, float** p, const float* v, size_t n) {
  VXG_ARG(v != nullptr, "missing dense parameter");
  return upload(E, p, v, n * 4);
}

// rel_pos_table (encoder.rs:760-776) for t frames, computed on the host (libm), cached per t.
const std::vector<float>& pos_table(vxg_encoder* E, int t) {
  auto it = E->pos_cache.find(t);
  if (it != E->pos_cache.end()) return it->second;
  const int d = E->d, np = 2 * t - 1, half = d / 2;
  std::vector<float> out((size_t)np * d), inv(half);
  for (int i = 0; i < half; i++) inv[i] = 1.0f / powf(10000.0f, 2.0f * (float)i / (float)d);
  for (int r = 0; r < np; r++) {
    const float p = (float)((int64_t)t - 1 - r);
    for (int i = 0; i < half; i++) {
      const float f = inv[i] * p;
      out[(size_t)r * d + 2 * i] = sinf(f);
      out[(size_t)r * d + 2 * i + 1] = cosf(f);
    }
  }
  if (E->pos_cache.size() > 64) E->pos_cache.clear();
  return E->pos_cache.emplace(t, std::move(out)).first->second;
}

void free_ws(vxg_encoder* E) {
  float** fs[] = {&E->x, &E->v, &E->qkv, &E->g, &E->relk, &E->pos, &E->as, &E->hs, &E->ctxs, &E->poss, &E->feats};
  for (auto f : fs) {
    cudaFree(*f);
    *f = nullptr;
  }
  int8_t** is[] = {&E->aq, &E->hq, &E->ctxq, &E->posq};
  for (auto q : is) {
    cudaFree(*q);
    *q = nullptr;
  }
  cudaFree(E->attn_ws);
  cudaFree(E->sub_ws);
  cudaFree(E->dtab);
  E->attn_ws = E->sub_ws = nullptr;
  E->dtab = nullptr;
  E->cap_rows = E->cap_np = E->cap_tab = E->cap_attn = E->cap_subws = E->cap_in = 0;
}

#define WS_ALLOC(ptr, bytes)                                              \
  do {                                                                    \
    cudaFree(ptr);                                                        \
    ptr = nullptr;                                                        \
    cudaError_t e_ = cudaMalloc((void**)&(ptr), std::max<size_t>(bytes, 256)); \
    if (e_ != cudaSuccess) return cuda_fail(e_, "workspace cudaMalloc");  \
  } while (0)

vxg_status ensure_ws(vxg_encoder* E, size_t rows, size_t tmax, const BatchPlan& b, size_t sub_ws, size_t in_rows) {
  const size_t d = E->d, np = 2 * tmax - 1;
  if (rows > E->cap_rows) {
    const size_t r = rows + rows / 4;
    WS_ALLOC(E->x, r * d * 4);
    WS_ALLOC(E->v, r * d * 4);
    WS_ALLOC(E->qkv, r * 3 * d * 4);
    WS_ALLOC(E->g, r * d * 4);  // GLU outputs of pointwise_conv1
    WS_ALLOC(E->aq, r * 2 * d);
    WS_ALLOC(E->as, r * (2 * d / E->group) * 4);
    WS_ALLOC(E->hq, r * E->ff);
    WS_ALLOC(E->hs, r * (E->ff / E->group) * 4);
    WS_ALLOC(E->ctxq, r * d);
    WS_ALLOC(E->ctxs, r * (d / 128) * 4);
    E->cap_rows = r;
  }
  if (np > E->cap_np) {
    const size_t n = np + np / 4;
    WS_ALLOC(E->relk, n * d * 4);
    WS_ALLOC(E->pos, n * d * 4);
    WS_ALLOC(E->posq, n * d);
    WS_ALLOC(E->poss, n * (d / E->group) * 4);
    E->cap_np = n;
  }
  const size_t att = attention_ws_bytes(b.rows, b.tmax, b.n_utt, E->heads, b.Mv);
  if (att > E->cap_attn) {
    WS_ALLOC(E->attn_ws, att + att / 4);
    E->cap_attn = att + att / 4;
  }
  if (b.tab.size() > E->cap_tab) {
    WS_ALLOC(E->dtab, (b.tab.size() + 1024) * 4);
    E->cap_tab = b.tab.size() + 1024;
  }
  if (sub_ws > E->cap_subws) {
    WS_ALLOC(E->sub_ws, sub_ws + sub_ws / 4);
    E->cap_subws = sub_ws + sub_ws / 4;
  }
  (void)in_rows;
  return VXG_OK;
}

vxg_status gemm(vxg_encoder* E, const TernDev& W, const int8_t* x, const float* sx, int M, float* y) {
  ProfScope ps(E, VXG_PROF_GEMM, 2.0 * M * W.out * W.in);
  return gemm_launch(W.packed, x, sx, W.w, W.s, M, W.out, W.in, W.group, VXG_EP_STORE, 0.0f, nullptr, y, nullptr,
                     nullptr, nullptr, E->stream);
}

// q|k|v projection: the attention's per-head int8 Q (with bias_u, bias_v) and K written by the GEMM epilogue straight
// into the attention workspace; only v reaches y as f32.
vxg_status gemm_qk(vxg_encoder* E, const TernDev& W, const int8_t* x, const float* sx, int M, float* y,
                   const QkQuant& qk) {
  ProfScope ps(E, VXG_PROF_GEMM, 2.0 * M * W.out * W.in);
  return gemm_launch(W.packed, x, sx, W.w, W.s, M, W.out, W.in, W.group, kGemmQKQuant, 0.0f, nullptr, y, nullptr,
                     nullptr, nullptr, E->stream, &qk);
}

// pointwise_conv1 with the GLU in its epilogue (interleaved weight rows): y = glu(W x) [M, N/2].
vxg_status gemm_glu(vxg_encoder* E, const TernDev& W, const int8_t* x, const float* sx, int M, float* y) {
  ProfScope ps(E, VXG_PROF_GEMM, 2.0 * M * W.out * W.in);
  return gemm_launch(W.packed, x, sx, W.w, W.s, M, W.out, W.in, W.group, kGemmGlu, 0.0f, nullptr, y, nullptr,
                     nullptr, nullptr, E->stream);
}

// linear1 of a feed-forward block: SiLU and the per-group int8 quantisation for linear2 fused into the GEMM.
vxg_status gemm_silu_q(vxg_encoder* E, const TernDev& W, const int8_t* x, const float* sx, int M, int8_t* q,
                       float* qs) {
  ProfScope ps(E, VXG_PROF_GEMM, 2.0 * M * W.out * W.in);
  return gemm_launch(W.packed, x, sx, W.w, W.s, M, W.out, W.in, W.group, kGemmSiluQuant, 0.0f, nullptr, nullptr, q,
                     qs, nullptr, E->stream);
}

// The 24 layers on x (stacked rows of the plan), result in `out` (may be x).
//
// Every residual update of the reference (x = fma(s, v, x) in the AddScaled epilogues of ff*.linear2, o_proj and
// pointwise_conv2) is applied by the LayerNorm pass that reads x next: the GEMM stores v, and that pass computes the
// same fma before normalising, so the residual stream makes one trip through HBM per update.
vxg_status run_layers(vxg_encoder* E, const BatchPlan& b, float* out) {
  const int M = b.rows, d = E->d, G = E->group, tmax = b.tmax, np = 2 * tmax - 1;
  cudaStream_t st = E->stream;
  vxg_status s;
  // relative positions: table for tmax, quantised once per forward (QuantAct::quantize_layout)
  const std::vector<float>& pt = pos_table(E, tmax);
  VXG_CUDA(cudaMemcpyAsync(E->pos, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice, st));
  {
    ProfScope ps(E, VXG_PROF_QUANT);
    if ((s = vxg_quantize_rows(E->pos, np, d, G, E->posq, E->poss, st)) != VXG_OK) return s;
  }
  VXG_CUDA(cudaMemcpyAsync(E->dtab, b.tab.data(), b.tab.size() * 4, cudaMemcpyHostToDevice, st));
  const float scaling = 1.0f / sqrtf((float)(d / E->heads));
  float pending = 0.0f;  // scale of the residual update waiting in E->v (0: none)
  // residual add (if pending) -> [LayerNorm g0 -> x] -> LayerNorm g1 -> int8 for the next GEMM
  auto lnq = [&](const float* g0, const float* b0, const float* g1, const float* b1) -> vxg_status {
    ProfScope ps(E, VXG_PROF_LNQ);
    const float* v = pending != 0.0f ? E->v : nullptr;
    const vxg_status r = ln_quant_run(E->x, v, pending, v && !g0 ? E->x : nullptr, M, d, g0, b0, g0 ? E->x : nullptr,
                                      g1, b1, G, E->aq, E->as, st);
    pending = 0.0f;
    return r;
  };
  for (int l = 0; l < E->n_layers; l++) {
    const LayerDev& L = E->layers[l];
    const LayerDev* P = l > 0 ? &E->layers[l - 1] : nullptr;
    // feed-forward 1 (with the previous layer's norm_out first)
    if ((s = lnq(P ? P->ln[4][0] : nullptr, P ? P->ln[4][1] : nullptr, L.ln[0][0], L.ln[0][1])) != VXG_OK) return s;
    if ((s = gemm_silu_q(E, L.ff1_1, E->aq, E->as, M, E->hq, E->hs)) != VXG_OK) return s;
    if ((s = gemm(E, L.ff1_2, E->hq, E->hs, M, E->v)) != VXG_OK) return s;
    pending = 0.5f;
    // attention
    if ((s = lnq(nullptr, nullptr, L.ln[1][0], L.ln[1][1])) != VXG_OK) return s;
    QkQuant qk = attention_qk_buffers(b, E->heads, E->attn_ws);
    qk.bu = L.bias_u;
    qk.bv = L.bias_v;
    if ((s = gemm_qk(E, L.qkv, E->aq, E->as, M, E->qkv, qk)) != VXG_OK) return s;
    if ((s = gemm(E, L.relk, E->posq, E->poss, np, E->relk)) != VXG_OK) return s;
    {
      ProfScope ps(E, VXG_PROF_ATTN);
      if ((s = attention_run(b, E->dtab, E->qkv, 3 * d, E->relk, L.bias_u, L.bias_v, E->heads, scaling, nullptr,
                             E->ctxq, E->ctxs, E->attn_ws, E->cap_attn, st, true)) != VXG_OK)
        return s;
    }
    if ((s = gemm(E, L.o, E->ctxq, E->ctxs, M, E->v)) != VXG_OK) return s;
    pending = 1.0f;
    // conv module
    if ((s = lnq(nullptr, nullptr, L.ln[2][0], L.ln[2][1])) != VXG_OK) return s;
    if ((s = gemm_glu(E, L.pw1, E->aq, E->as, M, E->g)) != VXG_OK) return s;
    {
      ProfScope ps(E, VXG_PROF_CONV);
      if ((s = conv_run(b, E->dtab, E->g, d, L.dw_t, L.dw_b, d, E->k, nullptr, E->aq, E->as, st, true)) != VXG_OK)
        return s;
    }
    if ((s = gemm(E, L.pw2, E->aq, E->as, M, E->v)) != VXG_OK) return s;
    pending = 1.0f;
    // feed-forward 2
    if ((s = lnq(nullptr, nullptr, L.ln[3][0], L.ln[3][1])) != VXG_OK) return s;
    if ((s = gemm_silu_q(E, L.ff2_1, E->aq, E->as, M, E->hq, E->hs)) != VXG_OK) return s;
    if ((s = gemm(E, L.ff2_2, E->hq, E->hs, M, E->v)) != VXG_OK) return s;
    pending = 0.5f;
  }
  const LayerDev& last = E->layers.back();
  ProfScope ps(E, VXG_PROF_LNQ);
  return ln_quant_run(E->x, E->v, pending, nullptr, M, d, last.ln[4][0], last.ln[4][1], out, nullptr, nullptr, G,
                      nullptr, nullptr, st);
}

}  // namespace

vxg_encoder::~vxg_encoder() {
  if (device >= 0) cudaSetDevice(device);
  if (stream) cudaStreamSynchronize(stream);
  for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
  free_ws(this);
  for (void* p : allocs) cudaFree(p);
  if (host_pin) cudaFreeHost(host_pin);
  if (copy_stream) cudaStreamSynchronize(copy_stream), cudaStreamDestroy(copy_stream);
  if (stream) cudaStreamDestroy(stream);
}

extern "C" {

vxg_status vxg_encoder_create(const vxg_encoder_desc* desc, int device, vxg_encoder** out) {
  clear_error();
  VXG_ARG(desc && out && desc->layers && desc->sub, "NULL argument");
  VXG_ARG(desc->d_model % 128 == 0 && desc->heads > 0 && desc->d_model / desc->heads == 128,
          "d_model must be heads x 128");
  VXG_ARG(desc->n_layers > 0 && desc->conv_kernel % 2 == 1 && desc->sub_channels == 256 && desc->n_mels % 8 == 0,
          "unsupported encoder configuration");
  VXG_ARG(desc->weight_format == VXG_WEIGHTS_2BIT || desc->weight_format == VXG_WEIGHTS_INT8, "bad weight format");
  *out = nullptr;
  VXG_CUDA(cudaSetDevice(device));
  vxg_encoder* E = new vxg_encoder();
  E->device = device;
  E->d = desc->d_model;
  E->ff = desc->ff;
  E->heads = desc->heads;
  E->k = desc->conv_kernel;
  E->n_layers = desc->n_layers;
  E->n_mels = desc->n_mels;
  E->sub_ch = desc->sub_channels;
  E->packed = desc->weight_format == VXG_WEIGHTS_2BIT;
  auto fail = [&](vxg_status s) {
    delete E;
    return s;
  };
  cudaError_t ce = cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) return fail(cuda_fail(ce, "cudaStreamCreate"));
  const int d = E->d, k = E->k;
  E->layers.resize(E->n_layers);
  vxg_status s;
  for (int l = 0; l < E->n_layers; l++) {
    const vxg_layer_weights& W = desc->layers[l];
    LayerDev& L = E->layers[l];
    const vxg_ternary_tensor qkv[3] = {W.q_proj, W.k_proj, W.v_proj};
    if ((s = load_tern(E, &L.ff1_1, &W.ff1_linear1, 1)) != VXG_OK || (s = load_tern(E, &L.ff1_2, &W.ff1_linear2, 1)) != VXG_OK ||
        (s = load_tern(E, &L.qkv, qkv, 3)) != VXG_OK || (s = load_tern(E, &L.o, &W.o_proj, 1)) != VXG_OK ||
        (s = load_tern(E, &L.relk, &W.relative_k_proj, 1)) != VXG_OK ||
        (s = load_tern(E, &L.pw1, &W.pointwise_conv1, 1, true)) != VXG_OK ||
        (s = load_tern(E, &L.pw2, &W.pointwise_conv2, 1)) != VXG_OK ||
        (s = load_tern(E, &L.ff2_1, &W.ff2_linear1, 1)) != VXG_OK || (s = load_tern(E, &L.ff2_2, &W.ff2_linear2, 1)) != VXG_OK)
      return fail(s);
    const float* lnp[5][2] = {{W.norm_ff1_w, W.norm_ff1_b}, {W.norm_attn_w, W.norm_attn_b},
                              {W.norm_conv_w, W.norm_conv_b}, {W.norm_ff2_w, W.norm_ff2_b},
                              {W.norm_out_w, W.norm_out_b}};
    for (int i = 0; i < 5; i++)
      for (int j = 0; j < 2; j++)
        if ((s = load_vec(E, &L.ln[i][j], lnp[i][j], d)) != VXG_OK) return fail(s);
    if ((s = load_vec(E, &L.bias_u, W.bias_u, d)) != VXG_OK || (s = load_vec(E, &L.bias_v, W.bias_v, d)) != VXG_OK)
      return fail(s);
    std::vector<float> dw_t((size_t)k * d), dw_b(d);
    if ((s = vxg_fold_bn(W.dw_weight, W.bn_weight, W.bn_bias, W.bn_mean, W.bn_var, d, k, dw_t.data(), dw_b.data())) !=
        VXG_OK)
      return fail(s);
    if ((s = load_vec(E, &L.dw_t, dw_t.data(), dw_t.size())) != VXG_OK || (s = load_vec(E, &L.dw_b, dw_b.data(), d)) != VXG_OK)
      return fail(s);
  }
  {  // Subsampling::load (subsampling.rs:31-96): tap-major convs, [out][in] pointwise, channels-last linear
    const vxg_subsampling_weights& S = *desc->sub;
    const int c = E->sub_ch, f3 = E->n_mels / 8;
    auto tap = [&](const float* w) {
      std::vector<float> t((size_t)9 * c);
      for (int ch = 0; ch < c; ch++)
        for (int tp = 0; tp < 9; tp++) t[(size_t)tp * c + ch] = w[(size_t)ch * 9 + tp];
      return t;
    };
    std::vector<float> lin((size_t)d * c * f3);
    for (int o = 0; o < d; o++)
      for (int ch = 0; ch < c; ch++)
        for (int f = 0; f < f3; f++) lin[(size_t)o * c * f3 + (size_t)f * c + ch] = S.lin_w[(size_t)o * c * f3 + (size_t)ch * f3 + f];
    std::vector<float> t0 = tap(S.conv0_w), t1 = tap(S.dw1_w), t2 = tap(S.dw2_w);
    const float* src[12] = {t0.data(), S.conv0_b, t1.data(), S.dw1_b, S.pw1_w, S.pw1_b,
                            t2.data(), S.dw2_b, S.pw2_w, S.pw2_b, lin.data(), S.lin_b};
    const size_t n[12] = {(size_t)9 * c, (size_t)c, (size_t)9 * c, (size_t)c, (size_t)c * c, (size_t)c,
                          (size_t)9 * c, (size_t)c, (size_t)c * c, (size_t)c, lin.size(), (size_t)d};
    for (int i = 0; i < 12; i++)
      if ((s = load_vec(E, &E->sub[i], src[i], n[i])) != VXG_OK) return fail(s);
  }
  *out = E;
  return VXG_OK;
}

void vxg_encoder_destroy(vxg_encoder* e) { delete e; }

}  // extern "C"

namespace {

// Forward with E->mu held: device feats (stacked) -> device out (stacked; NULL = E->x, valid until the next call).
// One host copy of a batch's staging: the bytes [dst, dst + bytes) <- [src, src + bytes).
struct HostCopy {
  void* dst;
  const void* src;
  size_t bytes;
};

// Copy the parts of `jobs` (laid out back to back in the staging buffer `stage`, as jobs[0] first) that fall in
// the staging byte range [b0, b1), on the encoder's copy threads (at most 16 with the caller). parallel_copy fills the staging buffer (jobs' dst are
// inside it), parallel_copy_from drains it (jobs' src are inside it).
void copy_range(CopyPool& pool, const std::vector<HostCopy>& jobs, size_t b0, size_t b1, bool into_stage,
                char* stage_w, const char* stage_r) {
  if (b1 <= b0) return;
  std::vector<std::pair<char*, const char*>> segs;  // (dst, src) pieces with lengths below
  std::vector<size_t> lens;
  size_t at = 0;
  for (const HostCopy& j : jobs) {
    const size_t s0 = std::max(at, b0), s1 = std::min(at + j.bytes, b1);
    if (s0 < s1) {
      if (into_stage)
        segs.push_back({stage_w + s0, static_cast<const char*>(j.src) + (s0 - at)});
      else
        segs.push_back({static_cast<char*>(j.dst) + (s0 - at), stage_r + s0});
      lens.push_back(s1 - s0);
    }
    at += j.bytes;
  }
  const size_t total = b1 - b0;
  const int nt = (int)std::max<size_t>(1, std::min<size_t>((size_t)pool.workers() + 1, total >> 20));
  auto work = [&](size_t w0, size_t w1) {  // byte range of the concatenated pieces
    size_t pos = 0;
    for (size_t i = 0; i < segs.size(); i++) {
      const size_t p0 = std::max(pos, w0), p1 = std::min(pos + lens[i], w1);
      if (p0 < p1) std::memcpy(segs[i].first + (p0 - pos), segs[i].second + (p0 - pos), p1 - p0);
      pos += lens[i];
    }
  };
  if (nt <= 1) {
    work(0, total);
    return;
  }
  pool.run(nt, [&](int i) { work(total * i / nt, total * (i + 1) / nt); });
}
void parallel_copy(CopyPool& pool, const std::vector<HostCopy>& jobs, char* stage, size_t b0, size_t b1) {
  copy_range(pool, jobs, b0, b1, true, stage, nullptr);
}
void parallel_copy_from(CopyPool& pool, const std::vector<HostCopy>& jobs, const char* stage, size_t b0, size_t b1) {
  copy_range(pool, jobs, b0, b1, false, nullptr, stage);
}

// `order`: run after the work already queued on `caller` and make work queued on `caller` later wait for this
// forward (caller 0 is the legacy default stream, as everywhere in CUDA). The host-buffer entry orders its own copies
// on the encoder's stream instead.
vxg_status forward_locked(vxg_encoder* E, const float* feats, const int* t_in, int n, float* out, int* t_e,
                          cudaStream_t caller, bool order) {
  std::vector<int> te(n);
  int tmax = 0;
  for (int u = 0; u < n; u++) {
    VXG_ARG(t_in[u] > 0, "empty utterance %d", u);
    te[u] = vxg_sub_out_frames(t_in[u]);
    tmax = std::max(tmax, te[u]);
    if (t_e) t_e[u] = te[u];
  }
  BatchPlan b;
  batch_plan(b, te.data(), n, tmax);
  vxg_status s = ensure_ws(E, b.rows, tmax, b, vxg_subsampling_workspace_bytes(t_in, n, E->n_mels), 0);
  if (s != VXG_OK) return s;
  cudaEvent_t ev = nullptr;
  if (order) {  // order after the caller's stream, run on ours, then make the caller's stream wait for us
    VXG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    VXG_CUDA(cudaEventRecord(ev, caller));
    VXG_CUDA(cudaStreamWaitEvent(E->stream, ev, 0));
  }
  float* const* sw = E->sub;
  {
    ProfScope ps(E, VXG_PROF_SUB);
    if ((s = vxg_subsampling(feats, t_in, n, E->n_mels, sw[0], sw[1], sw[2], sw[3], sw[4], sw[5], sw[6], sw[7],
                             sw[8], sw[9], sw[10], sw[11], E->d, E->x, E->sub_ws, E->cap_subws, E->stream)) != VXG_OK)
      return s;
  }
  if ((s = run_layers(E, b, out ? out : E->x)) != VXG_OK) return s;
  if (order) {
    VXG_CUDA(cudaEventRecord(ev, E->stream));
    VXG_CUDA(cudaStreamWaitEvent(caller, ev, 0));
    VXG_CUDA(cudaEventDestroy(ev));
  }
  return VXG_OK;
}

// Whether [p, p + bytes) is page-locked host memory this context can copy with the DMA engines directly (both ends
// checked: a cudaHostRegister'd range may cover only part of a buffer).
bool host_pinned(const void* p, size_t bytes) {
  for (const char* q : {static_cast<const char*>(p), static_cast<const char*>(p) + (bytes ? bytes - 1 : 0)}) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, q) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (a.type != cudaMemoryTypeHost) return false;
  }
  return true;
}

// Host-buffer forward whose inputs are page-locked: the utterances are cut into up to four groups of consecutive
// utterances with similar frame counts; group g's feats go to the device on the copy stream while the encoder's
// stream runs the subsampling front end of group g - 1, so the input transfer hides behind the front end. The
// layers then run on the whole stacked batch, as in forward_locked.
vxg_status forward_pinned_in(vxg_encoder* E, const float* const* feats, const int* t_in, int n) {
  std::vector<int> te(n);
  int tmax = 0;
  size_t in_rows = 0;
  for (int u = 0; u < n; u++) {
    te[u] = vxg_sub_out_frames(t_in[u]);
    tmax = std::max(tmax, te[u]);
    in_rows += t_in[u];
  }
  BatchPlan b;
  batch_plan(b, te.data(), n, tmax);
  vxg_status s = ensure_ws(E, b.rows, tmax, b, vxg_subsampling_workspace_bytes(t_in, n, E->n_mels), 0);
  if (s != VXG_OK) return s;
  if (!E->copy_stream) VXG_CUDA(cudaStreamCreateWithFlags(&E->copy_stream, cudaStreamNonBlocking));
  constexpr int kGroups = 4;
  std::vector<int> cut{0};  // group g = utterances [cut[g], cut[g + 1])
  {
    size_t acc = 0;
    for (int u = 0; u < n; u++) {
      acc += t_in[u];
      if ((int)cut.size() < kGroups && acc * kGroups >= in_rows * cut.size() && u + 1 < n) cut.push_back(u + 1);
    }
    cut.push_back(n);
  }
  const int ng = (int)cut.size() - 1;
  cudaEvent_t ev[kGroups] = {};
  s = VXG_OK;
  size_t in_off = 0, out_off = 0;
  for (int g = 0; g < ng && s == VXG_OK; g++) {
    const int u0 = cut[g], u1 = cut[g + 1];
    size_t gin = 0, gout = 0;
    cudaError_t ce = cudaEventCreateWithFlags(&ev[g], cudaEventDisableTiming);
    for (int u = u0; u < u1 && ce == cudaSuccess; u++) {
      const size_t bytes = (size_t)t_in[u] * E->n_mels * 4;
      ce = cudaMemcpyAsync(E->feats + (in_off + gin) * E->n_mels, feats[u], bytes, cudaMemcpyHostToDevice,
                           E->copy_stream);
      gin += t_in[u];
      gout += te[u];
    }
    if (ce == cudaSuccess) ce = cudaEventRecord(ev[g], E->copy_stream);
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(E->stream, ev[g], 0);
    if (ce != cudaSuccess) {
      s = cuda_fail(ce, "input copy");
      break;
    }
    ProfScope ps(E, VXG_PROF_SUB);
    float* const* sw = E->sub;
    s = vxg_subsampling(E->feats + in_off * E->n_mels, t_in + u0, u1 - u0, E->n_mels, sw[0], sw[1], sw[2], sw[3], sw[4],
                        sw[5], sw[6], sw[7], sw[8], sw[9], sw[10], sw[11], E->d, E->x + out_off * E->d, E->sub_ws,
                        E->cap_subws, E->stream);
    in_off += gin;
    out_off += gout;
  }
  for (int g = 0; g < kGroups; g++)
    if (ev[g]) cudaEventDestroy(ev[g]);
  if (s != VXG_OK) {
    cudaStreamSynchronize(E->copy_stream);  // no copy may still read the caller's buffers after we return
    return s;
  }
  return run_layers(E, b, E->x);
}

vxg_status check_status() {
  int code = 0;
  int* st = device_status();
  if (!st) return VXG_OK;
  VXG_CUDA(cudaMemcpy(&code, st, sizeof(int), cudaMemcpyDeviceToHost));
  if (code) {
    cudaMemset(st, 0, sizeof(int));
    set_error("a kernel reported device status 0x%x (bounded wait expired)", code);
    return VXG_ERR_TIMEOUT;
  }
  return VXG_OK;
}

// Encoder frames of a host-buffer forward (stacked in E->x) to page-locked caller buffers, one DMA per utterance.
vxg_status copy_out_direct(vxg_encoder* E, float* const* outs, const int* t_e, int n) {
  size_t r = 0;
  for (int u = 0; u < n; u++) {
    VXG_CUDA(cudaMemcpyAsync(outs[u], E->x + r * E->d, (size_t)t_e[u] * E->d * 4, cudaMemcpyDeviceToHost, E->stream));
    r += t_e[u];
  }
  VXG_CUDA(cudaStreamSynchronize(E->stream));
  return check_status();
}

// The same through the pinned staging buffer, in chunks: each chunk's host copy (on the copy threads) overlaps the
// next chunk's transfer.
vxg_status copy_out_staged(vxg_encoder* E, float* const* outs, const int* t_e, int n, size_t out_rows) {
  if (!E->copy_pool)
    E->copy_pool = std::make_unique<CopyPool>((int)std::min(15u, std::max(1u, std::thread::hardware_concurrency()) - 1));
  constexpr int kChunks = 4;
  std::vector<HostCopy> out_jobs;
  size_t r = 0;
  for (int u = 0; u < n; u++) {
    out_jobs.push_back({outs[u], E->host_pin + r * E->d, (size_t)t_e[u] * E->d * 4});
    r += t_e[u];
  }
  const size_t out_bytes = out_rows * E->d * 4;
  cudaEvent_t done[kChunks];
  for (int c = 0; c < kChunks; c++) {
    const size_t b0 = out_bytes * c / kChunks / 16 * 16, b1 = c + 1 == kChunks ? out_bytes : out_bytes * (c + 1) / kChunks / 16 * 16;
    VXG_CUDA(cudaEventCreateWithFlags(&done[c], cudaEventDisableTiming));
    if (b1 > b0)
      VXG_CUDA(cudaMemcpyAsync(reinterpret_cast<char*>(E->host_pin) + b0, reinterpret_cast<char*>(E->x) + b0, b1 - b0,
                               cudaMemcpyDeviceToHost, E->stream));
    VXG_CUDA(cudaEventRecord(done[c], E->stream));
  }
  for (int c = 0; c < kChunks; c++) {
    const size_t b0 = out_bytes * c / kChunks / 16 * 16, b1 = c + 1 == kChunks ? out_bytes : out_bytes * (c + 1) / kChunks / 16 * 16;
    const cudaError_t e = cudaEventSynchronize(done[c]);
    if (e != cudaSuccess) {
      for (int k = c; k < kChunks; k++) cudaEventDestroy(done[k]);
      return cuda_fail(e, "cudaEventSynchronize");
    }
    cudaEventDestroy(done[c]);
    parallel_copy_from(*E->copy_pool, out_jobs, reinterpret_cast<const char*>(E->host_pin), b0, b1);
  }
  return check_status();
}

}  // namespace

extern "C" {

vxg_status vxg_encoder_forward_device(vxg_encoder* E, const float* feats, const int* t_in, int n, float* out,
                                      int* t_e, void* stream) {
  clear_error();
  VXG_ARG(E && feats && t_in && out && n > 0, "NULL argument");
  std::lock_guard<std::mutex> lk(E->mu);
  VXG_CUDA(cudaSetDevice(E->device));
  return forward_locked(E, feats, t_in, n, out, t_e, (cudaStream_t)stream, true);
}

vxg_status vxg_encoder_forward_layers_device(vxg_encoder* E, const float* x, const int* t, int n, float* out,
                                             void* stream) {
  clear_error();
  VXG_ARG(E && x && t && out && n > 0, "NULL argument");
  std::lock_guard<std::mutex> lk(E->mu);
  VXG_CUDA(cudaSetDevice(E->device));
  int tmax = 0;
  for (int u = 0; u < n; u++) {
    VXG_ARG(t[u] > 0, "empty utterance %d", u);
    tmax = std::max(tmax, t[u]);
  }
  BatchPlan b;
  batch_plan(b, t, n, tmax);
  vxg_status s = ensure_ws(E, b.rows, tmax, b, 0, 0);
  if (s != VXG_OK) return s;
  VXG_CUDA(cudaStreamSynchronize((cudaStream_t)stream));  // x was produced on the caller's stream (0: legacy)
  VXG_CUDA(cudaMemcpyAsync(E->x, x, (size_t)b.rows * E->d * 4, cudaMemcpyDeviceToDevice, E->stream));
  if ((s = run_layers(E, b, out)) != VXG_OK) return s;
  VXG_CUDA(cudaStreamSynchronize(E->stream));
  return check_status();
}

vxg_status vxg_encoder_subsample_device(vxg_encoder* E, const float* feats, const int* t_in, int n, float* out,
                                        int* t_e, void* stream) {
  clear_error();
  VXG_ARG(E && feats && t_in && out && n > 0, "NULL argument");
  for (int u = 0; u < n; u++) {
    VXG_ARG(t_in[u] > 0, "empty utterance %d", u);
    if (t_e) t_e[u] = vxg_sub_out_frames(t_in[u]);
  }
  std::lock_guard<std::mutex> lk(E->mu);
  VXG_CUDA(cudaSetDevice(E->device));
  const size_t ws = vxg_subsampling_workspace_bytes(t_in, n, E->n_mels);
  if (ws > E->cap_subws) {
    WS_ALLOC(E->sub_ws, ws + ws / 4);
    E->cap_subws = ws + ws / 4;
  }
  cudaStream_t caller = (cudaStream_t)stream;
  cudaEvent_t ev = nullptr;
  VXG_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  VXG_CUDA(cudaEventRecord(ev, caller));
  VXG_CUDA(cudaStreamWaitEvent(E->stream, ev, 0));
  float* const* sw = E->sub;
  vxg_status s = vxg_subsampling(feats, t_in, n, E->n_mels, sw[0], sw[1], sw[2], sw[3], sw[4], sw[5], sw[6], sw[7],
                                 sw[8], sw[9], sw[10], sw[11], E->d, out, E->sub_ws, E->cap_subws, E->stream);
  if (s == VXG_OK) {
    VXG_CUDA(cudaEventRecord(ev, E->stream));
    VXG_CUDA(cudaStreamWaitEvent(caller, ev, 0));
  }
  cudaEventDestroy(ev);
  return s;
}

vxg_status vxg_encoder_forward_batch(vxg_encoder* E, const float* const* feats, const int* t_in, int n,
                                     float* const* outs, int* t_e) {
  clear_error();
  VXG_ARG(E && feats && t_in && outs && t_e && n > 0, "NULL argument");
  size_t in_rows = 0, out_rows = 0;
  for (int u = 0; u < n; u++) {
    VXG_ARG(feats[u] && outs[u] && t_in[u] > 0, "utterance %d: NULL buffer or empty", u);
    in_rows += t_in[u];
    out_rows += vxg_sub_out_frames(t_in[u]);
  }
  std::lock_guard<std::mutex> lk(E->mu);
  VXG_CUDA(cudaSetDevice(E->device));
  const size_t need = std::max(in_rows * E->n_mels, out_rows * E->d);
  if (need > E->cap_host) {
    if (E->host_pin) cudaFreeHost(E->host_pin);
    E->host_pin = nullptr;
    E->cap_host = 0;
    VXG_CUDA(cudaMallocHost(&E->host_pin, (need + need / 4) * 4));
    E->cap_host = need + need / 4;
  }
  if (in_rows > E->cap_in) {
    cudaFree(E->feats);
    E->feats = nullptr;
    E->cap_in = 0;
    cudaError_t e = cudaMalloc(&E->feats, (in_rows + in_rows / 4) * E->n_mels * 4);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    E->cap_in = in_rows + in_rows / 4;
  }
  // Page-locked caller buffers are copied by the DMA engines directly (inputs overlapped with the front end);
  // others go through the encoder's pinned staging buffer.
  bool in_pinned = true, out_pinned = true;
  for (int u = 0; u < n; u++) {
    in_pinned = in_pinned && host_pinned(feats[u], (size_t)t_in[u] * E->n_mels * 4);
    out_pinned = out_pinned && host_pinned(outs[u], (size_t)vxg_sub_out_frames(t_in[u]) * E->d * 4);
  }
  if (in_pinned) {
    for (int u = 0; u < n; u++) t_e[u] = vxg_sub_out_frames(t_in[u]);
    vxg_status s = forward_pinned_in(E, feats, t_in, n);
    if (s != VXG_OK) return s;
    if (out_pinned) return copy_out_direct(E, outs, t_e, n);
    return copy_out_staged(E, outs, t_e, n, out_rows);
  }
  // Host <-> pinned staging runs on several threads and in chunks, so each chunk's copy engine transfer overlaps
  // the host copy of the next one.
  if (!E->copy_pool)
    E->copy_pool = std::make_unique<CopyPool>((int)std::min(15u, std::max(1u, std::thread::hardware_concurrency()) - 1));
  constexpr int kChunks = 4;
  std::vector<HostCopy> in_jobs;
  size_t r = 0;
  for (int u = 0; u < n; u++) {  // stack into pinned memory
    in_jobs.push_back({E->host_pin + r * E->n_mels, feats[u], (size_t)t_in[u] * E->n_mels * 4});
    r += t_in[u];
  }
  const size_t in_bytes = in_rows * E->n_mels * 4;
  for (int c = 0; c < kChunks; c++) {
    const size_t b0 = in_bytes * c / kChunks / 16 * 16, b1 = c + 1 == kChunks ? in_bytes : in_bytes * (c + 1) / kChunks / 16 * 16;
    parallel_copy(*E->copy_pool, in_jobs, reinterpret_cast<char*>(E->host_pin), b0, b1);
    if (b1 > b0)
      VXG_CUDA(cudaMemcpyAsync(reinterpret_cast<char*>(E->feats) + b0, reinterpret_cast<char*>(E->host_pin) + b0,
                               b1 - b0, cudaMemcpyHostToDevice, E->stream));
  }
  vxg_status s = forward_locked(E, E->feats, t_in, n, nullptr, t_e, nullptr, false);
  if (s != VXG_OK) return s;
  if (out_pinned) return copy_out_direct(E, outs, t_e, n);
  return copy_out_staged(E, outs, t_e, n, out_rows);
}

vxg_status vxg_encoder_forward_feats(vxg_encoder* E, const float* feats, int t_in, float* out, size_t out_cap,
                                     int* t_e) {
  clear_error();
  VXG_ARG(E && feats && out && t_e && t_in > 0, "NULL argument");
  const int te = vxg_sub_out_frames(t_in);
  if (out_cap < (size_t)te * E->d) {
    set_error("output buffer holds %zu floats, %d x %d needed", out_cap, te, E->d);
    return VXG_ERR_ARG;
  }
  const float* f[1] = {feats};
  float* o[1] = {out};
  return vxg_encoder_forward_batch(E, f, &t_in, 1, o, t_e);
}

int vxg_encoder_out_frames(int t_in) { return vxg_sub_out_frames(t_in); }

vxg_status vxg_encoder_set_profiling(vxg_encoder* E, int on) {
  clear_error();
  VXG_ARG(E, "NULL encoder");
  std::lock_guard<std::mutex> lk(E->mu);
  E->profile = on != 0;
  return VXG_OK;
}

vxg_status vxg_encoder_profile(vxg_encoder* E, double* ms, int* launches, double* gemm_ops) {
  clear_error();
  VXG_ARG(E && ms && launches && gemm_ops, "NULL argument");
  std::lock_guard<std::mutex> lk(E->mu);
  VXG_CUDA(cudaSetDevice(E->device));
  VXG_CUDA(cudaStreamSynchronize(E->stream));
  for (const auto& e : E->evs) {
    float t = 0.0f;
    VXG_CUDA(cudaEventElapsedTime(&t, e.a, e.b));
    E->prof_ms[e.cls] += t;
    E->prof_n[e.cls] += 1;
    if (e.cls == VXG_PROF_GEMM) E->prof_gemm_ops += e.ops;
  }
  E->evs.clear();
  E->ev_used = 0;
  for (int c = 0; c < VXG_PROF_CLASSES; c++) {
    ms[c] = E->prof_ms[c];
    launches[c] = E->prof_n[c];
    E->prof_ms[c] = 0.0;
    E->prof_n[c] = 0;
  }
  *gemm_ops = E->prof_gemm_ops;
  E->prof_gemm_ops = 0.0;
  return VXG_OK;
}

}  // extern "C"
