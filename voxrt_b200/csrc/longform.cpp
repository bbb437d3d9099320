// Long-form / streaming transcription: LongForm (crates/voxrt/src/longform.rs) and Transcriber::transcribe_long
// (crates/voxrt/src/transcriber.rs:356-420) over this library's GPU frontend, encoder, VAD head and TDT decoder.
//
// The state machine is the reference's: audio accumulates in `pending` (absolute sample base_sample onward); every
// complete block of block_samples (plus ctx_samples of look-ahead) gets VAD probabilities computed over the block
// with up to ctx_samples of context on each side (whole frames on the left), keeping only the block's own frames;
// after each push the probability track is segmented and the leading segments that no future audio can change are
// closed, transcribed (unless collect_only) and dropped from the buffers. flush() runs the VAD on the remaining
// partial block and closes everything; a short stream that never closed a segment is transcribed whole.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "common.h"
#include "tdt.h"

namespace vxg {
namespace vad {
size_t segment(const float* p, int t, const vxg_segment_cfg& cfg, std::vector<vxg_vad_segment>& out);
}
}  // namespace vxg

using namespace vxg;

namespace {
// Device memory grown on demand and kept (a long-form stream reuses it for every VAD block and segment).
// Device scratch from the library's memory pool, stream-ordered on the legacy stream that every copy and entry
// here runs on: a pool keeps its memory between calls, where cudaMalloc / cudaFree of large buffers now and then
// stall behind the driver's bookkeeping.
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  int dev = -1;  // device of p
  void release() {
    if (!p) return;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev) cudaSetDevice(dev);
    cudaFreeAsync(p, nullptr);
    if (cur != dev && cur >= 0) cudaSetDevice(cur);
    p = nullptr;
    cap = 0;
  }
  ~DevBuf() { release(); }
  vxg_status need(size_t bytes) {
    if (bytes <= cap) return VXG_OK;
    release();
    VXG_CUDA(cudaGetDevice(&dev));
    cudaMemPool_t pool = scratch_pool();
    VXG_CUDA(pool ? cudaMallocFromPoolAsync(&p, std::max<size_t>(bytes, 256), pool, nullptr)
                  : cudaMallocAsync(&p, std::max<size_t>(bytes, 256), nullptr));
    cap = bytes;
    return VXG_OK;
  }
  template <class T>
  T* as(size_t byte_off = 0) const {
    return reinterpret_cast<T*>(static_cast<char*>(p) + byte_off);
  }
};

}  // namespace

struct vxg_longform {
  vxg_frontend* fe = nullptr;
  vxg_encoder* enc = nullptr;
  vxg_vad* vad = nullptr;
  vxg_tdt* dec = nullptr;
  vxg_vad_block_fn fn = nullptr;
  void* user = nullptr;
  vxg_longform_cfg cfg{};
  int device = -1, n_mels = 0, d_model = 0;
  std::vector<float> pending;  // audio from base_sample onward
  long long base_sample = 0, next_block = 0, total = 0, max_pending = 0;
  std::vector<float> probs;  // VAD probabilities from the frame at base_sample onward
  std::vector<vxg_emission> emissions;
  std::vector<long long> ranges;  // every closed segment's absolute sample range, in order
  bool emitted = false;
  DevBuf blk, seg;  // VAD-block and segment scratch
  // Offline use (transcribe_long): every block's probabilities computed in one batch ahead of the state machine,
  // for the window [lo, hi) the block would have if no earlier cut clipped its left context; a block whose window
  // matches takes these, any other is computed when the machine reaches it.
  struct Pre {
    long long lo, hi;
    std::vector<float> p;  // all frames of the window
  };
  std::vector<std::pair<long long, Pre>> pre;  // by block start, in order
};

namespace {

size_t up256(size_t b) { return (b + 255) / 256 * 256; }

vxg_status component_info(vxg_longform* L) {
  int d = 0, sr = 0, nm = 0;
  VXG_ARG(vxg_vad_info(L->vad, &d, nullptr, nullptr, nullptr) == VXG_OK, "bad VAD handle");
  VXG_ARG(vxg_frontend_info(L->fe, &sr, &nm) == VXG_OK, "bad frontend handle");
  VXG_ARG(sr == L->cfg.sample_rate, "frontend sample rate %d differs from the config's %d", sr, L->cfg.sample_rate);
  L->d_model = d;
  L->n_mels = nm;
  return VXG_OK;
}

// VAD probabilities of frames [skip, skip + want) of the audio block samples[0 .. n): the GPU frontend, the
// encoder's subsampling front end, the VAD head (vad_block_at, longform.rs:101-115).
vxg_status gpu_block_probs(vxg_longform* L, const float* samples, long long n, long long skip, long long want,
                           std::vector<float>& out) {
  const int t_in = vxg_frontend_frames(n);
  VXG_ARG(t_in > 0, "VAD block of %lld samples has no frames", n);
  const int te = vxg_encoder_out_frames(t_in);
  VXG_ARG(te >= 2, "VAD block of %lld samples gives %d encoder frame(s); at least 2 are needed", n, te);
  VXG_CUDA(cudaSetDevice(L->device));
  cudaStream_t st = nullptr;  // the legacy stream orders the copies and the entries below
  DevBuf& buf = L->blk;
  const size_t b_s = up256(sizeof(float) * n), b_f = up256(sizeof(float) * (size_t)t_in * L->n_mels),
               b_x = up256(sizeof(float) * (size_t)te * L->d_model), b_p = up256(sizeof(float) * te);
  vxg_status s = buf.need(b_s + b_f + b_x + b_p);
  if (s != VXG_OK) return s;
  float* d_s = buf.as<float>(0);
  float* d_f = buf.as<float>(b_s);
  float* d_x = buf.as<float>(b_s + b_f);
  float* d_p = buf.as<float>(b_s + b_f + b_x);
  VXG_CUDA(cudaMemcpy(d_s, samples, sizeof(float) * n, cudaMemcpyHostToDevice));
  const long long ns = n;
  int nf = 0, tex = 0;
  if ((s = vxg_frontend_device(L->fe, d_s, &ns, 1, 1, d_f, &nf, st)) != VXG_OK) return s;
  if ((s = vxg_encoder_subsample_device(L->enc, d_f, &nf, 1, d_x, &tex, st)) != VXG_OK) return s;
  if ((s = vxg_vad_probs_device(L->vad, d_x, &tex, 1, d_p, st)) != VXG_OK) return s;
  std::vector<float> p(tex);
  VXG_CUDA(cudaMemcpy(p.data(), d_p, sizeof(float) * tex, cudaMemcpyDeviceToHost));
  for (long long i = skip; i < std::min<long long>(skip + want, tex); i++) out.push_back(p[i]);
  return VXG_OK;
}

// The window of the block at absolute samples [start, end): whole frames of left context down to lo, right context
// up to hi (vad_block_at, longform.rs:104-107), with `base` the first sample still buffered and `total` received.
void block_window(const vxg_longform_cfg& c, long long start, long long end, long long base, long long total,
                  long long* lo, long long* hi) {
  const long long spf = c.samples_per_frame;
  long long l = std::max(std::max(start - c.ctx_samples, 0LL), base);
  *lo = start - ((start - l) / spf) * spf;
  *hi = std::min(end + c.ctx_samples, total);
}

vxg_status block_probs(vxg_longform* L, long long start, long long end) {
  const long long spf = L->cfg.samples_per_frame;
  long long lo = 0, hi = 0;
  block_window(L->cfg, start, end, L->base_sample, L->total, &lo, &hi);
  const float* block = L->pending.data() + (lo - L->base_sample);
  const long long skip = (start - lo) / spf, want = (end - start) / spf;
  for (const auto& e : L->pre)
    if (e.first == start && e.second.lo == lo && e.second.hi == hi) {
      const auto& p = e.second.p;
      for (long long i = skip; i < std::min<long long>(skip + want, (long long)p.size()); i++) L->probs.push_back(p[i]);
      return VXG_OK;
    }
  if (L->fn) {
    std::vector<float> p(want);
    const long long got = L->fn(L->user, block, hi - lo, skip, want, p.data());
    VXG_ARG(got >= 0 && got <= want, "VAD callback returned %lld for %lld frames", got, want);
    L->probs.insert(L->probs.end(), p.begin(), p.begin() + got);
    return VXG_OK;
  }
  return gpu_block_probs(L, block, hi - lo, skip, want, L->probs);
}

// Every VAD block of a whole recording d_rec[0 .. n) (on the device) in one batch (frontend, subsampling, head over the stacked
// windows), each window as the streaming machine would cut it if no earlier cut clipped its left context: the
// blocks push() computes (whole blocks with their right context available) and those flush() computes.
vxg_status precompute_blocks(vxg_longform* L, const float* d_rec, long long n) {
  const vxg_longform_cfg& c = L->cfg;
  std::vector<long long> starts, los, his;
  long long next = 0;
  while (next + c.block_samples + c.ctx_samples <= n) {  // push: full blocks once their right context arrived
    starts.push_back(next);
    next += c.block_samples;
  }
  while (next < n) {  // flush: the rest, blocks of at least one frame
    const long long end = std::min(next + c.block_samples, n);
    if (end - next >= c.samples_per_frame) starts.push_back(next);
    next = end;
  }
  std::vector<long long> lens;
  std::vector<int> t_in;
  long long ns = 0, nf = 0, ne = 0;
  for (long long st : starts) {
    const long long end = std::min(st + c.block_samples, n);
    long long lo = 0, hi = 0;
    block_window(c, st, end, 0, n, &lo, &hi);
    los.push_back(lo);
    his.push_back(hi);
    lens.push_back(hi - lo);
    t_in.push_back(vxg_frontend_frames(hi - lo));
    if (t_in.back() <= 0 || vxg_encoder_out_frames(t_in.back()) < 2) return VXG_OK;  // left to the per-block path
    ns += hi - lo;
    nf += t_in.back();
    ne += vxg_encoder_out_frames(t_in.back());
  }
  const int nb = (int)starts.size();
  if (nb == 0) return VXG_OK;
  VXG_CUDA(cudaSetDevice(L->device));
  const size_t b_s = up256(sizeof(float) * ns), b_f = up256(sizeof(float) * nf * L->n_mels),
               b_x = up256(sizeof(float) * ne * L->d_model), b_p = up256(sizeof(float) * ne);
  DevBuf& buf = L->blk;
  vxg_status s = buf.need(b_s + b_f + b_x + b_p);
  if (s != VXG_OK) return s;
  float* d_s = buf.as<float>(0);
  float* d_f = buf.as<float>(b_s);
  float* d_x = buf.as<float>(b_s + b_f);
  float* d_p = buf.as<float>(b_s + b_f + b_x);
  long long o = 0;
  for (int i = 0; i < nb; i++) {
    VXG_CUDA(cudaMemcpyAsync(d_s + o, d_rec + los[i], sizeof(float) * lens[i], cudaMemcpyDeviceToDevice, nullptr));
    o += lens[i];
  }
  std::vector<int> nfr(nb), te(nb);
  cudaStream_t st = nullptr;
  if ((s = vxg_frontend_device(L->fe, d_s, lens.data(), nb, 1, d_f, nfr.data(), st)) != VXG_OK) return s;
  if ((s = vxg_encoder_subsample_device(L->enc, d_f, nfr.data(), nb, d_x, te.data(), st)) != VXG_OK) return s;
  if ((s = vxg_vad_probs_device(L->vad, d_x, te.data(), nb, d_p, st)) != VXG_OK) return s;
  std::vector<float> p(ne);
  VXG_CUDA(cudaMemcpy(p.data(), d_p, sizeof(float) * ne, cudaMemcpyDeviceToHost));
  long long q = 0;
  L->pre.clear();
  for (int i = 0; i < nb; i++) {
    L->pre.push_back({starts[i], {los[i], his[i], std::vector<float>(p.begin() + q, p.begin() + q + te[i])}});
    q += te[i];
  }
  return VXG_OK;
}

// Frontend + encoder + projection + greedy decode of n audio pieces on the GPU (transcribe_one's arithmetic for each
// piece; the pieces share token-stacked forwards and one lockstep decode). Emissions of piece i are appended with
// frame + base_frame[i].
vxg_status transcribe_pieces(vxg_frontend* fe, vxg_encoder* enc, vxg_tdt* dec, int device, int n_mels, int d_model,
                             int hidden, int max_symbols, const std::vector<const float*>& pieces,
                             const std::vector<long long>& lens, const std::vector<long long>& base_frame,
                             std::vector<vxg_emission>& out, DevBuf& buf, bool dev_pieces = false) {
  const int n = (int)pieces.size();
  if (n == 0) return VXG_OK;
  VXG_CUDA(cudaSetDevice(device));
  std::vector<int> t_in(n), te(n);
  long long ns = 0, nf = 0, ne = 0;
  for (int i = 0; i < n; i++) {
    t_in[i] = vxg_frontend_frames(lens[i]);
    VXG_ARG(t_in[i] > 0, "segment %d of %lld samples has no frames", i, lens[i]);
    te[i] = vxg_encoder_out_frames(t_in[i]);
    VXG_ARG(te[i] >= 2, "segment %d of %lld samples gives %d encoder frame(s); at least 2 are needed", i, lens[i],
            te[i]);
    ns += lens[i];
    nf += t_in[i];
    ne += te[i];
  }
  std::vector<size_t> cap(n);
  size_t ncap = 0;
  for (int i = 0; i < n; i++) ncap += (cap[i] = (size_t)te[i] * max_symbols + 16);
  const size_t b_s = up256(sizeof(float) * ns), b_f = up256(sizeof(float) * nf * n_mels),
               b_x = up256(sizeof(float) * ne * d_model), b_p = up256(sizeof(float) * ne * hidden),
               b_e = up256(sizeof(vxg_emission) * ncap), b_n = up256(sizeof(int) * n);
  vxg_status s = buf.need(b_s + b_f + b_x + b_p + b_e + b_n);
  if (s != VXG_OK) return s;
  size_t o = 0;
  float* d_s = buf.as<float>(o);
  float* d_f = buf.as<float>(o += b_s);
  float* d_x = buf.as<float>(o += b_f);
  float* d_p = buf.as<float>(o += b_x);
  vxg_emission* d_e = buf.as<vxg_emission>(o += b_p);
  int* d_n = buf.as<int>(o += b_e);
  long long so = 0;
  for (int i = 0; i < n; i++) {
    VXG_CUDA(cudaMemcpyAsync(d_s + so, pieces[i], sizeof(float) * lens[i],
                             dev_pieces ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, nullptr));
    so += lens[i];
  }
  cudaStream_t st = nullptr;
  if ((s = vxg_frontend_device(fe, d_s, lens.data(), n, 1, d_f, nullptr, st)) != VXG_OK) return s;
  if ((s = vxg_encoder_forward_device(enc, d_f, t_in.data(), n, d_x, nullptr, st)) != VXG_OK) return s;
  if ((s = vxg_tdt_project_device(dec, d_x, (int)ne, d_p, st)) != VXG_OK) return s;
  if ((s = vxg_tdt_greedy_device(dec, n, d_p, te.data(), d_e, cap.data(), d_n, st)) != VXG_OK) return s;
  std::vector<vxg_emission> em(ncap);
  std::vector<int> cnt(n);
  VXG_CUDA(cudaMemcpy(em.data(), d_e, sizeof(vxg_emission) * ncap, cudaMemcpyDeviceToHost));
  VXG_CUDA(cudaMemcpy(cnt.data(), d_n, sizeof(int) * n, cudaMemcpyDeviceToHost));
  size_t eo = 0;
  for (int i = 0; i < n; i++) {
    VXG_ARG((size_t)cnt[i] <= cap[i], "segment %d: %d emissions exceed the bound", i, cnt[i]);
    for (int k = 0; k < cnt[i]; k++) {
      vxg_emission e = em[eo + k];
      e.frame += (int32_t)base_frame[i];
      out.push_back(e);
    }
    eo += cap[i];
  }
  return VXG_OK;
}

struct DecInfo {
  int hidden = 0, max_symbols = 0;
};

DecInfo dec_info(const vxg_tdt* d) { return DecInfo{d->d.hidden, d->d.max_symbols}; }

// Transcribe pending samples [a, b) frames (emit, longform.rs:170-193).
vxg_status emit(vxg_longform* L, long long a, long long b, std::vector<long long>& closed) {
  L->emitted = true;
  const long long spf = L->cfg.samples_per_frame;
  const long long s0 = a * spf, s1 = std::min<long long>(b * spf, (long long)L->pending.size());
  for (long long v : {L->base_sample + s0, L->base_sample + s1}) {
    closed.push_back(v);
    L->ranges.push_back(v);
  }
  if (L->cfg.collect_only) return VXG_OK;
  const DecInfo di = dec_info(L->dec);
  return transcribe_pieces(L->fe, L->enc, L->dec, L->device, L->n_mels, L->d_model, di.hidden, di.max_symbols,
                           {L->pending.data() + s0}, {s1 - s0}, {(L->base_sample + s0) / spf}, L->emissions, L->seg);
}

// drain (longform.rs:117-167).
vxg_status drain(vxg_longform* L, bool fin, std::vector<long long>& closed) {
  const long long spf = L->cfg.samples_per_frame;
  if (L->probs.empty()) {
    if (fin && (long long)L->pending.size() >= spf) return emit(L, 0, (long long)L->pending.size() / spf, closed);
    return VXG_OK;
  }
  std::vector<vxg_vad_segment> segs;
  vad::segment(L->probs.data(), (int)L->probs.size(), L->cfg.seg, segs);
  const long long known = (long long)L->probs.size();
  size_t nclosed = 0;
  for (size_t i = 0; i < segs.size(); i++) {
    const bool is_closed =
        fin || (i + 1 < segs.size() && segs[i + 1].end + L->cfg.seg.min_pause_frames <= known) ||
        (segs[i].end - segs[i].start >= L->cfg.seg.max_frames && known >= segs[i].end + 63);
    if (!is_closed) break;
    nclosed = i + 1;
  }
  if (nclosed == 0) return VXG_OK;
  for (size_t i = 0; i < nclosed; i++) {
    const vxg_status s = emit(L, segs[i].start, segs[i].end, closed);
    if (s != VXG_OK) return s;
  }
  // drop audio and probabilities before the next segment's start (or the last closed end when final)
  const long long cut_frame = nclosed < segs.size() ? segs[nclosed].start : segs[nclosed - 1].end;
  const long long cut_sample = std::min<long long>(cut_frame * spf, (long long)L->pending.size());
  L->pending.erase(L->pending.begin(), L->pending.begin() + cut_sample);
  L->base_sample += cut_sample;
  L->probs.erase(L->probs.begin(), L->probs.begin() + std::min<long long>(cut_frame, (long long)L->probs.size()));
  return VXG_OK;
}

vxg_status write_closed(const std::vector<long long>& closed, long long* ranges, size_t cap, size_t* n_closed) {
  const size_t n = closed.size() / 2;
  if (n_closed) *n_closed = n;
  for (size_t i = 0; i < std::min(n, cap); i++) {
    ranges[2 * i] = closed[2 * i];
    ranges[2 * i + 1] = closed[2 * i + 1];
  }
  return VXG_OK;
}

vxg_status check_cfg(const vxg_longform_cfg* c) {
  VXG_ARG(c->block_samples > 0 && c->ctx_samples >= 0 && c->samples_per_frame > 0 && c->sample_rate > 0,
          "bad long-form config");
  VXG_ARG(c->block_samples % c->samples_per_frame == 0, "block_samples must be whole frames");
  VXG_ARG(c->seg.max_frames >= 2 && c->seg.min_pause_frames >= 0 && c->seg.min_frames >= 0 && c->seg.pad_frames >= 0,
          "bad segment config");
  return VXG_OK;
}

}  // namespace

extern "C" {

void vxg_longform_cfg_default(vxg_longform_cfg* c) {
  if (!c) return;
  vxg_segment_cfg_default(&c->seg);
  c->block_samples = 10 * 16000;
  c->ctx_samples = 16 * 1280;
  c->samples_per_frame = 1280;
  c->sample_rate = 16000;
  c->long_form_threshold_s = 30.0;
  c->collect_only = 0;
}

vxg_status vxg_longform_create(vxg_frontend* fe, vxg_encoder* enc, vxg_vad* vad, vxg_tdt* dec,
                               const vxg_longform_cfg* cfg, vxg_longform** out) {
  clear_error();
  VXG_ARG(fe && enc && vad && out && cfg, "NULL argument");
  VXG_ARG(dec || cfg->collect_only, "a decoder is needed unless collect_only");
  vxg_status s = check_cfg(cfg);
  if (s != VXG_OK) return s;
  auto* L = new vxg_longform();
  L->fe = fe, L->enc = enc, L->vad = vad, L->dec = dec, L->cfg = *cfg;
  int dev = -1;
  cudaGetDevice(&dev);
  L->device = dev;
  if ((s = component_info(L)) != VXG_OK) {
    delete L;
    return s;
  }
  *out = L;
  return VXG_OK;
}

vxg_status vxg_longform_create_with_vad(vxg_vad_block_fn fn, void* user, const vxg_longform_cfg* cfg,
                                        vxg_longform** out) {
  clear_error();
  VXG_ARG(fn && out && cfg, "NULL argument");
  vxg_status s = check_cfg(cfg);
  if (s != VXG_OK) return s;
  auto* L = new vxg_longform();
  L->fn = fn, L->user = user, L->cfg = *cfg;
  L->cfg.collect_only = 1;
  *out = L;
  return VXG_OK;
}

void vxg_longform_destroy(vxg_longform* lf) { delete lf; }

vxg_status vxg_longform_push(vxg_longform* L, const float* samples, long long n, long long* ranges, size_t cap,
                             size_t* n_closed) {
  clear_error();
  VXG_ARG(L && n >= 0 && (samples || n == 0) && (ranges || cap == 0), "bad arguments");
  L->pending.insert(L->pending.end(), samples, samples + n);
  L->total += n;
  L->max_pending = std::max(L->max_pending, (long long)L->pending.size());
  while (L->next_block + L->cfg.block_samples + L->cfg.ctx_samples <= L->total) {
    const vxg_status s = block_probs(L, L->next_block, L->next_block + L->cfg.block_samples);
    if (s != VXG_OK) return s;
    L->next_block += L->cfg.block_samples;
  }
  std::vector<long long> closed;
  const vxg_status s = drain(L, false, closed);
  write_closed(closed, ranges, cap, n_closed);
  return s;
}

vxg_status vxg_longform_flush(vxg_longform* L, long long* ranges, size_t cap, size_t* n_closed) {
  clear_error();
  VXG_ARG(L && (ranges || cap == 0), "bad arguments");
  std::vector<long long> closed;
  const bool short_stream = (double)L->total / L->cfg.sample_rate <= L->cfg.long_form_threshold_s;
  if (!L->cfg.collect_only && !L->emitted && L->base_sample == 0 && short_stream) {
    // the whole-clip path, as Transcriber::transcribe_long takes for audio of this length
    L->emitted = true;
    vxg_status s = VXG_OK;
    if (!L->pending.empty()) {
      const DecInfo di = dec_info(L->dec);
      s = transcribe_pieces(L->fe, L->enc, L->dec, L->device, L->n_mels, L->d_model, di.hidden, di.max_symbols,
                            {L->pending.data()}, {(long long)L->pending.size()}, {0}, L->emissions, L->seg);
    }
    closed = {0, L->total};
    L->ranges.insert(L->ranges.end(), closed.begin(), closed.end());
    L->base_sample = L->total;
    L->next_block = L->total;
    L->pending.clear();
    L->probs.clear();
    write_closed(closed, ranges, cap, n_closed);
    return s;
  }
  while (L->next_block < L->total) {
    const long long end = std::min(L->next_block + L->cfg.block_samples, L->total);
    if (end - L->next_block >= L->cfg.samples_per_frame) {
      const vxg_status s = block_probs(L, L->next_block, end);
      if (s != VXG_OK) return s;
    }
    L->next_block = end;
  }
  const vxg_status s = drain(L, true, closed);
  write_closed(closed, ranges, cap, n_closed);
  return s;
}

vxg_status vxg_longform_emissions(const vxg_longform* L, vxg_emission* out, size_t cap, size_t* n) {
  clear_error();
  VXG_ARG(L && n && (out || cap == 0), "bad arguments");
  *n = L->emissions.size();
  std::copy(L->emissions.begin(), L->emissions.begin() + std::min(cap, L->emissions.size()), out);
  return VXG_OK;
}

vxg_status vxg_longform_ranges(const vxg_longform* L, long long* ranges, size_t cap, size_t* n) {
  clear_error();
  VXG_ARG(L && n && (ranges || cap == 0), "bad arguments");
  return write_closed(L->ranges, ranges, cap, n);
}

vxg_status vxg_longform_stats(const vxg_longform* L, long long* max_pending, long long* base_sample,
                              long long* n_probs) {
  clear_error();
  VXG_ARG(L, "NULL argument");
  if (max_pending) *max_pending = L->max_pending;
  if (base_sample) *base_sample = L->base_sample;
  if (n_probs) *n_probs = (long long)L->probs.size();
  return VXG_OK;
}

vxg_status vxg_transcribe_long(vxg_frontend* fe, vxg_encoder* enc, vxg_vad* vad, vxg_tdt* dec, const float* samples,
                               long long n, const vxg_longform_cfg* cfg, vxg_emission* out, size_t cap,
                               size_t* n_out, long long* ranges, size_t rcap, size_t* n_ranges) {
  clear_error();
  VXG_ARG(fe && enc && vad && dec && cfg && n_out && n >= 0 && (samples || n == 0) && (out || cap == 0) &&
              (ranges || rcap == 0),
          "bad arguments");
  vxg_status s = check_cfg(cfg);
  if (s != VXG_OK) return s;
  int dev = -1;
  VXG_CUDA(cudaGetDevice(&dev));
  int d_model = 0;
  VXG_ARG(vxg_vad_info(vad, &d_model, nullptr, nullptr, nullptr) == VXG_OK, "bad VAD handle");
  const DecInfo di = dec_info(dec);
  std::vector<long long> rg;
  DevBuf rec;  // the whole recording on the device (long recordings): VAD windows and segments are cut from it
  if ((double)n / cfg->sample_rate <= cfg->long_form_threshold_s) {
    if (n > 0) rg = {0, n};
  } else {
    if ((s = rec.need(sizeof(float) * (size_t)n)) != VXG_OK) return s;
    VXG_CUDA(cudaMemcpy(rec.p, samples, sizeof(float) * (size_t)n, cudaMemcpyHostToDevice));
    vxg_longform_cfg c = *cfg;
    c.collect_only = 1;
    vxg_longform* L = nullptr;
    if ((s = vxg_longform_create(fe, enc, vad, nullptr, &c, &L)) != VXG_OK) return s;
    s = precompute_blocks(L, rec.as<float>(), n);
    const long long chunk = 10LL * cfg->sample_rate;  // transcriber.rs:362-364
    for (long long a = 0; a < n && s == VXG_OK; a += chunk) {
      size_t k = 0;
      s = vxg_longform_push(L, samples + a, std::min(chunk, n - a), nullptr, 0, &k);
    }
    size_t k = 0;
    if (s == VXG_OK) s = vxg_longform_flush(L, nullptr, 0, &k);
    rg = L->ranges;
    vxg_longform_destroy(L);
    if (s != VXG_OK) return s;
  }
  const size_t nr = rg.size() / 2;
  if (n_ranges) *n_ranges = nr;
  for (size_t i = 0; i < std::min(nr, rcap); i++) ranges[2 * i] = rg[2 * i], ranges[2 * i + 1] = rg[2 * i + 1];
  std::vector<const float*> pieces;
  std::vector<long long> lens, base;
  const float* src = rec.p ? rec.as<float>() : samples;
  for (size_t i = 0; i < nr; i++) {
    pieces.push_back(src + rg[2 * i]);
    lens.push_back(rg[2 * i + 1] - rg[2 * i]);
    base.push_back(rg[2 * i] / cfg->samples_per_frame);
  }
  std::vector<vxg_emission> em;
  int sr = 0, n_mels = 0;
  VXG_ARG(vxg_frontend_info(fe, &sr, &n_mels) == VXG_OK, "bad frontend handle");
  DevBuf buf;
  s = transcribe_pieces(fe, enc, dec, dev, n_mels, d_model, di.hidden, di.max_symbols, pieces, lens, base, em, buf,
                        rec.p != nullptr);
  *n_out = em.size();
  std::copy(em.begin(), em.begin() + std::min(cap, em.size()), out);
  return s;
}

}  // extern "C"
