// thrush-ternary-v2 model directories: config.json + ternary.json + model.safetensors, read on the host, checked
// the way the reference checks them, and handed to the encoder and decoder loaders.
//
// Reference: ModelFile::open / tensor / validate (crates/voxrt/src/format.rs:88-309), the loaders that read it
// (Encoder::load_with encoder.rs:787-806 with TernaryLinear::load_stacked ternary_linear.rs:59-99 for q|k|v,
// Decoder::load decoder.rs:57-110) and load_f32 / load_f16_bits (tensor.rs:20-37, :505-525).
//
// The safetensors file is memory-mapped read-only; ternary qweight / f16 scale tensors are passed to the encoder as
// pointers into the mapping, dense tensors stored as f16 are widened to f32 (exactly) into buffers the model owns.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.h"

namespace vxg {
namespace model {

// ------------------------------------------------------------------------------------------------ JSON
// A small recursive-descent JSON reader (objects, arrays, strings with escapes, numbers, literals): enough for the
// two config files and the safetensors header.
struct Json {
  enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* get(const std::string& k) const {
    if (kind != OBJ) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

class JsonParser {
 public:
  JsonParser(const char* s, size_t n) : p_(s), e_(s + n) {}
  bool parse(Json& out, std::string& err) {
    if (!value(out, 0)) {
      err = err_.empty() ? "malformed JSON" : err_;
      return false;
    }
    ws();
    if (p_ != e_) {
      err = "trailing characters after JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* e_;
  std::string err_;

  void ws() {
    while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) p_++;
  }
  bool fail(const char* m) {
    if (err_.empty()) err_ = m;
    return false;
  }
  bool lit(const char* w) {
    const size_t n = strlen(w);
    if ((size_t)(e_ - p_) < n || strncmp(p_, w, n) != 0) return false;
    p_ += n;
    return true;
  }
  static void utf8(std::string& s, unsigned cp) {
    if (cp < 0x80) {
      s += (char)cp;
    } else if (cp < 0x800) {
      s += (char)(0xC0 | (cp >> 6));
      s += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      s += (char)(0xE0 | (cp >> 12));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    } else {
      s += (char)(0xF0 | (cp >> 18));
      s += (char)(0x80 | ((cp >> 12) & 0x3F));
      s += (char)(0x80 | ((cp >> 6) & 0x3F));
      s += (char)(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(unsigned& v) {
    if (e_ - p_ < 4) return false;
    v = 0;
    for (int i = 0; i < 4; i++) {
      const char c = *p_++;
      v <<= 4;
      if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
      else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
      else return false;
    }
    return true;
  }
  bool string(std::string& s) {
    if (p_ >= e_ || *p_ != '"') return fail("expected a string");
    p_++;
    while (p_ < e_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') {
        s += c;
        continue;
      }
      if (p_ >= e_) return fail("unterminated escape");
      c = *p_++;
      switch (c) {
        case '"': s += '"'; break;
        case '\\': s += '\\'; break;
        case '/': s += '/'; break;
        case 'b': s += '\b'; break;
        case 'f': s += '\f'; break;
        case 'n': s += '\n'; break;
        case 'r': s += '\r'; break;
        case 't': s += '\t'; break;
        case 'u': {
          unsigned cp;
          if (!hex4(cp)) return fail("bad \\u escape");
          if (cp >= 0xD800 && cp < 0xDC00 && e_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
            p_ += 2;
            unsigned lo;
            if (!hex4(lo)) return fail("bad \\u escape");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          utf8(s, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p_ >= e_) return fail("unterminated string");
    p_++;
    return true;
  }
  bool value(Json& v, int depth) {
    if (depth > 64) return fail("JSON nested too deeply");
    ws();
    if (p_ >= e_) return fail("unexpected end of JSON");
    const char c = *p_;
    if (c == '{') {
      p_++;
      v.kind = Json::OBJ;
      ws();
      if (p_ < e_ && *p_ == '}') {
        p_++;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!string(k)) return false;
        ws();
        if (p_ >= e_ || *p_ != ':') return fail("expected ':'");
        p_++;
        Json child;
        if (!value(child, depth + 1)) return false;
        v.obj.emplace_back(std::move(k), std::move(child));
        ws();
        if (p_ < e_ && *p_ == ',') {
          p_++;
          continue;
        }
        if (p_ < e_ && *p_ == '}') {
          p_++;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      p_++;
      v.kind = Json::ARR;
      ws();
      if (p_ < e_ && *p_ == ']') {
        p_++;
        return true;
      }
      for (;;) {
        Json child;
        if (!value(child, depth + 1)) return false;
        v.arr.push_back(std::move(child));
        ws();
        if (p_ < e_ && *p_ == ',') {
          p_++;
          continue;
        }
        if (p_ < e_ && *p_ == ']') {
          p_++;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v.kind = Json::STR;
      return string(v.str);
    }
    if (lit("true")) {
      v.kind = Json::BOOL;
      v.b = true;
      return true;
    }
    if (lit("false")) {
      v.kind = Json::BOOL;
      return true;
    }
    if (lit("null")) return true;
    // number
    std::string num;
    while (p_ < e_ && (isdigit((unsigned char)*p_) || *p_ == '-' || *p_ == '+' || *p_ == '.' || *p_ == 'e' || *p_ == 'E'))
      num += *p_++;
    if (num.empty()) return fail("unexpected character in JSON");
    char* end = nullptr;
    v.num = strtod(num.c_str(), &end);
    if (!end || *end) return fail("bad number");
    v.kind = Json::NUM;
    return true;
  }
};

static bool read_file(const std::string& path, std::string& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  char buf[65536];
  size_t n;
  while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.append(buf, n);
  fclose(f);
  return true;
}

// f16 bit pattern -> f32, exact (normals, subnormals, infinities, NaN payload kept in the high mantissa bits).
static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400u));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

enum DType { F16, BF16, F32, U8, I8, OTHER };
static DType dtype_of(const std::string& s) {
  if (s == "F16") return F16;
  if (s == "BF16") return BF16;
  if (s == "F32") return F32;
  if (s == "U8") return U8;
  if (s == "I8") return I8;
  return OTHER;
}
static const char* dtype_name(DType d) {
  switch (d) {
    case F16: return "F16";
    case BF16: return "BF16";
    case F32: return "F32";
    case U8: return "U8";
    case I8: return "I8";
    default: return "other";
  }
}

struct Tensor {
  DType dtype = OTHER;
  std::vector<size_t> shape;
  const uint8_t* data = nullptr;
  size_t bytes = 0;
};

struct QModule {
  std::string name;
  int out = 0, in = 0, group = 0;
  bool has_bias = false;
};

}  // namespace model
}  // namespace vxg

using namespace vxg;
using namespace vxg::model;

struct vxg_model {
  std::string dir;
  // config.json (format.rs:13-41)
  int hidden = 0, ff = 0, n_layers = 0, heads = 0, n_mels = 0, conv_kernel = 0, sub_channels = 0, sub_kernel = 0;
  int sub_stride = 0, sub_factor = 0, blank = 0, dec_hidden = 0, dec_layers = 0, max_symbols = 0, vocab = 0;
  int group = 0;
  std::vector<int> durations;
  // ternary.json (format.rs:43-72)
  std::vector<QModule> qmodules;
  int vad_d_model = 0, vad_hidden = 0, vad_kernel = 0;
  double vad_frame_seconds = 0.0;
  // model.safetensors
  void* map = nullptr;
  size_t map_bytes = 0;
  std::map<std::string, Tensor> tensors;
  std::vector<std::unique_ptr<std::vector<float>>> owned;  // f16 tensors widened to f32

  ~vxg_model() {
    if (map) munmap(map, map_bytes);
  }
  const Tensor* find(const std::string& n) const {
    auto it = tensors.find(n);
    return it == tensors.end() ? nullptr : &it->second;
  }
  // load_f32 (tensor.rs:20-37): the tensor as f32 (F16 / BF16 widened exactly), checked against `shape`
  const float* f32(const std::string& n, const std::vector<size_t>& shape) {
    const Tensor* t = find(n);
    if (!t) {
      set_error("missing tensor %s", n.c_str());
      return nullptr;
    }
    if (t->shape != shape) {
      set_error("%s: unexpected shape", n.c_str());
      return nullptr;
    }
    if (t->dtype == F32) return reinterpret_cast<const float*>(t->data);
    if (t->dtype != F16 && t->dtype != BF16) {
      set_error("%s: expected a float tensor, got %s", n.c_str(), dtype_name(t->dtype));
      return nullptr;
    }
    size_t count = 1;
    for (size_t d : shape) count *= d;
    auto v = std::make_unique<std::vector<float>>(count);
    const uint16_t* h = reinterpret_cast<const uint16_t*>(t->data);
    for (size_t i = 0; i < count; i++) {
      if (t->dtype == F16) {
        (*v)[i] = f16_to_f32(h[i]);
      } else {
        const uint32_t bits = (uint32_t)h[i] << 16;
        memcpy(&(*v)[i], &bits, 4);
      }
    }
    owned.push_back(std::move(v));
    return owned.back()->data();
  }
  // load_f16_bits (tensor.rs:505-525)
  const uint16_t* f16(const std::string& n, const std::vector<size_t>& shape) {
    const Tensor* t = find(n);
    if (!t) {
      set_error("missing tensor %s", n.c_str());
      return nullptr;
    }
    if (t->dtype != F16 || t->shape != shape) {
      set_error("%s: expected F16 of the model's shape", n.c_str());
      return nullptr;
    }
    return reinterpret_cast<const uint16_t*>(t->data);
  }
  const QModule* qmodule(const std::string& n) const {
    for (const auto& m : qmodules)
      if (m.name == n) return &m;
    return nullptr;
  }
};

namespace {

bool num_field(const Json* o, const char* k, int& out, std::string& err) {
  const Json* v = o ? o->get(k) : nullptr;
  if (!v || v->kind != Json::NUM) {
    err = std::string("missing number field ") + k;
    return false;
  }
  out = (int)v->num;
  return true;
}

// validate (format.rs:153-309): every tensor the loaders read exists with the expected dtype and shape
std::vector<std::string> validate(const vxg_model* m) {
  std::vector<std::string> problems, extra;
  auto shape_str = [](const std::vector<size_t>& s) {
    std::string r = "[";
    for (size_t i = 0; i < s.size(); i++) r += (i ? ", " : "") + std::to_string(s[i]);
    return r + "]";
  };
  auto expect = [&](const std::string& name, DType dt, const std::vector<size_t>& shape) {
    const Tensor* t = m->find(name);
    if (!t) {
      problems.push_back("missing " + name);
    } else if (t->dtype != dt || t->shape != shape) {
      problems.push_back(name + ": got " + dtype_name(t->dtype) + " " + shape_str(t->shape) + ", expected " +
                         dtype_name(dt) + " " + shape_str(shape));
    }
  };
  const size_t d = m->hidden, h = m->dec_hidden;
  for (const auto& q : m->qmodules) {
    expect(q.name + ".qweight", U8, {(size_t)q.out, (size_t)(q.in + 4) / 5});
    expect(q.name + ".scales", F16, {(size_t)q.out, (size_t)(q.in / q.group)});
    if (q.has_bias) expect(q.name + ".bias", F32, {(size_t)q.out});
    if (m->find(q.name + ".weight")) extra.push_back(q.name + ".weight present alongside qweight");
  }
  const size_t ch = m->sub_channels, k = m->sub_kernel;
  const std::pair<int, std::vector<size_t>> sub[] = {
      {0, {ch, 1, k, k}}, {2, {ch, 1, k, k}}, {3, {ch, ch, 1, 1}}, {5, {ch, 1, k, k}}, {6, {ch, ch, 1, 1}}};
  for (const auto& s : sub) {
    expect("encoder.subsampling.layers." + std::to_string(s.first) + ".weight", F16, s.second);
    expect("encoder.subsampling.layers." + std::to_string(s.first) + ".bias", F32, {ch});
  }
  const size_t sub_out = m->n_mels / m->sub_factor;
  expect("encoder.subsampling.linear.weight", F16, {d, ch * sub_out});
  expect("encoder.subsampling.linear.bias", F32, {d});
  for (int i = 0; i < m->n_layers; i++) {
    const std::string p = "encoder.layers." + std::to_string(i);
    for (const char* n : {"norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out",
                          "conv.norm"}) {
      expect(p + "." + n + ".weight", F32, {d});
      expect(p + "." + n + ".bias", F32, {d});
    }
    expect(p + ".conv.norm.running_mean", F32, {d});
    expect(p + ".conv.norm.running_var", F32, {d});
    expect(p + ".conv.depthwise_conv.weight", F16, {d, 1, (size_t)m->conv_kernel});
    expect(p + ".self_attn.bias_u", F16, {(size_t)m->heads, d / m->heads});
    expect(p + ".self_attn.bias_v", F16, {(size_t)m->heads, d / m->heads});
  }
  expect("encoder_projector.weight", F16, {h, d});
  expect("encoder_projector.bias", F32, {h});
  expect("decoder.embedding.weight", F16, {(size_t)m->vocab, h});
  for (int l = 0; l < m->dec_layers; l++) {
    const std::string s = std::to_string(l);
    expect("decoder.lstm.weight_ih_l" + s, F16, {4 * h, h});
    expect("decoder.lstm.weight_hh_l" + s, F16, {4 * h, h});
    expect("decoder.lstm.bias_ih_l" + s, F32, {4 * h});
    expect("decoder.lstm.bias_hh_l" + s, F32, {4 * h});
  }
  expect("decoder.decoder_projector.weight", F16, {h, h});
  expect("decoder.decoder_projector.bias", F32, {h});
  const size_t n_out = m->vocab + m->durations.size();
  expect("joint.head.weight", F16, {n_out, h});
  expect("joint.head.bias", F32, {n_out});
  const size_t vh = m->vad_hidden;
  expect("vad_head.proj.weight", F16, {vh, (size_t)m->vad_d_model, 1});
  expect("vad_head.proj.bias", F16, {vh});
  expect("vad_head.ctx.weight", F16, {vh, vh, (size_t)m->vad_kernel});
  expect("vad_head.ctx.bias", F16, {vh});
  expect("vad_head.out.weight", F16, {1, vh, 1});
  expect("vad_head.out.bias", F16, {1});
  problems.insert(problems.end(), extra.begin(), extra.end());
  return problems;
}

vxg_status open_model(const char* dir_c, vxg_model** out) {
  VXG_ARG(dir_c && out, "NULL argument");
  *out = nullptr;
  std::unique_ptr<vxg_model> m(new vxg_model());
  m->dir = dir_c;
  std::string text, err;
  Json cfg, tern;
  if (!read_file(m->dir + "/config.json", text)) {
    set_error("cannot read %s/config.json", dir_c);
    return VXG_ERR_ARG;
  }
  if (!JsonParser(text.data(), text.size()).parse(cfg, err)) {
    set_error("config.json: %s", err.c_str());
    return VXG_ERR_ARG;
  }
  text.clear();
  if (!read_file(m->dir + "/ternary.json", text)) {
    set_error("cannot read %s/ternary.json", dir_c);
    return VXG_ERR_ARG;
  }
  if (!JsonParser(text.data(), text.size()).parse(tern, err)) {
    set_error("ternary.json: %s", err.c_str());
    return VXG_ERR_ARG;
  }
  // ModelFile::open (format.rs:88-118): the format and naming must be the ones the loaders understand
  const Json* fmt = tern.get("format");
  if (!fmt || fmt->kind != Json::STR || fmt->str != "thrush-ternary-v2") {
    set_error("unsupported format %s, expected thrush-ternary-v2",
              fmt && fmt->kind == Json::STR ? fmt->str.c_str() : "(none)");
    return VXG_ERR_ARG;
  }
  const Json* names = tern.get("names");
  if (!names || names->kind != Json::STR || names->str != "hf") {
    set_error("unsupported tensor naming %s", names && names->kind == Json::STR ? names->str.c_str() : "(none)");
    return VXG_ERR_ARG;
  }
  const Json* ec = cfg.get("encoder_config");
  bool ok = num_field(ec, "hidden_size", m->hidden, err) && num_field(ec, "intermediate_size", m->ff, err) &&
            num_field(ec, "num_hidden_layers", m->n_layers, err) &&
            num_field(ec, "num_attention_heads", m->heads, err) && num_field(ec, "num_mel_bins", m->n_mels, err) &&
            num_field(ec, "conv_kernel_size", m->conv_kernel, err) &&
            num_field(ec, "subsampling_conv_channels", m->sub_channels, err) &&
            num_field(ec, "subsampling_conv_kernel_size", m->sub_kernel, err) &&
            num_field(ec, "subsampling_conv_stride", m->sub_stride, err) &&
            num_field(ec, "subsampling_factor", m->sub_factor, err) &&
            num_field(&cfg, "blank_token_id", m->blank, err) &&
            num_field(&cfg, "decoder_hidden_size", m->dec_hidden, err) &&
            num_field(&cfg, "num_decoder_layers", m->dec_layers, err) &&
            num_field(&cfg, "max_symbols_per_step", m->max_symbols, err) &&
            num_field(&cfg, "vocab_size", m->vocab, err) && num_field(&cfg, "ternary_group_size", m->group, err);
  if (!ok) {
    set_error("config.json: %s", err.c_str());
    return VXG_ERR_ARG;
  }
  const Json* durs = cfg.get("durations");
  if (!durs || durs->kind != Json::ARR) {
    set_error("config.json: missing durations");
    return VXG_ERR_ARG;
  }
  for (const auto& v : durs->arr) m->durations.push_back((int)v.num);
  const Json* qm = tern.get("quantized_modules");
  if (!qm || qm->kind != Json::ARR) {
    set_error("ternary.json: missing quantized_modules");
    return VXG_ERR_ARG;
  }
  for (const auto& e : qm->arr) {
    QModule q;
    const Json* n = e.get("name");
    const Json* hb = e.get("has_bias");
    if (!n || n->kind != Json::STR || !num_field(&e, "out_features", q.out, err) ||
        !num_field(&e, "in_features", q.in, err) || !num_field(&e, "group_size", q.group, err) || q.group <= 0) {
      set_error("ternary.json: bad quantized module entry");
      return VXG_ERR_ARG;
    }
    q.name = n->str;
    q.has_bias = hb && hb->kind == Json::BOOL && hb->b;
    m->qmodules.push_back(q);
  }
  const Json* vad = tern.get("vad_head");
  if (!num_field(vad, "d_model", m->vad_d_model, err) || !num_field(vad, "hidden", m->vad_hidden, err) ||
      !num_field(vad, "kernel", m->vad_kernel, err)) {
    set_error("ternary.json: vad_head: %s", err.c_str());
    return VXG_ERR_ARG;
  }
  const Json* fs = vad->get("frame_seconds");
  m->vad_frame_seconds = fs && fs->kind == Json::NUM ? fs->num : 0.0;
  // model.safetensors: u64 header length, JSON header {name: {dtype, shape, data_offsets}}, then the data
  const std::string st = m->dir + "/model.safetensors";
  const int fd = open(st.c_str(), O_RDONLY);
  if (fd < 0) {
    set_error("cannot open %s", st.c_str());
    return VXG_ERR_ARG;
  }
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size < 8) {
    close(fd);
    set_error("%s: too short", st.c_str());
    return VXG_ERR_ARG;
  }
  m->map_bytes = (size_t)sb.st_size;
  m->map = mmap(nullptr, m->map_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m->map == MAP_FAILED) {
    m->map = nullptr;
    set_error("cannot map %s", st.c_str());
    return VXG_ERR_ARG;
  }
  const uint8_t* base = static_cast<const uint8_t*>(m->map);
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | base[i];
  if (hlen > m->map_bytes - 8) {
    set_error("%s: header length %llu past the end of the file", st.c_str(), (unsigned long long)hlen);
    return VXG_ERR_ARG;
  }
  Json hdr;
  if (!JsonParser(reinterpret_cast<const char*>(base + 8), hlen).parse(hdr, err) || hdr.kind != Json::OBJ) {
    set_error("%s: header: %s", st.c_str(), err.empty() ? "not an object" : err.c_str());
    return VXG_ERR_ARG;
  }
  const uint8_t* data = base + 8 + hlen;
  const size_t data_bytes = m->map_bytes - 8 - hlen;
  for (const auto& kv : hdr.obj) {
    if (kv.first == "__metadata__") continue;
    const Json* dt = kv.second.get("dtype");
    const Json* sh = kv.second.get("shape");
    const Json* off = kv.second.get("data_offsets");
    if (!dt || dt->kind != Json::STR || !sh || sh->kind != Json::ARR || !off || off->kind != Json::ARR ||
        off->arr.size() != 2) {
      set_error("%s: bad header entry %s", st.c_str(), kv.first.c_str());
      return VXG_ERR_ARG;
    }
    Tensor t;
    t.dtype = dtype_of(dt->str);
    size_t count = 1;
    for (const auto& v : sh->arr) {
      t.shape.push_back((size_t)v.num);
      count *= (size_t)v.num;
    }
    const size_t b0 = (size_t)off->arr[0].num, b1 = (size_t)off->arr[1].num;
    const size_t esz = (t.dtype == F32) ? 4 : (t.dtype == F16 || t.dtype == BF16) ? 2 : 1;
    if (b1 < b0 || b1 > data_bytes || (t.dtype != OTHER && b1 - b0 != count * esz)) {
      set_error("%s: tensor %s: data offsets do not match its shape", st.c_str(), kv.first.c_str());
      return VXG_ERR_ARG;
    }
    t.data = data + b0;
    t.bytes = b1 - b0;
    m->tensors[kv.first] = t;
  }
  *out = m.release();
  return VXG_OK;
}

}  // namespace

extern "C" {

vxg_status vxg_model_open(const char* dir, vxg_model** out) {
  clear_error();
  try {
    return open_model(dir, out);
  } catch (const std::exception& e) {
    set_error("model open: %s", e.what());
    return VXG_ERR_ARG;
  }
}

void vxg_model_close(vxg_model* m) { delete m; }

int vxg_model_validate(const vxg_model* m, char* buf, size_t cap) {
  clear_error();
  if (!m) return -1;
  const std::vector<std::string> p = validate(m);
  std::string all;
  for (const auto& s : p) all += s + "\n";
  if (buf && cap) {
    const size_t n = std::min(cap - 1, all.size());
    memcpy(buf, all.data(), n);
    buf[n] = 0;
  }
  return (int)p.size();
}

vxg_status vxg_model_config(const vxg_model* m, vxg_model_cfg* c) {
  clear_error();
  VXG_ARG(m && c, "NULL argument");
  c->d_model = m->hidden;
  c->ff = m->ff;
  c->n_layers = m->n_layers;
  c->heads = m->heads;
  c->n_mels = m->n_mels;
  c->conv_kernel = m->conv_kernel;
  c->sub_channels = m->sub_channels;
  c->group = m->group;
  c->dec_hidden = m->dec_hidden;
  c->dec_layers = m->dec_layers;
  c->vocab = m->vocab;
  c->blank = m->blank;
  c->max_symbols = m->max_symbols;
  c->n_durations = (int)m->durations.size();
  c->vad_hidden = m->vad_hidden;
  c->vad_kernel = m->vad_kernel;
  c->vad_frame_seconds = m->vad_frame_seconds;
  return VXG_OK;
}

vxg_status vxg_model_tensor(const vxg_model* m, const char* name, int* dtype, int64_t* shape, int* ndim,
                            const void** data, size_t* bytes) {
  clear_error();
  VXG_ARG(m && name && dtype && shape && ndim && data && bytes, "NULL argument");
  const Tensor* t = m->find(name);
  if (!t) {
    set_error("missing tensor %s", name);
    return VXG_ERR_ARG;
  }
  *dtype = (int)t->dtype;
  *ndim = (int)std::min<size_t>(t->shape.size(), 8);
  for (int i = 0; i < *ndim; i++) shape[i] = (int64_t)t->shape[i];
  *data = t->data;
  *bytes = t->bytes;
  return VXG_OK;
}

vxg_status vxg_model_tensor_f32(vxg_model* m, const char* name, float* out, size_t count) {
  clear_error();
  VXG_ARG(m && name && out, "NULL argument");
  const Tensor* t = m->find(name);
  if (!t) {
    set_error("missing tensor %s", name);
    return VXG_ERR_ARG;
  }
  size_t n = 1;
  for (size_t d : t->shape) n *= d;
  VXG_ARG(count == n, "%s holds %zu elements, not %zu", name, n, count);
  const float* f = m->f32(name, t->shape);
  if (!f) return VXG_ERR_ARG;
  memcpy(out, f, n * sizeof(float));
  if (t->dtype != F32) m->owned.pop_back();  // the widened copy was made for this call only
  return VXG_OK;
}

vxg_status vxg_encoder_create_from_model(vxg_model* m, int weight_format, int device, vxg_encoder** out) {
  clear_error();
  VXG_ARG(m && out, "NULL argument");
  const std::vector<std::string> problems = validate(m);
  if (!problems.empty()) {
    set_error("model %s does not validate (%zu problems), first: %s", m->dir.c_str(), problems.size(),
              problems[0].c_str());
    return VXG_ERR_ARG;
  }
  const size_t d = m->hidden, ch = m->sub_channels, k = m->sub_kernel;
  std::vector<vxg_layer_weights> L(m->n_layers);
  auto tern = [&](const std::string& name, vxg_ternary_tensor& t) -> bool {
    const QModule* q = m->qmodule(name);
    const Tensor* qw = m->find(name + ".qweight");
    const Tensor* sc = m->find(name + ".scales");
    if (!q || !qw || !sc) {
      set_error("ternary module %s missing", name.c_str());
      return false;
    }
    t.qweight = qw->data;
    t.scales = reinterpret_cast<const uint16_t*>(sc->data);
    t.out = q->out;
    t.in = q->in;
    t.group = q->group;
    return true;
  };
  auto vec = [&](const std::string& n, const std::vector<size_t>& s, const float*& dst) -> bool {
    dst = m->f32(n, s);
    return dst != nullptr;
  };
  for (int i = 0; i < m->n_layers; i++) {
    const std::string p = "encoder.layers." + std::to_string(i);
    vxg_layer_weights& w = L[i];
    const bool ok =
        tern(p + ".feed_forward1.linear1", w.ff1_linear1) && tern(p + ".feed_forward1.linear2", w.ff1_linear2) &&
        tern(p + ".self_attn.q_proj", w.q_proj) && tern(p + ".self_attn.k_proj", w.k_proj) &&
        tern(p + ".self_attn.v_proj", w.v_proj) && tern(p + ".self_attn.o_proj", w.o_proj) &&
        tern(p + ".self_attn.relative_k_proj", w.relative_k_proj) &&
        tern(p + ".conv.pointwise_conv1", w.pointwise_conv1) && tern(p + ".conv.pointwise_conv2", w.pointwise_conv2) &&
        tern(p + ".feed_forward2.linear1", w.ff2_linear1) && tern(p + ".feed_forward2.linear2", w.ff2_linear2) &&
        vec(p + ".norm_feed_forward1.weight", {d}, w.norm_ff1_w) && vec(p + ".norm_feed_forward1.bias", {d}, w.norm_ff1_b) &&
        vec(p + ".norm_self_att.weight", {d}, w.norm_attn_w) && vec(p + ".norm_self_att.bias", {d}, w.norm_attn_b) &&
        vec(p + ".norm_conv.weight", {d}, w.norm_conv_w) && vec(p + ".norm_conv.bias", {d}, w.norm_conv_b) &&
        vec(p + ".norm_feed_forward2.weight", {d}, w.norm_ff2_w) && vec(p + ".norm_feed_forward2.bias", {d}, w.norm_ff2_b) &&
        vec(p + ".norm_out.weight", {d}, w.norm_out_w) && vec(p + ".norm_out.bias", {d}, w.norm_out_b) &&
        vec(p + ".self_attn.bias_u", {(size_t)m->heads, d / m->heads}, w.bias_u) &&
        vec(p + ".self_attn.bias_v", {(size_t)m->heads, d / m->heads}, w.bias_v) &&
        vec(p + ".conv.depthwise_conv.weight", {d, 1, (size_t)m->conv_kernel}, w.dw_weight) &&
        vec(p + ".conv.norm.weight", {d}, w.bn_weight) && vec(p + ".conv.norm.bias", {d}, w.bn_bias) &&
        vec(p + ".conv.norm.running_mean", {d}, w.bn_mean) && vec(p + ".conv.norm.running_var", {d}, w.bn_var);
    if (!ok) return VXG_ERR_ARG;
  }
  vxg_subsampling_weights S;
  const std::string sp = "encoder.subsampling.";
  const bool sok = vec(sp + "layers.0.weight", {ch, 1, k, k}, S.conv0_w) && vec(sp + "layers.0.bias", {ch}, S.conv0_b) &&
                   vec(sp + "layers.2.weight", {ch, 1, k, k}, S.dw1_w) && vec(sp + "layers.2.bias", {ch}, S.dw1_b) &&
                   vec(sp + "layers.3.weight", {ch, ch, 1, 1}, S.pw1_w) && vec(sp + "layers.3.bias", {ch}, S.pw1_b) &&
                   vec(sp + "layers.5.weight", {ch, 1, k, k}, S.dw2_w) && vec(sp + "layers.5.bias", {ch}, S.dw2_b) &&
                   vec(sp + "layers.6.weight", {ch, ch, 1, 1}, S.pw2_w) && vec(sp + "layers.6.bias", {ch}, S.pw2_b) &&
                   vec(sp + "linear.weight", {d, ch * (size_t)(m->n_mels / m->sub_factor)}, S.lin_w) &&
                   vec(sp + "linear.bias", {d}, S.lin_b);
  if (!sok) return VXG_ERR_ARG;
  vxg_encoder_desc desc;
  desc.d_model = m->hidden;
  desc.ff = m->ff;
  desc.heads = m->heads;
  desc.conv_kernel = m->conv_kernel;
  desc.n_layers = m->n_layers;
  desc.n_mels = m->n_mels;
  desc.sub_channels = m->sub_channels;
  desc.weight_format = weight_format;
  desc.layers = L.data();
  desc.sub = &S;
  return vxg_encoder_create(&desc, device, out);
}

vxg_status vxg_tdt_create_from_model(vxg_model* m, int device, vxg_tdt** out) {
  clear_error();
  VXG_ARG(m && out, "NULL argument");
  VXG_ARG(m->dec_layers >= 1 && m->dec_layers <= 4, "decoder with %d LSTM layers unsupported", m->dec_layers);
  const size_t h = m->dec_hidden, d = m->hidden, n_out = m->vocab + m->durations.size();
  vxg_tdt_desc t;
  memset(&t, 0, sizeof t);
  t.hidden = m->dec_hidden;
  t.vocab = m->vocab;
  t.n_durations = (int)m->durations.size();
  t.blank = m->blank;
  t.max_symbols = m->max_symbols;
  t.d_model = m->hidden;
  t.n_layers = m->dec_layers;
  t.durations = m->durations.data();
  t.device = device;
  bool ok = (t.embedding = m->f32("decoder.embedding.weight", {(size_t)m->vocab, h})) != nullptr;
  for (int l = 0; ok && l < m->dec_layers; l++) {
    const std::string s = std::to_string(l);
    ok = (t.w_ih[l] = m->f16("decoder.lstm.weight_ih_l" + s, {4 * h, h})) != nullptr &&
         (t.w_hh[l] = m->f16("decoder.lstm.weight_hh_l" + s, {4 * h, h})) != nullptr &&
         (t.b_ih[l] = m->f32("decoder.lstm.bias_ih_l" + s, {4 * h})) != nullptr &&
         (t.b_hh[l] = m->f32("decoder.lstm.bias_hh_l" + s, {4 * h})) != nullptr;
  }
  ok = ok && (t.proj_w = m->f16("decoder.decoder_projector.weight", {h, h})) != nullptr &&
       (t.proj_b = m->f32("decoder.decoder_projector.bias", {h})) != nullptr &&
       (t.head_w = m->f16("joint.head.weight", {n_out, h})) != nullptr &&
       (t.head_b = m->f32("joint.head.bias", {n_out})) != nullptr &&
       (t.enc_w = m->f32("encoder_projector.weight", {h, d})) != nullptr &&
       (t.enc_b = m->f32("encoder_projector.bias", {h})) != nullptr;
  if (!ok) return VXG_ERR_ARG;
  return vxg_tdt_create(&t, out);
}

vxg_status vxg_vad_create_from_model(vxg_model* m, int device, vxg_vad** out) {  // VadHead::load (vad.rs:21-36)
  clear_error();
  VXG_ARG(m && out, "NULL argument");
  const size_t h = m->vad_hidden, d = m->vad_d_model, k = m->vad_kernel;
  VXG_ARG(h > 0 && d > 0 && k > 0, "model has no VAD head");
  vxg_vad_desc v;
  memset(&v, 0, sizeof v);
  v.d_model = (int)d;
  v.hidden = (int)h;
  v.kernel = (int)k;
  v.frame_seconds = m->vad_frame_seconds;
  v.device = device;
  const float* ob = nullptr;
  const bool ok = (v.proj_w = m->f32("vad_head.proj.weight", {h, d, 1})) != nullptr &&
                  (v.proj_b = m->f32("vad_head.proj.bias", {h})) != nullptr &&
                  (v.ctx_w = m->f32("vad_head.ctx.weight", {h, h, k})) != nullptr &&
                  (v.ctx_b = m->f32("vad_head.ctx.bias", {h})) != nullptr &&
                  (v.out_w = m->f32("vad_head.out.weight", {1, h, 1})) != nullptr &&
                  (ob = m->f32("vad_head.out.bias", {1})) != nullptr;
  if (!ok) return VXG_ERR_ARG;
  v.out_b = ob[0];
  return vxg_vad_create(&v, out);
}

}  // extern "C"
