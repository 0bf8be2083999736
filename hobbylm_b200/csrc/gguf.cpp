// GGUF v3 reader, dequantizers, Config::from_gguf and the load-time Q8 re-quantization.
//
// Follows hobby-rs/src/gguf.rs (header parse 166-212, alignment 202-208, F32 view 215-235, typed
// load 250-269, half_to_f32 329-341, type sizes 349-359, Q8_0/F16/Q5_0/Q4_K/Q6_K dequant 361-468),
// hobby-rs/src/config.rs:35-98 (keys and defaults) and hobby-rs/src/quant.rs:78-102 (per-32 block
// re-quantization with f32 scales, round half away from zero, clamp to +-127).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>

#include "hg_host.h"

namespace hg {

namespace {

struct Reader {
  const uint8_t* b;
  size_t n, p;
  const uint8_t* take(size_t k) {
    if (k > n - p) throw Error(HG_ERR_FORMAT, "GGUF: unexpected end of file");
    const uint8_t* r = b + p;
    p += k;
    return r;
  }
  template <class T>
  T get() {
    T v;
    std::memcpy(&v, take(sizeof(T)), sizeof(T));
    return v;
  }
  std::string str() {
    uint64_t k = get<uint64_t>();
    const uint8_t* s = take(k);
    return std::string(reinterpret_cast<const char*>(s), k);
  }
};

GgufMeta read_scalar(Reader& r, uint32_t ty) {
  GgufMeta m;
  switch (ty) {
    case 0: m.kind = GgufMeta::U32; m.u = r.get<uint8_t>(); break;
    case 1: m.kind = GgufMeta::I32; m.i = (int8_t)r.get<uint8_t>(); break;
    case 2: m.kind = GgufMeta::U32; m.u = r.get<uint16_t>(); break;
    case 3: m.kind = GgufMeta::I32; m.i = r.get<int16_t>(); break;
    case 4: m.kind = GgufMeta::U32; m.u = r.get<uint32_t>(); break;
    case 5: m.kind = GgufMeta::I32; m.i = r.get<int32_t>(); break;
    case 6: m.kind = GgufMeta::F32; m.f = r.get<float>(); break;
    case 7: m.kind = GgufMeta::BOOL; m.u = r.get<uint8_t>() != 0; break;
    case 8: m.kind = GgufMeta::STR; m.s = r.str(); break;
    case 10: m.kind = GgufMeta::U64; m.u = r.get<uint64_t>(); break;
    case 11: m.kind = GgufMeta::I32; m.i = (int32_t)r.get<uint64_t>(); break;  // gguf.rs:121
    case 12: m.kind = GgufMeta::F32; m.f = (float)r.get<double>(); break;
    default: throw Error(HG_ERR_FORMAT, "GGUF: unsupported metadata scalar type " + std::to_string(ty));
  }
  return m;
}

GgufMeta read_value(Reader& r, uint32_t ty) {
  if (ty != 9) return read_scalar(r, ty);
  uint32_t at = r.get<uint32_t>();
  uint64_t n = r.get<uint64_t>();
  GgufMeta m;
  m.arr_len = n;
  if (at == 8) {
    m.kind = GgufMeta::ARR_STR;
    for (uint64_t i = 0; i < n; i++) r.str();
  } else if (at == 4 || at == 5 || at == 6) {
    m.kind = at == 6 ? GgufMeta::ARR_F32 : GgufMeta::ARR_I32;
    if (n > r.n) throw Error(HG_ERR_FORMAT, "GGUF: unexpected end of file");
    r.take(n * 4);
  } else {
    for (uint64_t i = 0; i < n; i++) read_scalar(r, at);
    m.kind = GgufMeta::OTHER;
  }
  return m;
}

inline float half_to_f32(uint16_t h) {  // gguf.rs:329-341
  int sign = (h >> 15) & 1, ex = (h >> 10) & 0x1f;
  float mant = (float)(h & 0x3ff), v;
  if (ex == 0) v = mant * std::ldexp(1.0f, -24);
  else if (ex == 0x1f) v = (h & 0x3ff) ? NAN : INFINITY;
  else v = (1.0f + mant / 1024.0f) * std::ldexp(1.0f, ex - 15);
  return sign ? -v : v;
}
inline float half_at(const uint8_t* b) {
  uint16_t h;
  std::memcpy(&h, b, 2);
  return half_to_f32(h);
}

}  // namespace

uint64_t GgufTensor::n_elems() const {
  uint64_t n = 1;
  for (uint64_t v : ne) n *= v;
  return n;
}

Gguf::Gguf(const char* path) {
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) throw Error(HG_ERR_IO, std::string("opening ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    throw Error(HG_ERR_IO, std::string("stat ") + path);
  }
  size_ = (size_t)st.st_size;
  if (size_ == 0) {
    ::close(fd);
    throw Error(HG_ERR_FORMAT, "GGUF: unexpected end of file");
  }
  void* p = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (p == MAP_FAILED) throw Error(HG_ERR_IO, std::string("mmap ") + path);
  map_ = static_cast<const uint8_t*>(p);
  try {
    Reader r{map_, size_, 0};
    if (r.get<uint32_t>() != 0x46554747u) throw Error(HG_ERR_FORMAT, "not a GGUF file (bad magic)");
    uint32_t version = r.get<uint32_t>();
    if (version != 3)
      throw Error(HG_ERR_FORMAT, "unsupported GGUF version " + std::to_string(version) + " (expected 3)");
    uint64_t n_tensors = r.get<uint64_t>(), n_meta = r.get<uint64_t>();
    for (uint64_t i = 0; i < n_meta; i++) {
      std::string key = r.str();
      uint32_t ty = r.get<uint32_t>();
      meta_[key] = read_value(r, ty);
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
      std::string name = r.str();
      uint32_t nd = r.get<uint32_t>();
      if (nd > 8) throw Error(HG_ERR_FORMAT, "GGUF: tensor `" + name + "` has too many dims");
      GgufTensor t;
      for (uint32_t k = 0; k < nd; k++) t.ne.push_back(r.get<uint64_t>());
      t.type = r.get<uint32_t>();
      t.offset = r.get<uint64_t>();
      tensors_[name] = t;
    }
    size_t align = 32;
    auto it = meta_.find("general.alignment");
    if (it != meta_.end() && it->second.kind == GgufMeta::U32 && it->second.u > 0) align = it->second.u;
    data_start_ = (r.p + align - 1) / align * align;
  } catch (...) {
    munmap((void*)map_, size_);
    map_ = nullptr;
    throw;
  }
}

Gguf::~Gguf() {
  if (map_) munmap((void*)map_, size_);
}

const GgufTensor* Gguf::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}

const uint8_t* Gguf::raw(const std::string& name, size_t* nbytes) const {
  const GgufTensor* t = tensor(name);
  if (!t) throw Error(HG_ERR_MISSING, "tensor `" + name + "` not found");
  size_t nb = ggml_type_nbytes(t->type, t->n_elems());
  size_t off = data_start_ + t->offset;
  if (off > size_ || nb > size_ - off) throw Error(HG_ERR_FORMAT, "tensor `" + name + "` extends past end of file");
  *nbytes = nb;
  return map_ + off;
}

std::vector<float> Gguf::f32(const std::string& name) const {
  const GgufTensor* t = tensor(name);
  if (!t) throw Error(HG_ERR_MISSING, "tensor `" + name + "` not found in GGUF");
  if (t->type != 0)
    throw Error(HG_ERR_FORMAT, "tensor `" + name + "` is ggml_type " + std::to_string(t->type) +
                                   " (expected F32=0)");
  size_t nb;
  const uint8_t* b = raw(name, &nb);
  std::vector<float> v(t->n_elems());
  std::memcpy(v.data(), b, nb);
  return v;
}

std::vector<float> Gguf::load(const std::string& name) const {
  const GgufTensor* t = tensor(name);
  if (!t) throw Error(HG_ERR_MISSING, "tensor `" + name + "` not found");
  size_t nb;
  const uint8_t* b = raw(name, &nb);
  std::vector<float> v(t->n_elems());
  if (t->type == 0) std::memcpy(v.data(), b, nb);
  else ggml_dequant(t->type, b, v.size(), v.data());
  return v;
}

bool Gguf::get_u32(const std::string& k, uint32_t* out) const {  // gguf.rs:272-279
  auto it = meta_.find(k);
  if (it == meta_.end()) return false;
  const GgufMeta& m = it->second;
  if (m.kind == GgufMeta::U32 || m.kind == GgufMeta::U64) *out = (uint32_t)m.u;
  else if (m.kind == GgufMeta::I32) *out = (uint32_t)m.i;
  else return false;
  return true;
}
bool Gguf::get_f32(const std::string& k, float* out) const {  // gguf.rs:280-286
  auto it = meta_.find(k);
  if (it == meta_.end()) return false;
  const GgufMeta& m = it->second;
  if (m.kind == GgufMeta::F32) *out = m.f;
  else if (m.kind == GgufMeta::U32) *out = (float)(uint32_t)m.u;
  else return false;
  return true;
}
bool Gguf::get_bool(const std::string& k, bool* out) const {
  auto it = meta_.find(k);
  if (it == meta_.end() || it->second.kind != GgufMeta::BOOL) return false;
  *out = it->second.u != 0;
  return true;
}
bool Gguf::get_str(const std::string& k, std::string* out) const {
  auto it = meta_.find(k);
  if (it == meta_.end() || it->second.kind != GgufMeta::STR) return false;
  *out = it->second.s;
  return true;
}
bool Gguf::has_str_array(const std::string& k) const {
  auto it = meta_.find(k);
  return it != meta_.end() && it->second.kind == GgufMeta::ARR_STR;
}

size_t ggml_type_nbytes(uint32_t type, size_t n) {  // gguf.rs:349-359
  switch (type) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 6: return (n / 32) * 22;
    case 8: return (n / 32) * 34;
    case 12: return (n / 256) * 144;
    case 14: return (n / 256) * 210;
    default: throw Error(HG_ERR_FORMAT, "unsupported ggml_type " + std::to_string(type));
  }
}

void ggml_dequant(uint32_t type, const uint8_t* b, size_t n, float* y) {
  switch (type) {
    case 1:  // F16
      for (size_t i = 0; i < n; i++) y[i] = half_at(b + 2 * i);
      return;
    case 8:  // Q8_0: {f16 d, 32 x i8} -> q * d (gguf.rs:365-375)
#pragma omp parallel for schedule(static)
      for (int64_t blk = 0; blk < (int64_t)(n / 32); blk++) {
        const uint8_t* p = b + blk * 34;
        float d = half_at(p);
        for (int j = 0; j < 32; j++) y[blk * 32 + j] = (float)(int8_t)p[2 + j] * d;
      }
      return;
    case 6:  // Q5_0 (gguf.rs:377-395)
      for (size_t blk = 0; blk < n / 32; blk++) {
        const uint8_t* p = b + blk * 22;
        float d = half_at(p);
        uint32_t qh;
        std::memcpy(&qh, p + 2, 4);
        const uint8_t* qs = p + 6;
        for (int j = 0; j < 16; j++) {
          uint8_t h0 = (uint8_t)(((qh >> j) << 4) & 0x10), h1 = (uint8_t)((qh >> (j + 12)) & 0x10);
          y[blk * 32 + j] = (float)((int)((qs[j] & 0x0F) | h0) - 16) * d;
          y[blk * 32 + 16 + j] = (float)((int)((qs[j] >> 4) | h1) - 16) * d;
        }
      }
      return;
    case 12: {  // Q4_K (gguf.rs:397-437)
      auto sm = [](int j, const uint8_t* sc, uint8_t* d, uint8_t* m) {
        if (j < 4) {
          *d = sc[j] & 63;
          *m = sc[j + 4] & 63;
        } else {
          *d = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
          *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
        }
      };
      size_t yi = 0;
      for (size_t blk = 0; blk < n / 256; blk++) {
        const uint8_t* p = b + blk * 144;
        float d = half_at(p), dmin = half_at(p + 2);
        const uint8_t *scales = p + 4, *qs = p + 16;
        for (int r = 0, is = 0; r < 4; r++, is += 2, qs += 32) {
          uint8_t s1, m1, s2, m2;
          sm(is, scales, &s1, &m1);
          sm(is + 1, scales, &s2, &m2);
          float d1 = d * (float)s1, mm1 = dmin * (float)m1, d2 = d * (float)s2, mm2 = dmin * (float)m2;
          for (int l = 0; l < 32; l++) y[yi++] = d1 * (float)(qs[l] & 0xF) - mm1;
          for (int l = 0; l < 32; l++) y[yi++] = d2 * (float)(qs[l] >> 4) - mm2;
        }
      }
      return;
    }
    case 14:  // Q6_K (gguf.rs:439-468)
      for (size_t blk = 0; blk < n / 256; blk++) {
        const uint8_t* p = b + blk * 210;
        const uint8_t *ql = p, *qh = p + 128, *sc = p + 192;
        float d = half_at(p + 208);
        for (int half = 0; half < 2; half++) {
          float* yb = y + blk * 256 + half * 128;
          int qlb = half * 64, qhb = half * 32, scb = half * 8;
          for (int l = 0; l < 32; l++) {
            int is = l / 16;
            int q1 = (int)((ql[qlb + l] & 0xF) | (((qh[qhb + l] >> 0) & 3) << 4)) - 32;
            int q2 = (int)((ql[qlb + l + 32] & 0xF) | (((qh[qhb + l] >> 2) & 3) << 4)) - 32;
            int q3 = (int)((ql[qlb + l] >> 4) | (((qh[qhb + l] >> 4) & 3) << 4)) - 32;
            int q4 = (int)((ql[qlb + l + 32] >> 4) | (((qh[qhb + l] >> 6) & 3) << 4)) - 32;
            auto s = [&](int k) { return (float)(int8_t)sc[scb + is + k]; };
            yb[l] = d * s(0) * (float)q1;
            yb[l + 32] = d * s(2) * (float)q2;
            yb[l + 64] = d * s(4) * (float)q3;
            yb[l + 96] = d * s(6) * (float)q4;
          }
        }
      }
      return;
    default: throw Error(HG_ERR_FORMAT, "unsupported ggml_type " + std::to_string(type));
  }
}

hg_config config_from_gguf(const Gguf& g) {  // config.rs:35-98
  hg_config c{};
  std::string arch;
  if (!g.get_str("general.architecture", &arch)) throw Error(HG_ERR_MISSING, "missing general.architecture");
  auto key = [&](const char* s) { return arch + "." + s; };
  auto req = [&](const char* s) -> int32_t {
    uint32_t v;
    if (!g.get_u32(key(s), &v)) throw Error(HG_ERR_MISSING, "missing metadata `" + arch + "." + s + "`");
    return (int32_t)v;
  };
  auto opt = [&](const char* s, int32_t dflt) -> int32_t {
    uint32_t v;
    return g.get_u32(key(s), &v) ? (int32_t)v : dflt;
  };
  uint32_t v;
  if (g.get_u32(key("attention.key_length"), &v)) {
    c.head_dim = (int32_t)v;
  } else {
    uint32_t d = 0, h = 1;
    g.get_u32(key("embedding_length"), &d);
    g.get_u32(key("attention.head_count"), &h);
    c.head_dim = (int32_t)(d / std::max<uint32_t>(h, 1));
  }
  const GgufTensor* te = g.tensor("token_embd.weight");
  if (te && te->ne.size() > 1) c.vocab_size = (int32_t)te->ne[1];
  else if (g.get_u32(key("vocab_size"), &v)) c.vocab_size = (int32_t)v;
  else throw Error(HG_ERR_MISSING, "cannot determine vocab_size");
  c.gating_sigmoid = 1;
  if (g.get_u32(key("expert_gating_func"), &v) && v == 1) c.gating_sigmoid = 0;
  c.d_model = req("embedding_length");
  c.n_layers = req("block_count");
  c.n_dense = opt("leading_dense_block_count", 1);
  c.n_heads = req("attention.head_count");
  c.n_kv_heads = req("attention.head_count_kv");
  c.dense_ffn = req("feed_forward_length");
  c.expert_ffn = req("expert_feed_forward_length");
  c.n_experts = req("expert_count");
  c.top_k = req("expert_used_count");
  c.n_shared = opt("expert_shared_count", 0);
  c.context_length = opt("context_length", 8192);
  float f;
  c.rms_eps = g.get_f32(key("attention.layer_norm_rms_epsilon"), &f) ? f : 1e-5f;
  c.rope_theta = g.get_f32(key("rope.freq_base"), &f) ? f : 1e6f;
  c.expert_weights_scale = g.get_f32(key("expert_weights_scale"), &f) ? f : 1.0f;
  bool b;
  c.expert_weights_norm = g.get_bool(key("expert_weights_norm"), &b) ? (int32_t)b : 0;
  c.eos_token = 50256;
  if (g.get_u32("tokenizer.ggml.eos_token_id", &v)) c.eos_token = (int32_t)v;
  c.diffusion = g.get_bool("diffusion.enabled", &b) ? (int32_t)b : 0;
  c.mask_token_id = g.get_u32("diffusion.mask_token_id", &v) ? (int32_t)v : 50257;
  c.block_size = g.get_u32("diffusion.block_size", &v) ? (int32_t)v : 32;
  return c;
}

int host_q8_ss(int64_t cols) { return (int)(((cols / 32) + 3) & ~3LL); }

static inline int host_q8_pos(int k, int nb) {
  int b = k >> 5, j = k & 31, l = j >> 2, bj = j & 3, nc = nb >> 2;
  if (b < nc * 4) return (b >> 2) * 128 + l * 16 + (b & 3) * 4 + bj;
  return nc * 128 + (b - nc * 4) * 32 + l * 4 + bj;
}

void q8_pack_rows(const float* w, int64_t rows, int64_t cols, int8_t* qs, float* sc) {
  if (cols % 32 != 0) throw Error(HG_ERR_FORMAT, "Q8 needs cols divisible by 32 (got " + std::to_string(cols) + ")");
  int nb = (int)(cols / 32), ss = host_q8_ss(cols);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; r++) {
    const float* wr = w + r * cols;
    int8_t* qr = qs + r * cols;
    float* sr = sc + r * ss;
    for (int b = 0; b < nb; b++) {
      const float* x = wr + b * 32;
      float amax = 0.0f;
      for (int j = 0; j < 32; j++) amax = std::fmax(amax, std::fabs(x[j]));
      float d = amax / 127.0f;
      float id = d > 0.0f ? 1.0f / d : 0.0f;
      sr[b] = d;
      for (int j = 0; j < 32; j++) {
        float q = std::round(x[j] * id);
        q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
        qr[host_q8_pos(b * 32 + j, nb)] = (int8_t)q;
      }
    }
    for (int b = nb; b < ss; b++) sr[b] = 0.0f;
  }
}

void rope_tables(int head_dim, int max_pos, float theta, float* cos_out, float* sin_out) {  // ops.rs:139-154
  int half = head_dim / 2;
#pragma omp parallel for schedule(static)
  for (int p = 0; p < max_pos; p++)
    for (int i = 0; i < half; i++) {
      double inv_freq = std::pow((double)theta, -(2.0 * (double)i) / (double)head_dim);
      double ang = (double)p * inv_freq;
      cos_out[(size_t)p * half + i] = (float)std::cos(ang);
      sin_out[(size_t)p * half + i] = (float)std::sin(ang);
    }
}

}  // namespace hg
