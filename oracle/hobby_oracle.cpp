// TEST INFRASTRUCTURE ONLY — CPU oracle for the hobby-rs decode path.
//
// Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and `--impl reference`)
// load this library, and only as the checker / timed CPU baseline. The product (hobbylm_b200) never
// links, imports or calls anything under oracle/.
//
// What it is: a C++ restatement of the AVX2 CPU path of hobby-rs (harishsg993010/HobbyLM). The
// reference is Rust and cannot be built in this environment (no cargo/rustc, crates not vendored),
// so this file is the stand-in. Each function cites the reference file:line it follows.
//
//   gguf.rs   GGUF v3 reader + F16/Q8_0/Q5_0/Q4_K/Q6_K dequant          (Gguf::open 166-212, load 250-269)
//   config.rs Config::from_gguf, same keys and defaults                  (35-98)
//   quant.rs  Q8Tensor::quantize (78-102), matvec + AVX2 lane order (106-136, 44-67), matmul (144-193)
//   ops.rs    dot (wide f32x8, 4 accumulators, 7-36), rmsnorm (85-95), softmax (112-128),
//             sigmoid/silu (75-82), Rope in f64 (139-166)
//   model.rs  Model::load (79-131), forward/forward_x (152-184), attention (186-238), ffn (240-327),
//             prefill (340-370), attn_prefill (372-439), ffn_prefill (653-750), norm_head (753-763),
//             diffusion forward_bidir (441-470), run_block (472-510), attn_block_cached (512-587),
//             attn_bidir (589-640)
//   lib.rs    Engine::generate (107-162); diffusion: num_transfer (66-73), diffusion_block (164-209),
//             score_block (221-263), generate_diffusion_cached (265-407) / _uncached (409-495);
//             sample.rs argmax (53-64), sample (66-112), gumbel_argmax (29-47), Rng (3-22)
//
// Arithmetic pins (built with -ffp-contract=off so only the explicit fmaf/_mm256_fmadd_ps fuse,
// matching Rust, which never contracts):
//   * f32::exp and f32::ln are platform-defined in Rust. The oracle pins them to (float)exp((double)x)
//     and (float)log((double)x) (ln appears only in the diffusion Gumbel sampler), the
//     correctly rounded value with overwhelming probability. glibc 2.39 expf agrees with it on
//     99.992% of finite inputs in [-104, 89]; `hor_set_exp_mode(1)` switches to libm expf so the
//     difference can be measured.
//   * `wide` 0.7.33 (f32x8::mul_add = vfmadd, reduce_add = ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7))) is an
//     un-vendored crate: the reduce order is assumed from its published AVX implementation
//     (parity unpinned at that boundary; the same tree is pinned for quant.rs:61-65).
//   * sort_unstable_by on the router's 36 selection scores leaves the order of exactly equal
//     scores unspecified; the oracle breaks such ties by ascending expert id.

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <unordered_map>
#include <vector>
#include <algorithm>
#include <stdexcept>
#include <chrono>
#if defined(__AVX2__)
#include <immintrin.h>
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

namespace hor {

static thread_local std::string g_err;
static int g_exp_mode = 0;  // 0: (float)exp((double)x); 1: libm expf

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

static inline float fexp(float x) {
  if (g_exp_mode == 1) return expf(x);
  return (float)exp((double)x);
}
// f32::ln (the diffusion Gumbel sampler, sample.rs:36-46), pinned like fexp.
static inline float flog(float x) {
  if (g_exp_mode == 1) return logf(x);
  return (float)log((double)x);
}

// ---------------------------------------------------------------------------------------------
// gguf.rs
// ---------------------------------------------------------------------------------------------
enum MetaKind { M_U32, M_I32, M_F32, M_U64, M_BOOL, M_STR, M_ARRSTR, M_ARRI32, M_ARRF32, M_OTHER };
struct Meta {
  MetaKind kind = M_OTHER;
  uint32_t u32 = 0;
  int32_t i32 = 0;
  float f32 = 0;
  uint64_t u64 = 0;
  bool b = false;
  std::string s;
  std::vector<std::string> arrs;
  std::vector<int32_t> arri;
  std::vector<float> arrf;
};
struct TensorInfo {
  std::vector<uint64_t> ne;
  uint32_t type = 0;
  uint64_t offset = 0;
  uint64_t n_elems() const {
    uint64_t n = 1;
    for (auto v : ne) n *= v;
    return n;
  }
};

struct Cur {
  const uint8_t* b;
  size_t n, p = 0;
  const uint8_t* take(size_t k) {
    if (p + k > n || p + k < p) throw Error("GGUF: unexpected end of file");
    const uint8_t* r = b + p;
    p += k;
    return r;
  }
  template <class T> T rd() {
    T v;
    memcpy(&v, take(sizeof(T)), sizeof(T));
    return v;
  }
  std::string gstr() {
    uint64_t k = rd<uint64_t>();
    const uint8_t* s = take(k);
    return std::string((const char*)s, k);
  }
};

static Meta read_scalar(Cur& c, uint32_t ty) {
  Meta m;
  switch (ty) {
    case 0: m.kind = M_U32; m.u32 = c.rd<uint8_t>(); break;
    case 1: m.kind = M_I32; m.i32 = (int8_t)c.rd<uint8_t>(); break;
    case 2: m.kind = M_U32; m.u32 = c.rd<uint16_t>(); break;
    case 3: m.kind = M_I32; m.i32 = c.rd<int16_t>(); break;
    case 4: m.kind = M_U32; m.u32 = c.rd<uint32_t>(); break;
    case 5: m.kind = M_I32; m.i32 = c.rd<int32_t>(); break;
    case 6: m.kind = M_F32; m.f32 = c.rd<float>(); break;
    case 7: m.kind = M_BOOL; m.b = c.rd<uint8_t>() != 0; break;
    case 8: m.kind = M_STR; m.s = c.gstr(); break;
    case 10: m.kind = M_U64; m.u64 = c.rd<uint64_t>(); break;
    case 11: m.kind = M_I32; m.i32 = (int32_t)c.rd<uint64_t>(); break;
    case 12: m.kind = M_F32; m.f32 = (float)c.rd<double>(); break;
    default: throw Error("GGUF: unsupported metadata scalar type " + std::to_string(ty));
  }
  return m;
}

static Meta read_value(Cur& c, uint32_t ty) {
  if (ty != 9) return read_scalar(c, ty);
  uint32_t at = c.rd<uint32_t>();
  uint64_t n = c.rd<uint64_t>();
  Meta m;
  if (at == 8) {
    m.kind = M_ARRSTR;
    for (uint64_t i = 0; i < n; i++) m.arrs.push_back(c.gstr());
  } else if (at == 5 || at == 4) {
    m.kind = M_ARRI32;
    for (uint64_t i = 0; i < n; i++) m.arri.push_back(c.rd<int32_t>());
  } else if (at == 6) {
    m.kind = M_ARRF32;
    for (uint64_t i = 0; i < n; i++) m.arrf.push_back(c.rd<float>());
  } else {
    for (uint64_t i = 0; i < n; i++) read_scalar(c, at);
    m.kind = M_OTHER;
  }
  return m;
}

static inline float half_to_f32(uint16_t h) {  // gguf.rs:329-341
  int sign = (h >> 15) & 1;
  int ex = (h >> 10) & 0x1f;
  float mant = (float)(h & 0x3ff);
  float val;
  if (ex == 0) val = mant * ldexpf(1.0f, -24);
  else if (ex == 0x1f) val = (h & 0x3ff) == 0 ? INFINITY : NAN;
  else val = (1.0f + mant / 1024.0f) * ldexpf(1.0f, ex - 15);
  return sign ? -val : val;
}
static inline float rd_half(const uint8_t* b, size_t i) {
  uint16_t h;
  memcpy(&h, b + i, 2);
  return half_to_f32(h);
}

static size_t type_nbytes(uint32_t ty, size_t n) {  // gguf.rs:349-359
  switch (ty) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 6: return (n / 32) * 22;
    case 8: return (n / 32) * 34;
    case 12: return (n / 256) * 144;
    case 14: return (n / 256) * 210;
    default: throw Error("type_nbytes: unsupported ggml_type " + std::to_string(ty));
  }
}

static void dequant_q8_0(const uint8_t* b, size_t n, float* y) {  // gguf.rs:365-375
  for (size_t blk = 0; blk < n / 32; blk++) {
    size_t o = blk * 34;
    float d = rd_half(b, o);
    for (int j = 0; j < 32; j++) y[blk * 32 + j] = (float)(int8_t)b[o + 2 + j] * d;
  }
}
static void dequant_f16(const uint8_t* b, size_t n, float* y) {
  for (size_t i = 0; i < n; i++) y[i] = rd_half(b, i * 2);
}
static void dequant_q5_0(const uint8_t* b, size_t n, float* y) {  // gguf.rs:377-395
  for (size_t blk = 0; blk < n / 32; blk++) {
    size_t o = blk * 22;
    float d = rd_half(b, o);
    uint32_t qh;
    memcpy(&qh, b + o + 2, 4);
    const uint8_t* qs = b + o + 6;
    for (int j = 0; j < 16; j++) {
      uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10);
      uint8_t xh1 = (uint8_t)((qh >> (j + 12)) & 0x10);
      int x0 = (int)((qs[j] & 0x0F) | xh0) - 16;
      int x1 = (int)((qs[j] >> 4) | xh1) - 16;
      y[blk * 32 + j] = (float)x0 * d;
      y[blk * 32 + 16 + j] = (float)x1 * d;
    }
  }
}
static void scale_min_k4(int j, const uint8_t* sc, uint8_t* d, uint8_t* m) {
  if (j < 4) {
    *d = sc[j] & 63;
    *m = sc[j + 4] & 63;
  } else {
    *d = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
    *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
}
static void dequant_q4_k(const uint8_t* b, size_t n, float* y) {  // gguf.rs:408-437
  size_t yi = 0;
  for (size_t blk = 0; blk < n / 256; blk++) {
    size_t o = blk * 144;
    float d = rd_half(b, o), dmin = rd_half(b, o + 2);
    const uint8_t* scales = b + o + 4;
    const uint8_t* qs = b + o + 16;
    int is = 0;
    size_t q = 0;
    for (int r = 0; r < 4; r++) {
      uint8_t sc1, m1, sc2, m2;
      scale_min_k4(is, scales, &sc1, &m1);
      float d1 = d * (float)sc1, mm1 = dmin * (float)m1;
      scale_min_k4(is + 1, scales, &sc2, &m2);
      float d2 = d * (float)sc2, mm2 = dmin * (float)m2;
      for (int l = 0; l < 32; l++) y[yi++] = d1 * (float)(qs[q + l] & 0xF) - mm1;
      for (int l = 0; l < 32; l++) y[yi++] = d2 * (float)(qs[q + l] >> 4) - mm2;
      q += 32;
      is += 2;
    }
  }
}
static void dequant_q6_k(const uint8_t* b, size_t n, float* y) {  // gguf.rs:439-468
  for (size_t blk = 0; blk < n / 256; blk++) {
    size_t o = blk * 210;
    const uint8_t* ql = b + o;
    const uint8_t* qh = b + o + 128;
    const uint8_t* sc = b + o + 192;
    float d = rd_half(b, o + 208);
    size_t ybase = blk * 256;
    for (int half = 0; half < 2; half++) {
      size_t yb = ybase + half * 128;
      int qlb = half * 64, qhb = half * 32, scb = half * 8;
      for (int l = 0; l < 32; l++) {
        int is = l / 16;
        int q1 = (int)((ql[qlb + l] & 0xF) | (((qh[qhb + l] >> 0) & 3) << 4)) - 32;
        int q2 = (int)((ql[qlb + l + 32] & 0xF) | (((qh[qhb + l] >> 2) & 3) << 4)) - 32;
        int q3 = (int)((ql[qlb + l] >> 4) | (((qh[qhb + l] >> 4) & 3) << 4)) - 32;
        int q4 = (int)((ql[qlb + l + 32] >> 4) | (((qh[qhb + l] >> 6) & 3) << 4)) - 32;
        auto s = [&](int k) { return (float)(int8_t)sc[scb + is + k]; };
        y[yb + l] = d * s(0) * (float)q1;
        y[yb + l + 32] = d * s(2) * (float)q2;
        y[yb + l + 64] = d * s(4) * (float)q3;
        y[yb + l + 96] = d * s(6) * (float)q4;
      }
    }
  }
}

struct Gguf {
  const uint8_t* map = nullptr;
  size_t size = 0;
  size_t data_start = 0;
  std::unordered_map<std::string, Meta> meta;
  std::unordered_map<std::string, TensorInfo> tensors;

  ~Gguf() {
    if (map) munmap((void*)map, size);
  }
  void open(const char* path) {  // gguf.rs:166-212
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) throw Error(std::string("opening ") + path);
    struct stat st;
    fstat(fd, &st);
    size = (size_t)st.st_size;
    if (size == 0) {
      ::close(fd);
      throw Error("GGUF: unexpected end of file");
    }
    void* p = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (p == MAP_FAILED) throw Error("mmap failed");
    map = (const uint8_t*)p;
    Cur c{map, size};
    if (c.rd<uint32_t>() != 0x46554747u) throw Error("not a GGUF file (bad magic)");
    uint32_t version = c.rd<uint32_t>();
    if (version != 3) throw Error("unsupported GGUF version " + std::to_string(version) + " (expected 3)");
    uint64_t n_tensors = c.rd<uint64_t>();
    uint64_t n_meta = c.rd<uint64_t>();
    for (uint64_t i = 0; i < n_meta; i++) {
      std::string key = c.gstr();
      uint32_t ty = c.rd<uint32_t>();
      meta[key] = read_value(c, ty);
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
      std::string name = c.gstr();
      uint32_t nd = c.rd<uint32_t>();
      TensorInfo t;
      for (uint32_t k = 0; k < nd; k++) t.ne.push_back(c.rd<uint64_t>());
      t.type = c.rd<uint32_t>();
      t.offset = c.rd<uint64_t>();
      tensors[name] = t;
    }
    size_t align = 32;
    auto it = meta.find("general.alignment");
    if (it != meta.end() && it->second.kind == M_U32) align = it->second.u32;
    data_start = (c.p + align - 1) / align * align;
  }
  const TensorInfo* info(const std::string& n) const {
    auto it = tensors.find(n);
    return it == tensors.end() ? nullptr : &it->second;
  }
  std::vector<float> f32(const std::string& name) const {  // gguf.rs:215-235
    const TensorInfo* t = info(name);
    if (!t) throw Error("tensor `" + name + "` not found in GGUF");
    if (t->type != 0)
      throw Error("tensor `" + name + "` is ggml_type " + std::to_string(t->type) +
                  " (expected F32=0); this engine is F32-only for now");
    size_t n = t->n_elems();
    size_t off = data_start + t->offset;
    if (off + n * 4 > size) throw Error("tensor `" + name + "` out of file bounds");
    std::vector<float> v(n);
    memcpy(v.data(), map + off, n * 4);
    return v;
  }
  std::vector<float> load(const std::string& name) const {  // gguf.rs:250-269
    const TensorInfo* t = info(name);
    if (!t) throw Error("tensor `" + name + "` not found");
    size_t n = t->n_elems();
    if (t->type == 0) return f32(name);
    size_t nbytes = type_nbytes(t->type, n);
    size_t off = data_start + t->offset;
    if (off + nbytes > size) throw Error("tensor `" + name + "` out of file bounds");
    const uint8_t* b = map + off;
    std::vector<float> v(n);
    switch (t->type) {
      case 1: dequant_f16(b, n, v.data()); break;
      case 6: dequant_q5_0(b, n, v.data()); break;
      case 8: dequant_q8_0(b, n, v.data()); break;
      case 12: dequant_q4_k(b, n, v.data()); break;
      case 14: dequant_q6_k(b, n, v.data()); break;
      default: throw Error("tensor `" + name + "`: unsupported ggml_type " + std::to_string(t->type));
    }
    return v;
  }
  bool get_u32(const std::string& k, uint32_t* out) const {
    auto it = meta.find(k);
    if (it == meta.end()) return false;
    const Meta& m = it->second;
    if (m.kind == M_U32) *out = m.u32;
    else if (m.kind == M_I32) *out = (uint32_t)m.i32;
    else if (m.kind == M_U64) *out = (uint32_t)m.u64;
    else return false;
    return true;
  }
  bool get_f32(const std::string& k, float* out) const {
    auto it = meta.find(k);
    if (it == meta.end()) return false;
    const Meta& m = it->second;
    if (m.kind == M_F32) *out = m.f32;
    else if (m.kind == M_U32) *out = (float)m.u32;
    else return false;
    return true;
  }
  bool get_bool(const std::string& k, bool* out) const {
    auto it = meta.find(k);
    if (it == meta.end() || it->second.kind != M_BOOL) return false;
    *out = it->second.b;
    return true;
  }
  bool get_str(const std::string& k, std::string* out) const {
    auto it = meta.find(k);
    if (it == meta.end() || it->second.kind != M_STR) return false;
    *out = it->second.s;
    return true;
  }
};

// ---------------------------------------------------------------------------------------------
// config.rs
// ---------------------------------------------------------------------------------------------
struct Config {
  std::string arch;
  int d_model, n_layers, n_dense, n_heads, n_kv_heads, head_dim, dense_ffn, expert_ffn;
  int n_experts, top_k, n_shared, vocab_size, context_length;
  float rms_eps, rope_theta, expert_weights_scale;
  bool expert_weights_norm, gating_sigmoid;
  bool diffusion;  // config.rs:92-94 (keys without the architecture prefix)
  int mask_token_id, block_size;
  int q_dim() const { return n_heads * head_dim; }
  int kv_dim() const { return n_kv_heads * head_dim; }
  bool is_moe(int l) const { return l >= n_dense; }
};

static Config config_from_gguf(const Gguf& g) {  // config.rs:35-98
  Config c;
  if (!g.get_str("general.architecture", &c.arch)) throw Error("missing general.architecture");
  auto k = [&](const char* s) { return c.arch + "." + s; };
  auto u = [&](const char* s) -> int {
    uint32_t v;
    if (!g.get_u32(k(s), &v)) throw Error(std::string("missing metadata `") + c.arch + "." + s + "`");
    return (int)v;
  };
  auto uo = [&](const char* s, int dflt) -> int {
    uint32_t v;
    return g.get_u32(k(s), &v) ? (int)v : dflt;
  };
  uint32_t v;
  if (g.get_u32(k("attention.key_length"), &v)) {
    c.head_dim = (int)v;
  } else {
    uint32_t d = 0, h = 1;
    g.get_u32(k("embedding_length"), &d);
    g.get_u32(k("attention.head_count"), &h);
    c.head_dim = (int)(d / std::max<uint32_t>(h, 1));
  }
  const TensorInfo* te = g.info("token_embd.weight");
  if (te && te->ne.size() > 1) c.vocab_size = (int)te->ne[1];
  else if (g.get_u32(k("vocab_size"), &v)) c.vocab_size = (int)v;
  else throw Error("cannot determine vocab_size");
  uint32_t gf;
  c.gating_sigmoid = true;
  if (g.get_u32(k("expert_gating_func"), &gf)) c.gating_sigmoid = (gf == 1) ? false : true;
  c.d_model = u("embedding_length");
  c.n_layers = u("block_count");
  c.n_dense = uo("leading_dense_block_count", 1);
  c.n_heads = u("attention.head_count");
  c.n_kv_heads = u("attention.head_count_kv");
  c.dense_ffn = u("feed_forward_length");
  c.expert_ffn = u("expert_feed_forward_length");
  c.n_experts = u("expert_count");
  c.top_k = u("expert_used_count");
  c.n_shared = uo("expert_shared_count", 0);
  c.context_length = uo("context_length", 8192);
  float f;
  c.rms_eps = g.get_f32(k("attention.layer_norm_rms_epsilon"), &f) ? f : 1e-5f;
  c.rope_theta = g.get_f32(k("rope.freq_base"), &f) ? f : 1e6f;
  c.expert_weights_scale = g.get_f32(k("expert_weights_scale"), &f) ? f : 1.0f;
  bool b;
  c.expert_weights_norm = g.get_bool(k("expert_weights_norm"), &b) ? b : false;
  c.diffusion = g.get_bool("diffusion.enabled", &b) ? b : false;
  c.mask_token_id = g.get_u32("diffusion.mask_token_id", &v) ? (int)v : 50257;
  c.block_size = g.get_u32("diffusion.block_size", &v) ? (int)v : 32;
  return c;
}

// ---------------------------------------------------------------------------------------------
// ops.rs
// ---------------------------------------------------------------------------------------------
// 8-lane horizontal sum in the order of the SSE hsum (quant.rs:61-65) and wide's reduce_add.
static inline float hsum8(const float* a) {
  float s0 = a[0] + a[4], s1 = a[1] + a[5], s2 = a[2] + a[6], s3 = a[3] + a[7];
  float t0 = s0 + s2, t1 = s1 + s3;
  return t0 + t1;
}

// ops.rs:7-36: four f32x8 FMA accumulators over 32-float strides, an 8-wide tail, then
// ((a0+a1)+(a2+a3)).reduce_add() and a scalar mul-add tail.
float dot(const float* a, const float* b, int n) {
  int i = 0;
  int main_ = n - n % 32;
  float s;
#if defined(__AVX2__) && defined(__FMA__)
  __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
  for (; i < main_; i += 32) {
    a0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), a0);
    a1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8), a1);
    a2 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 16), _mm256_loadu_ps(b + i + 16), a2);
    a3 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i + 24), _mm256_loadu_ps(b + i + 24), a3);
  }
  for (; i + 8 <= n; i += 8) a0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), a0);
  __m256 t = _mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3));
  alignas(32) float lanes[8];
  _mm256_store_ps(lanes, t);
  s = hsum8(lanes);
#else
  float acc[4][8] = {};
  for (; i < main_; i += 32)
    for (int m = 0; m < 4; m++)
      for (int l = 0; l < 8; l++) acc[m][l] = fmaf(a[i + 8 * m + l], b[i + 8 * m + l], acc[m][l]);
  for (; i + 8 <= n; i += 8)
    for (int l = 0; l < 8; l++) acc[0][l] = fmaf(a[i + l], b[i + l], acc[0][l]);
  float lanes[8];
  for (int l = 0; l < 8; l++) lanes[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
  s = hsum8(lanes);
#endif
  for (; i < n; i++) s += a[i] * b[i];
  return s;
}

static inline float sigmoid(float x) { return 1.0f / (1.0f + fexp(-x)); }
static inline float silu(float x) { return x * sigmoid(x); }

void rmsnorm(const float* x, const float* w, float eps, float* out, int n) {  // ops.rs:85-95
  float ss = 0.0f;
  for (int i = 0; i < n; i++) ss += x[i] * x[i];
  float scale = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

void softmax(float* x, int n) {  // ops.rs:112-128
  float m = -INFINITY;
  for (int i = 0; i < n; i++)
    if (x[i] > m) m = x[i];
  float sum = 0.0f;
  for (int i = 0; i < n; i++) {
    x[i] = fexp(x[i] - m);
    sum += x[i];
  }
  float inv = 1.0f / sum;
  for (int i = 0; i < n; i++) x[i] *= inv;
}

struct Rope {  // ops.rs:131-166
  int head_dim = 0, half = 0, max_pos = 0;
  std::vector<float> cos_, sin_;
  void init(int hd, int mp, float theta) {
    head_dim = hd;
    half = hd / 2;
    max_pos = mp;
    cos_.assign((size_t)mp * half, 0.0f);
    sin_.assign((size_t)mp * half, 0.0f);
    for (int p = 0; p < mp; p++)
      for (int i = 0; i < half; i++) {
        double inv_freq = pow((double)theta, -(2.0 * (double)i) / (double)hd);
        double ang = (double)p * inv_freq;
        cos_[(size_t)p * half + i] = (float)cos(ang);
        sin_[(size_t)p * half + i] = (float)sin(ang);
      }
  }
  void apply(float* v, int pos) const {
    if (pos < 0 || pos >= max_pos) throw Error("rope position out of range");
    size_t base = (size_t)pos * half;
    for (int i = 0; i < half; i++) {
      float c = cos_[base + i], s = sin_[base + i];
      float x1 = v[i], x2 = v[half + i];
      v[i] = x1 * c - x2 * s;
      v[half + i] = x2 * c + x1 * s;
    }
  }
};

static void norm_head(float* v, const float* w, float eps, int n) {  // model.rs:753-763
  float ss = 0.0f;
  for (int i = 0; i < n; i++) ss += v[i] * v[i];
  float scale = 1.0f / sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; i++) v[i] = v[i] * scale * w[i];
}

// ---------------------------------------------------------------------------------------------
// quant.rs
// ---------------------------------------------------------------------------------------------
// Per-32 block int8 quantization: amax, d = amax/127, id = d>0 ? 1/d : 0, q = clamp(round(x*id)).
// Shared by weight re-quantization (quant.rs:85-100) and activation quantization (quant.rs:112-123).
static inline void quant_block(const float* x, int8_t* q, float* d_out) {
  float amax = 0.0f;
  for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[j]));
  float d = amax / 127.0f;
  float id = d > 0.0f ? 1.0f / d : 0.0f;
  *d_out = d;
  for (int j = 0; j < 32; j++) {
    float r = roundf(x[j] * id);
    r = r < -127.0f ? -127.0f : (r > 127.0f ? 127.0f : r);
    q[j] = (int8_t)r;
  }
}

// quant.rs:44-67. Eight i32 lane partials per block (lane l sums bytes 4l..4l+3), scaled by
// sw[b]*dx[b] and FMA-accumulated across blocks in f32 lanes, then hsum8.
static inline float qrow_dot(const int8_t* qw, const int8_t* qa, const float* sw, const float* dx, int nb) {
#if defined(__AVX2__) && defined(__FMA__)
  const __m256i ones = _mm256_set1_epi16(1);
  __m256 acc = _mm256_setzero_ps();
  for (int b = 0; b < nb; b++) {
    __m256i w = _mm256_loadu_si256((const __m256i*)(qw + (size_t)b * 32));
    __m256i a = _mm256_loadu_si256((const __m256i*)(qa + (size_t)b * 32));
    __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(w, w), _mm256_sign_epi8(a, w));
    __m256i p32 = _mm256_madd_epi16(p16, ones);
    acc = _mm256_fmadd_ps(_mm256_set1_ps(sw[b] * dx[b]), _mm256_cvtepi32_ps(p32), acc);
  }
  alignas(32) float lanes[8];
  _mm256_store_ps(lanes, acc);
  return hsum8(lanes);
#else
  float lanes[8] = {};
  for (int b = 0; b < nb; b++) {
    float sd = sw[b] * dx[b];
    for (int l = 0; l < 8; l++) {
      int p = 0;
      for (int j = 0; j < 4; j++) p += (int)qw[b * 32 + 4 * l + j] * (int)qa[b * 32 + 4 * l + j];
      lanes[l] = fmaf(sd, (float)p, lanes[l]);
    }
  }
  return hsum8(lanes);
#endif
}

struct Q8Tensor {
  int out = 0, in = 0, nb = 0;
  std::vector<float> scales;  // [out*nb]
  std::vector<int8_t> qs;     // [out*in]

  void quantize(const float* w, int out_, int in_) {  // quant.rs:78-102
    if (in_ % 32 != 0) throw Error("Q8_0 needs in_ divisible by 32");
    out = out_;
    in = in_;
    nb = in_ / 32;
    scales.assign((size_t)out * nb, 0.0f);
    qs.assign((size_t)out * in, 0);
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out; o++)
      for (int b = 0; b < nb; b++)
        quant_block(w + (size_t)o * in + (size_t)b * 32, &qs[(size_t)o * in + (size_t)b * 32],
                    &scales[(size_t)o * nb + b]);
  }

  void matvec(const float* x, float* y) const {  // quant.rs:106-136
    std::vector<int8_t> qx(in);
    std::vector<float> dx(nb);
    for (int b = 0; b < nb; b++) quant_block(x + (size_t)b * 32, &qx[(size_t)b * 32], &dx[b]);
    auto work = [&](int o) {
      y[o] = qrow_dot(&qs[(size_t)o * in], qx.data(), &scales[(size_t)o * nb], dx.data(), nb);
    };
    if (out >= 64) {
#pragma omp parallel for schedule(static)
      for (int o = 0; o < out; o++) work(o);
    } else {
      for (int o = 0; o < out; o++) work(o);
    }
  }

  void matmul(const float* x, float* y, int tn) const {  // quant.rs:144-193
    std::vector<int8_t> qx((size_t)tn * in);
    std::vector<float> dx((size_t)tn * nb);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tn; t++)
      for (int b = 0; b < nb; b++)
        quant_block(x + (size_t)t * in + (size_t)b * 32, &qx[(size_t)t * in + (size_t)b * 32],
                    &dx[(size_t)t * nb + b]);
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out; o++) {
      const int8_t* qw = &qs[(size_t)o * in];
      const float* sw = &scales[(size_t)o * nb];
      for (int t = 0; t < tn; t++) {
        const int8_t* qxr = &qx[(size_t)t * in];
        const float* dxr = &dx[(size_t)t * nb];
        float acc = 0.0f;
        for (int b = 0; b < nb; b++) {
          int isum = 0;
          for (int j = 0; j < 32; j++) isum += (int)qw[b * 32 + j] * (int)qxr[b * 32 + j];
          acc += sw[b] * dxr[b] * (float)isum;
        }
        y[(size_t)t * out + o] = acc;
      }
    }
  }
  size_t bytes() const { return scales.size() * 4 + qs.size(); }
};

// ops.rs:40-53 (parallel over rows when out >= 64; no numeric effect)
static void f32_matvec(const float* w, const float* x, float* y, int out, int in) {
  if (out >= 64) {
#pragma omp parallel for schedule(static)
    for (int o = 0; o < out; o++) y[o] = dot(w + (size_t)o * in, x, in);
  } else {
    for (int o = 0; o < out; o++) y[o] = dot(w + (size_t)o * in, x, in);
  }
}
// ops.rs:58-72
static void f32_matmul(const float* w, const float* x, float* y, int tn, int in, int out) {
#pragma omp parallel for schedule(static)
  for (int o = 0; o < out; o++)
    for (int t = 0; t < tn; t++) y[(size_t)t * out + o] = dot(w + (size_t)o * in, x + (size_t)t * in, in);
}

struct Mat {  // quant.rs:198-247
  bool q8 = false;
  int out = 0, in = 0;
  std::vector<float> w;
  Q8Tensor q;
  void build(std::vector<float>&& src, int out_, int in_, bool quant) {
    if (src.size() != (size_t)out_ * in_) throw Error("matrix element count mismatch");
    out = out_;
    in = in_;
    q8 = quant;
    if (quant) {
      q.quantize(src.data(), out_, in_);
    } else {
      w = std::move(src);
    }
  }
  void matvec(const float* x, float* y) const {
    if (q8) q.matvec(x, y);
    else f32_matvec(w.data(), x, y, out, in);
  }
  void matmul(const float* x, float* y, int tn) const {
    if (q8) q.matmul(x, y, tn);
    else f32_matmul(w.data(), x, y, tn, in, out);
  }
  size_t bytes() const { return q8 ? q.bytes() : w.size() * 4; }
};

// ---------------------------------------------------------------------------------------------
// model.rs
// ---------------------------------------------------------------------------------------------
struct Moe {
  Mat gate_inp;  // (n_exp, d) f32
  std::vector<float> bias;
  std::vector<Mat> gate_exps, up_exps, down_exps;
  Mat gate_sh, up_sh, down_sh;
};
struct Layer {
  std::vector<float> attn_norm, attn_q_norm, attn_k_norm, ffn_norm;
  Mat attn_qkv, attn_output;
  bool moe = false;
  Mat gate, up, down;  // dense
  Moe m;
};

struct KvCache {  // model.rs:60-75
  std::vector<std::vector<float>> k, v;
  int len = 0;
};

// Router selection of one token (model.rs:270-293 / 678-699): returns (expert ids in rank order,
// gate weights) and writes the selection scores.
static void route(const Config& c, const float* logits, const float* bias, int* topk, float* w) {
  int ne = c.n_experts;
  std::vector<float> scores(ne);
  if (c.gating_sigmoid) {
    for (int e = 0; e < ne; e++) scores[e] = sigmoid(logits[e]);
  } else {
    for (int e = 0; e < ne; e++) scores[e] = logits[e];
    softmax(scores.data(), ne);
  }
  std::vector<std::pair<int, float>> order(ne);
  for (int e = 0; e < ne; e++) order[e] = {e, scores[e] + bias[e]};
  std::stable_sort(order.begin(), order.end(),
                   [](const std::pair<int, float>& a, const std::pair<int, float>& b) { return a.second > b.second; });
  for (int r = 0; r < c.top_k; r++) {
    topk[r] = order[r].first;
    w[r] = scores[order[r].first];
  }
  if (c.expert_weights_norm) {
    float s = -0.0f;
    for (int r = 0; r < c.top_k; r++) s = s + w[r];
    s = s + 1e-9f;
    for (int r = 0; r < c.top_k; r++) w[r] /= s;
  }
}

struct Model {
  Config cfg;
  Rope rope;
  std::vector<float> token_embd, output_norm;
  Mat output;
  std::vector<Layer> layers;
  // debug capture of the last forward's routing: [layer][top_k]
  std::vector<int> last_sel;
  std::vector<float> last_selw;

  void load(const Gguf& g, const Config& c, bool quant) {  // model.rs:79-131
    cfg = c;
    int d = c.d_model, f = c.expert_ffn;
    rope.init(c.head_dim, c.context_length, c.rope_theta);
    layers.resize(c.n_layers);
    for (int i = 0; i < c.n_layers; i++) {
      Layer& L = layers[i];
      std::string p = "blk." + std::to_string(i) + ".";
      auto nt = [&](const char* s) { return g.f32(p + s); };
      auto mt = [&](Mat& m, const char* s, int out, int in) { m.build(g.load(p + s), out, in, quant); };
      auto split = [&](std::vector<Mat>& v, const char* s, int a, int b) {
        std::vector<float> src = g.load(p + s);
        size_t ab = (size_t)a * b;
        if (src.size() < (size_t)c.n_experts * ab) throw Error("expert tensor too small");
        v.resize(c.n_experts);
        for (int e = 0; e < c.n_experts; e++) {
          std::vector<float> sl(src.begin() + e * ab, src.begin() + (e + 1) * ab);
          v[e].build(std::move(sl), a, b, quant);
        }
      };
      if (c.is_moe(i)) {
        L.moe = true;
        L.m.gate_inp.build(g.load(p + "ffn_gate_inp.weight"), c.n_experts, d, false);
        L.m.bias = nt("exp_probs_b.bias");
        split(L.m.gate_exps, "ffn_gate_exps.weight", f, d);
        split(L.m.up_exps, "ffn_up_exps.weight", f, d);
        split(L.m.down_exps, "ffn_down_exps.weight", d, f);
        mt(L.m.gate_sh, "ffn_gate_shexp.weight", f, d);
        mt(L.m.up_sh, "ffn_up_shexp.weight", f, d);
        mt(L.m.down_sh, "ffn_down_shexp.weight", d, f);
      } else {
        int df = c.dense_ffn;
        mt(L.gate, "ffn_gate.weight", df, d);
        mt(L.up, "ffn_up.weight", df, d);
        mt(L.down, "ffn_down.weight", d, df);
      }
      L.attn_norm = nt("attn_norm.weight");
      mt(L.attn_qkv, "attn_qkv.weight", c.q_dim() + 2 * c.kv_dim(), d);
      L.attn_q_norm = nt("attn_q_norm.weight");
      L.attn_k_norm = nt("attn_k_norm.weight");
      mt(L.attn_output, "attn_output.weight", d, c.q_dim());
      L.ffn_norm = nt("ffn_norm.weight");
    }
    output.build(g.load("output.weight"), c.vocab_size, d, quant);
    token_embd = g.load("token_embd.weight");
    if (token_embd.size() < (size_t)c.vocab_size * d) throw Error("token_embd too small");
    output_norm = g.f32("output_norm.weight");
    last_sel.assign((size_t)c.n_layers * c.top_k, -1);
    last_selw.assign((size_t)c.n_layers * c.top_k, 0.0f);
  }

  size_t weight_bytes() const {  // model.rs:134-149
    size_t b = output.bytes();
    for (auto& L : layers) {
      b += L.attn_qkv.bytes() + L.attn_output.bytes();
      if (!L.moe) b += L.gate.bytes() + L.up.bytes() + L.down.bytes();
      else {
        for (auto& e : L.m.gate_exps) b += e.bytes();
        for (auto& e : L.m.up_exps) b += e.bytes();
        for (auto& e : L.m.down_exps) b += e.bytes();
        b += L.m.gate_sh.bytes() + L.m.up_sh.bytes() + L.m.down_sh.bytes();
      }
    }
    return b;
  }

  void new_cache(KvCache& kc) const {
    kc.k.assign(cfg.n_layers, {});
    kc.v.assign(cfg.n_layers, {});
    for (int l = 0; l < cfg.n_layers; l++) {
      kc.k[l].reserve((size_t)cfg.context_length * cfg.kv_dim());
      kc.v[l].reserve((size_t)cfg.context_length * cfg.kv_dim());
    }
    kc.len = 0;
  }

  // model.rs:186-238
  void attention(const Layer& L, const float* h, int li, int pos, KvCache& cache, float* proj) const {
    const Config& c = cfg;
    int hd = c.head_dim, qd = c.q_dim(), kvd = c.kv_dim(), rep = c.n_heads / c.n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    std::vector<float> qkv(qd + 2 * kvd);
    L.attn_qkv.matvec(h, qkv.data());
    float* q = qkv.data();
    float* k = q + qd;
    float* v = k + kvd;
    for (int hq = 0; hq < c.n_heads; hq++) {
      norm_head(q + hq * hd, L.attn_q_norm.data(), c.rms_eps, hd);
      rope.apply(q + hq * hd, pos);
    }
    for (int hk = 0; hk < c.n_kv_heads; hk++) {
      norm_head(k + hk * hd, L.attn_k_norm.data(), c.rms_eps, hd);
      rope.apply(k + hk * hd, pos);
    }
    cache.k[li].insert(cache.k[li].end(), k, k + kvd);
    cache.v[li].insert(cache.v[li].end(), v, v + kvd);
    const float* kc = cache.k[li].data();
    const float* vc = cache.v[li].data();
    int n = pos + 1;
    if ((size_t)n * kvd > cache.k[li].size()) throw Error("kv cache shorter than pos+1");
    std::vector<float> out(qd, 0.0f), scores(n);
    for (int hq = 0; hq < c.n_heads; hq++) {
      int kvh = hq / rep;
      const float* qh = q + hq * hd;
      for (int t = 0; t < n; t++) scores[t] = dot(qh, kc + (size_t)t * kvd + kvh * hd, hd) * scale;
      softmax(scores.data(), n);
      float* oh = out.data() + hq * hd;
      for (int t = 0; t < n; t++) {
        const float* vt = vc + (size_t)t * kvd + kvh * hd;
        float p = scores[t];
        for (int di = 0; di < hd; di++) oh[di] += p * vt[di];
      }
    }
    L.attn_output.matvec(out.data(), proj);
  }

  // model.rs:240-327
  void ffn(const Layer& L, const float* h, float* out, int li) {
    const Config& c = cfg;
    int d = c.d_model;
    if (!L.moe) {
      int f = c.dense_ffn;
      std::vector<float> g(f), u(f);
      L.gate.matvec(h, g.data());
      L.up.matvec(h, u.data());
      for (int i = 0; i < f; i++) g[i] = silu(g[i]) * u[i];
      L.down.matvec(g.data(), out);
      return;
    }
    int f = c.expert_ffn, ne = c.n_experts;
    std::vector<float> logits(ne);
    L.m.gate_inp.matvec(h, logits.data());
    std::vector<int> topk(c.top_k);
    std::vector<float> w(c.top_k);
    route(c, logits.data(), L.m.bias.data(), topk.data(), w.data());
    if (li >= 0)
      for (int r = 0; r < c.top_k; r++) {
        last_sel[(size_t)li * c.top_k + r] = topk[r];
        last_selw[(size_t)li * c.top_k + r] = w[r];
      }
    for (int i = 0; i < d; i++) out[i] = 0.0f;
    std::vector<float> gb(f), ub(f), yb(d);
    for (int r = 0; r < c.top_k; r++) {
      int e = topk[r];
      L.m.gate_exps[e].matvec(h, gb.data());
      L.m.up_exps[e].matvec(h, ub.data());
      for (int i = 0; i < f; i++) gb[i] = silu(gb[i]) * ub[i];
      L.m.down_exps[e].matvec(gb.data(), yb.data());
      float sc = w[r] * c.expert_weights_scale;
      for (int i = 0; i < d; i++) out[i] += sc * yb[i];
    }
    if (c.n_shared > 0) {
      L.m.gate_sh.matvec(h, gb.data());
      L.m.up_sh.matvec(h, ub.data());
      for (int i = 0; i < f; i++) gb[i] = silu(gb[i]) * ub[i];
      L.m.down_sh.matvec(gb.data(), yb.data());
      for (int i = 0; i < d; i++) out[i] += yb[i];
    }
  }

  // model.rs:160-184
  void forward_x(std::vector<float> x, int pos, KvCache& cache, float* logits) {
    const Config& c = cfg;
    int d = c.d_model;
    std::vector<float> h(d), tmp(d);
    for (int li = 0; li < c.n_layers; li++) {
      const Layer& L = layers[li];
      rmsnorm(x.data(), L.attn_norm.data(), c.rms_eps, h.data(), d);
      attention(L, h.data(), li, pos, cache, tmp.data());
      for (int i = 0; i < d; i++) x[i] += tmp[i];
      rmsnorm(x.data(), L.ffn_norm.data(), c.rms_eps, h.data(), d);
      ffn(L, h.data(), tmp.data(), li);
      for (int i = 0; i < d; i++) x[i] += tmp[i];
    }
    cache.len = pos + 1;
    rmsnorm(x.data(), output_norm.data(), c.rms_eps, h.data(), d);
    output.matvec(h.data(), logits);
  }
  void forward(uint32_t token, int pos, KvCache& cache, float* logits) {  // model.rs:152-156
    int d = cfg.d_model;
    if ((int64_t)token >= cfg.vocab_size) throw Error("token id out of range");
    std::vector<float> x(token_embd.begin() + (size_t)token * d, token_embd.begin() + (size_t)(token + 1) * d);
    forward_x(std::move(x), pos, cache, logits);
  }

  // model.rs:372-439
  void attn_prefill(const Layer& L, const float* h, int li, int base, int tn, KvCache& cache, float* proj) const {
    const Config& c = cfg;
    int hd = c.head_dim, qd = c.q_dim(), kvd = c.kv_dim(), qw = qd + 2 * kvd, rep = c.n_heads / c.n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    std::vector<float> qkv((size_t)tn * qw);
    L.attn_qkv.matmul(h, qkv.data(), tn);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tn; t++) {
      float* row = qkv.data() + (size_t)t * qw;
      int pos = base + t;
      for (int hq = 0; hq < c.n_heads; hq++) {
        norm_head(row + hq * hd, L.attn_q_norm.data(), c.rms_eps, hd);
        rope.apply(row + hq * hd, pos);
      }
      for (int hk = 0; hk < c.n_kv_heads; hk++) {
        norm_head(row + qd + hk * hd, L.attn_k_norm.data(), c.rms_eps, hd);
        rope.apply(row + qd + hk * hd, pos);
      }
    }
    for (int t = 0; t < tn; t++) {
      const float* row = qkv.data() + (size_t)t * qw;
      cache.k[li].insert(cache.k[li].end(), row + qd, row + qd + kvd);
      cache.v[li].insert(cache.v[li].end(), row + qd + kvd, row + qw);
    }
    const float* kc = cache.k[li].data();
    const float* vc = cache.v[li].data();
    std::vector<float> o((size_t)tn * qd, 0.0f);
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < tn; t++) {
      int n = base + t + 1;
      const float* qrow = qkv.data() + (size_t)t * qw;
      std::vector<float> scores(n);
      float* orow = o.data() + (size_t)t * qd;
      for (int hq = 0; hq < c.n_heads; hq++) {
        int kvh = hq / rep;
        const float* qh = qrow + hq * hd;
        for (int j = 0; j < n; j++) scores[j] = dot(qh, kc + (size_t)j * kvd + kvh * hd, hd) * scale;
        softmax(scores.data(), n);
        float* oh = orow + hq * hd;
        for (int j = 0; j < n; j++) {
          const float* vt = vc + (size_t)j * kvd + kvh * hd;
          float p = scores[j];
          for (int di = 0; di < hd; di++) oh[di] += p * vt[di];
        }
      }
    }
    L.attn_output.matmul(o.data(), proj, tn);
  }

  // model.rs:653-750
  void ffn_prefill(const Layer& L, const float* h, int tn, float* out) const {
    const Config& c = cfg;
    int d = c.d_model, f = c.expert_ffn;
    if (!L.moe) {
      int df = c.dense_ffn;
      std::vector<float> g((size_t)tn * df), u((size_t)tn * df);
      L.gate.matmul(h, g.data(), tn);
      L.up.matmul(h, u.data(), tn);
      for (size_t i = 0; i < (size_t)tn * df; i++) g[i] = silu(g[i]) * u[i];
      L.down.matmul(g.data(), out, tn);
      return;
    }
    int ne = c.n_experts;
    std::vector<float> logits((size_t)tn * ne);
    L.m.gate_inp.matmul(h, logits.data(), tn);
    std::vector<std::vector<std::pair<int, float>>> assign(ne);
    std::vector<int> topk(c.top_k);
    std::vector<float> w(c.top_k);
    for (int t = 0; t < tn; t++) {
      route(c, logits.data() + (size_t)t * ne, L.m.bias.data(), topk.data(), w.data());
      for (int r = 0; r < c.top_k; r++) assign[topk[r]].push_back({t, w[r] * c.expert_weights_scale});
    }
    for (size_t i = 0; i < (size_t)tn * d; i++) out[i] = 0.0f;
    for (int e = 0; e < ne; e++) {
      auto& rows = assign[e];
      int m = (int)rows.size();
      if (m == 0) continue;
      std::vector<float> xe((size_t)m * d), ge((size_t)m * f), ue((size_t)m * f), ye((size_t)m * d);
      for (int i = 0; i < m; i++) memcpy(&xe[(size_t)i * d], h + (size_t)rows[i].first * d, d * 4);
      L.m.gate_exps[e].matmul(xe.data(), ge.data(), m);
      L.m.up_exps[e].matmul(xe.data(), ue.data(), m);
      for (size_t i = 0; i < (size_t)m * f; i++) ge[i] = silu(ge[i]) * ue[i];
      L.m.down_exps[e].matmul(ge.data(), ye.data(), m);
      for (int i = 0; i < m; i++) {
        int t = rows[i].first;
        float wt = rows[i].second;
        for (int k = 0; k < d; k++) out[(size_t)t * d + k] += wt * ye[(size_t)i * d + k];
      }
    }
    if (c.n_shared > 0) {
      std::vector<float> gs((size_t)tn * f), us((size_t)tn * f), ys((size_t)tn * d);
      L.m.gate_sh.matmul(h, gs.data(), tn);
      L.m.up_sh.matmul(h, us.data(), tn);
      for (size_t i = 0; i < (size_t)tn * f; i++) gs[i] = silu(gs[i]) * us[i];
      L.m.down_sh.matmul(gs.data(), ys.data(), tn);
      for (size_t i = 0; i < (size_t)tn * d; i++) out[i] += ys[i];
    }
  }

  // model.rs:340-370
  void prefill(const float* inputs, int tn, KvCache& cache, float* logits) {
    const Config& c = cfg;
    int d = c.d_model;
    int base = cache.len;
    std::vector<float> x(inputs, inputs + (size_t)tn * d), h((size_t)tn * d), tmp((size_t)tn * d);
    for (int li = 0; li < c.n_layers; li++) {
      const Layer& L = layers[li];
#pragma omp parallel for schedule(static)
      for (int t = 0; t < tn; t++)
        rmsnorm(&x[(size_t)t * d], L.attn_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
      attn_prefill(L, h.data(), li, base, tn, cache, tmp.data());
      for (size_t i = 0; i < (size_t)tn * d; i++) x[i] += tmp[i];
#pragma omp parallel for schedule(static)
      for (int t = 0; t < tn; t++)
        rmsnorm(&x[(size_t)t * d], L.ffn_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
      ffn_prefill(L, h.data(), tn, tmp.data());
      for (size_t i = 0; i < (size_t)tn * d; i++) x[i] += tmp[i];
    }
    cache.len = base + tn;
    std::vector<float> hl(d);
    rmsnorm(&x[(size_t)(tn - 1) * d], output_norm.data(), c.rms_eps, hl.data(), d);
    output.matvec(hl.data(), logits);
  }

  // QK-norm + RoPE of the q and k heads of tn qkv rows at positions base + t (model.rs:529-542).
  void qk_norm_rope_rows(const Layer& L, float* qkv, int tn, int base) const {
    const Config& c = cfg;
    int hd = c.head_dim, qd = c.q_dim(), kvd = c.kv_dim(), qw = qd + 2 * kvd;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tn; t++) {
      float* row = qkv + (size_t)t * qw;
      for (int hq = 0; hq < c.n_heads; hq++) {
        norm_head(row + hq * hd, L.attn_q_norm.data(), c.rms_eps, hd);
        rope.apply(row + hq * hd, base + t);
      }
      for (int hk = 0; hk < c.n_kv_heads; hk++) {
        norm_head(row + qd + hk * hd, L.attn_k_norm.data(), c.rms_eps, hd);
        rope.apply(row + qd + hk * hd, base + t);
      }
    }
  }

  // model.rs:512-587 (attn_block_cached): the b block queries attend to the cached prefix keys
  // (0..base) and then to every block key (bidirectional). bk / bv receive the block's K / V rows.
  void attn_block_cached(const Layer& L, const float* h, int li, const KvCache& cache, int base, int b, float* proj,
                         float* bk, float* bv) const {
    const Config& c = cfg;
    int hd = c.head_dim, qd = c.q_dim(), kvd = c.kv_dim(), qw = qd + 2 * kvd, rep = c.n_heads / c.n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    std::vector<float> qkv((size_t)b * qw);
    L.attn_qkv.matmul(h, qkv.data(), b);
    qk_norm_rope_rows(L, qkv.data(), b, base);
    for (int t = 0; t < b; t++) {
      const float* row = qkv.data() + (size_t)t * qw;
      memcpy(bk + (size_t)t * kvd, row + qd, kvd * 4);
      memcpy(bv + (size_t)t * kvd, row + qd + kvd, kvd * 4);
    }
    const float* pk = cache.k[li].data();
    const float* pv = cache.v[li].data();
    const int n = base + b;
    std::vector<float> o((size_t)b * qd, 0.0f);
#pragma omp parallel for schedule(dynamic, 2)
    for (int t = 0; t < b; t++) {
      const float* qrow = qkv.data() + (size_t)t * qw;
      std::vector<float> scores(n);
      float* orow = o.data() + (size_t)t * qd;
      for (int hq = 0; hq < c.n_heads; hq++) {
        int kvh = hq / rep;
        const float* qh = qrow + hq * hd;
        for (int j = 0; j < base; j++) scores[j] = dot(qh, pk + (size_t)j * kvd + kvh * hd, hd) * scale;
        for (int j = 0; j < b; j++) scores[base + j] = dot(qh, bk + (size_t)j * kvd + kvh * hd, hd) * scale;
        softmax(scores.data(), n);
        float* oh = orow + hq * hd;
        for (int j = 0; j < base; j++) {
          const float* vt = pv + (size_t)j * kvd + kvh * hd;
          float p = scores[j];
          for (int di = 0; di < hd; di++) oh[di] += p * vt[di];
        }
        for (int j = 0; j < b; j++) {
          const float* vt = bv + (size_t)j * kvd + kvh * hd;
          float p = scores[base + j];
          for (int di = 0; di < hd; di++) oh[di] += p * vt[di];
        }
      }
    }
    L.attn_output.matmul(o.data(), proj, b);
  }

  // model.rs:472-510 (run_block): b residual rows at positions base.. against the frozen prefix of
  // `cache` (which is not modified). logits (may be null): [b][vocab] through output.matmul.
  // bk / bv: [n_layers][b * kv_dim] block K / V, appended by the caller when the block is final.
  void run_block(const float* inputs, int b, const KvCache& cache, int base, float* logits,
                 std::vector<std::vector<float>>& bk, std::vector<std::vector<float>>& bv) const {
    const Config& c = cfg;
    int d = c.d_model, kvd = c.kv_dim();
    if (cache.len < base) throw Error("run_block base beyond the cached prefix");
    std::vector<float> x(inputs, inputs + (size_t)b * d), h((size_t)b * d), tmp((size_t)b * d);
    bk.assign(c.n_layers, std::vector<float>((size_t)b * kvd));
    bv.assign(c.n_layers, std::vector<float>((size_t)b * kvd));
    for (int li = 0; li < c.n_layers; li++) {
      const Layer& L = layers[li];
#pragma omp parallel for schedule(static)
      for (int t = 0; t < b; t++)
        rmsnorm(&x[(size_t)t * d], L.attn_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
      attn_block_cached(L, h.data(), li, cache, base, b, tmp.data(), bk[li].data(), bv[li].data());
      for (size_t i = 0; i < (size_t)b * d; i++) x[i] += tmp[i];
#pragma omp parallel for schedule(static)
      for (int t = 0; t < b; t++)
        rmsnorm(&x[(size_t)t * d], L.ffn_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
      ffn_prefill(L, h.data(), b, tmp.data());
      for (size_t i = 0; i < (size_t)b * d; i++) x[i] += tmp[i];
    }
    if (!logits) return;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < b; t++) rmsnorm(&x[(size_t)t * d], output_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
    output.matmul(h.data(), logits, b);
  }

  // model.rs:589-640 (attn_bidir): every query attends to every key, RoPE at position t, no cache.
  void attn_bidir(const Layer& L, const float* h, int tn, float* proj) const {
    const Config& c = cfg;
    int hd = c.head_dim, qd = c.q_dim(), kvd = c.kv_dim(), qw = qd + 2 * kvd, rep = c.n_heads / c.n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    std::vector<float> qkv((size_t)tn * qw);
    L.attn_qkv.matmul(h, qkv.data(), tn);
    qk_norm_rope_rows(L, qkv.data(), tn, 0);
    std::vector<float> kbuf((size_t)tn * kvd), vbuf((size_t)tn * kvd);
    for (int t = 0; t < tn; t++) {
      const float* row = qkv.data() + (size_t)t * qw;
      memcpy(&kbuf[(size_t)t * kvd], row + qd, kvd * 4);
      memcpy(&vbuf[(size_t)t * kvd], row + qd + kvd, kvd * 4);
    }
    std::vector<float> o((size_t)tn * qd, 0.0f);
#pragma omp parallel for schedule(dynamic, 2)
    for (int t = 0; t < tn; t++) {
      const float* qrow = qkv.data() + (size_t)t * qw;
      std::vector<float> scores(tn);
      float* orow = o.data() + (size_t)t * qd;
      for (int hq = 0; hq < c.n_heads; hq++) {
        int kvh = hq / rep;
        const float* qh = qrow + hq * hd;
        for (int j = 0; j < tn; j++) scores[j] = dot(qh, &kbuf[(size_t)j * kvd + kvh * hd], hd) * scale;
        softmax(scores.data(), tn);
        float* oh = orow + hq * hd;
        for (int j = 0; j < tn; j++) {
          const float* vt = &vbuf[(size_t)j * kvd + kvh * hd];
          float p = scores[j];
          for (int di = 0; di < hd; di++) oh[di] += p * vt[di];
        }
      }
    }
    L.attn_output.matmul(o.data(), proj, tn);
  }

  // model.rs:441-470 (forward_bidir): logits [tn][vocab] of every position of a bidirectional pass.
  void forward_bidir(const float* inputs, int tn, float* logits) const {
    const Config& c = cfg;
    int d = c.d_model;
    std::vector<float> x(inputs, inputs + (size_t)tn * d), h((size_t)tn * d), tmp((size_t)tn * d);
    for (int li = 0; li < c.n_layers; li++) {
      const Layer& L = layers[li];
#pragma omp parallel for schedule(static)
      for (int t = 0; t < tn; t++)
        rmsnorm(&x[(size_t)t * d], L.attn_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
      attn_bidir(L, h.data(), tn, tmp.data());
      for (size_t i = 0; i < (size_t)tn * d; i++) x[i] += tmp[i];
#pragma omp parallel for schedule(static)
      for (int t = 0; t < tn; t++)
        rmsnorm(&x[(size_t)t * d], L.ffn_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
      ffn_prefill(L, h.data(), tn, tmp.data());
      for (size_t i = 0; i < (size_t)tn * d; i++) x[i] += tmp[i];
    }
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tn; t++) rmsnorm(&x[(size_t)t * d], output_norm.data(), c.rms_eps, &h[(size_t)t * d], d);
    output.matmul(h.data(), logits, tn);
  }
};

// sample.rs
struct Rng {
  uint64_t s;
  explicit Rng(uint64_t seed) : s(seed < 1 ? 1 : seed) {}
  uint64_t next_u64() {
    uint64_t x = s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    s = x;
    return x * 0x2545F4914F6CDD1Dull;
  }
  float next_f32() { return (float)(next_u64() >> 40) / (float)(1ull << 24); }
};
static uint32_t argmax(const float* v, int n) {  // sample.rs:53-64
  int best = 0;
  float bv = -INFINITY;
  for (int i = 0; i < n; i++)
    if (v[i] > bv) {
      bv = v[i];
      best = i;
    }
  return (uint32_t)best;
}
static uint32_t sample(const float* logits, int n, float temp, float top_p, Rng& rng) {  // sample.rs:66-112
  if (temp <= 0.0f) return argmax(logits, n);
  std::vector<std::pair<int, float>> probs(n);
  for (int i = 0; i < n; i++) probs[i] = {i, logits[i] / temp};
  float m = -INFINITY;
  for (auto& p : probs) m = fmaxf(m, p.second);
  float sum = 0.0f;
  for (auto& p : probs) {
    p.second = fexp(p.second - m);
    sum += p.second;
  }
  for (auto& p : probs) p.second /= sum;
  if (top_p > 0.0f && top_p < 1.0f) {
    std::stable_sort(probs.begin(), probs.end(),
                     [](const std::pair<int, float>& a, const std::pair<int, float>& b) { return a.second > b.second; });
    float cum = 0.0f;
    size_t cut = probs.size();
    for (size_t i = 0; i < probs.size(); i++) {
      cum += probs[i].second;
      if (cum >= top_p) {
        cut = i + 1;
        break;
      }
    }
    probs.resize(cut);
    float s = -0.0f;
    for (auto& p : probs) s = s + p.second;
    for (auto& p : probs) p.second /= s;
  }
  float r = rng.next_f32();
  float cum = 0.0f;
  for (auto& p : probs) {
    cum += p.second;
    if (r < cum) return (uint32_t)p.first;
  }
  return probs.empty() ? 0 : (uint32_t)probs.back().first;
}

struct Engine {
  Gguf g;
  Config cfg;
  Model model;
  uint32_t eos = 50256;
};

// sample.rs:29-47: Gumbel-max over the finite logits; temp <= 0 is the plain argmax.
static uint32_t gumbel_argmax(const float* logits, int n, float temp, Rng& rng) {
  if (temp <= 0.0f) return argmax(logits, n);
  int best = 0;
  float bv = -INFINITY;
  for (int i = 0; i < n; i++) {
    float l = logits[i];
    if (!std::isfinite(l)) continue;
    float u = std::clamp(rng.next_f32(), 1e-9f, 1.0f - 1e-9f);
    float val = l / temp + -flog(-flog(u));
    if (val > bv) {
      bv = val;
      best = i;
    }
  }
  return (uint32_t)best;
}

// lib.rs:66-73: n unmask events spread over `steps` (sums to n).
static std::vector<int> num_transfer(int n, int steps) {
  int base = n / steps;
  std::vector<int> out(steps, base);
  for (int i = 0; i < n - base * steps; i++) out[i] += 1;
  return out;
}

// DiffOpts (lib.rs:43-63).
struct DiffOpts {
  int gen_len = 128, block = 32, steps = 32;
  float temp = 0.0f, rep_penalty = 1.4f;
  int remask_steps = 0;
  float remask_frac = 0.3f;
  uint64_t seed = 1234;
  bool cached = true;
  float threshold = 0.0f;
};

// lib.rs:221-263 (score_block): per block row, ids >= valid banned, the presence penalty over the
// committed ids and the block's own non-mask ids, a Gumbel / greedy pick, and the softmax
// probabilities of the pick (pconf) and of the row's current id (cconf).
static void score_block(const float* all, int V, const uint32_t* blk, int blk_len, const uint32_t* committed,
                        int n_committed, int valid, uint32_t mask, float rep_penalty, float temp, Rng& rng,
                        uint32_t* pred, float* pconf, float* cconf) {
  std::vector<char> present(valid, 0);
  if (rep_penalty != 1.0f) {
    for (int i = 0; i < n_committed + blk_len; i++) {
      uint32_t id = i < n_committed ? committed[i] : blk[i - n_committed];
      if (id != mask && (int64_t)id < valid) present[id] = 1;
    }
  }
  std::vector<float> row(V);
  for (int i = 0; i < blk_len; i++) {
    memcpy(row.data(), all + (size_t)i * V, (size_t)V * 4);
    for (int l = valid; l < V; l++) row[l] = -INFINITY;
    if (rep_penalty != 1.0f)
      for (int t = 0; t < valid; t++)
        if (present[t]) {
          float l = row[t];
          row[t] = l > 0.0f ? l / rep_penalty : l * rep_penalty;
        }
    uint32_t p = gumbel_argmax(row.data(), V, temp, rng);
    softmax(row.data(), V);
    pred[i] = p;
    pconf[i] = row[p];
    cconf[i] = row[blk[i]];
  }
}

static void embed_rows(const Engine& e, const uint32_t* ids, int n, std::vector<float>& out) {
  const int d = e.cfg.d_model;
  out.resize((size_t)n * d);
  for (int t = 0; t < n; t++) {
    if ((int64_t)ids[t] >= e.cfg.vocab_size) throw Error("token id out of range");
    memcpy(&out[(size_t)t * d], &e.model.token_embd[(size_t)ids[t] * d], d * 4);
  }
}

// lib.rs:265-407 (generate_diffusion_cached) over token ids; the per-block text stream becomes
// the committed ids up to the first eos. Returns the generated count; out receives the ids.
static int diffusion_cached(Engine& e, const uint32_t* prompt, int p, const DiffOpts& o, std::vector<uint32_t>& out) {
  const Config& c = e.cfg;
  const int V = c.vocab_size, valid = std::min(50257, V);
  const uint32_t mask = (uint32_t)c.mask_token_id;
  Rng rng(o.seed);
  out.clear();
  if (p == 0) return 0;
  const int gen_len = std::min(o.gen_len, std::max(c.context_length - (p + o.block), 1));
  KvCache cache;
  e.model.new_cache(cache);
  std::vector<float> rows;
  std::vector<std::vector<float>> bk, bv;
  embed_rows(e, prompt, p, rows);
  e.model.run_block(rows.data(), p, cache, 0, nullptr, bk, bv);
  for (int li = 0; li < c.n_layers; li++) {
    cache.k[li].insert(cache.k[li].end(), bk[li].begin(), bk[li].end());
    cache.v[li].insert(cache.v[li].end(), bv[li].begin(), bv[li].end());
  }
  cache.len = p;
  std::vector<uint32_t> committed(prompt, prompt + p);
  int b0 = p;
  while (b0 < p + gen_len) {
    const int b1 = std::min(b0 + o.block, p + gen_len), blk_len = b1 - b0, base = b0;
    std::vector<uint32_t> blk(blk_len, mask), pred(blk_len);
    std::vector<float> all((size_t)blk_len * V), pconf(blk_len), cconf(blk_len);
    auto step = [&]() {
      embed_rows(e, blk.data(), blk_len, rows);
      e.model.run_block(rows.data(), blk_len, cache, base, all.data(), bk, bv);
      score_block(all.data(), V, blk.data(), blk_len, committed.data(), (int)committed.size(), valid, mask,
                  o.rep_penalty, o.temp, rng, pred.data(), pconf.data(), cconf.data());
    };
    auto any_masked = [&]() { return std::find(blk.begin(), blk.end(), mask) != blk.end(); };
    if (o.threshold > 0.0f) {
      for (int it = 0; it < std::max(blk_len, 1); it++) {
        if (!any_masked()) break;
        step();
        bool any = false;
        int best = -1;
        for (int i = 0; i < blk_len; i++) {
          if (blk[i] != mask) continue;
          if (best < 0 || !(pconf[i] < pconf[best])) best = i;  // Iterator::max_by keeps the last maximum
        }
        for (int i = 0; i < blk_len; i++)
          if (blk[i] == mask && pconf[i] >= o.threshold) {
            blk[i] = pred[i];
            any = true;
          }
        if (!any) blk[best] = pred[best];
      }
    } else {
      const int sb = std::max((int)roundf((float)(o.steps * blk_len) / (float)gen_len), 1);
      for (int k_step : num_transfer(blk_len, sb)) {
        step();
        std::vector<std::pair<int, float>> cand;
        for (int i = 0; i < blk_len; i++)
          if (blk[i] == mask) cand.push_back({i, pconf[i]});
        if (cand.empty()) break;
        std::stable_sort(cand.begin(), cand.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
        for (int r = 0; r < std::min(k_step, (int)cand.size()); r++) blk[cand[r].first] = pred[cand[r].first];
      }
      if (any_masked()) {
        step();
        for (int i = 0; i < blk_len; i++)
          if (blk[i] == mask) blk[i] = pred[i];
      }
    }
    for (int it = 0; it < o.remask_steps; it++) {
      step();
      const int r = std::max((int)((float)blk_len * o.remask_frac), 1);
      std::vector<std::pair<int, float>> idx(blk_len);
      for (int i = 0; i < blk_len; i++) idx[i] = {i, cconf[i]};
      std::stable_sort(idx.begin(), idx.end(), [](const auto& a, const auto& b) { return a.second < b.second; });
      for (int q = 0; q < std::min(r, blk_len); q++) blk[idx[q].first] = mask;
      step();
      for (int i = 0; i < blk_len; i++)
        if (blk[i] == mask) blk[i] = pred[i];
    }
    // finalize: the block's K / V join the cache
    embed_rows(e, blk.data(), blk_len, rows);
    e.model.run_block(rows.data(), blk_len, cache, base, nullptr, bk, bv);
    for (int li = 0; li < c.n_layers; li++) {
      cache.k[li].insert(cache.k[li].end(), bk[li].begin(), bk[li].end());
      cache.v[li].insert(cache.v[li].end(), bv[li].begin(), bv[li].end());
    }
    cache.len = b1;
    committed.insert(committed.end(), blk.begin(), blk.end());
    int endpos = (int)committed.size();
    bool hit = false;
    for (int i = p; i < (int)committed.size(); i++)
      if (committed[i] == e.eos) {
        endpos = i;
        hit = true;
        break;
      }
    out.assign(committed.begin() + p, committed.begin() + endpos);
    if (hit) return endpos - p;
    b0 = b1;
  }
  return gen_len;
}

// lib.rs:409-495 (generate_diffusion_uncached): every step re-runs the canvas x[0..b1]
// bidirectionally (diffusion_block, lib.rs:164-209).
static int diffusion_uncached(Engine& e, const uint32_t* prompt, int p, const DiffOpts& o,
                              std::vector<uint32_t>& out) {
  const Config& c = e.cfg;
  const int V = c.vocab_size, valid = std::min(50257, V);
  const uint32_t mask = (uint32_t)c.mask_token_id;
  Rng rng(o.seed);
  out.clear();
  const int gen_len = std::min(o.gen_len, std::max(c.context_length - p, 1));
  std::vector<uint32_t> x(prompt, prompt + p);
  x.resize((size_t)p + gen_len, mask);
  std::vector<float> rows, all;
  int b0 = p;
  while (b0 < p + gen_len) {
    const int b1 = std::min(b0 + o.block, p + gen_len), blk_len = b1 - b0;
    std::vector<uint32_t> pred(blk_len);
    std::vector<float> pconf(blk_len), cconf(blk_len);
    auto step = [&]() {
      embed_rows(e, x.data(), b1, rows);
      all.resize((size_t)b1 * V);
      e.model.forward_bidir(rows.data(), b1, all.data());
      score_block(all.data() + (size_t)b0 * V, V, x.data() + b0, blk_len, x.data(), b0, valid, mask, o.rep_penalty,
                  o.temp, rng, pred.data(), pconf.data(), cconf.data());
    };
    const int sb = std::max((int)roundf((float)(o.steps * blk_len) / (float)gen_len), 1);
    for (int k_step : num_transfer(blk_len, sb)) {
      step();
      std::vector<std::pair<int, float>> cand;
      for (int i = 0; i < blk_len; i++)
        if (x[b0 + i] == mask) cand.push_back({i, pconf[i]});
      if (cand.empty()) break;
      std::stable_sort(cand.begin(), cand.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
      for (int r = 0; r < std::min(k_step, (int)cand.size()); r++) x[b0 + cand[r].first] = pred[cand[r].first];
    }
    bool any = false;
    for (int i = 0; i < blk_len; i++) any = any || x[b0 + i] == mask;
    if (any) {
      step();
      for (int i = 0; i < blk_len; i++)
        if (x[b0 + i] == mask) x[b0 + i] = pred[i];
    }
    for (int it = 0; it < o.remask_steps; it++) {
      step();
      const int r = std::max((int)((float)blk_len * o.remask_frac), 1);
      std::vector<std::pair<int, float>> idx(blk_len);
      for (int i = 0; i < blk_len; i++) idx[i] = {i, cconf[i]};
      std::stable_sort(idx.begin(), idx.end(), [](const auto& a, const auto& b) { return a.second < b.second; });
      for (int q = 0; q < std::min(r, blk_len); q++) x[b0 + idx[q].first] = mask;
      step();
      for (int i = 0; i < blk_len; i++)
        if (x[b0 + i] == mask) x[b0 + i] = pred[i];
    }
    int endpos = b1;
    bool hit = false;
    for (int i = p; i < b1; i++)
      if (x[i] == e.eos) {
        endpos = i;
        hit = true;
        break;
      }
    out.assign(x.begin() + p, x.begin() + endpos);
    if (hit) return endpos - p;
    b0 = b1;
  }
  return gen_len;
}

}  // namespace hor

using namespace hor;

// ---------------------------------------------------------------------------------------------
// C API (ctypes). Every entry returns 0 on success, -1 on error (message in hor_last_error()).
// ---------------------------------------------------------------------------------------------
#define HOR_TRY(...)                  \
  try {                               \
    __VA_ARGS__;                      \
    return 0;                         \
  } catch (const std::exception& e) { \
    g_err = e.what();                 \
    return -1;                        \
  }

extern "C" {

const char* hor_last_error() { return g_err.c_str(); }
void hor_set_exp_mode(int m) { g_exp_mode = m; }
int hor_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
void hor_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

// lib.rs:85-92 (quant: 1 = Q8 re-quantization as `--quant q8`, 0 = F32 as `--quant f32`)
int hor_engine_load(const char* path, int quant, void** out) {
  HOR_TRY({
    Engine* e = new Engine();
    try {
      e->g.open(path);
      e->cfg = config_from_gguf(e->g);
      uint32_t eos;
      if (e->g.get_u32("tokenizer.ggml.eos_token_id", &eos)) e->eos = eos;
      e->model.load(e->g, e->cfg, quant != 0);
    } catch (...) {
      delete e;
      throw;
    }
    *out = e;
  })
}
void hor_engine_free(void* e) { delete (Engine*)e; }

// int fields: d_model n_layers n_dense n_heads n_kv_heads head_dim dense_ffn expert_ffn n_experts
// top_k n_shared vocab_size context_length expert_weights_norm gating_sigmoid eos diffusion
// mask_token_id block_size ; floats: rms_eps rope_theta expert_weights_scale
int hor_engine_config(void* ep, int32_t* ints, float* floats) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    const Config& c = e->cfg;
    int32_t v[19] = {c.d_model, c.n_layers, c.n_dense, c.n_heads, c.n_kv_heads, c.head_dim,
                     c.dense_ffn, c.expert_ffn, c.n_experts, c.top_k, c.n_shared, c.vocab_size,
                     c.context_length, (int)c.expert_weights_norm, (int)c.gating_sigmoid, (int)e->eos,
                     (int)c.diffusion, c.mask_token_id, c.block_size};
    memcpy(ints, v, sizeof(v));
    floats[0] = c.rms_eps;
    floats[1] = c.rope_theta;
    floats[2] = c.expert_weights_scale;
  })
}
uint64_t hor_engine_weight_bytes(void* ep) { return ((Engine*)ep)->model.weight_bytes(); }

int hor_cache_new(void* ep, void** out) {
  HOR_TRY({
    KvCache* kc = new KvCache();
    ((Engine*)ep)->model.new_cache(*kc);
    *out = kc;
  })
}
void hor_cache_free(void* c) { delete (KvCache*)c; }
int hor_cache_len(void* c) { return ((KvCache*)c)->len; }

// Raw per-layer K/V rows of the cache ([len][kv_dim] each), for comparisons.
int hor_cache_read(void* cp, int layer, float* k_out, float* v_out) {
  HOR_TRY({
    KvCache* kc = (KvCache*)cp;
    if (layer < 0 || layer >= (int)kc->k.size()) throw Error("layer out of range");
    memcpy(k_out, kc->k[layer].data(), kc->k[layer].size() * 4);
    memcpy(v_out, kc->v[layer].data(), kc->v[layer].size() * 4);
  })
}

// Model::prefill on token ids (embedding rows as inputs, lib.rs:118-126).
int hor_prefill(void* ep, void* cp, const uint32_t* ids, int n, float* logits) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    int d = e->cfg.d_model;
    if (n <= 0) throw Error("empty prefill");
    std::vector<float> in((size_t)n * d);
    for (int t = 0; t < n; t++) {
      if ((int64_t)ids[t] >= e->cfg.vocab_size) throw Error("token id out of range");
      memcpy(&in[(size_t)t * d], &e->model.token_embd[(size_t)ids[t] * d], d * 4);
    }
    e->model.prefill(in.data(), n, *(KvCache*)cp, logits);
  })
}

// Model::prefill (model.rs:340-370) on caller rows (n x d_model): the inputs lib.rs:118-121 builds
// from spliced modality embeddings and token embeddings.
int hor_prefill_embeds(void* ep, void* cp, const float* rows, int n, float* logits) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    if (n <= 0) throw Error("empty prefill");
    e->model.prefill(rows, n, *(KvCache*)cp, logits);
  })
}

// Model::forward_x (model.rs:160-184) from a caller row of d_model floats.
int hor_forward_x(void* ep, void* cp, const float* row, int pos, float* logits) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    e->model.forward_x(std::vector<float>(row, row + e->cfg.d_model), pos, *(KvCache*)cp, logits);
  })
}

int hor_forward(void* ep, void* cp, uint32_t token, int pos, float* logits) {
  HOR_TRY({ ((Engine*)ep)->model.forward(token, pos, *(KvCache*)cp, logits); })
}

// Routing of the last forward(): [n_layers][top_k] ids (-1 for dense layers) and gate weights.
// Model::run_block (model.rs:472-510) of n token ids at base = cache length: logits (may be null)
// [n][vocab]; commit != 0 appends the block's K / V to the cache as lib.rs:386-391 does.
int hor_run_block(void* ep, void* cp, const uint32_t* ids, int n, int commit, float* logits) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    KvCache& cache = *(KvCache*)cp;
    std::vector<float> rows;
    std::vector<std::vector<float>> bk, bv;
    embed_rows(*e, ids, n, rows);
    e->model.run_block(rows.data(), n, cache, cache.len, logits, bk, bv);
    if (commit) {
      for (int li = 0; li < e->cfg.n_layers; li++) {
        cache.k[li].insert(cache.k[li].end(), bk[li].begin(), bk[li].end());
        cache.v[li].insert(cache.v[li].end(), bv[li].begin(), bv[li].end());
      }
      cache.len += n;
    }
  })
}

// Model::forward_bidir (model.rs:441-470) of n token ids: logits [n][vocab].
int hor_forward_bidir(void* ep, const uint32_t* ids, int n, float* logits) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    std::vector<float> rows;
    embed_rows(*e, ids, n, rows);
    e->model.forward_bidir(rows.data(), n, logits);
  })
}

// Engine::generate_diffusion (lib.rs:211-220) on token ids. out_ids: room for gen_len ids; the
// generated count is written to *n_out.
int hor_generate_diffusion(void* ep, const uint32_t* ids, int n, int gen_len, int block, int steps, float temp,
                           float rep_penalty, int remask_steps, float remask_frac, uint64_t seed, int cached,
                           float threshold, uint32_t* out_ids, int* n_out) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    DiffOpts o;
    o.gen_len = gen_len;
    o.block = block > 0 ? block : std::max(e->cfg.block_size, 1);
    o.steps = steps;
    o.temp = temp;
    o.rep_penalty = rep_penalty;
    o.remask_steps = remask_steps;
    o.remask_frac = remask_frac;
    o.seed = seed;
    o.cached = cached != 0;
    o.threshold = threshold;
    std::vector<uint32_t> out;
    int cnt = o.cached ? diffusion_cached(*e, ids, n, o, out) : diffusion_uncached(*e, ids, n, o, out);
    std::copy(out.begin(), out.end(), out_ids);
    *n_out = cnt;
  })
}

// sample.rs:66-112 over n logits with the xorshift64* state in *state (advanced).
int hor_sample(const float* logits, int n, float temp, float top_p, uint64_t* state, uint32_t* out) {
  HOR_TRY({
    Rng rng(*state);
    *out = sample(logits, n, temp, top_p, rng);
    *state = rng.s;
  })
}

// lib.rs:221-263 (score_block) over blk_len rows of vocab logits, valid = min(50257, vocab).
int hor_score_block(const float* logits, int vocab, const uint32_t* blk, int blk_len, const uint32_t* committed,
                    int n_committed, uint32_t mask, float rep_penalty, float temp, uint64_t* state, uint32_t* pred,
                    float* pconf, float* cconf) {
  HOR_TRY({
    Rng rng(*state);
    score_block(logits, vocab, blk, blk_len, committed, n_committed, std::min(50257, vocab), mask, rep_penalty, temp,
                rng, pred, pconf, cconf);
    *state = rng.s;
  })
}

int hor_last_routing(void* ep, int32_t* sel, float* w) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    memcpy(sel, e->model.last_sel.data(), e->model.last_sel.size() * 4);
    if (w) memcpy(w, e->model.last_selw.data(), e->model.last_selw.size() * 4);
  })
}

// Engine::generate on token ids (lib.rs:107-162). Writes generated ids to out_ids (max_new), the
// logits each sampled token was chosen from to out_logits ([max_new][vocab], may be null), and the
// wall time of the forward() calls to *forward_s. Returns the count via *n_out.
static int generate_rows(Engine* e, const float* rows, int n_rows, const uint32_t* ids, int n, int max_new,
                         float temp, float top_p, uint64_t seed, float rep_penalty, uint32_t* out_ids,
                         float* out_logits, int* n_out, double* forward_s, double* prefill_s) {
  HOR_TRY({
    const Config& c = e->cfg;
    int V = c.vocab_size, d = c.d_model;
    *n_out = 0;
    if (forward_s) *forward_s = 0;
    if (n + n_rows <= 0) return 0;  // lib.rs:122-124
    KvCache cache;
    e->model.new_cache(cache);
    Rng rng(seed);
    // lib.rs:118-121: the caller's rows first, then the prompt's token embeddings
    std::vector<float> in((size_t)(n_rows + n) * d), logits(V);
    if (n_rows > 0) memcpy(in.data(), rows, (size_t)n_rows * d * 4);
    for (int t = 0; t < n; t++) {
      if ((int64_t)ids[t] >= V) throw Error("token id out of range");
      memcpy(&in[(size_t)(n_rows + t) * d], &e->model.token_embd[(size_t)ids[t] * d], d * 4);
    }
    n += n_rows;
    int pos = n;
    auto t0 = std::chrono::steady_clock::now();
    e->model.prefill(in.data(), n, cache, logits.data());
    if (prefill_s) *prefill_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    int valid = std::min(50257, V);
    std::vector<uint32_t> outv;
    double fs = 0;
    for (int it = 0; it < max_new; it++) {
      for (int i = valid; i < V; i++) logits[i] = -INFINITY;
      if (rep_penalty != 1.0f)
        for (uint32_t t : outv) {
          float& l = logits[t];
          l = l > 0.0f ? l / rep_penalty : l * rep_penalty;
        }
      if (out_logits) memcpy(out_logits + (size_t)it * V, logits.data(), (size_t)V * 4);
      uint32_t next = sample(logits.data(), V, temp, top_p, rng);
      if (next == e->eos) break;
      outv.push_back(next);
      out_ids[outv.size() - 1] = next;
      if (pos + 1 >= c.context_length) break;
      auto t1 = std::chrono::steady_clock::now();
      e->model.forward(next, pos, cache, logits.data());
      fs += std::chrono::duration<double>(std::chrono::steady_clock::now() - t1).count();
      pos += 1;
    }
    *n_out = (int)outv.size();
    if (forward_s) *forward_s = fs;
  })
}

int hor_generate(void* ep, const uint32_t* ids, int n, int max_new, float temp, float top_p, uint64_t seed,
                 float rep_penalty, uint32_t* out_ids, float* out_logits, int* n_out, double* forward_s,
                 double* prefill_s) {
  if (n <= 0) {
    *n_out = 0;
    if (forward_s) *forward_s = 0;
    return 0;
  }
  return generate_rows((Engine*)ep, nullptr, 0, ids, n, max_new, temp, top_p, seed, rep_penalty, out_ids, out_logits,
                       n_out, forward_s, prefill_s);
}

// Engine::generate with `embeds` (lib.rs:107-126): n_rows caller rows of d_model floats precede the
// prompt ids' embeddings in one prefill.
int hor_generate_embeds(void* ep, const float* rows, int n_rows, const uint32_t* ids, int n, int max_new, float temp,
                        float top_p, uint64_t seed, float rep_penalty, uint32_t* out_ids, int* n_out) {
  return generate_rows((Engine*)ep, rows, n_rows, ids, n, max_new, temp, top_p, seed, rep_penalty, out_ids, nullptr,
                       n_out, nullptr, nullptr);
}

// Append synthetic K/V rows ([n][kv_dim] per layer, all layers share the arrays) to a cache, for
// timing decode at a chosen context length without a CPU prefill.
int hor_cache_fill(void* ep, void* cp, const float* k, const float* v, int n) {
  HOR_TRY({
    Engine* e = (Engine*)ep;
    KvCache* kc = (KvCache*)cp;
    size_t m = (size_t)n * e->cfg.kv_dim();
    for (int l = 0; l < e->cfg.n_layers; l++) {
      kc->k[l].insert(kc->k[l].end(), k, k + m);
      kc->v[l].insert(kc->v[l].end(), v, v + m);
    }
    kc->len += n;
  })
}

// ---- op level ------------------------------------------------------------------------------
int hor_q8_quantize(const float* w, int out, int in, int8_t* qs, float* scales) {
  HOR_TRY({
    Q8Tensor t;
    t.quantize(w, out, in);
    memcpy(qs, t.qs.data(), t.qs.size());
    memcpy(scales, t.scales.data(), t.scales.size() * 4);
  })
}
// Activation quantization of one row (quant.rs:112-123).
int hor_q8_quant_act(const float* x, int n, int8_t* qx, float* dx) {
  HOR_TRY({
    if (n % 32) throw Error("n % 32 != 0");
    for (int b = 0; b < n / 32; b++) quant_block(x + b * 32, qx + b * 32, dx + b);
  })
}
int hor_q8_matvec(const int8_t* qs, const float* scales, int out, int in, const float* x, float* y) {
  HOR_TRY({
    Q8Tensor t;
    t.out = out;
    t.in = in;
    t.nb = in / 32;
    t.qs.assign(qs, qs + (size_t)out * in);
    t.scales.assign(scales, scales + (size_t)out * t.nb);
    t.matvec(x, y);
  })
}
int hor_q8_matmul(const int8_t* qs, const float* scales, int out, int in, const float* x, float* y, int tn) {
  HOR_TRY({
    Q8Tensor t;
    t.out = out;
    t.in = in;
    t.nb = in / 32;
    t.qs.assign(qs, qs + (size_t)out * in);
    t.scales.assign(scales, scales + (size_t)out * t.nb);
    t.matmul(x, y, tn);
  })
}
int hor_dequant(int type, const uint8_t* b, size_t n, float* y) {
  HOR_TRY({
    switch (type) {
      case 1: dequant_f16(b, n, y); break;
      case 6: dequant_q5_0(b, n, y); break;
      case 8: dequant_q8_0(b, n, y); break;
      case 12: dequant_q4_k(b, n, y); break;
      case 14: dequant_q6_k(b, n, y); break;
      default: throw Error("unsupported type");
    }
  })
}
float hor_dot(const float* a, const float* b, int n) { return dot(a, b, n); }
void hor_rmsnorm(const float* x, const float* w, float eps, float* out, int n) { rmsnorm(x, w, eps, out, n); }
float hor_expf(float x) { return fexp(x); }
float hor_sigmoid(float x) { return sigmoid(x); }
float hor_silu(float x) { return silu(x); }

// Standalone MoE layer (an Ffn::Moe) built from raw arrays, for the op-level config. Expert
// tensors are f32 in GGUF stacked order ([E][rows][cols]) and are re-quantized exactly as Model::load.
struct MoeOp {
  Config c;
  Layer L;
};
int hor_moe_create(int d, int f, int ne, int top_k, int n_shared, int gating_sigmoid, int weights_norm,
                   float weights_scale, const float* router, const float* bias, const float* gate_exps,
                   const float* up_exps, const float* down_exps, const float* gate_sh, const float* up_sh,
                   const float* down_sh, void** out) {
  HOR_TRY({
    MoeOp* op = new MoeOp();
    Config& c = op->c;
    c.d_model = d;
    c.expert_ffn = f;
    c.n_experts = ne;
    c.top_k = top_k;
    c.n_shared = n_shared;
    c.gating_sigmoid = gating_sigmoid != 0;
    c.expert_weights_norm = weights_norm != 0;
    c.expert_weights_scale = weights_scale;
    Layer& L = op->L;
    L.moe = true;
    L.m.gate_inp.build(std::vector<float>(router, router + (size_t)ne * d), ne, d, false);
    L.m.bias.assign(bias, bias + ne);
    auto split = [&](std::vector<Mat>& v, const float* src, int a, int b) {
      v.resize(ne);
      for (int e = 0; e < ne; e++)
        v[e].build(std::vector<float>(src + (size_t)e * a * b, src + (size_t)(e + 1) * a * b), a, b, true);
    };
    split(L.m.gate_exps, gate_exps, f, d);
    split(L.m.up_exps, up_exps, f, d);
    split(L.m.down_exps, down_exps, d, f);
    if (n_shared > 0) {
      L.m.gate_sh.build(std::vector<float>(gate_sh, gate_sh + (size_t)f * d), f, d, true);
      L.m.up_sh.build(std::vector<float>(up_sh, up_sh + (size_t)f * d), f, d, true);
      L.m.down_sh.build(std::vector<float>(down_sh, down_sh + (size_t)d * f), d, f, true);
    }
    *out = op;
  })
}
void hor_moe_free(void* p) { delete (MoeOp*)p; }
// mode 0: per-token ffn (decode, model.rs:256-324); mode 1: ffn_prefill over all T (model.rs:671-747).
// sel (optional, [T][top_k]) receives the routing of each token (mode 0 and 1 alike).
int hor_moe_run(void* p, const float* x, int T, int mode, float* y, int32_t* sel, float* selw) {
  HOR_TRY({
    MoeOp* op = (MoeOp*)p;
    const Config& c = op->c;
    int d = c.d_model, ne = c.n_experts;
    if (sel || selw) {
      std::vector<float> logits(ne);
      std::vector<int> tk(c.top_k);
      std::vector<float> w(c.top_k);
      for (int t = 0; t < T; t++) {
        op->L.m.gate_inp.matvec(x + (size_t)t * d, logits.data());
        route(c, logits.data(), op->L.m.bias.data(), tk.data(), w.data());
        for (int r = 0; r < c.top_k; r++) {
          if (sel) sel[(size_t)t * c.top_k + r] = tk[r];
          if (selw) selw[(size_t)t * c.top_k + r] = w[r];
        }
      }
    }
    Model m;  // only cfg is used by ffn / ffn_prefill
    m.cfg = c;
    if (mode == 0) {
      for (int t = 0; t < T; t++) m.ffn(op->L, x + (size_t)t * d, y + (size_t)t * d, -1);
    } else {
      m.ffn_prefill(op->L, x, T, y);
    }
  })
}
// One expert's SwiGLU output on one normed row (model.rs:300-305 for e >= 0, 313-318 for the shared
// expert, e = -1), unscaled: the unit of work an expert-parallel rank computes for another.
int hor_moe_expert(void* p, const float* x, int e, float* y) {
  HOR_TRY({
    MoeOp* op = (MoeOp*)p;
    const Config& c = op->c;
    const int f = c.expert_ffn;
    if (e < -1 || e >= c.n_experts || (e == -1 && c.n_shared == 0)) throw Error("bad expert");
    std::vector<float> gb(f), ub(f);
    const Mat& G = e < 0 ? op->L.m.gate_sh : op->L.m.gate_exps[e];
    const Mat& U = e < 0 ? op->L.m.up_sh : op->L.m.up_exps[e];
    const Mat& Dn = e < 0 ? op->L.m.down_sh : op->L.m.down_exps[e];
    G.matvec(x, gb.data());
    U.matvec(x, ub.data());
    for (int i = 0; i < f; i++) gb[i] = silu(gb[i]) * ub[i];
    Dn.matvec(gb.data(), y);
  })
}
// Router selection scores (sigmoid(W_r x) + bias) for one token, for margin reporting.
int hor_moe_sel_scores(void* p, const float* x, float* sel_scores) {
  HOR_TRY({
    MoeOp* op = (MoeOp*)p;
    const Config& c = op->c;
    std::vector<float> logits(c.n_experts);
    op->L.m.gate_inp.matvec(x, logits.data());
    for (int e = 0; e < c.n_experts; e++)
      sel_scores[e] = (c.gating_sigmoid ? sigmoid(logits[e]) : logits[e]) + op->L.m.bias[e];
  })
}

// One decode attention step of a single layer (model.rs:199-233 without the two matvecs):
// qkv ([q_dim + 2 kv_dim], pre-norm) is QK-normed and roped at `pos`, k/v are appended to the
// cache rows (k_cache/v_cache hold `pos` rows of [kv_dim] and room for one more), and the
// attention output ([q_dim]) is written to out. rope tables: [max_pos][hd/2] built by Rope::new.
struct RopeOp {
  Rope r;
};
int hor_rope_create(int hd, int max_pos, float theta, void** out) {
  HOR_TRY({
    RopeOp* r = new RopeOp();
    r->r.init(hd, max_pos, theta);
    *out = r;
  })
}
void hor_rope_free(void* p) { delete (RopeOp*)p; }
int hor_rope_tables(void* p, float* cos_out, float* sin_out) {
  HOR_TRY({
    RopeOp* r = (RopeOp*)p;
    memcpy(cos_out, r->r.cos_.data(), r->r.cos_.size() * 4);
    memcpy(sin_out, r->r.sin_.data(), r->r.sin_.size() * 4);
  })
}
int hor_attn_step(void* rope, int n_heads, int n_kv_heads, int hd, float eps, const float* q_norm,
                  const float* k_norm, float* qkv, int pos, float* k_cache, float* v_cache, float* out) {
  HOR_TRY({
    const Rope& R = ((RopeOp*)rope)->r;
    int qd = n_heads * hd, kvd = n_kv_heads * hd, rep = n_heads / n_kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    float* q = qkv;
    float* k = qkv + qd;
    float* v = k + kvd;
    for (int hq = 0; hq < n_heads; hq++) {
      norm_head(q + hq * hd, q_norm, eps, hd);
      R.apply(q + hq * hd, pos);
    }
    for (int hk = 0; hk < n_kv_heads; hk++) {
      norm_head(k + hk * hd, k_norm, eps, hd);
      R.apply(k + hk * hd, pos);
    }
    memcpy(k_cache + (size_t)pos * kvd, k, kvd * 4);
    memcpy(v_cache + (size_t)pos * kvd, v, kvd * 4);
    int n = pos + 1;
    std::vector<float> scores(n);
    for (int i = 0; i < qd; i++) out[i] = 0.0f;
    for (int hq = 0; hq < n_heads; hq++) {
      int kvh = hq / rep;
      const float* qh = q + hq * hd;
      for (int t = 0; t < n; t++) scores[t] = dot(qh, k_cache + (size_t)t * kvd + kvh * hd, hd) * scale;
      softmax(scores.data(), n);
      float* oh = out + hq * hd;
      for (int t = 0; t < n; t++) {
        const float* vt = v_cache + (size_t)t * kvd + kvh * hd;
        float pp = scores[t];
        for (int di = 0; di < hd; di++) oh[di] += pp * vt[di];
      }
    }
  })
}

}  // extern "C"
