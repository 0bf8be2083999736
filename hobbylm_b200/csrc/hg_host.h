// Host-side internals of the hobbygpu engine: errors, the GGUF reader, config and weight packing.
#pragma once
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/hobbygpu.h"

namespace hg {

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

void set_last_error(const std::string& msg);

// ---- GGUF v3 (hobby-rs/src/gguf.rs) ----
struct GgufMeta {
  enum Kind { U32, I32, F32, U64, BOOL, STR, ARR_STR, ARR_I32, ARR_F32, OTHER } kind = OTHER;
  uint64_t u = 0;  // U32 / U64 / BOOL
  int64_t i = 0;   // I32
  float f = 0;     // F32
  std::string s;
  size_t arr_len = 0;
};

struct GgufTensor {
  std::vector<uint64_t> ne;  // fastest-varying first
  uint32_t type = 0;
  uint64_t offset = 0;       // relative to the data section
  uint64_t n_elems() const;
};

class Gguf {
 public:
  explicit Gguf(const char* path);  // throws Error(HG_ERR_IO / HG_ERR_FORMAT)
  ~Gguf();
  Gguf(const Gguf&) = delete;
  Gguf& operator=(const Gguf&) = delete;

  const GgufTensor* tensor(const std::string& name) const;
  // F32 tensor copied out (gguf.rs:215-235: must be F32).
  std::vector<float> f32(const std::string& name) const;
  // Any supported type dequantized to f32 (gguf.rs:250-269).
  std::vector<float> load(const std::string& name) const;
  // Raw bytes of a tensor.
  const uint8_t* raw(const std::string& name, size_t* nbytes) const;

  bool get_u32(const std::string& k, uint32_t* out) const;
  bool get_f32(const std::string& k, float* out) const;
  bool get_bool(const std::string& k, bool* out) const;
  bool get_str(const std::string& k, std::string* out) const;
  bool has_str_array(const std::string& k) const;

 private:
  const uint8_t* map_ = nullptr;
  size_t size_ = 0;
  size_t data_start_ = 0;
  std::unordered_map<std::string, GgufMeta> meta_;
  std::unordered_map<std::string, GgufTensor> tensors_;
};

size_t ggml_type_nbytes(uint32_t type, size_t n);
void ggml_dequant(uint32_t type, const uint8_t* b, size_t n, float* y);

hg_config config_from_gguf(const Gguf& g);

// ---- Q8 re-quantization + lane-chunked packing (quant.rs:78-102) ----
// w: row-major f32 [rows][cols]; qs: [rows][cols] packed bytes; sc: [rows][q8_ss(nb)].
void q8_pack_rows(const float* w, int64_t rows, int64_t cols, int8_t* qs, float* sc);
int host_q8_ss(int64_t cols);

// RoPE cos/sin tables in f64 (ops.rs:139-154).
void rope_tables(int head_dim, int max_pos, float theta, float* cos_out, float* sin_out);

// ---- host-side token selection (sampler.cpp) ----
// xorshift64* (sample.rs:3-22); Rng::new(seed) keeps seed.max(1).
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
// f32::exp / f32::ln pinned to the correctly rounded double results.
float exp_pinned(float x);
float log_pinned(float x);
uint32_t host_argmax(const float* v, int n);
uint32_t host_sample(const float* logits, int n, float temp, float top_p, Rng& rng);
uint32_t gumbel_argmax(const float* l, int n, float temp, Rng& rng);
std::vector<int> num_transfer(int n, int steps);
void score_block(const float* all, int V, const uint32_t* blk, int blk_len, const uint32_t* committed,
                 int n_committed, int valid, uint32_t mask, float rep_penalty, float temp, Rng& rng, uint32_t* pred,
                 float* pconf, float* cconf, std::vector<float>& rows);

}  // namespace hg
