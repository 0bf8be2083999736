// Host-side token selection over logits copied from the GPU: sample.rs (argmax, temperature /
// top-p sampling, the Gumbel-max sampler of the diffusion decode, the xorshift64* RNG) and the
// diffusion block scoring of lib.rs. No GPU work; exported for callers and tests as hg_host_*.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "hg_host.h"

namespace hg {

float exp_pinned(float x) { return (float)std::exp((double)x); }
float log_pinned(float x) { return (float)std::log((double)x); }

// sample.rs:53-64: the first maximum wins.
uint32_t host_argmax(const float* v, int n) {
  int best = 0;
  float bv = -INFINITY;
  for (int i = 0; i < n; i++)
    if (v[i] > bv) {
      bv = v[i];
      best = i;
    }
  return (uint32_t)best;
}

// Ids of n probabilities (all >= 0) in descending order, equal values by ascending id: the order
// of a stable descending sort. Non-negative floats order like their bit patterns, so the key
// (~bits << 16 | id) sorted ascending gives it; the keys start in id order, so an LSD radix sort
// needs only the two 16-bit digits of the probability. Longer inputs fall back to a stable sort.
static void order_desc(const float* p, int n, std::vector<int>& idx) {
  idx.resize(n);
  if (n > 65536) {
    for (int i = 0; i < n; i++) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [p](int a, int b) { return p[a] > p[b]; });
    return;
  }
  std::vector<uint64_t> a(n), b(n);
  for (int i = 0; i < n; i++) {
    uint32_t bits;
    std::memcpy(&bits, p + i, 4);
    a[i] = ((uint64_t)(0xFFFFFFFFu - bits) << 16) | (uint64_t)i;
  }
  std::vector<uint32_t> cnt(65536);
  for (int shift = 16; shift <= 32; shift += 16) {
    std::fill(cnt.begin(), cnt.end(), 0u);
    for (int i = 0; i < n; i++) cnt[(a[i] >> shift) & 0xFFFF]++;
    uint32_t acc = 0;
    for (auto& c : cnt) {
      uint32_t v = c;
      c = acc;
      acc += v;
    }
    for (int i = 0; i < n; i++) b[cnt[(a[i] >> shift) & 0xFFFF]++] = a[i];
    a.swap(b);
  }
  for (int i = 0; i < n; i++) idx[i] = (int)(a[i] & 0xFFFF);
}

// sample.rs:66-112: softmax of logits / temp, then (0 < top_p < 1) the smallest prefix of the
// probabilities in descending order (ties by id) whose running sum reaches top_p, renormalised,
// and one uniform draw walked over it. The exponentials and divisions run in parallel; every sum
// keeps the reference's order (the denominator by id, the nucleus sums in sorted order).
uint32_t host_sample(const float* logits, int n, float temp, float top_p, Rng& rng) {
  if (temp <= 0.0f) return host_argmax(logits, n);
  std::vector<float> p(n);
  float m = -INFINITY;
#pragma omp parallel for reduction(max : m) schedule(static)
  for (int i = 0; i < n; i++) {
    p[i] = logits[i] / temp;
    m = std::fmax(m, p[i]);
  }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; i++) p[i] = exp_pinned(p[i] - m);
  float sum = 0.0f;
  for (int i = 0; i < n; i++) sum += p[i];
#pragma omp parallel for schedule(static)
  for (int i = 0; i < n; i++) p[i] /= sum;
  if (top_p > 0.0f && top_p < 1.0f) {
    std::vector<int> idx;
    order_desc(p.data(), n, idx);
    float cum = 0.0f;
    int cut = n;
    for (int j = 0; j < n; j++) {
      cum += p[idx[j]];
      if (cum >= top_p) {
        cut = j + 1;
        break;
      }
    }
    float s = -0.0f;
    for (int j = 0; j < cut; j++) s = s + p[idx[j]];
    float r = rng.next_f32(), c2 = 0.0f;
    for (int j = 0; j < cut; j++) {
      c2 += p[idx[j]] / s;
      if (r < c2) return (uint32_t)idx[j];
    }
    return (uint32_t)idx[cut - 1];
  }
  float r = rng.next_f32(), cum = 0.0f;
  for (int i = 0; i < n; i++) {
    cum += p[i];
    if (r < cum) return (uint32_t)i;
  }
  return (uint32_t)(n - 1);
}

// sample.rs:29-47: Gumbel-max over the finite logits; temp <= 0 is the plain argmax.
uint32_t gumbel_argmax(const float* l, int n, float temp, Rng& rng) {
  if (temp <= 0.0f) return host_argmax(l, n);
  int best = 0;
  float bv = -INFINITY;
  for (int i = 0; i < n; i++) {
    if (!std::isfinite(l[i])) continue;
    float u = std::clamp(rng.next_f32(), 1e-9f, 1.0f - 1e-9f);
    float val = l[i] / temp + -log_pinned(-log_pinned(u));
    if (val > bv) {
      bv = val;
      best = i;
    }
  }
  return (uint32_t)best;
}

// lib.rs:66-73: n unmask events spread over `steps` (sums to n).
std::vector<int> num_transfer(int n, int steps) {
  const int base = n / steps;
  std::vector<int> out(steps, base);
  for (int i = 0; i < n - base * steps; i++) out[i] += 1;
  return out;
}

// lib.rs:221-263 (score_block): per block row, ids >= valid banned, the presence penalty over the
// committed ids and the block's own non-mask ids, a Gumbel / greedy pick, and the softmax
// probabilities (ops.rs:112-128) of the pick (pconf) and of the row's current id (cconf). Rows are
// independent except for the Gumbel draws, which take one RNG stream row after row.
void score_block(const float* all, int V, const uint32_t* blk, int blk_len, const uint32_t* committed,
                 int n_committed, int valid, uint32_t mask, float rep_penalty, float temp, Rng& rng, uint32_t* pred,
                 float* pconf, float* cconf, std::vector<float>& rows) {
  std::vector<char> present(valid, 0);
  if (rep_penalty != 1.0f)
    for (int i = 0; i < n_committed + blk_len; i++) {
      uint32_t id = i < n_committed ? committed[i] : blk[i - n_committed];
      if (id != mask && (int64_t)id < valid) present[id] = 1;
    }
  rows.resize((size_t)blk_len * V);
#pragma omp parallel for schedule(static)
  for (int i = 0; i < blk_len; i++) {
    float* row = rows.data() + (size_t)i * V;
    memcpy(row, all + (size_t)i * V, (size_t)V * 4);
    for (int l = valid; l < V; l++) row[l] = -INFINITY;
    if (rep_penalty != 1.0f)
      for (int t = 0; t < valid; t++)
        if (present[t]) {
          float l = row[t];
          row[t] = l > 0.0f ? l / rep_penalty : l * rep_penalty;
        }
    if (temp <= 0.0f) pred[i] = host_argmax(row, V);
  }
  if (temp > 0.0f) {
    // gumbel_argmax row after row: the draws, one per finite logit, are taken in that order
    // first (the cheap sequential part); the two logarithms per draw and the argmax then run in
    // parallel with the same first-maximum rule.
    std::vector<size_t> off(blk_len + 1, 0);
    for (int i = 0; i < blk_len; i++) {
      const float* row = rows.data() + (size_t)i * V;
      size_t c = 0;
      for (int k = 0; k < V; k++) c += std::isfinite(row[k]) ? 1 : 0;
      off[i + 1] = off[i] + c;
    }
    std::vector<float> u(off[blk_len]);
    for (size_t j = 0; j < u.size(); j++) u[j] = std::clamp(rng.next_f32(), 1e-9f, 1.0f - 1e-9f);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < blk_len; i++) {
      const float* row = rows.data() + (size_t)i * V;
      size_t j = off[i];
      int best = 0;
      float bv = -INFINITY;
      for (int k = 0; k < V; k++) {
        if (!std::isfinite(row[k])) continue;
        const float val = row[k] / temp + -log_pinned(-log_pinned(u[j++]));
        if (val > bv) {
          bv = val;
          best = k;
        }
      }
      pred[i] = (uint32_t)best;
    }
  }
#pragma omp parallel for schedule(static)
  for (int i = 0; i < blk_len; i++) {
    const float* row = rows.data() + (size_t)i * V;
    float m = -INFINITY;
    for (int k = 0; k < V; k++)
      if (row[k] > m) m = row[k];
    float sum = 0.0f;
    for (int k = 0; k < V; k++) sum += exp_pinned(row[k] - m);
    const float inv = 1.0f / sum;
    pconf[i] = exp_pinned(row[pred[i]] - m) * inv;
    cconf[i] = exp_pinned(row[blk[i]] - m) * inv;
  }
}

}  // namespace hg

using namespace hg;

extern "C" {

int hg_host_sample(const float* logits, int n, float temp, float top_p, uint64_t* rng_state, uint32_t* out) {
  try {
    if (!logits || !rng_state || !out || n <= 0) throw Error(HG_ERR_INVALID, "bad argument");
    Rng rng(*rng_state);
    *out = host_sample(logits, n, temp, top_p, rng);
    *rng_state = rng.s;
    return HG_OK;
  } catch (const Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  } catch (const std::exception& ex) {
    set_last_error(ex.what());
    return HG_ERR_INVALID;
  }
}

int hg_host_score_block(const float* logits, int vocab, const uint32_t* blk, int blk_len, const uint32_t* committed,
                        int n_committed, uint32_t mask, float rep_penalty, float temp, uint64_t* rng_state,
                        uint32_t* pred, float* pconf, float* cconf) {
  try {
    if (!logits || !blk || !rng_state || !pred || !pconf || !cconf || vocab <= 0 || blk_len <= 0 ||
        n_committed < 0 || (n_committed > 0 && !committed))
      throw Error(HG_ERR_INVALID, "bad argument");
    for (int i = 0; i < blk_len; i++)
      if ((int64_t)blk[i] >= vocab) throw Error(HG_ERR_TOKEN, "block id out of range");
    Rng rng(*rng_state);
    std::vector<float> rows;
    score_block(logits, vocab, blk, blk_len, committed, n_committed, std::min(50257, vocab), mask, rep_penalty, temp,
                rng, pred, pconf, cconf, rows);
    *rng_state = rng.s;
    return HG_OK;
  } catch (const Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  } catch (const std::exception& ex) {
    set_last_error(ex.what());
    return HG_ERR_INVALID;
  }
}

}  // extern "C"
