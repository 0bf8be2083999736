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

// sample.rs:66-112: softmax of logits / temp, then (0 < top_p < 1) the smallest prefix of the
// probabilities in descending order (ties by id) whose running sum reaches top_p, renormalised,
// and one uniform draw walked over it.
uint32_t host_sample(const float* logits, int n, float temp, float top_p, Rng& rng) {
  if (temp <= 0.0f) return host_argmax(logits, n);
  std::vector<std::pair<int, float>> pr(n);
  float m = -INFINITY;
  for (int i = 0; i < n; i++) {
    pr[i] = {i, logits[i] / temp};
    m = std::fmax(m, pr[i].second);
  }
  float sum = 0.0f;
  for (auto& p : pr) {
    p.second = exp_pinned(p.second - m);
    sum += p.second;
  }
  for (auto& p : pr) p.second /= sum;
  if (top_p > 0.0f && top_p < 1.0f) {
    std::stable_sort(pr.begin(), pr.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
    float cum = 0.0f;
    size_t cut = pr.size();
    for (size_t i = 0; i < pr.size(); i++) {
      cum += pr[i].second;
      if (cum >= top_p) {
        cut = i + 1;
        break;
      }
    }
    pr.resize(cut);
    float s = -0.0f;
    for (auto& p : pr) s = s + p.second;
    for (auto& p : pr) p.second /= s;
  }
  float r = rng.next_f32(), cum = 0.0f;
  for (auto& p : pr) {
    cum += p.second;
    if (r < cum) return (uint32_t)p.first;
  }
  return pr.empty() ? 0 : (uint32_t)pr.back().first;
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
  if (temp > 0.0f)
    for (int i = 0; i < blk_len; i++) pred[i] = gumbel_argmax(rows.data() + (size_t)i * V, V, temp, rng);
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
