// Token sampling on the GPU for Engine::generate (sample.rs:66-112, lib.rs:125-142): the
// repetition penalty over the generated ids, temperature, top-p and the xorshift64* draw, in the
// same arithmetic as the host sampler (sampler.cpp), so the ids are identical and only the chosen
// id leaves the GPU per token.
//
// One CTA of SMP_THREADS threads per call. The element-wise steps (mask, penalty, division by the
// temperature, exponentials, normalisation) run in parallel; every sum keeps the reference's
// order and runs in one thread: the softmax denominator over ids 0..V-1, the nucleus running sum
// and its renormalising sum over the probabilities in descending order (ties by ascending id), and
// the draw's running sum. That order comes from a bitonic sort of the host sampler's keys
// ((~bits(p) << 16) | id: distinct, so any correct sort gives the one stable order).
#include <cstdint>

#include "hg_launch.h"

namespace hg {

constexpr int SMP_THREADS = 1024;
constexpr int SMP_SORT = 65536;  // sort width: vocabularies up to 65,536 ids

struct SampleArgs {
  const float* logits;  // [V] the step's logits (device)
  int V, valid;         // ids >= valid are masked (the 50,257-id rule)
  float temp, top_p, rep_penalty;
  int32_t* counts;      // [V] how often each id was generated so far (the penalty's history)
  float* p;             // [V] scratch: scaled logits, then probabilities
  unsigned long long* keys;  // [SMP_SORT] scratch for the top-p order
  unsigned long long* rng;   // xorshift64* state
  uint32_t* next;       // the chosen id
};

__device__ __forceinline__ float rng_f32(unsigned long long& s) {  // Rng::next_f32 (hg_host.h)
  unsigned long long x = s;
  x ^= x >> 12;
  x ^= x << 25;
  x ^= x >> 27;
  s = x;
  const unsigned long long y = x * 0x2545F4914F6CDD1Dull;
  return __fdiv_rn(__uint2float_rn((uint32_t)(y >> 40)), 16777216.0f);  // exact: 24 bits / 2^24
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(SampleArgs a) {
  __shared__ float red_f[SMP_THREADS / 32];
  __shared__ unsigned long long red_k[SMP_THREADS / 32];
  __shared__ float bcast;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, V = a.V;
  const bool penalty = a.rep_penalty != 1.0f;
  // ---- mask + repetition penalty (lib.rs:130-139: applied once per occurrence in the history) ----
  auto logit = [&](int i) -> float {
    float l = i < a.valid ? a.logits[i] : -INFINITY;
    if (penalty) {
      const int c = a.counts[i];
      for (int k = 0; k < c; k++) l = l > 0.0f ? __fdiv_rn(l, a.rep_penalty) : __fmul_rn(l, a.rep_penalty);
    }
    return l;
  };
  if (a.temp <= 0.0f) {
    // argmax of the penalised logits, the first maximum winning (sample.rs:53-64)
    unsigned long long best = 0ull;
    for (int i = tid; i < V; i += SMP_THREADS) best = max(best, argmax_key(logit(i), (uint32_t)i));
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0) red_k[warp] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = 0ull;
      for (int w = 0; w < SMP_THREADS / 32; w++) b = max(b, red_k[w]);
      const uint32_t id = 0xffffffffu - (uint32_t)(b & 0xffffffffull);
      *a.next = id;
      a.counts[id] += 1;
    }
    return;
  }
  // ---- softmax of logits / temp (sample.rs:76-86) ----
  float m = -INFINITY;
  for (int i = tid; i < V; i += SMP_THREADS) {
    const float x = __fdiv_rn(logit(i), a.temp);
    a.p[i] = x;
    m = fmaxf(m, x);
  }
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red_f[warp] = m;
  __syncthreads();
  if (tid == 0) {
    float mm = -INFINITY;
    for (int w = 0; w < SMP_THREADS / 32; w++) mm = fmaxf(mm, red_f[w]);
    bcast = mm;
  }
  __syncthreads();
  m = bcast;
  for (int i = tid; i < V; i += SMP_THREADS) a.p[i] = exp_cr(__fsub_rn(a.p[i], m));
  __syncthreads();
  if (tid == 0) {  // the denominator, in id order
    float sum = 0.0f;
    for (int i = 0; i < V; i++) sum = fadd(sum, a.p[i]);
    bcast = sum;
  }
  __syncthreads();
  const float sum = bcast;
  for (int i = tid; i < V; i += SMP_THREADS) a.p[i] = __fdiv_rn(a.p[i], sum);
  __syncthreads();
  unsigned long long s = *a.rng;
  if (a.top_p > 0.0f && a.top_p < 1.0f) {
    // ---- nucleus (sample.rs:88-104): probabilities in descending order, ties by ascending id ----
    for (int i = tid; i < SMP_SORT; i += SMP_THREADS)
      a.keys[i] = i < V ? ((unsigned long long)(0xffffffffu - __float_as_uint(a.p[i])) << 16) | (unsigned long long)i
                        : ~0ull;  // padding sorts last
    __syncthreads();
    for (int k = 2; k <= SMP_SORT; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < SMP_SORT; i += SMP_THREADS) {
          const int ij = i ^ j;
          if (ij > i) {
            const unsigned long long x = a.keys[i], y = a.keys[ij];
            if (((i & k) == 0) == (x > y)) {  // ascending block: keep x <= y; descending: x >= y
              a.keys[i] = y;
              a.keys[ij] = x;
            }
          }
        }
        __syncthreads();
      }
    if (tid == 0) {
      int cut = V;
      float cum = 0.0f;
      for (int j = 0; j < V; j++) {
        cum = fadd(cum, a.p[(int)(a.keys[j] & 0xffffull)]);
        if (cum >= a.top_p) {
          cut = j + 1;
          break;
        }
      }
      float sn = -0.0f;
      for (int j = 0; j < cut; j++) sn = fadd(sn, a.p[(int)(a.keys[j] & 0xffffull)]);
      const float r = rng_f32(s);
      float c2 = 0.0f;
      int id = (int)(a.keys[cut - 1] & 0xffffull);
      for (int j = 0; j < cut; j++) {
        const int ij = (int)(a.keys[j] & 0xffffull);
        c2 = fadd(c2, __fdiv_rn(a.p[ij], sn));
        if (r < c2) {
          id = ij;
          break;
        }
      }
      *a.next = (uint32_t)id;
      a.counts[id] += 1;
      *a.rng = s;
    }
    return;
  }
  if (tid == 0) {  // the draw over ids in order (sample.rs:105-111)
    const float r = rng_f32(s);
    float cum = 0.0f;
    int id = V - 1;
    for (int i = 0; i < V; i++) {
      cum = fadd(cum, a.p[i]);
      if (r < cum) {
        id = i;
        break;
      }
    }
    *a.next = (uint32_t)id;
    a.counts[id] += 1;
    *a.rng = s;
  }
}

bool sample_usable(int V) { return V >= 1 && V <= SMP_SORT; }

size_t sample_scratch_bytes(int V) {
  return (size_t)V * 4 /* counts */ + (size_t)V * 4 /* p */ + (size_t)SMP_SORT * 8 /* keys */ + 8 /* rng */ + 8;
}

// scratch: [keys SMP_SORT x 8 B][rng 8 B][next id 8 B][counts V x 4 B][p V x 4 B]
uint32_t* sample_next_ptr(void* scratch) {
  return reinterpret_cast<uint32_t*>(static_cast<char*>(scratch) + (size_t)SMP_SORT * 8 + 8);
}

void launch_sample(const float* logits, int V, int valid, float temp, float top_p, float rep_penalty, void* scratch,
                   cudaStream_t st) {
  char* b = static_cast<char*>(scratch);
  SampleArgs a{};
  a.logits = logits;
  a.V = V;
  a.valid = valid;
  a.temp = temp;
  a.top_p = top_p;
  a.rep_penalty = rep_penalty;
  a.keys = reinterpret_cast<unsigned long long*>(b);
  a.rng = reinterpret_cast<unsigned long long*>(b + (size_t)SMP_SORT * 8);
  a.counts = reinterpret_cast<int32_t*>(b + (size_t)SMP_SORT * 8 + 16);
  a.p = reinterpret_cast<float*>(b + (size_t)SMP_SORT * 8 + 16 + (size_t)V * 4);
  a.next = sample_next_ptr(scratch);
  k_sample<<<1, SMP_THREADS, 0, st>>>(a);
}

// the scratch's history counts (zero) and RNG state (Rng(seed): a zero seed becomes 1)
void sample_reset(void* scratch, int V, unsigned long long seed, cudaStream_t st, unsigned long long* h_state) {
  char* b = static_cast<char*>(scratch);
  *h_state = seed < 1 ? 1 : seed;
  cudaMemcpyAsync(b + (size_t)SMP_SORT * 8, h_state, 8, cudaMemcpyHostToDevice, st);
  cudaMemsetAsync(b + (size_t)SMP_SORT * 8 + 16, 0, (size_t)V * 4, st);
}

}  // namespace hg
