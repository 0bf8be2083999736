// The hobbygpu engine: GGUF load + one-time HBM upload, paged KV pool, decode steps (CUDA graphs
// per batch size), exact chunked prefill, Engine::generate, and the C ABI (include/hobbygpu.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <mutex>
#include <numeric>
#include <random>
#include <string>
#include <unordered_set>
#include <vector>

#include "hg_ep.h"
#include "hg_host.h"
#include "hg_launch.h"

namespace hg {

// rows of one bidirectional pass (hg_run_block; the uncached diffusion canvas)
constexpr int PF_BLOCK_MAX = 1024;

static thread_local std::string g_last_error;
void set_last_error(const std::string& m) { g_last_error = m; }

#define HG_CUDA(call)                                                                               \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess)                                                                          \
      throw ::hg::Error(HG_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));           \
  } while (0)

// Device memory arena: one cudaMalloc, 256-byte aligned sub-allocations.
// A measuring arena (measure = true) hands out no memory and only sums the sizes, so a layout
// routine can run once to size the real allocation and once to carve it.
struct Arena {
  char* base = nullptr;
  size_t cap = 0, used = 0;
  bool measure = false;
  void init(size_t bytes) {
    cap = bytes;
    used = 0;
    measure = false;
    HG_CUDA(cudaMalloc((void**)&base, bytes));
  }
  template <class T>
  T* take(size_t n) {
    size_t b = (n * sizeof(T) + 255) & ~size_t(255);
    if (measure) {
      used += b;
      return nullptr;
    }
    if (used + b > cap) throw Error(HG_ERR_CUDA, "arena overflow");
    T* p = reinterpret_cast<T*>(base + used);
    used += b;
    return p;
  }
  void release() {
    if (base) cudaFree(base);
    base = nullptr;
  }
};

}  // namespace hg

using namespace hg;

struct hg_seq;

struct hg_engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  hg_config cfg{};
  Dims D{};
  Arena weights, work;
  uint64_t ref_weight_bytes = 0;
  float* embd = nullptr;
  float* out_norm = nullptr;
  Q8M lm;
  std::vector<LayerDev> layers;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  // KV pool
  float* kv = nullptr;
  long long page_stride = 0, layer_stride = 0;
  int n_pages = 0;
  std::vector<int> free_pages;
  int32_t* d_bt = nullptr;  // [max_rows][bt_stride]
  int bt_stride = 0, max_rows = 0;
  std::vector<int> free_rows;
  std::unordered_set<hg_seq*> live_seqs;  // detached (s->e = null) when the engine is freed
  // decode buffers
  int max_batch = 1;
  DecodeBufs buf{};
  int32_t* d_meta = nullptr;   // [3][max_batch]: tok, pos, bt_row
  int32_t* h_meta = nullptr;   // pinned
  unsigned long long* h_amax = nullptr;  // pinned [max_batch]
  int32_t* h_err = nullptr;    // pinned
  void* smp = nullptr;          // device sampling scratch (sample.cu), allocated by the first sampled generate
  uint32_t* h_smp = nullptr;    // pinned: the sampled id
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, int> graph_kernels;  // kernel nodes per step graph
  int32_t* d_gen = nullptr;          // [GEN_CAP][max_batch] generated ids ring
  int32_t* d_step = nullptr;         // ring step counter
  // prefill buffers
  int pf_rows = 0;
  struct Pf {
    float *x, *h, *qkv, *q, *o, *g, *u, *act, *y, *selw, *S, *inv;
    uint32_t* mkey;  // row maxima of the scores (order-preserving keys)
    int8_t *qa, *qact;
    float *sa, *sact;
    int32_t *ids, *sel, *ecount, *elist, *a_idx, *o_idx, *gm, *go, *gc;
  } pf{};
  int pf_tq = 4096;
  float* blk_logits = nullptr;  // [blk_logits_rows][vocab] logits of diffusion block rows
  int blk_logits_rows = 0;
  std::vector<int32_t> last_sel;  // [n_layers][max_batch][k] from the last decode step
  int last_T = 0;
  EpCtx* ep = nullptr;  // expert parallelism across ranks (hg_engine_ep_init), or none
  size_t device_bytes() const { return weights.cap + work.cap; }
};

struct hg_seq {
  hg_engine* e = nullptr;
  int row = -1;
  int len = 0;
  int max_ctx = 0;
  std::vector<int> pages;
};

namespace {

constexpr int GEN_CAP = 64;

template <class T>
T* dev_alloc(Arena& a, size_t n) {
  return a.take<T>(n);
}

void upload_q8(hg_engine* e, const Gguf& g, const std::string& name, int64_t count, int64_t rows, int64_t cols, Q8M* m,
               bool ref_counted = true) {
  int ss0 = host_q8_ss(cols);
  if (e->weights.measure) {
    const GgufTensor* t = g.tensor(name);
    if (!t) throw Error(HG_ERR_MISSING, "tensor `" + name + "` not found");
    e->weights.take<int8_t>((size_t)(count * rows * cols));
    e->weights.take<float>((size_t)(count * rows * ss0));
    return;
  }
  std::vector<float> w = g.load(name);
  if ((int64_t)w.size() != count * rows * cols)
    throw Error(HG_ERR_FORMAT, "tensor `" + name + "` has " + std::to_string(w.size()) + " elements, expected " +
                                   std::to_string(count * rows * cols));
  int ss = host_q8_ss(cols);
  std::vector<int8_t> qs((size_t)(count * rows * cols));
  std::vector<float> sc((size_t)(count * rows * ss));
  q8_pack_rows(w.data(), count * rows, cols, qs.data(), sc.data());
  int8_t* dq = dev_alloc<int8_t>(e->weights, qs.size());
  float* ds = dev_alloc<float>(e->weights, sc.size());
  HG_CUDA(cudaMemcpy(dq, qs.data(), qs.size(), cudaMemcpyHostToDevice));
  HG_CUDA(cudaMemcpy(ds, sc.data(), sc.size() * 4, cudaMemcpyHostToDevice));
  m->qs = dq;
  m->sc = ds;
  m->rows = (int)rows;
  m->cols = (int)cols;
  m->ss = ss;
  m->qs_mstride = rows * cols;
  m->sc_mstride = rows * ss;
  if (ref_counted) e->ref_weight_bytes += (uint64_t)(count * rows * cols) + (uint64_t)(count * rows * (cols / 32)) * 4;
}

float* upload_f32(hg_engine* e, const std::vector<float>& v) {
  float* d = dev_alloc<float>(e->weights, v.size());
  if (!e->weights.measure) HG_CUDA(cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return d;
}

void validate_cfg(const hg_config& c) {
  auto bad = [](const std::string& m) { throw Error(HG_ERR_FORMAT, m); };
  if (c.d_model <= 0 || c.d_model % 32) bad("embedding_length must be a positive multiple of 32");
  if (c.n_layers <= 0 || c.n_layers > MAX_LAYERS) bad("block_count out of range");
  if (c.n_heads <= 0 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads) bad("bad head counts");
  if (c.head_dim != 64 && c.head_dim != 128) bad("head_dim must be 64 or 128");
  int rep = c.n_heads / c.n_kv_heads;
  if (rep != 1 && rep != 2 && rep != 4) bad("GQA group size must be 1, 2 or 4");
  if (c.expert_ffn % 32 || c.dense_ffn % 32) bad("ffn widths must be multiples of 32");
  if (c.n_experts <= 0 || c.n_experts > 128) bad("expert_count out of range");
  if (c.top_k <= 0 || c.top_k > MAX_TOPK || c.top_k > c.n_experts) bad("expert_used_count out of range");
  if (c.context_length <= 0) bad("bad context_length");
  if (c.n_dense < 0 || c.n_dense > c.n_layers) bad("bad leading_dense_block_count");
}

void alloc_work(hg_engine* e) {
  const hg_config& c = e->cfg;
  const Dims& D = e->D;
  const int T = e->max_batch;
  const int d = c.d_model, qd = D.qd, qkvd = D.qkvd, k = c.top_k, ne = c.n_experts, f = c.expert_ffn;
  const int ss_d = host_q8_ss(d), ss_q = host_q8_ss(qd);
  const int act_stride = std::max(c.dense_ffn, (k + 1) * f);
  // prefill sizing
  const int PF = e->pf_rows;
  const int rep = c.n_heads / c.n_kv_heads;
  const size_t s_elems = (size_t)c.context_length * e->pf_tq * rep * c.n_kv_heads;  // every kv head's scores
  const size_t pf_act = std::max((size_t)PF * c.dense_ffn, (size_t)PF * (k + 1) * f);
  const size_t pf_act_s = std::max((size_t)PF * host_q8_ss(c.dense_ffn), (size_t)PF * (k + 1) * host_q8_ss(f));
  Arena& a = e->work;
  for (int pass = 0; pass < 2; pass++) {
  if (pass == 0) {
    a.measure = true;
    a.used = 0;
  } else {
    a.init(a.used + (1 << 20));
  }
  e->d_meta = a.take<int32_t>(3 * T);
  DecodeBufs& B = e->buf;
  B.T = T;
  B.tok = e->d_meta;
  B.pos = e->d_meta + T;
  B.bt_row = e->d_meta + 2 * T;
  B.bt = e->d_bt;
  B.bt_stride = e->bt_stride;
  B.x = a.take<float>((size_t)T * d);
  B.xin = a.take<float>((size_t)T * d);
  B.qa = a.take<int8_t>((size_t)T * d);
  B.sa = a.take<float>((size_t)T * ss_d);
  B.qkv = a.take<float>((size_t)T * qkvd);
  B.qo = a.take<int8_t>((size_t)T * qd);
  B.so = a.take<float>((size_t)T * ss_q);
  B.h2 = a.take<float>((size_t)T * d);
  B.qh = a.take<int8_t>((size_t)T * d);
  B.sh = a.take<float>((size_t)T * ss_d);
  B.sel = a.take<int32_t>((size_t)T * k);
  B.selw = a.take<float>((size_t)T * k);
  B.ecount = a.take<int32_t>(ne + 2);
  B.active = a.take<int32_t>(ne);
  B.elist = a.take<int32_t>((size_t)ne * T);
  B.act = a.take<float>((size_t)T * act_stride);
  B.act_stride = act_stride;
  B.ubuf = a.take<float>((size_t)T * act_stride);
  B.qact = a.take<int8_t>((size_t)T * act_stride);
  B.sact = a.take<float>((size_t)T * std::max(host_q8_ss(c.dense_ffn), (k + 1) * host_q8_ss(f)));
  B.y = a.take<float>((size_t)T * (k + 1) * d);
  B.s_stride = ((long long)c.context_length + 15) & ~15LL;
  B.S = a.take<float>((size_t)T * c.n_heads * B.s_stride);
  B.mkey = a.take<uint32_t>((size_t)T * c.n_heads);
  B.order = a.take<int32_t>((size_t)T);
  B.rinv = a.take<float>((size_t)T * c.n_heads);
  B.qn = a.take<float>((size_t)T * D.qd);
  B.logits = a.take<float>((size_t)T * c.vocab_size);
  B.amax = a.take<unsigned long long>(T);
  B.dbg_sel = a.take<int32_t>((size_t)c.n_layers * T * k);
  B.err = a.take<int32_t>(4);
  auto& P = e->pf;
  P.x = a.take<float>((size_t)PF * d);
  P.h = a.take<float>((size_t)PF * d);
  P.qkv = a.take<float>((size_t)PF * qkvd);
  P.q = a.take<float>((size_t)PF * qd);
  P.o = a.take<float>((size_t)PF * qd);
  P.g = a.take<float>(pf_act);
  P.u = a.take<float>(pf_act);
  P.act = a.take<float>(pf_act);
  P.y = a.take<float>((size_t)PF * (k + 1) * d);
  P.selw = a.take<float>((size_t)PF * k);
  P.S = a.take<float>(s_elems);
  P.inv = a.take<float>((size_t)e->pf_tq * rep * c.n_kv_heads);
  P.mkey = a.take<uint32_t>((size_t)e->pf_tq * rep * c.n_kv_heads);
  P.qa = a.take<int8_t>((size_t)PF * std::max(d, qd));
  P.qact = a.take<int8_t>(pf_act);
  P.sa = a.take<float>((size_t)PF * std::max(ss_d, ss_q));
  P.sact = a.take<float>(pf_act_s);
  P.ids = a.take<int32_t>(PF);
  P.sel = a.take<int32_t>((size_t)PF * k);
  P.ecount = a.take<int32_t>(ne);
  P.elist = a.take<int32_t>((size_t)ne * PF);
  P.a_idx = a.take<int32_t>((size_t)(ne + 1) * PF);
  P.o_idx = a.take<int32_t>((size_t)(ne + 1) * PF);
  P.gm = a.take<int32_t>(ne);
  P.go = a.take<int32_t>(ne);
  P.gc = a.take<int32_t>(ne);
  e->d_gen = a.take<int32_t>((size_t)GEN_CAP * T);
  e->d_step = a.take<int32_t>(4);
  }
  HG_CUDA(cudaMemset(a.base, 0, a.cap));
}

void load_engine(hg_engine* e, const char* path, const hg_engine_opts& o) {
  e->device = o.device;
  // the file is parsed and validated before any CUDA call, so format errors need no GPU
  Gguf g(path);
  hg_config c = config_from_gguf(g);
  // lib.rs:88 builds the tokenizer (tokenizer.rs:55-61 requires both arrays) before the model
  if (!g.has_str_array("tokenizer.ggml.tokens")) throw Error(HG_ERR_MISSING, "missing tokenizer.ggml.tokens");
  if (!g.has_str_array("tokenizer.ggml.merges")) throw Error(HG_ERR_MISSING, "missing tokenizer.ggml.merges");
  validate_cfg(c);
  for (const char* t : {"token_embd.weight", "output.weight", "output_norm.weight"})
    if (!g.tensor(t)) throw Error(HG_ERR_MISSING, std::string("tensor `") + t + "` not found");
  HG_CUDA(cudaSetDevice(e->device));
  HG_CUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  HG_CUDA(prepare_attn(c.head_dim, c.n_heads / c.n_kv_heads));
  HG_CUDA(prepare_tc());
  e->cfg = c;
  Dims& D = e->D;
  D.d = c.d_model;
  D.L = c.n_layers;
  D.nh = c.n_heads;
  D.nkv = c.n_kv_heads;
  D.hd = c.head_dim;
  D.qd = c.n_heads * c.head_dim;
  D.qkvd = D.qd + 2 * c.n_kv_heads * c.head_dim;
  D.f = c.expert_ffn;
  D.df = c.dense_ffn;
  D.ne = c.n_experts;
  D.k = c.top_k;
  D.nsh = c.n_shared;
  D.vocab = c.vocab_size;
  D.valid = std::min(50257, c.vocab_size);
  D.eps = c.rms_eps;
  D.wscale = c.expert_weights_scale;
  D.wnorm = c.expert_weights_norm;
  D.gsig = c.gating_sigmoid;
  D.max_pos = c.context_length;
  const int d = c.d_model, f = c.expert_ffn, df = c.dense_ffn, ne = c.n_experts, L = c.n_layers;
  // weights: one measuring pass sizes the arena, the second uploads
  for (int pass = 0; pass < 2; pass++) {
  if (pass == 0) {
    e->weights.measure = true;
    e->weights.used = 0;
  } else {
    e->weights.init(e->weights.used + (1 << 20));
    e->ref_weight_bytes = 0;
  }
  e->embd = upload_f32(e, g.load("token_embd.weight"));
  if (g.tensor("token_embd.weight")->n_elems() < (uint64_t)c.vocab_size * d)
    throw Error(HG_ERR_FORMAT, "token_embd too small");
  e->out_norm = upload_f32(e, g.f32("output_norm.weight"));
  upload_q8(e, g, "output.weight", 1, c.vocab_size, d, &e->lm);
  {
    std::vector<float> cs((size_t)c.context_length * (c.head_dim / 2)), sn(cs.size());
    rope_tables(c.head_dim, c.context_length, c.rope_theta, cs.data(), sn.data());
    e->rope_cos = upload_f32(e, cs);
    e->rope_sin = upload_f32(e, sn);
  }
  e->layers.resize(L);
  for (int i = 0; i < L; i++) {
    LayerDev& Ld = e->layers[i];
    std::memset(&Ld, 0, sizeof(Ld));
    std::string p = "blk." + std::to_string(i) + ".";
    auto nt = [&](const char* s, size_t n) {
      std::vector<float> v = g.f32(p + s);
      if (v.size() != n) throw Error(HG_ERR_FORMAT, "tensor `" + p + s + "` has the wrong size");
      return upload_f32(e, v);
    };
    Ld.attn_norm = nt("attn_norm.weight", d);
    Ld.q_norm = nt("attn_q_norm.weight", c.head_dim);
    Ld.k_norm = nt("attn_k_norm.weight", c.head_dim);
    Ld.ffn_norm = nt("ffn_norm.weight", d);
    upload_q8(e, g, p + "attn_qkv.weight", 1, D.qkvd, d, &Ld.qkv);
    upload_q8(e, g, p + "attn_output.weight", 1, d, D.qd, &Ld.wo);
    if (i >= c.n_dense) {
      Ld.moe = 1;
      std::vector<float> r = g.load(p + "ffn_gate_inp.weight");
      if (r.size() != (size_t)ne * d) throw Error(HG_ERR_FORMAT, "router has the wrong size");
      Ld.router = upload_f32(e, r);
      Ld.bias = nt("exp_probs_b.bias", ne);
      upload_q8(e, g, p + "ffn_gate_exps.weight", ne, f, d, &Ld.gate);
      upload_q8(e, g, p + "ffn_up_exps.weight", ne, f, d, &Ld.up);
      upload_q8(e, g, p + "ffn_down_exps.weight", ne, d, f, &Ld.down);
      // model.rs:99-101 loads the shared expert unconditionally
      upload_q8(e, g, p + "ffn_gate_shexp.weight", 1, f, d, &Ld.sgate);
      upload_q8(e, g, p + "ffn_up_shexp.weight", 1, f, d, &Ld.sup);
      upload_q8(e, g, p + "ffn_down_shexp.weight", 1, d, f, &Ld.sdown);
    } else {
      upload_q8(e, g, p + "ffn_gate.weight", 1, df, d, &Ld.gate);
      upload_q8(e, g, p + "ffn_up.weight", 1, df, d, &Ld.up);
      upload_q8(e, g, p + "ffn_down.weight", 1, d, df, &Ld.down);
    }
  }
  }
  // KV pool
  const long long blk = (long long)c.n_kv_heads * PAGE * c.head_dim;  // floats of one K (or V) page block
  e->layer_stride = 2 * blk;
  e->page_stride = (long long)L * 2 * blk;
  long long pool_tokens = o.kv_pool_tokens > 0 ? o.kv_pool_tokens : 2LL * c.context_length;
  e->n_pages = (int)((pool_tokens + PAGE - 1) / PAGE);
  HG_CUDA(cudaMalloc((void**)&e->kv, (size_t)e->n_pages * e->page_stride * 4));
  e->free_pages.resize(e->n_pages);
  std::iota(e->free_pages.rbegin(), e->free_pages.rend(), 0);  // pop_back hands out 0, 1, 2, ...
  if (o.kv_page_shuffle) {
    std::mt19937_64 rng(o.kv_page_shuffle);
    std::shuffle(e->free_pages.begin(), e->free_pages.end(), rng);
  }
  e->bt_stride = (c.context_length + PAGE - 1) / PAGE;
  e->max_batch = std::max(1, std::min(256, o.max_batch > 0 ? o.max_batch : 1));
  e->max_rows = std::max(e->max_batch, 8);
  HG_CUDA(cudaMalloc((void**)&e->d_bt, (size_t)e->max_rows * e->bt_stride * 4));
  HG_CUDA(cudaMemset(e->d_bt, 0, (size_t)e->max_rows * e->bt_stride * 4));
  for (int r = e->max_rows - 1; r >= 0; r--) e->free_rows.push_back(r);
  e->pf_rows = 4096;  // prefill rows per chunk: a chunk's attention launches hold rows x heads chains
  alloc_work(e);
  HG_CUDA(cudaMallocHost((void**)&e->h_meta, 3 * e->max_batch * 4));
  HG_CUDA(cudaMallocHost((void**)&e->h_amax, e->max_batch * 8));
  HG_CUDA(cudaMallocHost((void**)&e->h_err, 16));
  e->last_sel.assign((size_t)L * e->max_batch * c.top_k, -1);
  HG_CUDA(cudaDeviceSynchronize());
}

void free_engine(hg_engine* e) {
  if (!e) return;
  for (hg_seq* s : e->live_seqs) s->e = nullptr;  // their pages go with the pool below
  e->live_seqs.clear();
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);  // (their NCCL calls before the communicator)
  ep_destroy(e->ep);
  e->weights.release();
  e->work.release();
  if (e->kv) cudaFree(e->kv);
  if (e->d_bt) cudaFree(e->d_bt);
  if (e->blk_logits) cudaFree(e->blk_logits);
  if (e->h_meta) cudaFreeHost(e->h_meta);
  if (e->h_amax) cudaFreeHost(e->h_amax);
  if (e->h_err) cudaFreeHost(e->h_err);
  if (e->h_smp) cudaFreeHost(e->h_smp);
  if (e->smp) cudaFree(e->smp);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

// Make sure `s` has pages for positions [0, upto); new page ids are written to the device table.
void ensure_pages(hg_seq* s, int upto) {
  hg_engine* e = s->e;
  int need = (upto + PAGE - 1) / PAGE;
  if (need > e->bt_stride) throw Error(HG_ERR_CONTEXT, "position beyond context_length");
  int have = (int)s->pages.size();
  if (need <= have) return;
  if ((int)e->free_pages.size() < need - have) throw Error(HG_ERR_POOL_EXHAUSTED, "KV page pool exhausted");
  for (int i = have; i < need; i++) {
    s->pages.push_back(e->free_pages.back());
    e->free_pages.pop_back();
  }
  HG_CUDA(cudaMemcpyAsync(e->d_bt + (size_t)s->row * e->bt_stride + have, s->pages.data() + have, (need - have) * 4,
                          cudaMemcpyHostToDevice, e->stream));
}

// ---------------------------------------------------------------------------------------------
// Decode step
// ---------------------------------------------------------------------------------------------
AttnArgs make_attn_args(hg_engine* e, const DecodeBufs& B, int l) {
  const hg_config& c = e->cfg;
  const LayerDev& Ld = e->layers[l];
  AttnArgs A{};
  A.T = B.T;
  A.nh = c.n_heads;
  A.nkv = c.n_kv_heads;
  A.hd = c.head_dim;
  A.max_pos = c.context_length;
  A.bt_stride = e->bt_stride;
  A.eps = c.rms_eps;
  A.qkv = B.qkv;
  A.qkv_stride = e->D.qkvd;
  A.q_norm = Ld.q_norm;
  A.k_norm = Ld.k_norm;
  A.rope_cos = e->rope_cos;
  A.rope_sin = e->rope_sin;
  A.pos = B.pos;
  A.bt = B.bt;
  A.bt_row = B.bt_row;
  A.k_pool = e->kv + (long long)l * e->layer_stride;
  A.v_pool = A.k_pool + e->layer_stride / 2;
  A.page_stride = e->page_stride;
  A.S = B.S;
  A.s_stride = B.s_stride;
  A.mkey = B.mkey;
  A.order = B.order;
  A.rinv = B.rinv;
  A.qn = B.qn;
  A.out = nullptr;
  A.qo = B.qo;
  A.so = B.so;
  A.err = B.err;
  return A;
}

void record_decode(hg_engine* e, const DecodeBufs& B) {
  const Dims& D = e->D;
  cudaStream_t st = e->stream;
  for (int l = 0; l < D.L; l++) {
    const LayerDev& Ld = e->layers[l];
    int mode = l == 0 ? 0 : (e->layers[l - 1].moe ? 2 : 1);
    launch_pre_norm(D, B, mode, e->embd, Ld.attn_norm, B.qa, B.sa, nullptr, 1, 0, st);
    launch_mv_store(D, B, Ld.qkv, B.qa, B.sa, B.qkv, D.qkvd, st);
    AttnArgs A = make_attn_args(e, B, l);
    HG_CUDA(launch_attn_args(A, st));
    launch_mv_resid(D, B, Ld.wo, B.qo, B.so, st);
    launch_route(D, B, Ld, l, 0, st);
    if (e->ep && Ld.moe) ep_record_moe(e->ep, D, B, Ld, st);  // routed experts on their owners
    else launch_ffn(D, B, Ld, st);
  }
  int mode = e->layers[D.L - 1].moe ? 2 : 1;
  launch_pre_norm(D, B, mode, e->embd, e->out_norm, B.qa, B.sa, nullptr, 0, 1, st);
  launch_lmhead(D, B, e->lm, B.qa, B.sa, B.logits, st);
  // greedy feedback for device-driven multi-step decode; host-driven steps overwrite tok/pos
  launch_feedback(B, const_cast<int32_t*>(B.tok), const_cast<int32_t*>(B.pos), e->d_gen, GEN_CAP, e->d_step, st);
}

DecodeBufs step_bufs(hg_engine* e, int T) {
  DecodeBufs B = e->buf;
  B.T = T;
  B.tok = e->d_meta;
  B.pos = e->d_meta + T;
  B.bt_row = e->d_meta + 2 * T;
  return B;
}

// The step graph for T tokens (captured on first use).
cudaGraphExec_t step_graph(hg_engine* e, int T) {
  DecodeBufs B = step_bufs(e, T);
  cudaStream_t st = e->stream;
  auto it = e->graphs.find(T);
  if (it == e->graphs.end()) {
    cudaGraph_t graph;
    HG_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    try {
      record_decode(e, B);
    } catch (...) {
      cudaStreamEndCapture(st, &graph);
      throw;
    }
    HG_CUDA(cudaStreamEndCapture(st, &graph));
    size_t nodes = 0;
    HG_CUDA(cudaGraphGetNodes(graph, nullptr, &nodes));
    std::vector<cudaGraphNode_t> nv(nodes);
    HG_CUDA(cudaGraphGetNodes(graph, nv.data(), &nodes));
    int kernels = 0;
    for (auto nd : nv) {
      cudaGraphNodeType ty;
      HG_CUDA(cudaGraphNodeGetType(nd, &ty));
      kernels += ty == cudaGraphNodeTypeKernel;
    }
    cudaGraphExec_t exec;
    HG_CUDA(cudaGraphInstantiate(&exec, graph, 0));
    cudaGraphDestroy(graph);
    it = e->graphs.emplace(T, exec).first;
    e->graph_kernels[T] = kernels;
  }
  return it->second;
}

// One decode step for T tokens whose metadata is already in h_meta.
void decode_step(hg_engine* e, int T) {
  DecodeBufs B = step_bufs(e, T);
  cudaStream_t st = e->stream;
  HG_CUDA(cudaMemcpyAsync(e->d_meta, e->h_meta, 3 * T * 4, cudaMemcpyHostToDevice, st));
  HG_CUDA(cudaGraphLaunch(step_graph(e, T), st));
  HG_CUDA(cudaMemcpyAsync(e->h_amax, B.amax, T * 8, cudaMemcpyDeviceToHost, st));
  HG_CUDA(cudaMemcpyAsync(e->h_err, B.err, 4, cudaMemcpyDeviceToHost, st));
  e->last_T = T;
}

void finish_step(hg_engine* e) {
  HG_CUDA(cudaStreamSynchronize(e->stream));
  if (e->h_err[0] != 0) {
    int code = e->h_err[0];
    cudaMemsetAsync(e->buf.err, 0, 4, e->stream);
    cudaStreamSynchronize(e->stream);
    throw Error(code, code == HG_ERR_TOKEN ? "token id out of range" : "device-side error in decode step");
  }
}

uint32_t amax_index(unsigned long long key) { return 0xffffffffu - (uint32_t)(key & 0xffffffffull); }

void seq_check_step(hg_seq* s, uint32_t token) {
  hg_engine* e = s->e;
  if ((int64_t)token >= e->cfg.vocab_size) throw Error(HG_ERR_TOKEN, "token id out of range");
  if (s->len >= s->max_ctx) throw Error(HG_ERR_CONTEXT, "sequence is at its max context");
  ensure_pages(s, s->len + 1);
}

void forward(hg_engine* e, hg_seq* s, uint32_t token, float* logits, uint32_t* next) {
  seq_check_step(s, token);
  e->h_meta[0] = (int32_t)token;
  e->h_meta[1] = s->len;
  e->h_meta[2] = s->row;
  decode_step(e, 1);
  if (logits)
    HG_CUDA(cudaMemcpyAsync(logits, e->buf.logits, (size_t)e->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, e->stream));
  finish_step(e);
  s->len += 1;
  if (next) *next = amax_index(e->h_amax[0]);
}

// Model::forward_x (model.rs:160-184): one decode step from a caller row (d_model floats, host)
// instead of a token embedding; the step graph reads token -1 as "take row t of xin".
void forward_x(hg_engine* e, hg_seq* s, const float* row, float* logits, uint32_t* next) {
  if (s->len >= s->max_ctx) throw Error(HG_ERR_CONTEXT, "sequence is at its max context");
  ensure_pages(s, s->len + 1);
  HG_CUDA(cudaMemcpyAsync(const_cast<float*>(e->buf.xin), row, (size_t)e->cfg.d_model * 4, cudaMemcpyHostToDevice,
                          e->stream));
  e->h_meta[0] = -1;
  e->h_meta[1] = s->len;
  e->h_meta[2] = s->row;
  decode_step(e, 1);
  if (logits)
    HG_CUDA(cudaMemcpyAsync(logits, e->buf.logits, (size_t)e->cfg.vocab_size * 4, cudaMemcpyDeviceToHost, e->stream));
  finish_step(e);
  s->len += 1;
  if (next) *next = amax_index(e->h_amax[0]);
}

void decode_batch(hg_engine* e, hg_seq** seqs, int n, const uint32_t* tokens, uint32_t* next, float* logits) {
  if (n <= 0 || n > e->max_batch) throw Error(HG_ERR_INVALID, "batch size out of range (max_batch)");
  for (int i = 0; i < n; i++) {
    if (!seqs[i] || seqs[i]->e != e) throw Error(HG_ERR_INVALID, "sequence does not belong to this engine");
    for (int j = 0; j < i; j++)
      if (seqs[j] == seqs[i]) throw Error(HG_ERR_INVALID, "a sequence appears twice in one batch");
    seq_check_step(seqs[i], tokens[i]);
  }
  for (int i = 0; i < n; i++) {
    e->h_meta[i] = (int32_t)tokens[i];
    e->h_meta[n + i] = seqs[i]->len;
    e->h_meta[2 * n + i] = seqs[i]->row;
  }
  decode_step(e, n);
  if (logits)
    HG_CUDA(cudaMemcpyAsync(logits, e->buf.logits, (size_t)n * e->cfg.vocab_size * 4, cudaMemcpyDeviceToHost,
                            e->stream));
  finish_step(e);
  for (int i = 0; i < n; i++) {
    seqs[i]->len += 1;
    if (next) next[i] = amax_index(e->h_amax[i]);
  }
}

// K greedy steps for n sequences, driven on the device: the step graph is replayed back to back
// and its feedback kernel turns each argmax into the next input token.
void decode_greedy(hg_engine* e, hg_seq** seqs, int n, const uint32_t* tokens, int steps, uint32_t* out_ids) {
  if (n <= 0 || n > e->max_batch) throw Error(HG_ERR_INVALID, "batch size out of range (max_batch)");
  if (steps <= 0) return;
  for (int i = 0; i < n; i++) {
    if (!seqs[i] || seqs[i]->e != e) throw Error(HG_ERR_INVALID, "sequence does not belong to this engine");
    for (int j = 0; j < i; j++)
      if (seqs[j] == seqs[i]) throw Error(HG_ERR_INVALID, "a sequence appears twice in one batch");
    if ((int64_t)tokens[i] >= e->cfg.vocab_size) throw Error(HG_ERR_TOKEN, "token id out of range");
    if (seqs[i]->len + steps > seqs[i]->max_ctx) throw Error(HG_ERR_CONTEXT, "steps exceed the sequence's max context");
    ensure_pages(seqs[i], seqs[i]->len + steps);
  }
  for (int i = 0; i < n; i++) {
    e->h_meta[i] = (int32_t)tokens[i];
    e->h_meta[n + i] = seqs[i]->len;
    e->h_meta[2 * n + i] = seqs[i]->row;
  }
  cudaStream_t st = e->stream;
  HG_CUDA(cudaMemcpyAsync(e->d_meta, e->h_meta, 3 * n * 4, cudaMemcpyHostToDevice, st));
  HG_CUDA(cudaMemsetAsync(e->d_step, 0, 4, st));
  cudaGraphExec_t g = step_graph(e, n);
  std::vector<int32_t> ring((size_t)GEN_CAP * n);
  for (int k0 = 0; k0 < steps; k0 += GEN_CAP) {
    const int kn = std::min(GEN_CAP, steps - k0);
    for (int k = 0; k < kn; k++) HG_CUDA(cudaGraphLaunch(g, st));
    if (out_ids) {
      HG_CUDA(cudaMemcpyAsync(ring.data(), e->d_gen, ring.size() * 4, cudaMemcpyDeviceToHost, st));
      HG_CUDA(cudaStreamSynchronize(st));
      for (int k = 0; k < kn; k++)
        for (int i = 0; i < n; i++) out_ids[(size_t)(k0 + k) * n + i] = (uint32_t)ring[(size_t)k * n + i];
    }
  }
  HG_CUDA(cudaMemcpyAsync(e->h_err, e->buf.err, 4, cudaMemcpyDeviceToHost, st));
  e->last_T = n;
  finish_step(e);
  for (int i = 0; i < n; i++) seqs[i]->len += steps;
}

// ---------------------------------------------------------------------------------------------
// Prefill (exact reference order), chunked
// ---------------------------------------------------------------------------------------------
// One chunk of Model::prefill (model.rs:340-439). Its inputs are token ids (embedding rows looked
// up on the GPU) or, when embeds is given, tn caller rows of d_model floats (host memory).
// bidir: the rows form one diffusion block (Model::run_block, model.rs:472-587): each attends to
// the prefix and to all tn rows, and the sequence length is left unchanged.
void prefill_chunk(hg_engine* e, hg_seq* s, const uint32_t* ids, const float* embeds, int tn, bool bidir) {
  const hg_config& c = e->cfg;
  const Dims& D = e->D;
  auto& P = e->pf;
  cudaStream_t st = e->stream;
  const int d = c.d_model, base = s->len, k = c.top_k, ne = c.n_experts, f = c.expert_ffn;
  const int32_t* bt = e->d_bt + (size_t)s->row * e->bt_stride;
  if (embeds) {
    HG_CUDA(cudaMemcpyAsync(P.x, embeds, (size_t)tn * d * 4, cudaMemcpyHostToDevice, st));
  } else {
    std::vector<int32_t> h_ids(ids, ids + tn);
    HG_CUDA(cudaMemcpyAsync(P.ids, h_ids.data(), tn * 4, cudaMemcpyHostToDevice, st));
    launch_kp_embed(e->embd, P.ids, tn, d, c.vocab_size, P.x, e->buf.err, st);
  }
  for (int l = 0; l < c.n_layers; l++) {
    const LayerDev& Ld = e->layers[l];
    float* kb = e->kv + (long long)l * e->layer_stride;
    float* vb = kb + e->layer_stride / 2;
    launch_kp_norm(P.x, nullptr, tn, d, Ld.attn_norm, c.rms_eps, nullptr, P.qa, P.sa, st);
    launch_kp_matmul(mm_args(Ld.qkv, P.qa, P.sa, tn, P.qkv, D.qkvd, 0), tn, 1, st);
    launch_kp_qk_rope_append(P.qkv, tn, base, c.n_heads, c.n_kv_heads, c.head_dim, c.rms_eps, Ld.q_norm, Ld.k_norm,
                             e->rope_cos, e->rope_sin, bt, kb, vb, e->page_stride, P.q, st);
    for (int t0 = 0; t0 < tn; t0 += e->pf_tq) {
      int tq = std::min(e->pf_tq, tn - t0);
      launch_kp_attention(P.q, D.qd, t0, tq, base, bidir ? base + tn : 0, c.n_heads, c.n_kv_heads, c.head_dim, bt, kb,
                          vb, e->page_stride,
                          P.S, P.inv, P.mkey, P.o, st);
    }
    launch_kp_quant_rows(P.o, tn, D.qd, P.qa, P.sa, st);
    launch_kp_matmul(mm_args(Ld.wo, P.qa, P.sa, tn, P.x, d, 1), tn, 1, st);
    launch_kp_norm(P.x, nullptr, tn, d, Ld.ffn_norm, c.rms_eps, P.h, P.qa, P.sa, st);
    if (!Ld.moe) {
      const int df = c.dense_ffn;
      launch_kp_matmul(mm_args(Ld.gate, P.qa, P.sa, tn, P.g, df, 0), tn, 1, st);
      launch_kp_matmul(mm_args(Ld.up, P.qa, P.sa, tn, P.u, df, 0), tn, 1, st);
      launch_kp_swiglu(P.g, P.u, P.act, (long long)tn * df, st);
      launch_kp_quant_rows(P.act, tn, df, P.qact, P.sact, st);
      launch_kp_matmul(mm_args(Ld.down, P.qact, P.sact, tn, P.y, (k + 1) * d, 0), tn, 1, st);
      launch_kp_combine(P.x, P.y, P.sel, P.selw, tn, d, k, 0, c.n_shared, st);
      continue;
    }
    HG_CUDA(cudaMemsetAsync(P.ecount, 0, ne * 4, st));
    launch_kp_route(P.h, tn, d, Ld.router, Ld.bias, ne, k, c.gating_sigmoid, c.expert_weights_norm,
                    c.expert_weights_scale, P.sel, P.selw, P.ecount, P.elist, tn, st);
    launch_kp_expert_tables(P.ecount, ne, tn, P.gm, P.go, P.gc, st);
    launch_kp_entry_rows(P.elist, ne * tn, k, P.a_idx, P.o_idx, st);
    launch_kp_shared_rows(tn, k, P.o_idx + (size_t)ne * tn, st);
    const int rows_tot = tn * (k + 1);
    // gate / up: shared expert (all tokens, slot k) then routed experts grouped
    if (c.n_shared > 0) {
      MmArgs a = mm_args(Ld.sgate, P.qa, P.sa, tn, P.g, f, 0);
      a.o_idx = P.o_idx + (size_t)ne * tn;
      launch_kp_matmul(a, tn, 1, st);
      a.W = Ld.sup;
      a.out = P.u;
      launch_kp_matmul(a, tn, 1, st);
    }
    {
      MmArgs a = mm_args(Ld.gate, P.qa, P.sa, tn, P.g, f, 0);
      a.a_idx = P.a_idx;
      a.o_idx = P.o_idx;
      a.grp_mat = P.gm;
      a.grp_off = P.go;
      a.grp_cnt = P.gc;
      launch_kp_matmul(a, tn, ne, st);
      a.W = Ld.up;
      a.out = P.u;
      launch_kp_matmul(a, tn, ne, st);
    }
    launch_kp_swiglu(P.g, P.u, P.act, (long long)rows_tot * f, st);
    launch_kp_quant_rows(P.act, rows_tot, f, P.qact, P.sact, st);
    if (c.n_shared > 0) {
      MmArgs a = mm_args(Ld.sdown, P.qact, P.sact, tn, P.y, d, 0);
      a.a_idx = P.o_idx + (size_t)ne * tn;
      a.o_idx = P.o_idx + (size_t)ne * tn;
      launch_kp_matmul(a, tn, 1, st);
    }
    {
      MmArgs a = mm_args(Ld.down, P.qact, P.sact, tn, P.y, d, 0);
      a.a_idx = P.o_idx;
      a.o_idx = P.o_idx;
      a.grp_mat = P.gm;
      a.grp_off = P.go;
      a.grp_cnt = P.gc;
      launch_kp_matmul(a, tn, ne, st);
    }
    launch_kp_combine(P.x, P.y, P.sel, P.selw, tn, d, k, 1, c.n_shared, st);
  }
  if (!bidir) s->len += tn;
}

// Model::prefill over n inputs: token ids, or (ids == null) n rows of d_model floats in embeds.
void prefill(hg_engine* e, hg_seq* s, const uint32_t* ids, const float* embeds, int n, float* logits, uint32_t* next) {
  if (n <= 0) throw Error(HG_ERR_INVALID, "empty prefill");
  if (ids) {
    for (int i = 0; i < n; i++)
      if ((int64_t)ids[i] >= e->cfg.vocab_size) throw Error(HG_ERR_TOKEN, "token id out of range");
  }
  if (s->len + n > s->max_ctx) throw Error(HG_ERR_CONTEXT, "prompt exceeds the sequence's max context");
  ensure_pages(s, s->len + n);
  int last = 0;
  for (int c0 = 0; c0 < n; c0 += e->pf_rows) {
    int tn = std::min(e->pf_rows, n - c0);
    prefill_chunk(e, s, ids ? ids + c0 : nullptr, ids ? nullptr : embeds + (size_t)c0 * e->cfg.d_model, tn, false);
    last = tn;
  }
  // model.rs:365-369: exact norm of the last row, then the decode-style lm_head matvec
  const Dims& D = e->D;
  auto& P = e->pf;
  cudaStream_t st = e->stream;
  launch_kp_norm(P.x + (size_t)(last - 1) * D.d, nullptr, 1, D.d, e->out_norm, e->cfg.rms_eps, nullptr, e->buf.qa,
                 e->buf.sa, st);
  DecodeBufs B = e->buf;
  B.T = 1;
  HG_CUDA(cudaMemsetAsync(B.amax, 0, 8, st));
  launch_lmhead(D, B, e->lm, B.qa, B.sa, B.logits, st);
  HG_CUDA(cudaMemcpyAsync(e->h_amax, B.amax, 8, cudaMemcpyDeviceToHost, st));
  HG_CUDA(cudaMemcpyAsync(e->h_err, B.err, 4, cudaMemcpyDeviceToHost, st));
  if (logits) HG_CUDA(cudaMemcpyAsync(logits, B.logits, (size_t)D.vocab * 4, cudaMemcpyDeviceToHost, st));
  finish_step(e);
  if (next) *next = amax_index(e->h_amax[0]);
}

// Model::run_block (model.rs:472-510) of n token ids at positions len..len+n: each row attends to
// the sequence's prefix and to every row of the block, with the prefill arithmetic. The block's
// K/V rows go to its pages past len; commit makes them part of the prefix (lib.rs:386-391),
// otherwise the next call at the same position overwrites them. logits (host, may be null):
// [n_logits][vocab] of the last n_logits rows through output.matmul (model.rs:505-508).
void run_block(hg_engine* e, hg_seq* s, const uint32_t* ids, int n, int n_logits, bool commit, float* logits) {
  const hg_config& c = e->cfg;
  if (n <= 0 || n > PF_BLOCK_MAX) throw Error(HG_ERR_INVALID, "block rows out of range (1..1024 per bidirectional pass)");
  if (n_logits < 0 || n_logits > n) throw Error(HG_ERR_INVALID, "n_logits out of range");
  for (int i = 0; i < n; i++)
    if ((int64_t)ids[i] >= c.vocab_size) throw Error(HG_ERR_TOKEN, "token id out of range");
  if (s->len + n > s->max_ctx) throw Error(HG_ERR_CONTEXT, "block exceeds the sequence's max context");
  ensure_pages(s, s->len + n);
  prefill_chunk(e, s, ids, nullptr, n, true);
  cudaStream_t st = e->stream;
  if (n_logits > 0) {
    const Dims& D = e->D;
    auto& P = e->pf;
    if (e->blk_logits_rows < n_logits) {
      HG_CUDA(cudaStreamSynchronize(st));
      if (e->blk_logits) HG_CUDA(cudaFree(e->blk_logits));
      e->blk_logits = nullptr;
      e->blk_logits_rows = 0;
      HG_CUDA(cudaMalloc(&e->blk_logits, (size_t)n_logits * D.vocab * 4));
      e->blk_logits_rows = n_logits;
    }
    const int r0 = n - n_logits;
    launch_kp_norm(P.x + (size_t)r0 * D.d, nullptr, n_logits, D.d, e->out_norm, c.rms_eps, nullptr, P.qa, P.sa, st);
    launch_kp_matmul(mm_args(e->lm, P.qa, P.sa, n_logits, e->blk_logits, D.vocab, 0), n_logits, 1, st);
    if (logits)
      HG_CUDA(cudaMemcpyAsync(logits, e->blk_logits, (size_t)n_logits * D.vocab * 4, cudaMemcpyDeviceToHost, st));
  }
  HG_CUDA(cudaMemcpyAsync(e->h_err, e->buf.err, 4, cudaMemcpyDeviceToHost, st));
  finish_step(e);
  if (commit) s->len += n;
}

hg_seq* seq_create(hg_engine* e, int max_ctx) {
  if (max_ctx <= 0 || max_ctx > e->cfg.context_length) max_ctx = e->cfg.context_length;
  if (e->free_rows.empty()) throw Error(HG_ERR_POOL_EXHAUSTED, "too many live sequences");
  hg_seq* s = new hg_seq();
  s->e = e;
  s->row = e->free_rows.back();
  e->free_rows.pop_back();
  s->max_ctx = max_ctx;
  e->live_seqs.insert(s);
  return s;
}

void seq_free(hg_seq* s) {
  if (!s) return;
  if (hg_engine* e = s->e) {
    for (int p : s->pages) e->free_pages.push_back(p);
    e->free_rows.push_back(s->row);
    e->live_seqs.erase(s);
  }
  delete s;
}

// Engine::generate (lib.rs:107-162): n_rows caller rows of d_model floats (lib.rs:118-121's
// embeds; host memory) and then the n prompt ids are prefilled (two prefills over consecutive
// positions equal one), followed by the sampling loop.
int generate(hg_engine* e, const float* rows, int n_rows, const uint32_t* ids, int n, const hg_gen_opts* opts,
             hg_token_cb cb, void* user, uint32_t* out_ids) {
  hg_gen_opts o = opts ? *opts : hg_gen_opts{256, 0.0f, 0.95f, 1234, 1.0f};
  if (n < 0 || n_rows < 0) throw Error(HG_ERR_INVALID, "negative length");
  if (n + n_rows == 0) return 0;  // lib.rs:122-124
  std::unique_ptr<hg_seq, void (*)(hg_seq*)> s(seq_create(e, e->cfg.context_length), seq_free);
  const int V = e->cfg.vocab_size, valid = std::min(50257, V);
  // sampled tokens (temperature, top-p, repetition penalty) are drawn on the GPU (sample.cu) from
  // the step's logits in place; only vocabularies wider than the device sort use the host sampler
  const bool sampled = o.temp > 0.0f || o.rep_penalty != 1.0f;
  const bool dev_sample = sampled && sample_usable(V);
  const bool host_path = sampled && !dev_sample;
  std::vector<float> logits(host_path ? V : 0);
  Rng rng(o.seed);
  if (dev_sample) {
    if (!e->smp) HG_CUDA(cudaMalloc(&e->smp, sample_scratch_bytes(V)));
    if (!e->h_smp) HG_CUDA(cudaMallocHost((void**)&e->h_smp, 16));
    unsigned long long state = 0;
    sample_reset(e->smp, V, o.seed, e->stream, &state);
    HG_CUDA(cudaStreamSynchronize(e->stream));
  }
  uint32_t gpu_next = 0;
  if (n_rows > 0)
    prefill(e, s.get(), nullptr, rows, n_rows, n == 0 && host_path ? logits.data() : nullptr, &gpu_next);
  if (n > 0) prefill(e, s.get(), ids, nullptr, n, host_path ? logits.data() : nullptr, &gpu_next);
  int pos = n_rows + n, count = 0;
  std::vector<uint32_t> out;
  for (int it = 0; it < o.max_new; it++) {
    uint32_t next;
    if (dev_sample) {  // the last step's logits (row 0 of the step buffer) are still on the GPU
      launch_sample(e->buf.logits, V, valid, o.temp, o.top_p, o.rep_penalty, e->smp, e->stream);
      HG_CUDA(cudaGetLastError());
      HG_CUDA(cudaMemcpyAsync(e->h_smp, sample_next_ptr(e->smp), 4, cudaMemcpyDeviceToHost, e->stream));
      HG_CUDA(cudaStreamSynchronize(e->stream));
      next = e->h_smp[0];
    } else if (host_path) {
      for (int i = valid; i < V; i++) logits[i] = -INFINITY;
      if (o.rep_penalty != 1.0f)
        for (uint32_t t : out) {
          float& l = logits[t];
          l = l > 0.0f ? l / o.rep_penalty : l * o.rep_penalty;
        }
      next = host_sample(logits.data(), V, o.temp, o.top_p, rng);
    } else {
      next = gpu_next;
    }
    if (next == (uint32_t)e->cfg.eos_token) break;
    out.push_back(next);
    if (out_ids) out_ids[count] = next;
    count++;
    if (cb && !cb(next, user)) break;
    if (pos + 1 >= e->cfg.context_length) break;
    forward(e, s.get(), next, host_path ? logits.data() : nullptr, &gpu_next);
    pos += 1;
  }
  return count;
}

// ---------------------------------------------------------------------------------------------
// Diffusion decode (lib.rs:164-495): blocks of [MASK] ids filled over denoising passes of
// run_block on the GPU; each pass's block logits are scored on the host.
// ---------------------------------------------------------------------------------------------
// The unmasking passes shared by both paths for one block (lib.rs:304-384 / 425-471): `ids` are
// the block's current ids, `step` runs one scored pass over them.
template <class Step>
void fill_block(uint32_t* ids, int blk_len, int gen_len, uint32_t mask, const hg_diff_opts& o, bool threshold_mode,
                const uint32_t* pred, const float* pconf, const float* cconf, Step step) {
  auto any_masked = [&]() { return std::find(ids, ids + blk_len, mask) != ids + blk_len; };
  if (threshold_mode) {
    // Fast-dLLM confidence threshold (lib.rs:304-327): commit every masked row at or above it,
    // or else the most confident one (Iterator::max_by keeps the last of equal maxima).
    for (int it = 0; it < std::max(blk_len, 1); it++) {
      if (!any_masked()) break;
      step();
      int best = -1;
      for (int i = 0; i < blk_len; i++)
        if (ids[i] == mask && (best < 0 || !(pconf[i] < pconf[best]))) best = i;
      bool any = false;
      for (int i = 0; i < blk_len; i++)
        if (ids[i] == mask && pconf[i] >= o.threshold) {
          ids[i] = pred[i];
          any = true;
        }
      if (!any) ids[best] = pred[best];
    }
  } else {
    // fixed num_transfer schedule (lib.rs:328-354): the k most confident masked rows per pass
    const int sb = std::max((int)std::round((float)(o.steps * blk_len) / (float)gen_len), 1);
    for (int k_step : num_transfer(blk_len, sb)) {
      step();
      std::vector<std::pair<int, float>> cand;
      for (int i = 0; i < blk_len; i++)
        if (ids[i] == mask) cand.push_back({i, pconf[i]});
      if (cand.empty()) break;
      std::stable_sort(cand.begin(), cand.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
      for (int r = 0; r < std::min(k_step, (int)cand.size()); r++) ids[cand[r].first] = pred[cand[r].first];
    }
    if (any_masked()) {
      step();
      for (int i = 0; i < blk_len; i++)
        if (ids[i] == mask) ids[i] = pred[i];
    }
  }
  // low-confidence remasking (lib.rs:356-375)
  for (int it = 0; it < o.remask_steps; it++) {
    step();
    const int r = std::max((int)((float)blk_len * o.remask_frac), 1);
    std::vector<std::pair<int, float>> idx(blk_len);
    for (int i = 0; i < blk_len; i++) idx[i] = {i, cconf[i]};
    std::stable_sort(idx.begin(), idx.end(), [](const auto& a, const auto& b) { return a.second < b.second; });
    for (int q = 0; q < std::min(r, blk_len); q++) ids[idx[q].first] = mask;
    step();
    for (int i = 0; i < blk_len; i++)
      if (ids[i] == mask) ids[i] = pred[i];
  }
}

// Streams the generated ids up to the first eos (lib.rs:393-405 / 473-491, one call per block);
// returns false to stop, with *count set to the generated length.
bool stream_block(const std::vector<uint32_t>& ids, int p, int upto, uint32_t eos, int& emitted, hg_block_cb cb,
                  void* user, uint32_t* out_ids, int* count) {
  int endpos = upto;
  bool hit = false;
  for (int i = p; i < upto; i++)
    if (ids[i] == eos) {
      endpos = i;
      hit = true;
      break;
    }
  const int n_new = endpos - p - emitted;
  if (out_ids && n_new > 0) std::copy(ids.begin() + p + emitted, ids.begin() + endpos, out_ids + emitted);
  const int cont = cb ? cb(ids.data() + p + emitted, n_new, user) : 1;
  emitted = endpos - p;
  *count = endpos - p;
  return !(hit || !cont);
}

// lib.rs:265-407 (generate_diffusion_cached): the prompt is encoded bidirectionally into the
// sequence, then each block's passes run only the block against that frozen prefix.
int diffusion_cached(hg_engine* e, const uint32_t* prompt, int p, const hg_diff_opts& o, hg_block_cb cb, void* user,
                     uint32_t* out_ids) {
  const hg_config& c = e->cfg;
  const int V = c.vocab_size, valid = std::min(50257, V);
  const uint32_t mask = (uint32_t)c.mask_token_id;
  Rng rng(o.seed);
  if (p == 0) return 0;
  const int gen_len = std::min(o.gen_len, std::max(c.context_length - (p + o.block), 1));
  std::unique_ptr<hg_seq, void (*)(hg_seq*)> s(seq_create(e, c.context_length), seq_free);
  run_block(e, s.get(), prompt, p, 0, true, nullptr);
  std::vector<uint32_t> committed(prompt, prompt + p);
  std::vector<float> all, rows;
  int emitted = 0, count = 0;
  for (int b0 = p; b0 < p + gen_len;) {
    const int b1 = std::min(b0 + o.block, p + gen_len), blk_len = b1 - b0;
    std::vector<uint32_t> blk(blk_len, mask), pred(blk_len);
    std::vector<float> pconf(blk_len), cconf(blk_len);
    all.resize((size_t)blk_len * V);
    auto step = [&]() {
      run_block(e, s.get(), blk.data(), blk_len, blk_len, false, all.data());
      score_block(all.data(), V, blk.data(), blk_len, committed.data(), (int)committed.size(), valid, mask,
                  o.rep_penalty, o.temp, rng, pred.data(), pconf.data(), cconf.data(), rows);
    };
    fill_block(blk.data(), blk_len, gen_len, mask, o, o.threshold > 0.0f, pred.data(), pconf.data(), cconf.data(),
               step);
    run_block(e, s.get(), blk.data(), blk_len, 0, true, nullptr);  // finalize: the block joins the prefix
    committed.insert(committed.end(), blk.begin(), blk.end());
    if (!stream_block(committed, p, (int)committed.size(), (uint32_t)c.eos_token, emitted, cb, user, out_ids, &count))
      return count;
    b0 = b1;
  }
  return gen_len;
}

// lib.rs:409-495 (generate_diffusion_uncached): every pass re-runs the canvas x[0..b1] as one
// bidirectional block from position 0 (Model::forward_bidir, model.rs:441-470, is run_block on an
// empty prefix) and scores the active block's rows (diffusion_block, lib.rs:164-209).
int diffusion_uncached(hg_engine* e, const uint32_t* prompt, int p, const hg_diff_opts& o, hg_block_cb cb,
                       void* user, uint32_t* out_ids) {
  const hg_config& c = e->cfg;
  const int V = c.vocab_size, valid = std::min(50257, V);
  const uint32_t mask = (uint32_t)c.mask_token_id;
  Rng rng(o.seed);
  const int gen_len = std::min(o.gen_len, std::max(c.context_length - p, 1));
  std::vector<uint32_t> x(prompt, prompt + p);
  x.resize((size_t)p + std::max(gen_len, 0), mask);
  std::unique_ptr<hg_seq, void (*)(hg_seq*)> s(seq_create(e, c.context_length), seq_free);
  std::vector<float> all, rows;
  int emitted = 0, count = 0;
  for (int b0 = p; b0 < p + gen_len;) {
    const int b1 = std::min(b0 + o.block, p + gen_len), blk_len = b1 - b0;
    std::vector<uint32_t> pred(blk_len);
    std::vector<float> pconf(blk_len), cconf(blk_len);
    all.resize((size_t)blk_len * V);
    auto step = [&]() {
      run_block(e, s.get(), x.data(), b1, blk_len, false, all.data());
      score_block(all.data(), V, x.data() + b0, blk_len, x.data(), b0, valid, mask, o.rep_penalty, o.temp, rng,
                  pred.data(), pconf.data(), cconf.data(), rows);
    };
    fill_block(x.data() + b0, blk_len, gen_len, mask, o, false, pred.data(), pconf.data(), cconf.data(), step);
    if (!stream_block(x, p, b1, (uint32_t)c.eos_token, emitted, cb, user, out_ids, &count)) return count;
    b0 = b1;
  }
  return gen_len;
}

// Engine::generate_diffusion (lib.rs:211-220).
int generate_diffusion(hg_engine* e, const uint32_t* ids, int n, const hg_diff_opts* opts, hg_block_cb cb, void* user,
                       uint32_t* out_ids) {
  hg_diff_opts o = opts ? *opts : hg_diff_opts{128, 32, 32, 0.0f, 1.4f, 0, 0.3f, 1234, 1, 0.0f};
  if (o.block <= 0) o.block = std::max(e->cfg.block_size, 1);
  if (n < 0 || o.gen_len < 0) throw Error(HG_ERR_INVALID, "negative prompt or generation length");
  for (int i = 0; i < n; i++)
    if ((int64_t)ids[i] >= e->cfg.vocab_size) throw Error(HG_ERR_TOKEN, "token id out of range");
  if ((int64_t)e->cfg.mask_token_id >= e->cfg.vocab_size) throw Error(HG_ERR_TOKEN, "mask token id out of range");
  return o.cached ? diffusion_cached(e, ids, n, o, cb, user, out_ids)
                  : diffusion_uncached(e, ids, n, o, cb, user, out_ids);
}

}  // namespace


// ---------------------------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------------------------
#define HG_API_TRY(...)                                                \
  try {                                                                \
    __VA_ARGS__;                                                       \
    return HG_OK;                                                      \
  } catch (const ::hg::Error& ex_) {                                   \
    ::hg::set_last_error(ex_.what());                                  \
    return ex_.code;                                                   \
  } catch (const std::bad_alloc&) {                                    \
    ::hg::set_last_error("host out of memory");                        \
    return HG_ERR_INVALID;                                             \
  } catch (const std::exception& ex_) {                                \
    ::hg::set_last_error(ex_.what());                                  \
    return HG_ERR_INVALID;                                             \
  }

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

void need(bool ok, const char* what) {
  if (!ok) throw Error(HG_ERR_INVALID, what);
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

Q8M q8m(const int8_t* qs, const float* sc, int64_t count, int64_t rows, int64_t cols) {
  Q8M m;
  m.qs = qs;
  m.sc = sc;
  m.rows = (int)rows;
  m.cols = (int)cols;
  m.ss = host_q8_ss(cols);
  m.qs_mstride = rows * cols;
  m.sc_mstride = rows * m.ss;
  (void)count;
  return m;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// Scratch layout of hg_op_moe_ffn (device buffer supplied by the caller).
struct MoeScratch {
  size_t off_qh, off_sh, off_sel, off_selw, off_ecount, off_active, off_elist, off_act, off_ubuf, off_qact, off_sact,
      off_y, off_err, total;
};
MoeScratch moe_scratch_layout(const hg_moe_weights* w, int ntok) {
  MoeScratch s{};
  size_t o = 0;
  const int d = w->d_model, f = w->expert_ffn, k = w->top_k, ne = w->n_experts;
  auto take = [&](size_t bytes) {
    size_t r = o;
    o += align256(bytes);
    return r;
  };
  s.off_qh = take((size_t)ntok * d);
  s.off_sh = take((size_t)ntok * host_q8_ss(d) * 4);
  s.off_sel = take((size_t)ntok * k * 4);
  s.off_selw = take((size_t)ntok * k * 4);
  s.off_ecount = take((size_t)(ne + 2) * 4);
  s.off_active = take((size_t)ne * 4);
  s.off_elist = take((size_t)ne * ntok * 4);
  s.off_act = take((size_t)ntok * (k + 1) * f * 4);
  s.off_ubuf = take((size_t)ntok * (k + 1) * f * 4);
  s.off_qact = take((size_t)ntok * (k + 1) * f);
  s.off_sact = take((size_t)ntok * (k + 1) * host_q8_ss(f) * 4);
  s.off_y = take((size_t)ntok * (k + 1) * d * 4);
  s.off_err = take(16);
  s.total = o;
  return s;
}

size_t kv_s_stride(const hg_kv_attn_args* a) { return ((size_t)a->max_pos + 15) & ~size_t(15); }
size_t kv_scratch_bytes(const hg_kv_attn_args* a) {
  return align256((size_t)a->n_seqs * a->n_heads * kv_s_stride(a) * 4) +
         align256((size_t)a->n_seqs * a->n_heads * 4) +
         align256((size_t)a->n_seqs * a->n_heads * 4) + align256((size_t)a->n_seqs * a->n_heads * a->head_dim * 4) +
         align256((size_t)a->n_seqs * 4) + 256;
}

}  // namespace

extern "C" {

const char* hg_last_error(void) { return g_last_error.c_str(); }

int hg_engine_load_ex(const char* gguf_path, const hg_engine_opts* opts, hg_engine** out) {
  HG_API_TRY({
    need(gguf_path && out, "null argument");
    *out = nullptr;
    hg_engine_opts o{};
    if (opts) o = *opts;
    hg_engine* e = new hg_engine();
    try {
      load_engine(e, gguf_path, o);
    } catch (...) {
      free_engine(e);
      throw;
    }
    *out = e;
  })
}

int hg_engine_load(const char* gguf_path, int device, hg_engine** out) {
  hg_engine_opts o{};
  o.device = device;
  return hg_engine_load_ex(gguf_path, &o, out);
}

void hg_engine_free(hg_engine* e) { free_engine(e); }

int hg_engine_config(const hg_engine* e, hg_config* out) {
  HG_API_TRY({
    need(e && out, "null argument");
    *out = e->cfg;
  })
}

int hg_gguf_config(const char* gguf_path, hg_config* out) {
  HG_API_TRY({
    need(gguf_path && out, "null argument");
    Gguf g(gguf_path);
    *out = config_from_gguf(g);
  })
}

int hg_gguf_tensor_f32(const char* gguf_path, const char* name, float* out, int64_t n) {
  HG_API_TRY({
    need(gguf_path && name && out, "null argument");
    Gguf g(gguf_path);
    const GgufTensor* t = g.tensor(name);
    if (!t) throw Error(HG_ERR_MISSING, std::string("tensor `") + name + "` not found");
    need(n == (int64_t)t->n_elems(), "element count differs from the tensor's");
    std::vector<float> v = g.load(name);
    std::copy(v.begin(), v.end(), out);
  })
}

uint64_t hg_engine_weight_bytes(const hg_engine* e) { return e ? e->ref_weight_bytes : 0; }
uint32_t hg_engine_eos(const hg_engine* e) { return e ? (uint32_t)e->cfg.eos_token : 0; }
uint64_t hg_engine_device_bytes(const hg_engine* e) {
  return e ? (uint64_t)(e->device_bytes() + (size_t)e->n_pages * e->page_stride * 4) : 0;
}

int hg_seq_create(hg_engine* e, int max_ctx, hg_seq** out) {
  HG_API_TRY({
    need(e && out, "null argument");
    *out = seq_create(e, max_ctx);
  })
}

void hg_seq_free(hg_seq* s) { seq_free(s); }
int hg_seq_len(const hg_seq* s) { return s ? s->len : -1; }

int hg_prefill(hg_engine* e, hg_seq* s, const uint32_t* ids, int n, float* logits_or_null) {
  HG_API_TRY({
    need(e && s && ids && s->e == e, "bad argument");
    DeviceGuard g(e->device);
    prefill(e, s, ids, nullptr, n, logits_or_null, nullptr);
  })
}

int hg_prefill_embeds(hg_engine* e, hg_seq* s, const float* embeds, int n, float* logits_or_null) {
  HG_API_TRY({
    need(e && s && embeds && s->e == e, "bad argument");
    DeviceGuard g(e->device);
    prefill(e, s, nullptr, embeds, n, logits_or_null, nullptr);
  })
}

int hg_forward(hg_engine* e, hg_seq* s, uint32_t token, float* logits_or_null, uint32_t* argmax_or_null) {
  HG_API_TRY({
    need(e && s && s->e == e, "bad argument");
    DeviceGuard g(e->device);
    forward(e, s, token, logits_or_null, argmax_or_null);
  })
}

int hg_forward_x(hg_engine* e, hg_seq* s, const float* row, float* logits_or_null, uint32_t* argmax_or_null) {
  HG_API_TRY({
    need(e && s && row && s->e == e, "bad argument");
    DeviceGuard g(e->device);
    forward_x(e, s, row, logits_or_null, argmax_or_null);
  })
}

int hg_decode_batch(hg_engine* e, hg_seq** seqs, int n, const uint32_t* tokens, uint32_t* next_ids,
                    float* logits_or_null) {
  HG_API_TRY({
    need(e && seqs && tokens, "null argument");
    DeviceGuard g(e->device);
    decode_batch(e, seqs, n, tokens, next_ids, logits_or_null);
  })
}

int hg_generate(hg_engine* e, const uint32_t* ids, int n, const hg_gen_opts* opts, hg_token_cb cb, void* user,
                uint32_t* out_ids) {
  try {
    need(e && (ids || n == 0), "null argument");
    DeviceGuard g(e->device);
    if (n <= 0) return 0;
    return generate(e, nullptr, 0, ids, n, opts, cb, user, out_ids);
  } catch (const ::hg::Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  } catch (const std::exception& ex) {
    set_last_error(ex.what());
    return HG_ERR_INVALID;
  }
}

int hg_generate_embeds(hg_engine* e, const float* embeds, int n_embeds, const uint32_t* ids, int n,
                       const hg_gen_opts* opts, hg_token_cb cb, void* user, uint32_t* out_ids) {
  try {
    need(e && (embeds || n_embeds == 0) && (ids || n == 0), "null argument");
    DeviceGuard g(e->device);
    return generate(e, embeds, n_embeds, ids, n, opts, cb, user, out_ids);
  } catch (const ::hg::Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  } catch (const std::exception& ex) {
    set_last_error(ex.what());
    return HG_ERR_INVALID;
  }
}

int hg_run_block(hg_engine* e, hg_seq* s, const uint32_t* ids, int n, int n_logits, int commit,
                 float* logits_or_null) {
  HG_API_TRY({
    need(e && s && ids && s->e == e, "bad argument");
    DeviceGuard g(e->device);
    run_block(e, s, ids, n, n_logits, commit != 0, logits_or_null);
  })
}

int hg_generate_diffusion(hg_engine* e, const uint32_t* ids, int n, const hg_diff_opts* opts, hg_block_cb cb,
                          void* user, uint32_t* out_ids) {
  try {
    need(e && (ids || n == 0), "null argument");
    DeviceGuard g(e->device);
    return generate_diffusion(e, ids, n, opts, cb, user, out_ids);
  } catch (const ::hg::Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  } catch (const std::exception& ex) {
    set_last_error(ex.what());
    return HG_ERR_INVALID;
  }
}

int hg_decode_greedy(hg_engine* e, hg_seq** seqs, int n, const uint32_t* tokens, int steps, uint32_t* out_ids) {
  HG_API_TRY({
    need(e && seqs && tokens && steps >= 0, "bad argument");
    DeviceGuard g(e->device);
    decode_greedy(e, seqs, n, tokens, steps, out_ids);
  })
}

void* hg_engine_stream(const hg_engine* e) { return e ? (void*)e->stream : nullptr; }

int hg_ep_unique_id(void* out) {
  HG_API_TRY({
    need(out, "null argument");
    ep_unique_id(out);
  })
}

int hg_engine_ep_init(hg_engine* e, const void* nccl_id, int rank, int world) {
  HG_API_TRY({
    need(e && nccl_id, "null argument");
    need(!e->ep, "expert parallelism is already set up on this engine");
    DeviceGuard g(e->device);
    HG_CUDA(cudaStreamSynchronize(e->stream));
    // step graphs recorded before hold the local experts: drop them
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
    e->graph_kernels.clear();
    e->ep = ep_create(e->D, e->max_batch, e->device, nccl_id, rank, world);
  })
}

int hg_decode_kernel_count(hg_engine* e, int n) {
  try {
    need(e && n > 0 && n <= e->max_batch, "bad argument");
    DeviceGuard g(e->device);
    step_graph(e, n);
    return e->graph_kernels[n];
  } catch (const ::hg::Error& ex) {
    set_last_error(ex.what());
    return ex.code;
  }
}

int hg_debug_time_attention(hg_engine* e, hg_seq** seqs, int n, int iters, float* ms_scores, float* ms_out) {
  HG_API_TRY({
    need(e && seqs && n > 0 && n <= e->max_batch && iters > 0, "bad argument");
    DeviceGuard g(e->device);
    for (int i = 0; i < n; i++) {
      need(seqs[i] && seqs[i]->e == e && seqs[i]->len > 0, "sequences must have decoded at least one step");
      e->h_meta[i] = 0;
      e->h_meta[n + i] = seqs[i]->len - 1;  // re-run the last step: the append rewrites the same K/V row
      e->h_meta[2 * n + i] = seqs[i]->row;
    }
    cudaStream_t st = e->stream;
    HG_CUDA(cudaMemcpyAsync(e->d_meta, e->h_meta, 3 * n * 4, cudaMemcpyHostToDevice, st));
    DecodeBufs B = step_bufs(e, n);
    // the qkv buffer holds the last decode step's projections of the last layer
    AttnArgs A = make_attn_args(e, B, e->cfg.n_layers - 1);
    cudaEvent_t ev[3];
    for (auto& x : ev) HG_CUDA(cudaEventCreate(&x));
    float tot_s = 0, tot_o = 0;
    for (int it = 0; it < iters; it++) {
      HG_CUDA(cudaEventRecord(ev[0], st));
      HG_CUDA(launch_attn_scores_only(A, st));
      HG_CUDA(cudaEventRecord(ev[1], st));
      HG_CUDA(launch_attn_out_only(A, st));
      HG_CUDA(cudaEventRecord(ev[2], st));
      HG_CUDA(cudaEventSynchronize(ev[2]));
      float a, b;
      HG_CUDA(cudaEventElapsedTime(&a, ev[0], ev[1]));
      HG_CUDA(cudaEventElapsedTime(&b, ev[1], ev[2]));
      tot_s += a;
      tot_o += b;
    }
    for (auto& x : ev) cudaEventDestroy(x);
    if (ms_scores) *ms_scores = tot_s / iters;
    if (ms_out) *ms_out = tot_o / iters;
  })
}

int hg_debug_last_routing(hg_engine* e, int slot, int32_t* sel) {
  HG_API_TRY({
    need(e && sel, "null argument");
    need(slot >= 0 && slot < std::max(e->last_T, 1), "slot out of range");
    DeviceGuard g(e->device);
    const int L = e->cfg.n_layers, k = e->cfg.top_k, T = std::max(e->last_T, 1);
    std::vector<int32_t> all((size_t)L * T * k);
    HG_CUDA(cudaMemcpy(all.data(), e->buf.dbg_sel, all.size() * 4, cudaMemcpyDeviceToHost));
    for (int l = 0; l < L; l++)
      for (int r = 0; r < k; r++)
        sel[l * k + r] = e->layers[l].moe ? all[((size_t)l * T + slot) * k + r] : -1;
  })
}

int hg_q8_scale_stride(int64_t cols) { return host_q8_ss(cols); }

int hg_q8_pack(const float* w, int64_t rows, int64_t cols, int8_t* qs_out, float* scales_out) {
  HG_API_TRY({
    need(w && qs_out && scales_out && rows > 0 && cols > 0, "bad argument");
    q8_pack_rows(w, rows, cols, qs_out, scales_out);
  })
}

int hg_q8_unpack_qs(const int8_t* packed, int64_t rows, int64_t cols, int8_t* qs_out) {
  HG_API_TRY({
    need(packed && qs_out && cols % 32 == 0, "bad argument");
    int nb = (int)(cols / 32);
    for (int64_t r = 0; r < rows; r++)
      for (int64_t k = 0; k < cols; k++) qs_out[r * cols + k] = packed[r * cols + q8_pos((int)k, nb)];
  })
}

int hg_rope_tables(int head_dim, int max_pos, float theta, float* cos_out, float* sin_out) {
  HG_API_TRY({
    need(cos_out && sin_out && head_dim > 0 && max_pos > 0, "bad argument");
    rope_tables(head_dim, max_pos, theta, cos_out, sin_out);
  })
}

int hg_op_q8_matvec(const int8_t* qs, const float* scales, int64_t rows, int64_t cols, const float* x, float* y,
                    int ntok, void* stream) {
  HG_API_TRY({
    need(qs && scales && x && y && rows > 0 && cols > 0 && cols % 32 == 0 && ntok > 0, "bad argument");
    cudaStream_t st = as_stream(stream);
    const int ss = host_q8_ss(cols);
    int8_t* aq = nullptr;
    float* as = nullptr;
    HG_CUDA(cudaMallocAsync((void**)&aq, (size_t)ntok * cols, st));
    HG_CUDA(cudaMallocAsync((void**)&as, (size_t)ntok * ss * 4, st));
    launch_quant_rows(x, ntok, (int)cols, aq, as, st);
    HG_CUDA(prepare_tc());
    Dims D{};
    DecodeBufs B{};
    B.T = ntok;
    Q8M W = q8m(qs, scales, 1, rows, cols);
    launch_mv_store(D, B, W, aq, as, y, (int)rows, st);
    HG_CUDA(cudaGetLastError());
    HG_CUDA(cudaFreeAsync(aq, st));
    HG_CUDA(cudaFreeAsync(as, st));
  })
}

int hg_op_q8_matmul(const int8_t* qs, const float* scales, int64_t rows, int64_t cols, const float* x, float* y,
                    int ntok, void* stream) {
  HG_API_TRY({
    need(qs && scales && x && y && rows > 0 && cols > 0 && cols % 32 == 0 && ntok > 0, "bad argument");
    cudaStream_t st = as_stream(stream);
    const int ss = host_q8_ss(cols);
    int8_t* aq = nullptr;
    float* as = nullptr;
    HG_CUDA(cudaMallocAsync((void**)&aq, (size_t)ntok * cols, st));
    HG_CUDA(cudaMallocAsync((void**)&as, (size_t)ntok * ss * 4, st));
    launch_kp_quant_rows(x, ntok, (int)cols, aq, as, st);
    Q8M W = q8m(qs, scales, 1, rows, cols);
    launch_kp_matmul(mm_args(W, aq, as, ntok, y, (int)rows, 0), ntok, 1, st);
    HG_CUDA(cudaGetLastError());
    HG_CUDA(cudaFreeAsync(aq, st));
    HG_CUDA(cudaFreeAsync(as, st));
  })
}

size_t hg_op_moe_scratch_bytes(const hg_moe_weights* w, int ntok) {
  if (!w || ntok <= 0) return 0;
  return moe_scratch_layout(w, ntok).total;
}

int hg_op_moe_ffn(const hg_moe_weights* w, const float* x, int ntok, float* y, int32_t* sel_out, void* scratch,
                  void* stream) {
  HG_API_TRY({
    need(w && x && y && scratch && ntok > 0, "bad argument");
    need(w->d_model % 32 == 0 && w->expert_ffn % 32 == 0 && w->top_k > 0 && w->top_k <= MAX_TOPK &&
             w->top_k <= w->n_experts && w->n_experts <= 128,
         "unsupported MoE shape");
    cudaStream_t st = as_stream(stream);
    HG_CUDA(prepare_tc());
    const int d = w->d_model, f = w->expert_ffn, k = w->top_k, ne = w->n_experts;
    MoeScratch L = moe_scratch_layout(w, ntok);
    char* base = static_cast<char*>(scratch);
    Dims D{};
    D.d = d;
    D.f = f;
    D.df = f;
    D.ne = ne;
    D.k = k;
    D.nsh = w->n_shared > 0 ? 1 : 0;
    D.wscale = w->weights_scale;
    D.wnorm = w->weights_norm;
    D.gsig = w->gating_sigmoid;
    DecodeBufs B{};
    B.T = ntok;
    B.h2 = const_cast<float*>(x);
    B.qh = reinterpret_cast<int8_t*>(base + L.off_qh);
    B.sh = reinterpret_cast<float*>(base + L.off_sh);
    B.sel = reinterpret_cast<int32_t*>(base + L.off_sel);
    B.selw = reinterpret_cast<float*>(base + L.off_selw);
    B.ecount = reinterpret_cast<int32_t*>(base + L.off_ecount);
    B.active = reinterpret_cast<int32_t*>(base + L.off_active);
    B.elist = reinterpret_cast<int32_t*>(base + L.off_elist);
    B.act = reinterpret_cast<float*>(base + L.off_act);
    B.act_stride = (k + 1) * f;
    B.ubuf = reinterpret_cast<float*>(base + L.off_ubuf);
    B.qact = reinterpret_cast<int8_t*>(base + L.off_qact);
    B.sact = reinterpret_cast<float*>(base + L.off_sact);
    B.y = reinterpret_cast<float*>(base + L.off_y);
    B.err = reinterpret_cast<int32_t*>(base + L.off_err);
    LayerDev Ld{};
    Ld.moe = 1;
    Ld.router = w->router;
    Ld.bias = w->bias;
    Ld.gate = q8m(w->gate_qs, w->gate_sc, ne, f, d);
    Ld.up = q8m(w->up_qs, w->up_sc, ne, f, d);
    Ld.down = q8m(w->down_qs, w->down_sc, ne, d, f);
    if (D.nsh) {
      Ld.sgate = q8m(w->sh_gate_qs, w->sh_gate_sc, 1, f, d);
      Ld.sup = q8m(w->sh_up_qs, w->sh_up_sc, 1, f, d);
      Ld.sdown = q8m(w->sh_down_qs, w->sh_down_sc, 1, d, f);
    }
    HG_CUDA(cudaMemsetAsync(B.ecount, 0, (ne + 2) * 4, st));
    launch_route(D, B, Ld, 0, 1, st);
    launch_ffn(D, B, Ld, st);
    launch_moe_combine(D, B, y, st);
    if (sel_out) HG_CUDA(cudaMemcpyAsync(sel_out, B.sel, (size_t)ntok * k * 4, cudaMemcpyDeviceToDevice, st));
    HG_CUDA(cudaGetLastError());
  })
}

size_t hg_op_kv_attn_scratch_bytes(const hg_kv_attn_args* a) { return a ? kv_scratch_bytes(a) : 0; }

int hg_op_kv_attn(const hg_kv_attn_args* a, void* scratch, void* stream) {
  HG_API_TRY({
    need(a && scratch && a->qkv && a->out && a->k_pool && a->v_pool && a->pos && a->block_table, "null argument");
    need(a->n_seqs > 0 && a->n_seqs <= 256, "n_seqs must be in 1..256");
    need(a->n_heads > 0 && a->n_kv_heads > 0 && a->n_heads % a->n_kv_heads == 0, "bad head counts");
    cudaStream_t st = as_stream(stream);
    char* base = static_cast<char*>(scratch);
    {
      cudaError_t pe = prepare_attn(a->head_dim, a->n_heads / a->n_kv_heads);
      if (pe == cudaErrorInvalidValue) throw Error(HG_ERR_INVALID, "unsupported head_dim / GQA group");
      HG_CUDA(pe);
    }
    AttnArgs A{};
    A.T = a->n_seqs;
    A.nh = a->n_heads;
    A.nkv = a->n_kv_heads;
    A.hd = a->head_dim;
    A.max_pos = a->max_pos;
    A.bt_stride = a->bt_stride;
    A.eps = a->eps;
    A.qkv = a->qkv;
    A.qkv_stride = (a->n_heads + 2 * a->n_kv_heads) * a->head_dim;
    A.q_norm = a->q_norm;
    A.k_norm = a->k_norm;
    A.rope_cos = a->rope_cos;
    A.rope_sin = a->rope_sin;
    A.pos = a->pos;
    A.bt = a->block_table;
    A.bt_row = nullptr;
    A.k_pool = a->k_pool;
    A.v_pool = a->v_pool;
    A.page_stride = a->page_stride;
    A.s_stride = (long long)kv_s_stride(a);
    A.S = reinterpret_cast<float*>(base);
    const size_t s_bytes = align256((size_t)a->n_seqs * a->n_heads * A.s_stride * 4);
    A.mkey = reinterpret_cast<uint32_t*>(base + s_bytes);
    A.rinv = reinterpret_cast<float*>(base + s_bytes + align256((size_t)a->n_seqs * a->n_heads * 4));
    A.qn = reinterpret_cast<float*>(reinterpret_cast<char*>(A.rinv) + align256((size_t)a->n_seqs * a->n_heads * 4));
    A.order = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(A.qn) +
                                         align256((size_t)a->n_seqs * a->n_heads * a->head_dim * 4));
    A.err = nullptr;
    A.out = a->out;
    A.qo = nullptr;
    A.so = nullptr;
    cudaError_t err = launch_attn_args(A, st);
    if (err == cudaErrorInvalidValue) throw Error(HG_ERR_INVALID, "unsupported head_dim / GQA group");
    HG_CUDA(err);
  })
}

}  // extern "C"
