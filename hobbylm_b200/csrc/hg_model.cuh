// Device views of the model and the per-engine work buffers, shared by the kernels and the host.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "hg_device.cuh"

namespace hg {

constexpr int MAX_LAYERS = 64;
constexpr int MAX_TOPK = 16;
constexpr int PAGE = 16;       // positions per KV page

// One packed Q8 matrix, or a stack of `count` equally shaped matrices.
struct Q8M {
  const int8_t* qs = nullptr;  // [count][rows][cols] lane-chunked rows
  const float* sc = nullptr;   // [count][rows][ss]
  int rows = 0, cols = 0, ss = 0;
  long long qs_mstride = 0, sc_mstride = 0;  // bytes / floats between stacked matrices
  __host__ __device__ const int8_t* row_q(int m, int r) const { return qs + m * qs_mstride + (long long)r * cols; }
  __host__ __device__ const float* row_s(int m, int r) const { return sc + m * sc_mstride + (long long)r * ss; }
};

struct LayerDev {
  const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
  Q8M qkv, wo;
  int moe;
  Q8M gate, up, down;     // dense FFN (count 1) or routed-expert stacks (count n_experts)
  Q8M sgate, sup, sdown;  // shared expert (moe && n_shared > 0)
  const float* router;    // [n_experts][d] f32
  const float* bias;      // [n_experts]
};

struct Dims {
  int d, L, nh, nkv, hd, qkvd, qd, f, df, ne, k, nsh, vocab, valid;
  float eps, wscale;
  int wnorm, gsig, max_pos;
};

// Paged KV pool: page p, layer l: K block of kv head h at k + p*page_stride + l*layer_stride +
// h*16*hd; V block at the same offset from v.
struct KvPool {
  float* k;
  float* v;
  long long page_stride, layer_stride;
};

// Work buffers for a decode step of up to T tokens (sizes in engine.cu).
struct DecodeBufs {
  int T;                   // tokens in this step
  const int32_t* tok;      // [T]
  const int32_t* pos;      // [T] position of the new token (= sequence length before the step)
  const int32_t* bt;       // block tables [rows][bt_stride]
  const int32_t* bt_row;   // [T] row of each token's sequence in bt
  int bt_stride;
  float* x;                // [T][d] residual stream
  const float* xin;        // [T][d] caller rows: a token given as -1 starts from its row (forward_x)
  int8_t* qa;              // [T][d] quantized normed activations (attention / lm_head input)
  float* sa;               // [T][ss(d)]
  float* qkv;              // [T][qkvd]
  int8_t* qo;              // [T][qd] quantized attention output
  float* so;               // [T][ss(qd)]
  float* h2;               // [T][d] ffn-normed hidden (router input)
  int8_t* qh;              // [T][d] quantized ffn-normed hidden
  float* sh;               // [T][ss(d)]
  int32_t* sel;            // [T][k]
  float* selw;             // [T][k]
  int32_t* ecount;         // [ne + 2]: per-expert token counts, then the active-expert count
  int32_t* active;         // [ne] experts with at least one token this step (any order)
  int32_t* elist;          // [ne][T] packed (t * 32 + rank)
  float* act;              // [T][act_stride] SwiGLU activations per (token, slot)
  int act_stride;          // floats per token (max(dense_ffn, (k + 1) * expert_ffn))
  float* ubuf;             // [T][act_stride] up-projection outputs (tensor-core FFN), or null
  int8_t* qact;            // [T][act_stride] quantized SwiGLU activations (tensor-core FFN), or null
  float* sact;             // their per-32 scales: [T][slots][ss(width)]
  float* y;                // [T][k + 1][d] expert outputs per (token, slot)
  float* S;                // [T][nh][s_stride] attention scores / exp weights
  long long s_stride;
  float* rinv;             // [T][nh] 1 / softmax denominator
  float* qn;               // [T][nh][hd] QK-normed, roped q
  uint32_t* mkey;          // [T][nh] running maximum of the attention scores (order-preserving key)
  int32_t* order;          // [T] tokens by decreasing position (attention work order)
  float* logits;           // [T][vocab] or null
  unsigned long long* amax;// [T]
  int32_t* dbg_sel;        // [L][T][k] routing capture
  int32_t* err;            // device error flag (bounded waits / bad positions)
};

// Arguments of the split-K decode attention kernel (decode.cu).
struct AttnArgs {
  int T, nh, nkv, hd, max_pos, bt_stride;
  float eps;
  const float* qkv;  // [T][qkvd]
  int qkv_stride;
  const float* q_norm;
  const float* k_norm;
  const float* rope_cos;
  const float* rope_sin;
  const int32_t* pos;
  const int32_t* bt;
  const int32_t* bt_row;  // may be null: row = token index
  float* k_pool;
  float* v_pool;
  long long page_stride;
  float* S;        // [T][nh][s_stride] scores, then exp(score - max)
  long long s_stride;  // >= max_pos, multiple of 16
  float* rinv;     // [T][nh] 1 / softmax denominator
  float* qn;       // [T][nh][hd] QK-normed, roped q (k_qk_prep)
  uint32_t* mkey;  // [T][nh] maximum score per (token, head) as an order-preserving key (f2key)
  int32_t* order;  // [T] the tokens by decreasing position (k_qk_prep), or null: value sums and
                   // softmax take the longest sequences first
  float* out;      // [T][nh*hd] or null
  int8_t* qo;      // [T][nh*hd] or null
  float* so;       // [T][ss(nh*hd/32)]
  int32_t* err;
};

// Arguments of the prefill-order Q8 matmul (prefill.cu). Grouped launches take the matrix index,
// first list entry and entry count of group blockIdx.z from grp_*.
struct MmArgs {
  Q8M W;
  int mat;               // stacked matrix index (-1: from grp table)
  const int8_t* aq;
  const float* as;
  int nrows;             // activation rows
  const int32_t* a_idx;  // may be null
  float* out;
  int ostride;
  const int32_t* o_idx;  // may be null
  int mode;
  // grouped (expert) launches: grid.z = group; entries from the tables below
  const int32_t* grp_mat;    // [groups] stacked matrix index, -1 = skip
  const int32_t* grp_off;    // [groups] first entry
  const int32_t* grp_cnt;    // [groups] entry count
  int32_t* err;              // device error word (tensor-core path: HG_ERR_TIMEOUT), or null
};

}  // namespace hg
