// Decode-step kernels (Model::forward, hobby-rs/src/model.rs:152-327) for T tokens of T sequences.
//
// Per layer: pre_norm (residual update + RMSNorm + activation quantization) -> QKV Q8 matvec ->
// paged attention: scores with fused QK-norm/RoPE/KV append, then the softmax denominator and the
// probability-weighted value sums (which write the quantized attention output) -> output
// projection with the residual add fused -> ffn RMSNorm +
// router + top-k -> gate/up SwiGLU over active experts -> down projection. The MoE combine of a
// layer is folded into the next layer's pre_norm. Finally output norm + lm_head + greedy argmax.
//
// Arithmetic: the Q8 matvec (quant.rs:44-67, 106-136), the activation quantization (quant.rs:
// 112-123), the router dot (ops.rs:7-36), sigmoid/silu (ops.rs:75-82, exp pinned to
// (float)exp((double)x)), top-k (model.rs:282-293) and the rank-order combine (model.rs:300-323)
// reproduce the reference bit for bit given the same inputs, and so do the RMSNorm / QK-norm sums
// and the attention softmax / value sums, which run sequentially in position order like the
// reference's loops (one thread per chain).
#include <algorithm>
#include <cfloat>
#include <utility>

#include "hg_launch.h"

namespace hg {

// Steps of up to this many tokens launch their kernels with programmatic stream serialization
// (see pdl_wait in hg_device.cuh): their kernels are short, so hiding each launch and each
// kernel's weight-load latency behind the previous kernel pays. Larger steps run multi-wave grids,
// where early-launched CTAs would only hold SM slots while they wait; they launch normally.
constexpr int PDL_MAX_T = 64;

// Launch (programmatic when pdl); errors are left for cudaGetLastError like a <<<>>> launch.
template <typename... P, typename... Args>
static inline void launch_pdl(bool pdl, void (*kern)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------------------------------
// Block reductions
// ------------------------------------------------------------------------------------------
// Sequential f32 sum of squares of xs[0..n) (ops.rs:85-95 `ss += v * v`, no FMA) computed by one
// thread; every thread of the block receives the result. xs is 16-byte aligned and n % 16 == 0;
// the shared-memory loads run one 16-element group ahead of the adds, so the dependent add
// latency, not the load latency, sets the pace.
__device__ __forceinline__ float seq_sumsq_smem(const float* xs, int n) {
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int ng = n >> 4;
  float ss = 0.0f;
  float4 a[4], b[4];
  auto add4 = [&](const float4* v) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      ss = fadd(ss, fmul(v[i].x, v[i].x));
      ss = fadd(ss, fmul(v[i].y, v[i].y));
      ss = fadd(ss, fmul(v[i].z, v[i].z));
      ss = fadd(ss, fmul(v[i].w, v[i].w));
    }
  };
  if (ng > 0) {
#pragma unroll
    for (int i = 0; i < 4; i++) a[i] = x4[i];
  }
  int g = 0;
  for (; g + 1 < ng; g += 2) {
#pragma unroll
    for (int i = 0; i < 4; i++) b[i] = x4[(g + 1) * 4 + i];
    add4(a);
    if (g + 2 < ng) {
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = x4[(g + 2) * 4 + i];
    }
    add4(b);
  }
  if (g < ng) add4(a);
  return ss;
}

__device__ inline float seq_sumsq_block(const float* xs, int n, float* red) {
  __syncthreads();
  if (threadIdx.x == 0) red[0] = seq_sumsq_smem(xs, n);
  __syncthreads();
  return red[0];
}

// ------------------------------------------------------------------------------------------
// pre_norm: residual update, RMSNorm (ops.rs:85-95, sequential sum), quantization of the result.
// mode 0: x = token embedding; 1: x += y[t][0] (dense FFN); 2: x += MoE combine (model.rs:300-323,
// rank order then the shared expert); 3: x unchanged.
// ------------------------------------------------------------------------------------------
constexpr int PRE_NORM_THREADS = 1024;  // one element per thread up to d = 1024

__global__ void __launch_bounds__(PRE_NORM_THREADS) k_pre_norm(Dims D, DecodeBufs B, int mode, const float* __restrict__ embd,
                                                  const float* __restrict__ norm_w, int8_t* q_out, float* s_out,
                                                  float* h_out, int reset_moe, int reset_amax) {
  extern __shared__ float xs[];
  __shared__ float red[32];
  const int t = blockIdx.x, d = D.d;
  float* x = B.x + (size_t)t * d;
  // loads of data older than the previous kernel, issued before the wait: the norm gain, the
  // residual row (written by the output projection, three kernels back) and the MoE gate weights
  // (written by the router, two kernels back)
  const bool first = threadIdx.x < d;
  const float nw0 = first ? norm_w[threadIdx.x] : 0.0f;
  const float x0 = (mode != 0 && first) ? x[threadIdx.x] : 0.0f;
  float sc[MAX_TOPK];
#pragma unroll
  for (int r = 0; r < MAX_TOPK; r++) sc[r] = (mode == 2 && r < D.k) ? fmul(B.selw[t * D.k + r], D.wscale) : 0.0f;
  pdl_wait();
  pdl_trigger();
  if (mode == 0) {
    int tok = B.tok[t];
    const float* e;
    if (tok == -1 && B.xin) {  // Model::forward_x (model.rs:160): the caller's row instead of an embedding
      e = B.xin + (size_t)t * d;
    } else {
      if (tok < 0 || tok >= D.vocab) {
        if (threadIdx.x == 0) atomicExch(B.err, HG_ERR_TOKEN);
        tok = 0;
      }
      e = embd + (size_t)tok * d;
    }
    for (int i = threadIdx.x; i < d; i += blockDim.x) xs[i] = e[i];
  } else if (mode == 1) {
    const float* y = B.y + (size_t)t * (D.k + 1) * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) xs[i] = fadd(i == threadIdx.x ? x0 : x[i], y[i]);
  } else if (mode == 2) {
    const float* y = B.y + (size_t)t * (D.k + 1) * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
      float yv[MAX_TOPK + 1];  // every row's element loaded before the rank-order sum
#pragma unroll
      for (int r = 0; r <= MAX_TOPK; r++) yv[r] = (r < D.k || (r == D.k && D.nsh > 0)) ? y[r * d + i] : 0.0f;
      const float xi = i == threadIdx.x ? x0 : x[i];
      float o = 0.0f;
#pragma unroll
      for (int r = 0; r < MAX_TOPK; r++)
        if (r < D.k) o = fadd(o, fmul(sc[r], yv[r]));
      if (D.nsh > 0) {
#pragma unroll
        for (int r = 0; r <= MAX_TOPK; r++)
          if (r == D.k) o = fadd(o, yv[r]);
      }
      xs[i] = fadd(xi, o);
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) xs[i] = i == threadIdx.x ? x0 : x[i];
  }
  if (mode != 3)
    for (int i = threadIdx.x; i < d; i += blockDim.x) x[i] = xs[i];
  float ss = seq_sumsq_block(xs, d, red);
  float scale = __fdiv_rn(1.0f, __fsqrt_rn(fadd(__fdiv_rn(ss, (float)d), D.eps)));
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float h = fmul(fmul(xs[i], scale), i == threadIdx.x ? nw0 : norm_w[i]);
    xs[i] = h;
    if (h_out) h_out[(size_t)t * d + i] = h;
  }
  __syncthreads();
  quant_row_block(xs, d, q_out + (size_t)t * d, s_out + (size_t)t * q8_ss(d >> 5));
  if (reset_moe && t == 0)
    for (int i = threadIdx.x; i < D.ne + 2; i += blockDim.x) B.ecount[i] = 0;
  if (reset_amax && threadIdx.x == 0) B.amax[t] = 0ull;
}

// ------------------------------------------------------------------------------------------
// Q8 matvec over the step's tokens. ROWS rows x 8 lanes per CTA; activations of up to TT tokens
// are staged in shared memory. NB = blocks per row (0: runtime).
// ------------------------------------------------------------------------------------------
template <int NB>
struct Frag {
  static constexpr int NC = NB / 4, NT = NB % 4;
  int4 w[NC > 0 ? NC : 1];
  float4 s[NC > 0 ? NC : 1];
  int wt[NT > 0 ? NT : 1];
  float st[NT > 0 ? NT : 1];
  __device__ __forceinline__ void load(const int8_t* __restrict__ wq, const float* __restrict__ ws, int lane) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
      w[c] = __ldg(reinterpret_cast<const int4*>(wq + c * 128 + lane * 16));
      s[c] = __ldg(reinterpret_cast<const float4*>(ws + c * 4));
    }
#pragma unroll
    for (int t = 0; t < NT; t++) {
      wt[t] = __ldg(reinterpret_cast<const int*>(wq + NC * 128 + t * 32 + lane * 4));
      st[t] = __ldg(ws + NC * 4 + t);
    }
  }
  __device__ __forceinline__ float dot(const int8_t* aq, const float* as, int lane) const {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; c++) {
      int4 a = *reinterpret_cast<const int4*>(aq + c * 128 + lane * 16);
      float4 d = *reinterpret_cast<const float4*>(as + c * 4);
      acc = __fmaf_rn(fmul(s[c].x, d.x), (float)__dp4a(w[c].x, a.x, 0), acc);
      acc = __fmaf_rn(fmul(s[c].y, d.y), (float)__dp4a(w[c].y, a.y, 0), acc);
      acc = __fmaf_rn(fmul(s[c].z, d.z), (float)__dp4a(w[c].z, a.z, 0), acc);
      acc = __fmaf_rn(fmul(s[c].w, d.w), (float)__dp4a(w[c].w, a.w, 0), acc);
    }
#pragma unroll
    for (int t = 0; t < NT; t++) {
      int a = *reinterpret_cast<const int*>(aq + NC * 128 + t * 32 + lane * 4);
      acc = __fmaf_rn(fmul(st[t], as[NC * 4 + t]), (float)__dp4a(wt[t], a, 0), acc);
    }
    return acc;
  }
};

// Weight row of one (row, lane) thread, dotted with staged activations. Rows with NB <= 24 keep
// their words in registers across tokens; longer rows re-read them (L1) per token.
template <int NB>
struct RowDot {
  static constexpr bool REG = (NB > 0 && NB <= 24);
  Frag<REG ? NB : 4> f;
  const int8_t* wq;
  const float* ws;
  int nb;
  __device__ __forceinline__ void init(const int8_t* q, const float* s, int lane, int nb_) {
    wq = q;
    ws = s;
    nb = nb_;
    if constexpr (REG) f.load(q, s, lane);
  }
  __device__ __forceinline__ float dot(const int8_t* aq, const float* as, int lane) const {
    if constexpr (REG) return f.dot(aq, as, lane);
    else if constexpr (NB > 0) return q8_lane_dot<NB>(wq, ws, aq, as, lane);
    else return q8_lane_dot_rt(wq, ws, aq, as, lane, nb);
  }
};

// Copy n activation rows (cols bytes + ss floats each, contiguous per row in global) into smem.
__device__ inline void stage_rows(int8_t* aq_s, float* as_s, const int8_t* q, const float* s, const int* rows_idx,
                                  int n, int cols, int ss, long long qstride, long long sstride) {
  int vq = cols >> 4;  // int4 per row
  for (int i = threadIdx.x; i < n * vq; i += blockDim.x) {
    int r = i / vq, c = i - r * vq;
    long long src = rows_idx ? rows_idx[r] : r;
    reinterpret_cast<int4*>(aq_s + (size_t)r * cols)[c] = reinterpret_cast<const int4*>(q + src * qstride)[c];
  }
  for (int i = threadIdx.x; i < n * ss; i += blockDim.x) {
    int r = i / ss, c = i - r * ss;
    long long src = rows_idx ? rows_idx[r] : r;
    as_s[(size_t)r * ss + c] = s[src * sstride + c];
  }
}

enum { EPI_STORE = 0, EPI_RESID = 1, EPI_LMHEAD = 2 };

// Rows of one matrix against the tokens of chunk blockIdx.y (TY tokens; aq/as rows t, strides
// cols / ss), TT tokens staged in shared memory at a time; two tokens' dots are in flight per
// thread so their FMA chains overlap.
template <int NB, int ROWS, int TT, int EPI>
__global__ void __launch_bounds__(ROWS * 8) k_mv_tokens(Dims D, DecodeBufs B, Q8M W, const int8_t* __restrict__ aq,
                                                         const float* __restrict__ as, float* out, int ostride,
                                                         int ty) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int cols = W.cols, nb = cols >> 5, ss = W.ss;
  int8_t* aq_s = reinterpret_cast<int8_t*>(smem);
  float* as_s = reinterpret_cast<float*>(smem + (size_t)TT * cols);
  const int lane = threadIdx.x & 7, rl = threadIdx.x >> 3;
  const int row = blockIdx.x * ROWS + rl;
  const bool valid_row = row < W.rows;
  const int tbeg = blockIdx.y * ty, tend = min(B.T, tbeg + ty);
  RowDot<NB> rd;
  rd.init(W.row_q(0, valid_row ? row : 0), W.row_s(0, valid_row ? row : 0), lane, nb);  // weights: before the wait
  pdl_wait();
  pdl_trigger();
  if (tbeg >= tend) return;
  __shared__ unsigned long long best_s[TT > 0 ? TT : 1];
  auto emit = [&](int i, int t, float v) {
    if (EPI == EPI_STORE) {
      if (lane == 0 && valid_row) out[(size_t)t * ostride + row] = v;
    } else if (EPI == EPI_RESID) {
      if (lane == 0 && valid_row) {
        float* xp = B.x + (size_t)t * D.d + row;
        *xp = fadd(*xp, v);
      }
    } else {
      if (lane == 0 && valid_row && out) out[(size_t)t * ostride + row] = v;
      unsigned long long key = (valid_row && row < D.valid) ? argmax_key(v, (uint32_t)row) : 0ull;
      key = max(key, __shfl_xor_sync(0xffffffffu, key, 8));
      key = max(key, __shfl_xor_sync(0xffffffffu, key, 16));
      if ((threadIdx.x & 31) == 0) atomicMax(&best_s[i], key);
    }
  };
  for (int t0 = tbeg; t0 < tend; t0 += TT) {
    int n = min(TT, tend - t0);
    __syncthreads();
    stage_rows(aq_s, as_s, aq + (size_t)t0 * cols, as + (size_t)t0 * ss, nullptr, n, cols, ss, cols, ss);
    if (EPI == EPI_LMHEAD && threadIdx.x < TT) best_s[threadIdx.x] = 0ull;
    __syncthreads();
    int i = 0;
#pragma unroll 1
    for (; i + 1 < n; i += 2) {
      const float a0 = rd.dot(aq_s + (size_t)i * cols, as_s + (size_t)i * ss, lane);
      const float a1 = rd.dot(aq_s + (size_t)(i + 1) * cols, as_s + (size_t)(i + 1) * ss, lane);
      emit(i, t0 + i, hsum8_group(a0));
      emit(i + 1, t0 + i + 1, hsum8_group(a1));
    }
    if (i < n) emit(i, t0 + i, hsum8_group(rd.dot(aq_s + (size_t)i * cols, as_s + (size_t)i * ss, lane)));
    if (EPI == EPI_LMHEAD) {
      __syncthreads();
      if (threadIdx.x < n) atomicMax(&B.amax[t0 + threadIdx.x], best_s[threadIdx.x]);
    }
  }
}

// ------------------------------------------------------------------------------------------
// Router (model.rs:270-293): ffn RMSNorm, quantized copy for the experts, f32 router logits in
// the ops::dot order, sigmoid, selection score + bias, top-k by descending score (ties by lower
// id), gate weights = raw scores (optionally renormalized), expert token lists.
// ------------------------------------------------------------------------------------------
// prenormed != 0: B.h2 already holds the normed hidden state (op-level MoE entry point).
constexpr int ROUTE_THREADS = 1024;
constexpr int ROUTE_ROWS = 2;  // router rows per warp held in registers (covers 64 experts)

template <int NI>  // d / 32 (0: rows are read during the dot, any d)
__global__ void __launch_bounds__(ROUTE_THREADS) k_route(Dims D, DecodeBufs B, LayerDev Ld, int layer, int prenormed) {
  extern __shared__ float hs[];  // d floats
  __shared__ float red[32];
  __shared__ float logit_s[128], score_s[128], selsc_s[128];
  __shared__ int rank_e[MAX_TOPK];
  const int t = blockIdx.x, d = D.d;
  // this warp's router rows, loaded before the norm so their latency overlaps it
  const int rwarp = threadIdx.x >> 5, rlane = threadIdx.x & 31;
  float wr[ROUTE_ROWS][NI > 0 ? NI : 1];
  if (NI > 0 && Ld.moe) {
#pragma unroll
    for (int rr = 0; rr < ROUTE_ROWS; rr++) {
      const int e = rwarp + rr * (ROUTE_THREADS / 32);
#pragma unroll
      for (int i = 0; i < NI; i++) wr[rr][i] = e < D.ne ? Ld.router[(size_t)e * d + 32 * i + rlane] : 0.0f;
    }
  }
  // weights, before the wait; the gain only when this kernel normalizes (prenormed callers, such
  // as the op-level MoE entry, pass no gain)
  const float nw0 = (!prenormed && threadIdx.x < d) ? Ld.ffn_norm[threadIdx.x] : 0.0f;
  const float bias0 = (Ld.moe && threadIdx.x < D.ne) ? Ld.bias[threadIdx.x] : 0.0f;
  pdl_wait();
  pdl_trigger();
  if (prenormed) {
    for (int i = threadIdx.x; i < d; i += blockDim.x) hs[i] = B.h2[(size_t)t * d + i];
  } else {
    const float* x = B.x + (size_t)t * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) hs[i] = x[i];
    float ss = seq_sumsq_block(hs, d, red);
    float scale = __fdiv_rn(1.0f, __fsqrt_rn(fadd(__fdiv_rn(ss, (float)d), D.eps)));
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
      float h = fmul(fmul(hs[i], scale), i == threadIdx.x ? nw0 : Ld.ffn_norm[i]);
      hs[i] = h;
      B.h2[(size_t)t * d + i] = h;
    }
  }
  __syncthreads();
  quant_row_block(hs, d, B.qh + (size_t)t * d, B.sh + (size_t)t * q8_ss(d >> 5));
  if (!Ld.moe) return;
  const int ne = D.ne, k = D.k, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (NI > 0) {
#pragma unroll
    for (int rr = 0; rr < ROUTE_ROWS; rr++) {
      const int e = warp + rr * nw;
      if (e < ne) {
        float acc = 0.0f;  // ops::dot lane order, as dot_ref_warp
#pragma unroll
        for (int i = 0; i < NI; i++) acc = __fmaf_rn(wr[rr][i], hs[32 * i + rlane], acc);
        const float lg = dot_ref_warp_finish(acc);
        if (rlane == 0) logit_s[e] = lg;
      }
    }
  }
  for (int e = warp + (NI > 0 ? ROUTE_ROWS * nw : 0); e < ne; e += nw) {
    float lg = dot_ref_warp(Ld.router + (size_t)e * d, hs, d);
    if ((threadIdx.x & 31) == 0) logit_s[e] = lg;
  }
  __syncthreads();
  if (threadIdx.x == 0 && !D.gsig) {  // softmax gating (ops.rs:112-128), sequential
    float m = -INFINITY;
    for (int e = 0; e < ne; e++) m = logit_s[e] > m ? logit_s[e] : m;
    float sum = 0.0f;
    for (int e = 0; e < ne; e++) {
      score_s[e] = exp_cr(logit_s[e] - m);
      sum = fadd(sum, score_s[e]);
    }
    float inv = __fdiv_rn(1.0f, sum);
    for (int e = 0; e < ne; e++) score_s[e] = fmul(score_s[e], inv);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ne; e += blockDim.x) {
    float sc = D.gsig ? sigmoid_ref(logit_s[e]) : score_s[e];
    score_s[e] = sc;
    selsc_s[e] = fadd(sc, e == (int)threadIdx.x ? bias0 : Ld.bias[e]);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ne; e += blockDim.x) {
    float v = selsc_s[e];
    int r = 0;
    for (int j = 0; j < ne; j++) {
      float u = selsc_s[j];
      r += (u > v) || (u == v && j < e);
    }
    if (r < k) rank_e[r] = e;
  }
  __syncthreads();
  // rank r's selection by thread r: the k experts of a token are distinct, so their list slots
  // are claimed independently (the order of the active-expert list changes no result)
  if (threadIdx.x < k) {
    const int r = threadIdx.x, e = rank_e[r];
    float w = score_s[e];
    if (D.wnorm) {  // the weights' sum in rank order (model.rs:288-292)
      float s = -0.0f;
      for (int rr = 0; rr < k; rr++) s = fadd(s, score_s[rank_e[rr]]);
      s = fadd(s, 1e-9f);
      w = __fdiv_rn(w, s);
    }
    B.sel[t * k + r] = e;
    B.selw[t * k + r] = w;
    if (B.dbg_sel) B.dbg_sel[((size_t)layer * B.T + t) * k + r] = e;
    const int slot = atomicAdd(&B.ecount[e], 1);
    if (slot == 0) B.active[atomicAdd(&B.ecount[ne], 1)] = e;
    B.elist[(size_t)e * B.T + slot] = t * 32 + r;
  }
}

// ------------------------------------------------------------------------------------------
// SwiGLU gate/up (model.rs:243-255, 300-305, 313-318): blockIdx.y = slot group (0: shared expert
// or the dense FFN; 1 + i: i-th active routed expert). Each CTA covers PAIRS rows of gate and the
// same rows of up (16 lanes per pair) and writes act = silu(g) * u for every token of the group.
// ------------------------------------------------------------------------------------------
template <int NB, int PAIRS, int TT>
__global__ void __launch_bounds__(PAIRS * 16) k_ffn_up(Dims D, DecodeBufs B, LayerDev Ld, int ez, int sh) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int ent_s[TT];
  const int cols = D.d, nb = cols >> 5, ss = q8_ss(nb);
  // y < sh: group 0 (shared expert or dense FFN, all T tokens), chunk y of its entries (z == 0
  // only); y >= sh: routed group y - sh + 1, whose chunks are strided over the z CTAs
  const bool g0 = blockIdx.y < (unsigned)sh;
  const int grp = g0 ? 0 : (int)blockIdx.y - sh + 1, pair0 = blockIdx.x * PAIRS;
  const int cstep = g0 ? sh : (int)gridDim.z;
  const int lane = threadIdx.x & 7, rg = threadIdx.x >> 3, pr = rg >> 1, is_up = rg & 1;
  const int row = pair0 + pr;
  // group 0 (shared expert or dense FFN) has fixed weights: load them before the wait; the routed
  // groups' experts come from the router, the kernel just before this one
  RowDot<NB> rd;
  const bool fixed = g0 && blockIdx.z == 0 && !(Ld.moe && D.nsh == 0);
  const int fdim0 = Ld.moe ? D.f : D.df;
  if (fixed) {
    const Q8M M = Ld.moe ? (is_up ? Ld.sup : Ld.sgate) : (is_up ? Ld.up : Ld.gate);
    const int r = row < fdim0 ? row : 0;
    rd.init(M.row_q(0, r), M.row_s(0, r), lane, nb);
  }
  pdl_wait();
  pdl_trigger();
  int expert = 0, nent, fdim;
  if (grp == 0) {
    if (!fixed) return;
    nent = B.T;
    fdim = fdim0;
  } else {
    if (!Ld.moe || grp - 1 >= B.ecount[D.ne]) return;
    expert = B.active[grp - 1];
    nent = B.ecount[expert];
    fdim = D.f;
  }
  if (pair0 >= fdim) return;
  int8_t* aq_s = reinterpret_cast<int8_t*>(smem);
  float* as_s = reinterpret_cast<float*>(smem + (size_t)TT * cols);
  const bool valid_row = row < fdim;
  const int ebeg = (g0 ? (int)blockIdx.y : (int)blockIdx.z) * ez;
  if (ebeg >= nent) return;
  if (!fixed) {
    const Q8M M = is_up ? Ld.up : Ld.gate;
    rd.init(M.row_q(expert, valid_row ? row : 0), M.row_s(expert, valid_row ? row : 0), lane, nb);
  }
  // this CTA's chunks of ez entries (ez % TT == 0), TT entries at a time
  for (int e0 = ebeg; e0 < nent; e0 += (e0 + TT) % ez == 0 ? TT + (cstep - 1) * ez : TT) {
    int n = min(TT, nent - e0);
    __syncthreads();
    if (threadIdx.x < n) {
      int code = grp == 0 ? (e0 + threadIdx.x) * 32 : B.elist[(size_t)expert * B.T + e0 + threadIdx.x];
      ent_s[threadIdx.x] = code;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n * (cols >> 4); i += blockDim.x) {
      int r = i / (cols >> 4), c = i - r * (cols >> 4);
      int t = ent_s[r] >> 5;
      reinterpret_cast<int4*>(aq_s + (size_t)r * cols)[c] = reinterpret_cast<const int4*>(B.qh + (size_t)t * cols)[c];
    }
    for (int i = threadIdx.x; i < n * ss; i += blockDim.x) {
      int r = i / ss, c = i - r * ss;
      int t = ent_s[r] >> 5;
      as_s[(size_t)r * ss + c] = B.sh[(size_t)t * ss + c];
    }
    __syncthreads();
    auto emit = [&](int i, float v) {
      float u = __shfl_down_sync(0xffffffffu, v, 8);  // up row value from the neighbouring group
      if (!is_up && lane == 0 && valid_row) {
        int code = ent_s[i], t = code >> 5, r = code & 31;
        int slot = grp == 0 ? (Ld.moe ? D.k : 0) : r;
        B.act[(size_t)t * B.act_stride + (size_t)slot * fdim + row] = fmul(silu_ref(v), u);
      }
    };
    int i = 0;
#pragma unroll 1
    for (; i + 1 < n; i += 2) {
      const float a0 = rd.dot(aq_s + (size_t)i * cols, as_s + (size_t)i * ss, lane);
      const float a1 = rd.dot(aq_s + (size_t)(i + 1) * cols, as_s + (size_t)(i + 1) * ss, lane);
      emit(i, hsum8_group(a0));
      emit(i + 1, hsum8_group(a1));
    }
    if (i < n) emit(i, hsum8_group(rd.dot(aq_s + (size_t)i * cols, as_s + (size_t)i * ss, lane)));
  }
}

// ------------------------------------------------------------------------------------------
// Down projection: blockIdx.y = slot group as in k_ffn_up; the activation row of each (token,
// slot) is quantized in shared memory (quant.rs:112-123) and dotted with ROWS rows of the down
// matrix; y[t][slot][row] = result.
// ------------------------------------------------------------------------------------------
template <int NB, int ROWS, int TT>
__global__ void __launch_bounds__(ROWS * 8) k_ffn_down(Dims D, DecodeBufs B, LayerDev Ld, int ez, int sh) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int ent_s[TT];
  // the expert tables come from the router, two kernels back (readable before the wait); the
  // activations come from k_ffn_up, just before
  const bool g0 = blockIdx.y < (unsigned)sh;  // group / chunk mapping as in k_ffn_up
  const int grp = g0 ? 0 : (int)blockIdx.y - sh + 1;
  const int cstep = g0 ? sh : (int)gridDim.z;
  int expert = 0, nent = 0, fdim = 0;
  bool work = true;
  if (grp == 0) {
    work = blockIdx.z == 0 && !(Ld.moe && D.nsh == 0);
    nent = B.T;
    fdim = Ld.moe ? D.f : D.df;
  } else {
    work = Ld.moe && grp - 1 < B.ecount[D.ne];
    if (work) {
      expert = B.active[grp - 1];
      nent = B.ecount[expert];
      fdim = D.f;
    }
  }
  const int ebeg = (g0 ? (int)blockIdx.y : (int)blockIdx.z) * ez;
  if (!work || ebeg >= nent) {
    pdl_wait();
    pdl_trigger();
    return;
  }
  const Q8M W = (grp == 0 && Ld.moe) ? Ld.sdown : Ld.down;
  const int cols = fdim, nb = cols >> 5, ss = q8_ss(nb);
  int8_t* aq_s = reinterpret_cast<int8_t*>(smem);
  float* as_s = reinterpret_cast<float*>(smem + (size_t)TT * cols);
  const int lane = threadIdx.x & 7, rl = threadIdx.x >> 3;
  const int row = blockIdx.x * ROWS + rl;
  const bool valid_row = row < D.d;
  const int mi = grp == 0 ? 0 : expert;
  RowDot<NB> rd;
  rd.init(W.row_q(mi, valid_row ? row : 0), W.row_s(mi, valid_row ? row : 0), lane, nb);
  pdl_wait();
  pdl_trigger();
  // this CTA's chunks of ez entries (ez % TT == 0), TT entries at a time
  for (int e0 = ebeg; e0 < nent; e0 += (e0 + TT) % ez == 0 ? TT + (cstep - 1) * ez : TT) {
    int n = min(TT, nent - e0);
    __syncthreads();
    if (threadIdx.x < n) {
      int code = grp == 0 ? (e0 + threadIdx.x) * 32 : B.elist[(size_t)expert * B.T + e0 + threadIdx.x];
      ent_s[threadIdx.x] = code;
    }
    __syncthreads();
    // quantize each entry's activation row: warps take 32-blocks
    {
      int warp = threadIdx.x >> 5, wl = threadIdx.x & 31, nw = blockDim.x >> 5;
      for (int j = warp; j < n * nb; j += nw) {
        int r = j / nb, b = j - r * nb;
        int code = ent_s[r], t = code >> 5, rk = code & 31;
        int slot = grp == 0 ? (Ld.moe ? D.k : 0) : rk;
        const float* a = B.act + (size_t)t * B.act_stride + (size_t)slot * fdim;
        float dq;
        int8_t q = quant_lane(a[b * 32 + wl], &dq);
        aq_s[(size_t)r * cols + q8_pos(b * 32 + wl, nb)] = q;
        if (wl == 0) as_s[(size_t)r * ss + b] = dq;
      }
    }
    __syncthreads();
    auto emit = [&](int i, float v) {
      if (lane == 0 && valid_row) {
        int code = ent_s[i], t = code >> 5, rk = code & 31;
        int slot = grp == 0 ? (Ld.moe ? D.k : 0) : rk;
        B.y[((size_t)t * (D.k + 1) + slot) * D.d + row] = v;
      }
    };
    int i = 0;
#pragma unroll 1
    for (; i + 1 < n; i += 2) {
      const float a0 = rd.dot(aq_s + (size_t)i * cols, as_s + (size_t)i * ss, lane);
      const float a1 = rd.dot(aq_s + (size_t)(i + 1) * cols, as_s + (size_t)(i + 1) * ss, lane);
      emit(i, hsum8_group(a0));
      emit(i + 1, hsum8_group(a1));
    }
    if (i < n) emit(i, hsum8_group(rd.dot(aq_s + (size_t)i * cols, as_s + (size_t)i * ss, lane)));
  }
}

// ------------------------------------------------------------------------------------------
// Attention (model.rs:199-233) over a paged f32 KV pool, in the reference's arithmetic order.
//
// k_qk_prep: QK-norm (sequential sum, model.rs:753-763) + RoPE of each token's q heads into qn,
//   and of its k heads, appended with its v heads to their page slot; resets the score maxima.
// k_attn_scores: work units of 32 positions of one (token, kv head), dealt to CTAs in contiguous
//   runs. A unit's K rows (two pages) and the group's q rows are staged into shared memory by
//   cp.async (SC_SLOTS units in flight per CTA); one thread per (position, q head) computes
//   s = dot(q_h, k_j) * (1/sqrt(hd)) in the ops::dot order; per-(token, head) maxima are merged
//   with an atomic max on an order-preserving key.
// k_attn_softmax: per (token, q head): e_j = exp(s_j - max) (parallel), sum = sequential f32 sum
//   over j (one thread), inv = 1/sum (ops.rs:112-128).
// k_attn_pv / k_attn_pv_small: every (head, dim) chain accumulates o += (e_j * inv) * v_j[dim]
//   sequentially over j (model.rs:227-232), V and e staged through a cp.async ring; the result
//   is quantized per 32-block for the output projection (quant.rs:112-123).
// ------------------------------------------------------------------------------------------

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// per-head RMSNorm with a sequential sum (model.rs:753-763) + rotate-half RoPE (ops.rs:157-166)
// of one head vector by one warp. wv: this lane's gains (elements lane + 32 j); cv / sv: its cos /
// sin entries (lane + 32 j < HD / 2); buf: this warp's HD-float shared scratch (16-byte aligned),
// which receives the result.
template <int HD>
__device__ __forceinline__ void norm_rope_warp(const float* src, const float (&wv)[HD / 32], float eps,
                                               const float (&cv)[HD / 64], const float (&sv)[HD / 64], float* buf) {
  constexpr int HALF = HD / 2;
  const int lane = threadIdx.x & 31;
  for (int i = lane; i < HD; i += 32) buf[i] = src[i];
  __syncwarp();
  float scale = 0.0f;
  if (lane == 0) {
    const float ss = seq_sumsq_smem(buf, HD);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(fadd(__fdiv_rn(ss, (float)HD), eps)));
  }
  scale = __shfl_sync(0xffffffffu, scale, 0);
  float v[HD / 32];
#pragma unroll
  for (int j = 0; j < HD / 32; j++) v[j] = fmul(fmul(buf[lane + 32 * j], scale), wv[j]);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < HD / 32; j++) buf[lane + 32 * j] = v[j];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < HD / 64; j++) {
    const int i = lane + 32 * j;  // i < HALF
    const float x1 = buf[i], x2 = buf[i + HALF], c = cv[j], sn = sv[j];
    v[j] = __fsub_rn(fmul(x1, c), fmul(x2, sn));
    v[j + HD / 64] = fadd(fmul(x2, c), fmul(x1, sn));
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < HD / 64; j++) {
    buf[lane + 32 * j] = v[j];
    buf[lane + 32 * j + HALF] = v[j + HD / 64];
  }
  __syncwarp();
}

// A token's position is usable when its page is inside the block table and below max_pos;
// otherwise the token does no attention work and the step reports HG_ERR_CONTEXT.
__device__ __forceinline__ bool attn_pos_ok(const AttnArgs& A, int pos) {
  return pos >= 0 && pos < A.max_pos && pos / PAGE < A.bt_stride;
}

// QK-norm (sequential sum, model.rs:753-763) + RoPE of every q head of a token into qn, and of
// the token's k heads, appended with its v heads to their page slot (model.rs:199-210). One CTA
// per token, one warp per head (q heads first, then kv heads). Also resets the token's score
// maxima (read by k_attn_softmax two kernels later).
constexpr int ATT_MAX_T = 256;  // tokens of one attention call (engine batches and hg_op_kv_attn)

template <int HD>
__global__ void k_qk_prep(AttnArgs A) {
  extern __shared__ __align__(16) float prep_s[];  // one HD-float scratch per warp
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // everything but the qkv row is older than the previous kernel: the maxima (last read two
  // kernels ago), the position, the gains, the RoPE rows and the page slot are handled before the
  // wait
  for (int h = threadIdx.x; h < A.nh; h += blockDim.x) A.mkey[(size_t)t * A.nh + h] = 0u;
  if (A.order && blockIdx.x == 0) {
    // the tokens by decreasing position (ties by index), a permutation: the value sums and the
    // softmax hand their longest chains out first, so no SM ends up holding several of them
    __shared__ int pos_sh[ATT_MAX_T];
    for (int u = threadIdx.x; u < A.T; u += blockDim.x) pos_sh[u] = A.pos[u];
    __syncthreads();
    for (int u = threadIdx.x; u < A.T; u += blockDim.x) {
      const int pu = pos_sh[u];
      int r = 0;
      for (int v = 0; v < A.T; v++) {
        const int pv = pos_sh[v];
        r += (pv > pu) || (pv == pu && v < u);
      }
      A.order[r] = u;
    }
  }
  const int pos = A.pos[t];
  const bool ok = attn_pos_ok(A, pos);
  const bool is_q = warp < A.nh, is_k = !is_q && warp < A.nh + A.nkv;
  float wv[HD / 32], cv[HD / 64], sv[HD / 64];
  long long off = 0;
  if (ok && (is_q || is_k)) {
    const float* w = is_q ? A.q_norm : A.k_norm;
#pragma unroll
    for (int j = 0; j < HD / 32; j++) wv[j] = w[lane + 32 * j];
#pragma unroll
    for (int j = 0; j < HD / 64; j++) {
      cv[j] = A.rope_cos[(size_t)pos * (HD / 2) + lane + 32 * j];
      sv[j] = A.rope_sin[(size_t)pos * (HD / 2) + lane + 32 * j];
    }
    if (is_k) {
      const int* bt = A.bt + (size_t)(A.bt_row ? A.bt_row[t] : t) * A.bt_stride;
      off = (long long)bt[pos / PAGE] * A.page_stride + ((long long)(warp - A.nh) * PAGE + pos % PAGE) * HD;
    }
  }
  pdl_wait();
  pdl_trigger();
  if (!ok) {
    if (threadIdx.x == 0 && A.err) atomicExch(A.err, HG_ERR_CONTEXT);
    return;
  }
  const float* qkv = A.qkv + (size_t)t * A.qkv_stride;
  const int qd = A.nh * HD, kvd = A.nkv * HD;
  float* buf = prep_s + warp * HD;
  if (is_q) {
    norm_rope_warp<HD>(qkv + warp * HD, wv, A.eps, cv, sv, buf);
    float* dst = A.qn + ((size_t)t * A.nh + warp) * HD;
    for (int j = lane; j < HD; j += 32) dst[j] = buf[j];
  } else if (is_k) {
    const int kvh = warp - A.nh;
    norm_rope_warp<HD>(qkv + qd + kvh * HD, wv, A.eps, cv, sv, buf);
    for (int j = lane; j < HD; j += 32) {
      A.k_pool[off + j] = buf[j];
      A.v_pool[off + j] = qkv[qd + kvd + kvh * HD + j];
    }
  }
}

// Units of 32 positions (two pages) of the tokens, kv head by kv head: u_count[t] units per
// (token, kv head). prefix_s[t] = first unit of token t (nkv * sum of earlier counts);
// prefix_s[T] = total. Computed by warp 0 (T <= SC_MAX_T).
constexpr int ATT_UNIT = 32;
constexpr int SC_MAX_T = 1024;
constexpr int ATT_MAX_BT = 4096;  // block-table entries per sequence (contexts up to 65,536 positions)

__device__ __forceinline__ int attn_units_of(const AttnArgs& A, int t) {
  const int p = A.pos[t];
  return attn_pos_ok(A, p) ? (p + 1 + ATT_UNIT - 1) / ATT_UNIT : 0;
}

__device__ inline void attn_unit_prefix(const AttnArgs& A, int* prefix_s) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (A.T + 31) / 32, t0 = lane * per;
    int run = 0;
    for (int i = 0; i < per; i++) run += t0 + i < A.T ? attn_units_of(A, t0 + i) * A.nkv : 0;
    int incl = run;  // inclusive scan of the lanes' run totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int acc = incl - run;
    for (int i = 0; i < per; i++) {
      if (t0 + i < A.T) {
        prefix_s[t0 + i] = acc;
        acc += attn_units_of(A, t0 + i) * A.nkv;
      }
    }
    if (lane == 31) prefix_s[A.T] = incl;
  }
  __syncthreads();
}

// A CTA walks its contiguous run of units in order: (token, kv head, unit within the head).
struct UnitCursor {
  int t, kvh, s, nu;  // nu = units per (token, kv head) of token t
  __device__ void seek(const AttnArgs& A, const int* prefix_s, int u) {
    int lo = 0, hi = A.T - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix_s[mid] <= u) lo = mid;
      else hi = mid - 1;
    }
    t = lo;
    nu = (prefix_s[t + 1] - prefix_s[t]) / A.nkv;
    const int rem = u - prefix_s[t];
    kvh = nu > 0 ? rem / nu : 0;
    s = nu > 0 ? rem - kvh * nu : 0;
  }
  __device__ void next(const AttnArgs& A, const int* prefix_s) {
    if (++s < nu) return;
    s = 0;
    if (++kvh < A.nkv) return;
    kvh = 0;
    do {
      ++t;
      nu = t < A.T ? (prefix_s[t + 1] - prefix_s[t]) / A.nkv : 1;
    } while (nu == 0);
  }
};

constexpr int SC_SLOTS = 4;  // units in flight per scores CTA
constexpr int SC_WARPS = 8;  // 8 warps x 4 positions: one 32-position unit per pass

template <int HD, int REP>
struct ScoresShape {
  static constexpr int NT = 32 * SC_WARPS;
  static constexpr int CH = HD / 4;  // 16-byte chunks per K row
  static constexpr int E = HD / 32;  // ops::dot steps per accumulator lane
  static constexpr int SLOT = ATT_UNIT * HD + REP * HD;  // K rows of the unit, then the group's q rows
  static constexpr size_t SMEM = (size_t)SC_SLOTS * SLOT * 4;
};

// Thread mapping: a warp scores 4 positions of the unit (pp = lane / 8) for all REP q heads of the
// group; lane l = lane % 8 is SIMD lane l of the four ops::dot accumulators (ops.rs:7-36), so it
// holds elements 32e + 8m + l of q (registers, reloaded when the unit's (token, kv head) changes)
// and reads the same elements of its position's K row. K chunk c (16 bytes) of unit row r is
// stored at chunk c ^ ((r & 3) << 1): the four rows a warp reads at once then fall on distinct
// banks, so each 32-bit K load is one shared-memory wavefront shared by all REP heads.
template <int HD, int REP>
__global__ void __launch_bounds__(32 * SC_WARPS) k_attn_scores(AttnArgs A) {
  using S = ScoresShape<HD, REP>;
  constexpr int E = S::E;
  extern __shared__ __align__(16) float sc_smem[];
  float* ring = sc_smem;
  int* prefix_s = reinterpret_cast<int*>(sc_smem + SC_SLOTS * S::SLOT);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int l = lane & 7, pp = lane >> 3, r = warp * 4 + pp;  // r: row within the unit
  attn_unit_prefix(A, prefix_s);  // positions are older than the previous kernel
  pdl_wait();  // qn and the appended K rows come from k_qk_prep
  pdl_trigger();
  const long long total = prefix_s[A.T];
  const int u0 = (int)(total * blockIdx.x / gridDim.x), u1 = (int)(total * (blockIdx.x + 1) / gridDim.x);
  const int count = u1 - u0;
  if (count <= 0) return;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  UnitCursor ic, cc;  // issue / compute cursors
  ic.seek(A, prefix_s, u0);
  cc = ic;
  // this thread's copies of a unit: chunk c0 of rows rc + RPP k (k < CPT), i.e. two pages
  static_assert(S::NT % S::CH == 0 && ATT_UNIT % (S::NT / S::CH) == 0, "whole rows per pass");
  constexpr int RPP = S::NT / S::CH, CPT = ATT_UNIT / RPP;  // rows per pass, copies per thread
  const int c0 = tid % S::CH, rc = tid / S::CH;
  // the issue cursor's unit: its token's position and the unit's two page ids, fetched when the
  // cursor arrives there (one unit before they are used), so the copies never wait on the loads
  int f_pos = 0, f_p0 = 0, f_p1 = 0;
  auto fetch = [&]() {
    if (ic.t < A.T) {
      const int* bt = A.bt + (size_t)(A.bt_row ? A.bt_row[ic.t] : ic.t) * A.bt_stride;
      const int pg0 = ic.s * (ATT_UNIT / PAGE);
      f_pos = A.pos[ic.t];
      f_p0 = bt[pg0];
      f_p1 = pg0 + 1 < A.bt_stride ? bt[pg0 + 1] : f_p0;  // in the table; used only inside the sequence
    }
  };
  fetch();
  auto issue = [&](int i) {
    if (i < count) {
      float* slot = ring + (i % SC_SLOTS) * S::SLOT;
      const int npg = f_pos / PAGE + 1, pg0 = ic.s * (ATT_UNIT / PAGE);
      const float* kb = A.k_pool + (long long)ic.kvh * PAGE * HD + c0 * 4;
      const float* page0 = kb + (long long)f_p0 * A.page_stride;
      const float* page1 = pg0 + 1 < npg ? kb + (long long)f_p1 * A.page_stride : page0;
#pragma unroll
      for (int k = 0; k < CPT; k++) {
        const int row = rc + RPP * k;
        if (row < PAGE || pg0 + 1 < npg)
          cp_async16(slot + row * HD + ((c0 ^ ((row & 3) << 1)) << 2), (row < PAGE ? page0 : page1) + (row % PAGE) * HD);
      }
      const float* q = A.qn + ((size_t)ic.t * A.nh + ic.kvh * REP) * HD;
      for (int i2 = tid; i2 < REP * S::CH; i2 += S::NT) cp_async16(slot + ATT_UNIT * HD + i2 * 4, q + i2 * 4);
      ic.next(A, prefix_s);
      fetch();
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < SC_SLOTS - 1; k++) issue(k);
  // element 32e + 8m + l of unit row r lies in chunk 8e + 2m + l/4, stored at chunk
  // 8e + 2 (m ^ (r % 4)) + l/4: koff[m] + 32 e floats from the slot
  int koff[4];
#pragma unroll
  for (int m = 0; m < 4; m++) koff[m] = r * HD + ((2 * (m ^ (r & 3)) + (l >> 2)) << 2) + (l & 3);
  float qv[REP][E][4];
  float mx[REP];
#pragma unroll
  for (int h = 0; h < REP; h++) mx[h] = -INFINITY;  // running maxima over the current (token, kv head)
  for (int i = 0; i < count; i++) {
    cp_async_wait<SC_SLOTS - 2>();
    __syncthreads();  // unit i has landed for every thread; every thread is done with unit i - 1
    issue(i + SC_SLOTS - 1);
    const float* slot = ring + (i % SC_SLOTS) * S::SLOT;
    if (i == 0 || cc.s == 0) {  // a new (token, kv head): its q rows came with this unit
      const float* qs = slot + ATT_UNIT * HD;
#pragma unroll
      for (int h = 0; h < REP; h++)
#pragma unroll
        for (int e = 0; e < E; e++)
#pragma unroll
          for (int m = 0; m < 4; m++) qv[h][e][m] = qs[h * HD + 32 * e + 8 * m + l];
    }
    float kv[E][4];
#pragma unroll
    for (int m = 0; m < 4; m++) {
      const float* kr = slot + koff[m];
#pragma unroll
      for (int e = 0; e < E; e++) kv[e][m] = kr[32 * e];
    }
    const int n = A.pos[cc.t] + 1, j = cc.s * ATT_UNIT + r;
    float* srow = A.S + ((size_t)cc.t * A.nh + cc.kvh * REP) * A.s_stride + j;
#pragma unroll
    for (int h = 0; h < REP; h++) {
      float a[4];
#pragma unroll
      for (int m = 0; m < 4; m++) {
        float acc = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) acc = __fmaf_rn(qv[h][e][m], kv[e][m], acc);
        a[m] = acc;
      }
      const float sc = fmul(hsum8_group(fadd(fadd(a[0], a[1]), fadd(a[2], a[3]))), scale);
      if (j < n) {
        if (l == 0) srow[(size_t)h * A.s_stride] = sc;
        mx[h] = fmaxf(mx[h], sc);
      }
    }
    // the (token, kv head) run ends at the CTA's last unit or at its last unit in the head
    if (i + 1 == count || cc.s + 1 == cc.nu) {
#pragma unroll
      for (int h = 0; h < REP; h++) {
        float v = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 8));
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
        if (lane == 0 && v > -INFINITY) atomicMax(A.mkey + (size_t)cc.t * A.nh + cc.kvh * REP + h, f2key(v));
        mx[h] = -INFINITY;
      }
    }
    cc.next(A, prefix_s);
  }
  cp_async_wait<0>();  // no copy may land after the CTA exits
}

// ------------------------------------------------------------------------------------------
// Softmax denominator: one CTA per (token, q head). e = exp(s - max) goes back into S and the
// sequential denominator (ops.rs:118-122) is summed by one thread from shared memory while the
// other warps compute the next chunk's exponentials; 1/sum goes to rinv[t][h].
// ------------------------------------------------------------------------------------------
constexpr int SMX_ECH = 1024;   // softmax positions per chunk
constexpr int SMX_THREADS = 256;

// sum = (((sum + e0) + e1) + ...) over eb[0..cnt), loads issued one 16-position group ahead
__device__ __forceinline__ float seq_sum_smem(const float* eb, int cnt, float sum) {
  const float4* e4 = reinterpret_cast<const float4*>(eb);
  const int ng = cnt >> 4;
  float4 a[4], b[4];
  if (ng > 0) {
#pragma unroll
    for (int i = 0; i < 4; i++) a[i] = e4[i];
  }
  int g = 0;
  for (; g + 1 < ng; g += 2) {
#pragma unroll
    for (int i = 0; i < 4; i++) b[i] = e4[(g + 1) * 4 + i];
#pragma unroll
    for (int i = 0; i < 4; i++) sum = fadd(fadd(fadd(fadd(sum, a[i].x), a[i].y), a[i].z), a[i].w);
    if (g + 2 < ng) {
#pragma unroll
      for (int i = 0; i < 4; i++) a[i] = e4[(g + 2) * 4 + i];
    }
#pragma unroll
    for (int i = 0; i < 4; i++) sum = fadd(fadd(fadd(fadd(sum, b[i].x), b[i].y), b[i].z), b[i].w);
  }
  if (g < ng) {
#pragma unroll
    for (int i = 0; i < 4; i++) sum = fadd(fadd(fadd(fadd(sum, a[i].x), a[i].y), a[i].z), a[i].w);
  }
  for (int j = ng * 16; j < cnt; j++) sum = fadd(sum, eb[j]);
  return sum;
}

__global__ void __launch_bounds__(SMX_THREADS) k_attn_softmax(AttnArgs A) {
  constexpr int PER = (SMX_ECH + SMX_THREADS - 33) / (SMX_THREADS - 32);  // exps per thread (warps 1..)
  __shared__ __align__(16) float ebuf[2][SMX_ECH];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int rk = blockIdx.x / A.nh, h = blockIdx.x - rk * A.nh;
  const int t = A.order ? A.order[rk] : rk;  // written two kernels ago
  pdl_wait();
  pdl_trigger();
  const int pos = A.pos[t];
  if (!attn_pos_ok(A, pos)) return;  // flagged by k_qk_prep
  const int n = pos + 1;
  float* erow = A.S + ((size_t)t * A.nh + h) * A.s_stride;
  const float mrow = key2f(A.mkey[(size_t)t * A.nh + h]);
  const int nchunks = (n + SMX_ECH - 1) / SMX_ECH;
  {
    const int cnt = min(SMX_ECH, n);
    float sv[SMX_ECH / SMX_THREADS];
#pragma unroll
    for (int k = 0; k < SMX_ECH / SMX_THREADS; k++) {
      const int j = tid + k * SMX_THREADS;
      sv[k] = j < cnt ? erow[j] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < SMX_ECH / SMX_THREADS; k++) {
      const int j = tid + k * SMX_THREADS;
      if (j < cnt) {
        const float e = exp_cr(__fsub_rn(sv[k], mrow));
        ebuf[0][j] = e;
        erow[j] = e;
      }
    }
  }
  __syncthreads();
  float sum = 0.0f;
  for (int c = 0; c < nchunks; c++) {
    const int j0 = c * SMX_ECH, cnt = min(SMX_ECH, n - j0);
    if (tid == 0) {
      sum = seq_sum_smem(ebuf[c & 1], cnt, sum);
    } else if (warp > 0 && c + 1 < nchunks) {
      const int j1 = j0 + SMX_ECH, cn1 = min(SMX_ECH, n - j1), t1 = tid - 32;
      float* eb = ebuf[(c + 1) & 1];
      float sv[PER];
#pragma unroll
      for (int k = 0; k < PER; k++) {
        const int j = t1 + k * (SMX_THREADS - 32);
        sv[k] = j < cn1 ? erow[j1 + j] : 0.0f;
      }
#pragma unroll
      for (int k = 0; k < PER; k++) {
        const int j = t1 + k * (SMX_THREADS - 32);
        if (j < cn1) {
          const float e = exp_cr(__fsub_rn(sv[k], mrow));
          eb[j] = e;
          erow[j1 + j] = e;
        }
      }
    }
    __syncthreads();
  }
  if (tid == 0) A.rinv[(size_t)t * A.nh + h] = __fdiv_rn(1.0f, sum);
}

// ------------------------------------------------------------------------------------------
// Value sums. Both kernels stream a (token, kv head)'s V rows and the group's e rows (exp
// weights, from k_attn_softmax) in stages of PV_STAGE positions through a ring of cp.async
// copies, one CTA barrier per stage. Each stage's probabilities p = e * inv (ops.rs:124-126) are
// formed one stage ahead of the chains that use them, so a chain step is one shared-memory V
// load, one multiply and the dependent add.
//
// k_attn_pv (many (token, kv head) pairs): CTA = (token, kv head), thread = output dim, the
// REP chains of the group's q heads per thread sharing each V load.
// k_attn_pv_small (few pairs, down to one token): CTA = (token, kv head, 32-dim slice), warp = q
// head, lane = dim: one chain per thread, so a warp spends ~3 instructions per position and the
// chain's add latency sets the pace.
// ------------------------------------------------------------------------------------------
constexpr int PV_STAGE = 16;        // positions per stage (large kernel): one page
constexpr int PV_SLOTS = 4;         // ring slots (large kernel): 2 stages in flight ahead of the chain
constexpr int PVS_STAGE = 64;       // positions per stage (small kernel)
constexpr int PVS_SLOTS = 6;        // ring slots (small kernel)
constexpr int PV_SMALL_MAX_PAIRS = 48;  // (token, kv head) pairs up to which k_attn_pv_small runs

template <int HD, int REP>
struct PvShape {
  static constexpr int NT = HD;
  static constexpr int SLOT = PV_STAGE * HD + REP * PV_STAGE;  // V rows, then e rows
  static constexpr size_t SMEM = (size_t)PV_SLOTS * SLOT * 4;
};

// quantize the finished chain value o of (token t, output element hd) for the output projection
__device__ __forceinline__ void pv_emit(const AttnArgs& A, int t, int hd, float o) {
  const int qd = A.nh * A.hd, lane = threadIdx.x & 31;
  if (A.out) A.out[(size_t)t * qd + hd] = o;
  if (A.qo) {  // a warp holds one 32-block of the head
    float dq;
    int8_t q = quant_lane(o, &dq);
    const int nbq = qd >> 5;
    A.qo[(size_t)t * qd + q8_pos(hd, nbq)] = q;
    if (lane == 0) A.so[(size_t)t * q8_ss(nbq) + (hd >> 5)] = dq;
  }
}

template <int HD, int REP>
__global__ void __launch_bounds__(HD) k_attn_pv(AttnArgs A) {
  static_assert(HD % 32 == 0 && (REP == 1 || REP == 2 || REP == 4), "whole warps; GQA group of 1, 2 or 4");
  using S = PvShape<HD, REP>;
  extern __shared__ __align__(16) float pv_smem[];
  __shared__ __align__(16) float p_s[2][PV_STAGE][4];
  const int tid = threadIdx.x;
  const int rk = blockIdx.x / A.nkv, kvh = blockIdx.x - rk * A.nkv, h0 = kvh * REP;
  const int t = A.order ? A.order[rk] : rk;  // longest first; written three kernels ago
  const int pos = A.pos[t];  // positions and page ids are older than the previous kernel
  if (!attn_pos_ok(A, pos)) {  // flagged by k_qk_prep
    pdl_wait();
    pdl_trigger();
    return;
  }
  const int n = pos + 1, nst = (n + PV_STAGE - 1) / PV_STAGE, npg = pos / PAGE + 1;
  const int* bt = A.bt + (size_t)(A.bt_row ? A.bt_row[t] : t) * A.bt_stride;
  int* bt_s = reinterpret_cast<int*>(pv_smem + PV_SLOTS * S::SLOT);  // the sequence's page ids
  for (int i = tid; i < npg; i += S::NT) bt_s[i] = bt[i];
  __syncthreads();
  const float* vb = A.v_pool + (long long)kvh * PAGE * HD;
  const float* e0 = A.S + ((size_t)t * A.nh + h0) * A.s_stride;
  // page ids and V rows are older than the previous kernel; the e rows are not, so the ring is
  // filled after the wait
  pdl_wait();
  pdl_trigger();
  // 1/sum of the head of each (position, head) pair this thread forms p for in make_p
  constexpr int PK = (REP * PV_STAGE + S::NT - 1) / S::NT;
  float inv_k[PK];
#pragma unroll
  for (int k = 0; k < PK; k++) {
    const int i = tid + k * S::NT;
    inv_k[k] = i < REP * PV_STAGE ? A.rinv[(size_t)t * A.nh + h0 + i / PV_STAGE] : 0.0f;
  }
  auto issue = [&](int st) {
    if (st < nst) {
      float* slot = pv_smem + (st % PV_SLOTS) * S::SLOT;
#pragma unroll
      for (int i = tid; i < PV_STAGE * HD / 4; i += S::NT) {
        const int row = i / (HD / 4), c = i - row * (HD / 4), pg = st * (PV_STAGE / PAGE) + row / PAGE;
        if (pg < npg) cp_async16(slot + row * HD + c * 4, vb + (long long)bt_s[pg] * A.page_stride + (row % PAGE) * HD + c * 4);
      }
      if (tid < REP * PV_STAGE / 4) {  // e rows run to s_stride >= npg * PAGE
        const int r = tid / (PV_STAGE / 4), q = tid - r * (PV_STAGE / 4);
        if (st * PV_STAGE + q * 4 < npg * PAGE)
          cp_async16(slot + PV_STAGE * HD + r * PV_STAGE + q * 4, e0 + (size_t)r * A.s_stride + st * PV_STAGE + q * 4);
      }
    }
    cp_async_commit();
  };
  // p of stage st into p_s[st & 1] (threads cover (position, head) pairs)
  auto make_p = [&](int st) {
    if (st < nst) {
      const float* es = pv_smem + (st % PV_SLOTS) * S::SLOT + PV_STAGE * HD;
#pragma unroll
      for (int k = 0; k < PK; k++) {
        const int i = tid + k * S::NT, r = i / PV_STAGE, j = i - r * PV_STAGE;
        if (i < REP * PV_STAGE) p_s[st & 1][j][r] = fmul(es[r * PV_STAGE + j], inv_k[k]);
      }
    }
  };
#pragma unroll
  for (int k = 0; k < PV_SLOTS - 1; k++) issue(k);
  cp_async_wait<PV_SLOTS - 2>();
  __syncthreads();
  make_p(0);
  float o[REP];
#pragma unroll
  for (int r = 0; r < REP; r++) o[r] = 0.0f;
  for (int st = 0; st < nst; st++) {
    // stages <= st + 1 have landed (issued: up to st + PV_SLOTS - 2); p of stage st is in p_s
    cp_async_wait<PV_SLOTS - 3>();
    __syncthreads();  // also: every thread is done with stage st - 1 (its slot and p_s buffer)
    issue(st + PV_SLOTS - 1);
    make_p(st + 1);
    const float* vs = pv_smem + (st % PV_SLOTS) * S::SLOT + tid;
    const float4* pq = reinterpret_cast<const float4*>(&p_s[st & 1][0][0]);
    const int rows = min(PV_STAGE, n - st * PV_STAGE);
    auto step = [&](int j) {
      const float4 pj = pq[j];
      const float v = vs[j * HD];
      o[0] = fadd(o[0], fmul(pj.x, v));
      if (REP > 1) o[REP > 1 ? 1 : 0] = fadd(o[REP > 1 ? 1 : 0], fmul(pj.y, v));
      if (REP > 2) o[REP > 2 ? 2 : 0] = fadd(o[REP > 2 ? 2 : 0], fmul(pj.z, v));
      if (REP > 3) o[REP > 3 ? 3 : 0] = fadd(o[REP > 3 ? 3 : 0], fmul(pj.w, v));
    };
    if (rows == PV_STAGE) {
      // the stage's V and p values into registers first, then the dependent adds
      float vr[PV_STAGE];
      float4 pr[PV_STAGE];
#pragma unroll
      for (int j = 0; j < PV_STAGE; j++) {
        vr[j] = vs[j * HD];
        pr[j] = pq[j];
      }
#pragma unroll
      for (int j = 0; j < PV_STAGE; j++) {
        o[0] = fadd(o[0], fmul(pr[j].x, vr[j]));
        if (REP > 1) o[REP > 1 ? 1 : 0] = fadd(o[REP > 1 ? 1 : 0], fmul(pr[j].y, vr[j]));
        if (REP > 2) o[REP > 2 ? 2 : 0] = fadd(o[REP > 2 ? 2 : 0], fmul(pr[j].z, vr[j]));
        if (REP > 3) o[REP > 3 ? 3 : 0] = fadd(o[REP > 3 ? 3 : 0], fmul(pr[j].w, vr[j]));
      }
    } else {
      for (int j = 0; j < rows; j++) step(j);
    }
  }
  cp_async_wait<0>();
#pragma unroll
  for (int r = 0; r < REP; r++) pv_emit(A, t, (h0 + r) * HD + tid, o[r]);
}

// With only a few CTAs on the GPU (a handful of sequences) each must keep its own copies far ahead
// of its chain to cover DRAM latency: those launches use the deep ring.
constexpr int PVS_SLOTS_DEEP = 16;
constexpr int PVS_DEEP_MAX_PAIRS = 12;

template <int REP, int NSLOT>
struct PvSmallShape {
  static constexpr int NT = 32 * REP;
  static constexpr int SLOT = PVS_STAGE * 32 + REP * PVS_STAGE;  // V rows of the slice, then e rows
  static constexpr size_t SMEM = (size_t)NSLOT * SLOT * 4;
};

template <int HD, int REP, int PVS_SLOTS>
__global__ void __launch_bounds__(32 * REP) k_attn_pv_small(AttnArgs A) {
  static_assert(HD % 32 == 0 && (REP == 1 || REP == 2 || REP == 4), "32-dim slices; GQA group of 1, 2 or 4");
  using S = PvSmallShape<REP, PVS_SLOTS>;
  constexpr int DS = HD / 32;  // slices per head
  extern __shared__ __align__(16) float pv_smem[];
  __shared__ __align__(16) float p_s[REP][2][PVS_STAGE];  // per warp (head), double-buffered
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int slice = blockIdx.x % DS, tk = blockIdx.x / DS;
  const int rk = tk / A.nkv, kvh = tk - rk * A.nkv, h = kvh * REP + w, d = slice * 32 + lane;
  const int t = A.order ? A.order[rk] : rk;  // longest first; written three kernels ago
  const int pos = A.pos[t];
  if (!attn_pos_ok(A, pos)) {  // flagged by k_qk_prep
    pdl_wait();
    pdl_trigger();
    return;
  }
  const int n = pos + 1, nst = (n + PVS_STAGE - 1) / PVS_STAGE, npg = pos / PAGE + 1;
  const int* bt = A.bt + (size_t)(A.bt_row ? A.bt_row[t] : t) * A.bt_stride;
  int* bt_s = reinterpret_cast<int*>(pv_smem + PVS_SLOTS * S::SLOT);  // the sequence's page ids
  for (int i = tid; i < npg; i += S::NT) bt_s[i] = bt[i];
  __syncthreads();
  const float* vb = A.v_pool + (long long)kvh * PAGE * HD + slice * 32;
  const float* e0 = A.S + ((size_t)t * A.nh + kvh * REP) * A.s_stride;
  pdl_wait();
  pdl_trigger();
  const float inv = A.rinv[(size_t)t * A.nh + h];
  auto issue = [&](int st) {
    if (st < nst) {
      float* slot = pv_smem + (st % PVS_SLOTS) * S::SLOT;
#pragma unroll
      for (int i = tid; i < PVS_STAGE * 8; i += S::NT) {  // 8 chunks per 32-float row slice
        const int row = i >> 3, c = i & 7, pg = st * (PVS_STAGE / PAGE) + row / PAGE;
        if (pg < npg) cp_async16(slot + row * 32 + c * 4, vb + (long long)bt_s[pg] * A.page_stride + (row % PAGE) * HD + c * 4);
      }
      for (int i = tid; i < REP * PVS_STAGE / 4; i += S::NT) {
        const int r = i / (PVS_STAGE / 4), q = i - r * (PVS_STAGE / 4);
        if (st * PVS_STAGE + q * 4 < npg * PAGE)
          cp_async16(slot + PVS_STAGE * 32 + r * PVS_STAGE + q * 4, e0 + (size_t)r * A.s_stride + st * PVS_STAGE + q * 4);
      }
    }
    cp_async_commit();
  };
  // this warp's p of stage st (lane j covers positions j, j + 32)
  auto make_p = [&](int st) {
    if (st < nst) {
      const float* es = pv_smem + (st % PVS_SLOTS) * S::SLOT + PVS_STAGE * 32 + w * PVS_STAGE;
#pragma unroll
      for (int j = lane; j < PVS_STAGE; j += 32) p_s[w][st & 1][j] = fmul(es[j], inv);
    }
  };
#pragma unroll
  for (int k = 0; k < PVS_SLOTS - 1; k++) issue(k);
  cp_async_wait<PVS_SLOTS - 2>();
  __syncthreads();
  make_p(0);
  float o = 0.0f;
  for (int st = 0; st < nst; st++) {
    cp_async_wait<PVS_SLOTS - 3>();
    __syncthreads();  // stage st + 1 landed; every warp is done with stage st - 1
    issue(st + PVS_SLOTS - 1);
    make_p(st + 1);  // p_s[w][(st + 1) & 1] was last read by this warp's chain over stage st - 1
    __syncwarp();
    const float* vs = pv_smem + (st % PVS_SLOTS) * S::SLOT + lane;
    const float4* pq = reinterpret_cast<const float4*>(&p_s[w][st & 1][0]);
    const int rows = min(PVS_STAGE, n - st * PVS_STAGE);
    if (rows == PVS_STAGE) {
      // 16-position groups: the next group's V and p values are loaded into registers before the
      // current group's dependent adds, so the add chain never waits on shared memory
      constexpr int G = 16, NG = PVS_STAGE / G;
      float vr[2][G];
      float4 pr[2][G / 4];
      auto load = [&](int g, int b) {
#pragma unroll
        for (int k = 0; k < G; k++) vr[b][k] = vs[(g * G + k) * 32];
#pragma unroll
        for (int k = 0; k < G / 4; k++) pr[b][k] = pq[g * (G / 4) + k];
      };
      load(0, 0);
#pragma unroll
      for (int g = 0; g < NG; g++) {
        if (g + 1 < NG) load(g + 1, (g + 1) & 1);
        const int b = g & 1;
#pragma unroll
        for (int k = 0; k < G / 4; k++) {
          o = fadd(o, fmul(pr[b][k].x, vr[b][4 * k + 0]));
          o = fadd(o, fmul(pr[b][k].y, vr[b][4 * k + 1]));
          o = fadd(o, fmul(pr[b][k].z, vr[b][4 * k + 2]));
          o = fadd(o, fmul(pr[b][k].w, vr[b][4 * k + 3]));
        }
      }
    } else {
      for (int j = 0; j < rows; j++) o = fadd(o, fmul(p_s[w][st & 1][j], vs[j * 32]));
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  pv_emit(A, t, h * HD + d, o);
}

// ------------------------------------------------------------------------------------------
// Greedy feedback at the end of a decode step: each token's masked argmax (sample.rs:53-64)
// becomes its next input, the position advances, and the id is stored in a ring of generated ids
// (gen[(step % gen_cap) * T + t]) whose step counter lives in device memory.
// ------------------------------------------------------------------------------------------
__global__ void k_feedback(DecodeBufs B, int32_t* tok, int32_t* pos, int32_t* gen, int gen_cap, int32_t* step) {
  const int t = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int s = *step;
  __syncthreads();
  if (t < B.T) {
    const unsigned long long key = B.amax[t];
    const int32_t next = (int32_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    tok[t] = next;
    pos[t] = pos[t] + 1;
    gen[(size_t)(s % gen_cap) * B.T + t] = next;
  }
  __syncthreads();
  if (t == 0) *step = s + 1;
}

void launch_feedback(const DecodeBufs& B, int32_t* tok, int32_t* pos, int32_t* gen, int gen_cap, int32_t* step,
                     cudaStream_t st) {
  launch_pdl(B.T <= PDL_MAX_T, k_feedback, dim3(1), dim3(256), 0, st, B, tok, pos, gen, gen_cap, step);
}

// ------------------------------------------------------------------------------------------
// Row quantization of f32 activations (op-level entry points).
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_quant_rows(const float* x, int cols, int8_t* q, float* s) {
  const int t = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  quant_row_block(x + (size_t)t * cols, cols, q + (size_t)t * cols, s + (size_t)t * q8_ss(cols >> 5));
}

// ------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------
#define HG_NB_SWITCH(nb, ...)            \
  switch (nb) {                          \
    case 6: { constexpr int NB = 6; __VA_ARGS__; } break;   \
    case 10: { constexpr int NB = 10; __VA_ARGS__; } break; \
    case 16: { constexpr int NB = 16; __VA_ARGS__; } break; \
    case 24: { constexpr int NB = 24; __VA_ARGS__; } break; \
    case 48: { constexpr int NB = 48; __VA_ARGS__; } break; \
    case 72: { constexpr int NB = 72; __VA_ARGS__; } break; \
    default: { constexpr int NB = 0; __VA_ARGS__; } break;  \
  }

constexpr int MV_TY = 16;         // tokens per CTA of the batched matvec
constexpr int MV_TY_LMHEAD = 64;  // the lm_head has rows enough for many CTAs: fewer passes over its weights
constexpr int FFN_EZ = 16;   // (token, slot) entries per chunk of the batched expert kernels
constexpr int FFN_ZMAX = 4;  // chunk CTAs per (row tile, routed expert)

static inline size_t act_smem(int tt, int cols) { return (size_t)tt * cols + (size_t)tt * q8_ss(cols >> 5) * 4; }

template <int EPI>
static void launch_mv_tokens_t(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as,
                               float* out, int ostride, cudaStream_t st) {
  int nb = W.cols >> 5;
  // many tokens: the partials come from the tensor cores (tc.cu)
  if (tc_usable(W, B.T) && launch_mv_tc(D, B, W, aq, as, out, ostride, EPI, st)) return;
  if (B.T == 1) {
    constexpr int ROWS = 8, TT = 1;
    dim3 grid((W.rows + ROWS - 1) / ROWS);
    HG_NB_SWITCH(nb, launch_pdl(B.T <= PDL_MAX_T, k_mv_tokens<NB, ROWS, TT, EPI>, grid, dim3(ROWS * 8), act_smem(TT, W.cols), st, D, B, W, aq, as, out, ostride, 1));
  } else {
    constexpr int ROWS = 32, TT = 8;
    // token chunks of MV_TY tokens: enough CTAs for small matrices, weights re-read from L2 per chunk
    const int ty = EPI == EPI_LMHEAD ? MV_TY_LMHEAD : MV_TY;
    dim3 grid((W.rows + ROWS - 1) / ROWS, (B.T + ty - 1) / ty);
    HG_NB_SWITCH(nb, launch_pdl(B.T <= PDL_MAX_T, k_mv_tokens<NB, ROWS, TT, EPI>, grid, dim3(ROWS * 8), act_smem(TT, W.cols), st, D, B, W, aq, as, out, ostride, ty));
  }
}

void launch_mv_store(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* out,
                     int ostride, cudaStream_t st) {
  launch_mv_tokens_t<EPI_STORE>(D, B, W, aq, as, out, ostride, st);
}
void launch_mv_resid(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as,
                     cudaStream_t st) {
  launch_mv_tokens_t<EPI_RESID>(D, B, W, aq, as, nullptr, 0, st);
}
void launch_lmhead(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* logits,
                   cudaStream_t st) {
  launch_mv_tokens_t<EPI_LMHEAD>(D, B, W, aq, as, logits, D.vocab, st);
}

void launch_pre_norm(const Dims& D, const DecodeBufs& B, int mode, const float* embd, const float* norm_w,
                     int8_t* q_out, float* s_out, float* h_out, int reset_moe, int reset_amax, cudaStream_t st) {
  launch_pdl(B.T <= PDL_MAX_T, k_pre_norm, dim3(B.T), dim3(PRE_NORM_THREADS), D.d * sizeof(float), st, D, B, mode, embd, norm_w, q_out,
             s_out, h_out, reset_moe, reset_amax);
}

void launch_route(const Dims& D, const DecodeBufs& B, const LayerDev& L, int layer, int prenormed, cudaStream_t st) {
  const size_t sm = D.d * sizeof(float);
  const dim3 g(B.T), b(ROUTE_THREADS);
  if (D.d == 768) launch_pdl(B.T <= PDL_MAX_T, k_route<24>, g, b, sm, st, D, B, L, layer, prenormed);
  else if (D.d == 512) launch_pdl(B.T <= PDL_MAX_T, k_route<16>, g, b, sm, st, D, B, L, layer, prenormed);
  else launch_pdl(B.T <= PDL_MAX_T, k_route<0>, g, b, sm, st, D, B, L, layer, prenormed);
}

// MoE combine without a residual (op-level entry point): y_out[t] = rank-order combine.
__global__ void k_moe_combine(Dims D, DecodeBufs B, float* y_out) {
  const int t = blockIdx.x, d = D.d;
  pdl_wait();
  pdl_trigger();
  const float* y = B.y + (size_t)t * (D.k + 1) * d;
  float sc[MAX_TOPK];
  for (int r = 0; r < D.k; r++) sc[r] = fmul(B.selw[t * D.k + r], D.wscale);
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float o = 0.0f;
    for (int r = 0; r < D.k; r++) o = fadd(o, fmul(sc[r], y[r * d + i]));
    if (D.nsh > 0) o = fadd(o, y[D.k * d + i]);
    y_out[(size_t)t * d + i] = o;
  }
}
void launch_moe_combine(const Dims& D, const DecodeBufs& B, float* y_out, cudaStream_t st) {
  k_moe_combine<<<B.T, 256, 0, st>>>(D, B, y_out);
}

void launch_ffn(const Dims& D, const DecodeBufs& B, const LayerDev& L, cudaStream_t st) {
  if (ffn_tc_usable(D, B, L) && launch_ffn_tc(D, B, L, st)) return;  // many tokens: the tensor-core FFN (tc.cu)
  const int nrouted = L.moe ? (D.ne < B.T * D.k ? D.ne : B.T * D.k) : 0;
  launch_ffn_ex(D, B, L, true, nrouted, st);
}

void launch_ffn_ex(const Dims& D, const DecodeBufs& B, const LayerDev& L, bool group0, int nrouted, cudaStream_t st) {
  // group 0 (shared expert / dense FFN: T entries) over sh y-slices of one ez-entry chunk each; the
  // routed groups (at most T entries each, usually far fewer) after them, their chunks strided
  // over nz z-CTAs, so few routed CTAs find no work
  const int ez = B.T == 1 ? 1 : FFN_EZ, chunks = (B.T + ez - 1) / ez, sh = group0 ? chunks : 0;
  const int groups = sh + nrouted, nz = nrouted > 0 ? std::min(chunks, FFN_ZMAX) : 1;
  if (groups == 0) return;
  static_assert(FFN_EZ % 8 == 0, "whole TT-entry steps per chunk");
  const int fdim = L.moe ? D.f : D.df;
  const int nb_up = D.d >> 5;
  if (B.T == 1) {
    constexpr int PAIRS = 16, TT = 1;
    dim3 grid((fdim + PAIRS - 1) / PAIRS, groups, nz);
    HG_NB_SWITCH(nb_up, launch_pdl(B.T <= PDL_MAX_T, k_ffn_up<NB, PAIRS, TT>, grid, dim3(PAIRS * 16), act_smem(TT, D.d), st, D, B, L, ez, sh));
  } else {
    constexpr int PAIRS = 16, TT = 8;
    dim3 grid((fdim + PAIRS - 1) / PAIRS, groups, nz);
    HG_NB_SWITCH(nb_up, launch_pdl(B.T <= PDL_MAX_T, k_ffn_up<NB, PAIRS, TT>, grid, dim3(PAIRS * 16), act_smem(TT, D.d), st, D, B, L, ez, sh));
  }
  // dense layers and the shared expert use the down matrix of their own width
  const int nb_dn = fdim >> 5;
  if (B.T == 1) {
    constexpr int ROWS = 8, TT = 1;
    dim3 grid((D.d + ROWS - 1) / ROWS, groups, nz);
    HG_NB_SWITCH(nb_dn, launch_pdl(B.T <= PDL_MAX_T, k_ffn_down<NB, ROWS, TT>, grid, dim3(ROWS * 8), act_smem(TT, fdim), st, D, B, L, ez, sh));
  } else {
    constexpr int ROWS = 32, TT = 8;
    dim3 grid((D.d + ROWS - 1) / ROWS, groups, nz);
    HG_NB_SWITCH(nb_dn, launch_pdl(B.T <= PDL_MAX_T, k_ffn_down<NB, ROWS, TT>, grid, dim3(ROWS * 8), act_smem(TT, fdim), st, D, B, L, ez, sh));
  }
}

// SMs of each device (set by prepare_attn, before any capture)
static int g_attn_sms[64];

template <int HD, int REP>
static size_t scores_smem(int T) {
  return ScoresShape<HD, REP>::SMEM + (((size_t)T + 1) * 4 + 15) / 16 * 16;
}

// Units are dealt to the scores CTAs in contiguous runs, so the grid only needs to fill the GPU:
// every resident CTA slot, or one CTA per unit when there are fewer units than that.
template <int HD, int REP>
static int scores_grid(const AttnArgs& A, size_t smem) {
  int dev = 0, per_sm = 1;
  cudaGetDevice(&dev);
  const int sms = (dev >= 0 && dev < 64 && g_attn_sms[dev] > 0) ? g_attn_sms[dev] : 148;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_attn_scores<HD, REP>, 32 * SC_WARPS, smem);
  const long long units = (long long)A.T * A.nkv * ((A.max_pos + ATT_UNIT - 1) / ATT_UNIT);
  const long long g = std::min<long long>(units, (long long)sms * std::max(per_sm, 1));
  return (int)std::max<long long>(g, 1);
}

template <int HD, int REP>
static cudaError_t launch_attn_t(const AttnArgs& A, cudaStream_t st, int which) {
  const bool pdl = A.T <= PDL_MAX_T;
  if (which & 1) {
    const int nw = A.nh + A.nkv;
    launch_pdl(pdl, k_qk_prep<HD>, dim3(A.T), dim3(32 * nw), (size_t)nw * HD * 4, st, A);
    const size_t sm = scores_smem<HD, REP>(A.T);
    launch_pdl(pdl, k_attn_scores<HD, REP>, dim3(scores_grid<HD, REP>(A, sm)), dim3(32 * SC_WARPS), sm, st, A);
  }
  if (which & 2) {
    launch_pdl(pdl, k_attn_softmax, dim3(A.T * A.nh), dim3(SMX_THREADS), 0, st, A);
    if (A.T * A.nkv <= PVS_DEEP_MAX_PAIRS)
      launch_pdl(pdl, k_attn_pv_small<HD, REP, PVS_SLOTS_DEEP>, dim3(A.T * A.nkv * (HD / 32)), dim3(32 * REP),
                 PvSmallShape<REP, PVS_SLOTS_DEEP>::SMEM + (size_t)A.bt_stride * 4, st, A);
    else if (A.T * A.nkv <= PV_SMALL_MAX_PAIRS)
      launch_pdl(pdl, k_attn_pv_small<HD, REP, PVS_SLOTS>, dim3(A.T * A.nkv * (HD / 32)), dim3(32 * REP),
                 PvSmallShape<REP, PVS_SLOTS>::SMEM + (size_t)A.bt_stride * 4, st, A);
    else
      launch_pdl(pdl, k_attn_pv<HD, REP>, dim3(A.T * A.nkv), dim3(HD), PvShape<HD, REP>::SMEM + (size_t)A.bt_stride * 4,
                 st, A);
  }
  return cudaGetLastError();
}

static cudaError_t launch_attn_which(const AttnArgs& A, cudaStream_t st, int which) {
  int rep = A.nh / A.nkv;
  if (A.T < 1 || A.T > SC_MAX_T || A.bt_stride > ATT_MAX_BT || !A.rinv || !A.qn || !A.mkey || A.nh + A.nkv > 32 ||
      A.page_stride % 4 != 0)
    return cudaErrorInvalidValue;
  if (A.hd == 128 && rep == 4) return launch_attn_t<128, 4>(A, st, which);
  if (A.hd == 64 && rep == 4) return launch_attn_t<64, 4>(A, st, which);
  if (A.hd == 128 && rep == 2) return launch_attn_t<128, 2>(A, st, which);
  if (A.hd == 64 && rep == 2) return launch_attn_t<64, 2>(A, st, which);
  if (A.hd == 128 && rep == 1) return launch_attn_t<128, 1>(A, st, which);
  if (A.hd == 64 && rep == 1) return launch_attn_t<64, 1>(A, st, which);
  return cudaErrorInvalidValue;
}
cudaError_t launch_attn_scores_only(const AttnArgs& A, cudaStream_t st) { return launch_attn_which(A, st, 1); }
cudaError_t launch_attn_out_only(const AttnArgs& A, cudaStream_t st) { return launch_attn_which(A, st, 2); }

// Opt in to the kernels' dynamic shared memory and record the SM count on the current device
// (call before any launch or graph capture).
template <int HD, int REP>
static cudaError_t prepare_attn_t() {
  cudaError_t e = cudaFuncSetAttribute((const void*)k_attn_scores<HD, REP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)scores_smem<HD, REP>(SC_MAX_T));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void*)k_attn_pv<HD, REP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(PvShape<HD, REP>::SMEM + ATT_MAX_BT * 4));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void*)k_attn_pv_small<HD, REP, PVS_SLOTS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(PvSmallShape<REP, PVS_SLOTS>::SMEM + ATT_MAX_BT * 4));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void*)k_attn_pv_small<HD, REP, PVS_SLOTS_DEEP>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(PvSmallShape<REP, PVS_SLOTS_DEEP>::SMEM + ATT_MAX_BT * 4));
  return e;
}

cudaError_t prepare_attn(int hd, int rep) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) {
    e = cudaDeviceGetAttribute(&g_attn_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  if (hd == 128 && rep == 4) return prepare_attn_t<128, 4>();
  if (hd == 64 && rep == 4) return prepare_attn_t<64, 4>();
  if (hd == 128 && rep == 2) return prepare_attn_t<128, 2>();
  if (hd == 64 && rep == 2) return prepare_attn_t<64, 2>();
  if (hd == 128 && rep == 1) return prepare_attn_t<128, 1>();
  if (hd == 64 && rep == 1) return prepare_attn_t<64, 1>();
  return cudaErrorInvalidValue;
}

cudaError_t launch_attn_args(const AttnArgs& A, cudaStream_t st) { return launch_attn_which(A, st, 3); }

void launch_quant_rows(const float* x, int rows, int cols, int8_t* q, float* s, cudaStream_t st) {
  k_quant_rows<<<rows, 256, 0, st>>>(x, cols, q, s);
}

}  // namespace hg
