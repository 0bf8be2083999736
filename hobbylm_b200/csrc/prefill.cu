// Prefill kernels (Model::prefill, hobby-rs/src/model.rs:340-439, 653-750) in the reference's own
// arithmetic order, so the KV cache and the last-position logits match hobby-rs bit for bit
// (with exp pinned to (float)exp((double)x)):
//   * RMSNorm / QK-norm: sequential f32 sum of squares (ops.rs:85-95, model.rs:753-763);
//   * Q8 matmul: per output, blocks in order, acc += (sw*dx)*isum with an exact int32 block dot
//     (quant.rs:144-193);
//   * attention scores: ops::dot order (ops.rs:7-36) then * 1/sqrt(hd); softmax with a sequential
//     sum (ops.rs:112-128); values accumulated sequentially over positions (model.rs:426-432);
//   * MoE: routed experts accumulated per token in ascending expert id, then the shared expert
//     (model.rs:705-746).
// The prompt may be processed in chunks: every per-row step is row-local and attention reads the
// cache, so chunking does not change any result.
#include "hg_launch.h"

namespace hg {

// ------------------------------------------------------------------------------------------
// Exact RMSNorm of rows + quantization. One warp per row; lane 0 runs the sequential sum.
// in: [rows][d]; h_out (optional) [rows][d]; q/s quantized rows. Optional residual add first:
// if add != null: x = x + add (written back to in) before the norm.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) kp_norm_exact(float* in, const float* add, int rows, int d,
                                                     const float* __restrict__ w, float eps, float* h_out, int8_t* q,
                                                     float* s) {
  extern __shared__ float sq[];  // [4][d]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 4 + warp;
  if (r >= rows) return;
  float* x = in + (size_t)r * d;
  float* buf = sq + (size_t)warp * d;
  for (int i = lane; i < d; i += 32) {
    float v = x[i];
    if (add) {
      v = fadd(v, add[(size_t)r * d + i]);
      x[i] = v;
    }
    buf[i] = v;
  }
  __syncwarp();
  float scale = 0.0f;
  if (lane == 0) {
    float ss = 0.0f;
    for (int i = 0; i < d; i++) ss = fadd(ss, fmul(buf[i], buf[i]));
    scale = __fdiv_rn(1.0f, __fsqrt_rn(fadd(__fdiv_rn(ss, (float)d), eps)));
  }
  scale = __shfl_sync(0xffffffffu, scale, 0);
  for (int i = lane; i < d; i += 32) {
    float h = fmul(fmul(buf[i], scale), w[i]);
    buf[i] = h;
    if (h_out) h_out[(size_t)r * d + i] = h;
  }
  __syncwarp();
  const int nb = d >> 5;
  for (int b = 0; b < nb; b++) {
    float dq;
    int8_t qv = quant_lane(buf[b * 32 + lane], &dq);
    q[(size_t)r * d + q8_pos(b * 32 + lane, nb)] = qv;
    if (lane == 0) s[(size_t)r * q8_ss(nb) + b] = dq;
  }
}

// ------------------------------------------------------------------------------------------
// Q8 matmul in the prefill order. Tile: 64 output rows x 64 activation rows, 256 threads, each
// 4 x 4 outputs. K loop over 4-block chunks (128 bytes per row) then tail blocks.
// A rows: aq + arow(i) * cols (arow = a_idx ? a_idx[i] : i); out: out[orow(i) * ostride + o]
// (orow = o_idx ? o_idx[i] : i); mode 0 store, 1 add into out. Matrix m of a stack = mat.
// ------------------------------------------------------------------------------------------

__global__ void __launch_bounds__(256) kp_matmul(MmArgs a) {
  // rows padded to 144 bytes: rows r and r+1 start 4 banks apart (few shared-memory conflicts)
  __shared__ __align__(16) int8_t ws[64][144];
  __shared__ __align__(16) int8_t xs[64][144];
  __shared__ float wsc[64][4], xsc[64][4];
  int mat = a.mat, n = a.nrows, off = 0;
  if (a.grp_mat) {
    mat = a.grp_mat[blockIdx.z];
    if (mat < 0) return;
    off = a.grp_off[blockIdx.z];
    n = a.grp_cnt[blockIdx.z];
  }
  const int o0 = blockIdx.x * 64, r0 = blockIdx.y * 64;
  if (r0 >= n || o0 >= a.W.rows) return;
  const int cols = a.W.cols, nb = cols >> 5, ss = a.W.ss, nc = nb >> 2, nt = nb & 3;
  // thread (ty, tx): output rows ty + 16 i, activation rows tx + 16 j (i, j < 4)
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
  auto arow = [&](int i) -> long long {
    int e = off + r0 + i;
    return a.a_idx ? (long long)a.a_idx[e] : (long long)e;
  };
  for (int c = 0; c < nc + nt; c++) {
    const bool full = c < nc;
    const int bytes = full ? 128 : 32;
    const int boff = full ? c * 128 : nc * 128 + (c - nc) * 32;
    const int nblk = full ? 4 : 1;
    const int b0 = full ? c * 4 : nc * 4 + (c - nc);
    __syncthreads();
    // load tiles: 64 rows x bytes each
    for (int i = threadIdx.x; i < 64 * (bytes >> 4); i += 256) {
      int r = i / (bytes >> 4), v = i - r * (bytes >> 4);
      int o = o0 + r;
      int4 wv = make_int4(0, 0, 0, 0);
      if (o < a.W.rows) wv = *reinterpret_cast<const int4*>(a.W.row_q(mat, o) + boff + v * 16);
      reinterpret_cast<int4*>(&ws[r][0])[v] = wv;
      int4 xv = make_int4(0, 0, 0, 0);
      if (r0 + r < n) xv = *reinterpret_cast<const int4*>(a.aq + arow(r) * cols + boff + v * 16);
      reinterpret_cast<int4*>(&xs[r][0])[v] = xv;
    }
    for (int i = threadIdx.x; i < 64 * nblk; i += 256) {
      int r = i / nblk, k = i - r * nblk;
      int o = o0 + r;
      wsc[r][k] = o < a.W.rows ? a.W.row_s(mat, o)[b0 + k] : 0.0f;
      xsc[r][k] = (r0 + r < n) ? a.as[arow(r) * ss + b0 + k] : 0.0f;
    }
    __syncthreads();
    for (int k = 0; k < nblk; k++) {
      // word of (block k, lane l) inside this tile row
      int isum[4][4];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) isum[i][j] = 0;
#pragma unroll
      for (int l = 0; l < 8; l++) {
        const int woff = full ? l * 16 + k * 4 : l * 4;
        int wv[4], xv[4];
#pragma unroll
        for (int i = 0; i < 4; i++) wv[i] = *reinterpret_cast<const int*>(&ws[ty + 16 * i][woff]);
#pragma unroll
        for (int j = 0; j < 4; j++) xv[j] = *reinterpret_cast<const int*>(&xs[tx + 16 * j][woff]);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) isum[i][j] = __dp4a(wv[i], xv[j], isum[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++)
          acc[i][j] = fadd(acc[i][j], fmul(fmul(wsc[ty + 16 * i][k], xsc[tx + 16 * j][k]), (float)isum[i][j]));
    }
  }
#pragma unroll
  for (int j = 0; j < 4; j++) {
    int r = r0 + tx + 16 * j;
    if (r >= n) continue;
    int e = off + r;
    long long orow = a.o_idx ? (long long)a.o_idx[e] : (long long)e;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      int o = o0 + ty + 16 * i;
      if (o >= a.W.rows) continue;
      float* p = a.out + orow * a.ostride + o;
      *p = a.mode == 1 ? fadd(*p, acc[i][j]) : acc[i][j];
    }
  }
}

// ------------------------------------------------------------------------------------------
// QK-norm + RoPE + KV append for prefill rows (model.rs:386-407). One warp per (row, head);
// the norm sum is sequential in lane 0. q heads go to qo [rows][qd]; k/v rows to their pages.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) kp_qk_rope_append(const float* qkv, int rows, int base, int nh, int nkv, int hd,
                                                         float eps, const float* q_norm, const float* k_norm,
                                                         const float* rcos, const float* rsin, const int32_t* bt,
                                                         float* k_pool, float* v_pool, long long page_stride,
                                                         float* qo) {
  extern __shared__ float buf_all[];  // [4][hd]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = nh + 2 * nkv;
  const int item = blockIdx.x * 4 + warp;
  if (item >= rows * heads) return;
  const int r = item / heads, hh = item - r * heads, pos = base + r;
  const int qd = nh * hd, kvd = nkv * hd, half = hd / 2;
  const float* src = qkv + (size_t)r * (qd + 2 * kvd) + (size_t)hh * hd;
  float* buf = buf_all + warp * hd;
  const int pg = bt[pos / PAGE], slot = pos % PAGE;
  if (hh >= nh + nkv) {  // v head: plain append
    int kvh = hh - nh - nkv;
    float* dst = v_pool + (long long)pg * page_stride + ((long long)kvh * PAGE + slot) * hd;
    for (int i = lane; i < hd; i += 32) dst[i] = src[i];
    return;
  }
  const float* w = hh < nh ? q_norm : k_norm;
  for (int i = lane; i < hd; i += 32) buf[i] = src[i];
  __syncwarp();
  float scale = 0.0f;
  if (lane == 0) {
    float ss = 0.0f;
    for (int i = 0; i < hd; i++) ss = fadd(ss, fmul(buf[i], buf[i]));
    scale = __fdiv_rn(1.0f, __fsqrt_rn(fadd(__fdiv_rn(ss, (float)hd), eps)));
  }
  scale = __shfl_sync(0xffffffffu, scale, 0);
  for (int i = lane; i < hd; i += 32) buf[i] = fmul(fmul(buf[i], scale), w[i]);
  __syncwarp();
  const float* cs = rcos + (size_t)pos * half;
  const float* sn = rsin + (size_t)pos * half;
  float* dst;
  if (hh < nh) dst = qo + (size_t)r * qd + (size_t)hh * hd;
  else dst = k_pool + (long long)pg * page_stride + ((long long)(hh - nh) * PAGE + slot) * hd;
  for (int i = lane; i < half; i += 32) {
    float x1 = buf[i], x2 = buf[half + i], c = cs[i], s = sn[i];
    dst[i] = __fsub_rn(fmul(x1, c), fmul(x2, s));
    dst[half + i] = fadd(fmul(x2, c), fmul(x1, s));
  }
}

// ------------------------------------------------------------------------------------------
// Attention scores of query rows against positions, all kv heads in one launch (blockIdx.z =
// kv head g, scores of head g at S + g * s_head). Rows R = (t_local, head-in-group) flattened:
// R = t_local * rep + hr. S[j][R] = dot(q, k_j) * scale for j < base + t + 1 (causal), or for
// j < nfix when nfix > 0: every row attends to the same nfix keys, the diffusion block's prefix
// plus the whole block (model.rs:556-565).
//
// The ops::dot order (ops.rs:7-36): accumulator m (0..3) of SIMD lane l (0..7) is the chain
// c = fma(a[32i + 8m + l], b[...], c) over i = 0..HD/32-1 from 0, lane l sums (c0 + c1) + (c2 + c3),
// and the lanes meet in the tree ((t0+t4)+(t2+t6))+((t1+t5)+(t3+t7)). Shared memory keeps each
// row with the HD/32 elements of one (l, m) chain side by side, so a chain's operands are one
// vector load. CTA: 64 rows x a run of KP_KTILES tiles of 32 positions; a warp owns 4 positions
// of a tile (broadcast loads), a lane 2 rows (lane, lane + 32: coalesced stores).
// ------------------------------------------------------------------------------------------
constexpr int KP_SR = 64;      // rows per CTA
constexpr int KP_SJ = 32;      // positions per tile
constexpr int KP_KTILES = 8;   // tiles per CTA
// padded row length (floats): an odd number of vector widths, so lanes reading different rows
// at the same offset hit different banks
template <int HD>
constexpr int kp_row_stride() { return HD + (HD / 32 == 4 ? 4 : 2); }
template <int HD>
constexpr size_t kp_scores_smem() { return (size_t)(KP_SR + 2 * KP_SJ) * kp_row_stride<HD>() * sizeof(float); }

template <int NI> struct KpVec;
template <> struct KpVec<4> {
  float v[4];
  __device__ __forceinline__ void load(const float* p) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  }
};
template <> struct KpVec<2> {
  float v[2];
  __device__ __forceinline__ void load(const float* p) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    v[0] = t.x; v[1] = t.y;
  }
};

template <int HD>
__global__ void __launch_bounds__(256) kp_scores(const float* q, int qd, int t0, int tq, int base, int rep,
                                                 const int32_t* bt, const float* k_pool, long long page_stride,
                                                 float* S, long long s_head, int nR, int nfix, uint32_t* mkey) {
  constexpr int NI = HD / 32, RS = kp_row_stride<HD>();
  __shared__ uint32_t mred[KP_SR];  // this CTA's maxima of its rows (order-preserving keys)
  extern __shared__ __align__(16) float kp_sm[];
  float* qs = kp_sm;              // [KP_SR][RS]
  float* kbuf = kp_sm + KP_SR * RS;  // [2][KP_SJ][RS]: the tile being scored and the next one
  const int g = blockIdx.z;
  const int R0 = blockIdx.x * KP_SR, jt0 = blockIdx.y * KP_KTILES * KP_SJ;
  const int Rl = min(R0 + KP_SR - 1, nR - 1);
  const int lim_hi = nfix > 0 ? nfix : base + t0 + Rl / rep + 1;  // longest row of the tile
  if (jt0 >= lim_hi) return;
  float* Sg = S + (size_t)g * s_head;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // element e = 32 ii + 8 m + l of a row goes to (l * 4 + m) * NI + ii
  auto perm = [](int e) { return (((e & 7) * 4 + ((e >> 3) & 3)) * NI) + (e >> 5); };
  for (int i = tid; i < KP_SR * HD; i += 256) {
    const int rr = i / HD, e = i - rr * HD, R = R0 + rr;
    float v = 0.0f;
    if (R < nR) {
      const int tl = R / rep, hr = R - tl * rep;
      v = q[(size_t)(t0 + tl) * qd + (size_t)(g * rep + hr) * HD + e];
    }
    qs[rr * RS + perm(e)] = v;
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  int lim[2];
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int R = R0 + lane + 32 * k;
    lim[k] = R < nR ? (nfix > 0 ? nfix : base + t0 + R / rep + 1) : 0;
  }
  const float* qa0 = qs + lane * RS;
  const float* qa1 = qs + (lane + 32) * RS;
  if (tid < KP_SR) mred[tid] = 0u;  // ordered before use by the first tile's barrier
  float mx[2] = {-INFINITY, -INFINITY};
  // K tiles: thread tid holds 16-byte pieces c = tid + 256 i of the next tile in registers while
  // the current one is scored (piece c: position c / (HD / 4), elements 4 (c % (HD / 4)) .. + 3)
  constexpr int KQ = KP_SJ * HD / 4 / 256;
  float4 kr[KQ];
  auto load_k = [&](int j0) {
#pragma unroll
    for (int i = 0; i < KQ; i++) {
      const int c = tid + 256 * i, jj = c / (HD / 4), e4 = (c - jj * (HD / 4)) * 4, j = j0 + jj;
      kr[i] = j < lim_hi ? *reinterpret_cast<const float4*>(k_pool + (long long)bt[j / PAGE] * page_stride +
                                                            ((long long)g * PAGE + (j % PAGE)) * HD + e4)
                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  };
  auto store_k = [&](float* kb) {
#pragma unroll
    for (int i = 0; i < KQ; i++) {
      const int c = tid + 256 * i, jj = c / (HD / 4), e4 = (c - jj * (HD / 4)) * 4;
      float* row = kb + jj * RS;
      row[perm(e4)] = kr[i].x;
      row[perm(e4 + 1)] = kr[i].y;
      row[perm(e4 + 2)] = kr[i].z;
      row[perm(e4 + 3)] = kr[i].w;
    }
  };
  int ntile = 0;
  while (ntile < KP_KTILES && jt0 + ntile * KP_SJ < lim_hi) ntile++;
  load_k(jt0);
  for (int kt = 0; kt < ntile; kt++) {
    const int j0 = jt0 + kt * KP_SJ;
    float* ks = kbuf + (kt & 1) * KP_SJ * RS;
    store_k(ks);  // buffer kt % 2 was last read by tile kt - 2, before the previous barrier
    if (kt + 1 < ntile) load_k(j0 + KP_SJ);
    __syncthreads();
    // pairs (row lane + 32 r, position j0 + 4 warp + p)
    float A[2][4], Bt[2][4], Dt[2][4];
    constexpr int LORD[8] = {0, 4, 2, 6, 1, 5, 3, 7};
#pragma unroll
    for (int li = 0; li < 8; li++) {
      const int l = LORD[li];
      float pc[2][4], qc[2][4];
#pragma unroll
      for (int m = 0; m < 4; m++) {
        KpVec<NI> a[2], b[4];
        a[0].load(qa0 + (l * 4 + m) * NI);
        a[1].load(qa1 + (l * 4 + m) * NI);
#pragma unroll
        for (int p = 0; p < 4; p++) b[p].load(ks + (warp * 4 + p) * RS + (l * 4 + m) * NI);
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
          for (int p = 0; p < 4; p++) {
            float c = __fmaf_rn(a[r].v[0], b[p].v[0], 0.0f);
#pragma unroll
            for (int ii = 1; ii < NI; ii++) c = __fmaf_rn(a[r].v[ii], b[p].v[ii], c);
            if (m == 0) pc[r][p] = c;
            else if (m == 1) pc[r][p] = fadd(pc[r][p], c);
            else if (m == 2) qc[r][p] = c;
            else qc[r][p] = fadd(qc[r][p], c);
          }
      }
#pragma unroll
      for (int r = 0; r < 2; r++)
#pragma unroll
        for (int p = 0; p < 4; p++) {
          const float t = fadd(pc[r][p], qc[r][p]);  // lane l: (c0 + c1) + (c2 + c3)
          if (li == 0) A[r][p] = t;
          else if (li == 1) A[r][p] = fadd(A[r][p], t);             // t0 + t4
          else if (li == 2) Bt[r][p] = t;
          else if (li == 3) A[r][p] = fadd(A[r][p], fadd(Bt[r][p], t));  // (t0+t4)+(t2+t6)
          else if (li == 4) Bt[r][p] = t;
          else if (li == 5) Bt[r][p] = fadd(Bt[r][p], t);           // t1 + t5
          else if (li == 6) Dt[r][p] = t;
          else A[r][p] = fadd(A[r][p], fadd(Bt[r][p], fadd(Dt[r][p], t)));  // + ((t1+t5)+(t3+t7))
        }
    }
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int R = R0 + lane + 32 * r;
#pragma unroll
      for (int p = 0; p < 4; p++) {
        const int j = j0 + warp * 4 + p;
        if (j < lim[r]) {
          const float sv = fmul(A[r][p], scale);
          Sg[(size_t)j * nR + R] = sv;
          mx[r] = fmaxf(mx[r], sv);
        }
      }
    }
  }
  // row maxima for the softmax (any order gives the same maximum): the CTA's, then global
#pragma unroll
  for (int r = 0; r < 2; r++)
    if (mx[r] > -INFINITY) atomicMax(&mred[lane + 32 * r], f2key(mx[r]));
  __syncthreads();
  if (tid < KP_SR && R0 + tid < nR && mred[tid]) atomicMax(&mkey[(size_t)g * nR + R0 + tid], mred[tid]);
}

// Softmax of score rows (ops.rs:112-128), all kv heads (blockIdx.y = g). One thread per row: with
// the row maximum that kp_scores left in mkey, e = exp(s - max) is written back in place and
// summed in position order in a register chain (the reference's sequential sum);
// inv[g * nR + R] = 1 / sum. Row lengths as kp_scores. Lanes are consecutive rows, so every load
// and store is coalesced.
__global__ void __launch_bounds__(32) kp_softmax_rows(float* S, long long s_head, int nR, int rep, int base, int t0,
                                                      int nfix, const uint32_t* mkey, float* inv) {
  constexpr int U = 16;  // positions in flight per thread
  const int g = blockIdx.y, R = blockIdx.x * 32 + threadIdx.x;
  if (R >= nR) return;
  float* Sg = S + (size_t)g * s_head + R;
  const size_t st = (size_t)nR;
  const int n = nfix > 0 ? nfix : base + t0 + R / rep + 1;
  const float m = key2f(mkey[(size_t)g * nR + R]);  // the row's maximum score, from kp_scores
  float sum = 0.0f;
  int j = 0;
  if (j + U <= n) {
    float v[U];
#pragma unroll
    for (int u = 0; u < U; u++) v[u] = Sg[(j + u) * st];
    for (; j + U <= n; j += U) {
      float e[U];
#pragma unroll
      for (int u = 0; u < U; u++) e[u] = exp_cr(__fsub_rn(v[u], m));
      if (j + 2 * U <= n) {  // the next group's scores, loaded while this group's sum runs
#pragma unroll
        for (int u = 0; u < U; u++) v[u] = Sg[(j + U + u) * st];
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        Sg[(j + u) * st] = e[u];
        sum = fadd(sum, e[u]);
      }
    }
  }
  for (; j < n; j++) {
    const float e = exp_cr(__fsub_rn(Sg[j * st], m));
    Sg[j * st] = e;
    sum = fadd(sum, e);
  }
  inv[(size_t)g * nR + R] = __fdiv_rn(1.0f, sum);
}

// O[t][h][dd] = sum_j (e_j * inv) * v_j[dd], sequential in j (model.rs:426-432; 573-584 for a
// diffusion block, whose prefix-then-block order is position order), kv head g = blockIdx.y.
// CTA: 64 rows x HD dims; warp w owns rows 8w..8w+7, lane owns dims HD/32 * lane + 0..HD/32-1, so a
// thread runs 8 x HD/32 chains. Tiles of 32 positions are staged in shared memory, double
// buffered and loaded into registers a tile ahead: p = e * inv (ops.rs:124-126) formed once per
// (row, position), and 0 past the row's length -- adding fmul(0, v) = +-0 leaves a chain exactly
// unchanged (a chain that starts at +0 never holds -0), so the chains need no per-position test.
constexpr int KP_PR = 64;   // rows per CTA
constexpr int KP_PJ = 32;   // positions per tile
template <int HD>
constexpr size_t kp_pv_smem() { return (size_t)2 * KP_PJ * (KP_PR + HD) * sizeof(float); }

template <int HD>
__global__ void __launch_bounds__(256) kp_pv(const float* S, long long s_head, const float* inv, int nR, int rep,
                                             int base, int t0, int nfix, const int32_t* bt, const float* v_pool,
                                             long long page_stride, float* o, int qd) {
  constexpr int DPT = HD / 32;                 // dims per thread
  constexpr int VQ = KP_PJ * HD / 4 / 256;     // float4 pieces of a V tile per thread
  constexpr int SQ = KP_PJ * KP_PR / 256;      // probabilities of a tile per thread
  extern __shared__ __align__(16) float kp_pv_sm[];
  float* ps = kp_pv_sm;                        // [2][KP_PJ][KP_PR]
  float* vs = kp_pv_sm + 2 * KP_PJ * KP_PR;    // [2][KP_PJ][HD]
  const int g = blockIdx.y;
  const float* Sg = S + (size_t)g * s_head;
  const float* ig = inv + (size_t)g * nR;
  const int R0 = blockIdx.x * KP_PR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int Rlast = min(R0 + KP_PR - 1, nR - 1);
  const int nmax = nfix > 0 ? nfix : base + t0 + Rlast / rep + 1;
  // staging role: one row (tid % 64) of the probabilities
  const int sr = tid & (KP_PR - 1), sR = R0 + sr;
  const int slim = sR < nR ? (nfix > 0 ? nfix : base + t0 + sR / rep + 1) : 0;
  const float siv = sR < nR ? ig[sR] : 0.0f;
  float pr[SQ];
  float4 vr[VQ];
  auto load_tile = [&](int j0) {
#pragma unroll
    for (int q = 0; q < SQ; q++) {
      const int j = j0 + ((tid + 256 * q) >> 6);
      pr[q] = j < slim ? fmul(Sg[(size_t)j * nR + sR], siv) : 0.0f;
    }
#pragma unroll
    for (int q = 0; q < VQ; q++) {
      const int idx = tid + 256 * q, jj = idx / (HD / 4), c4 = idx - jj * (HD / 4), j = j0 + jj;
      vr[q] = j < nmax ? *reinterpret_cast<const float4*>(
                             v_pool + (long long)bt[j / PAGE] * page_stride + ((long long)g * PAGE + (j % PAGE)) * HD +
                             c4 * 4)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  };
  auto store_tile = [&](int b) {
    float* pb = ps + b * KP_PJ * KP_PR;
    float* vb = vs + b * KP_PJ * HD;
#pragma unroll
    for (int q = 0; q < SQ; q++) pb[((tid + 256 * q) >> 6) * KP_PR + sr] = pr[q];
#pragma unroll
    for (int q = 0; q < VQ; q++) reinterpret_cast<float4*>(vb)[tid + 256 * q] = vr[q];
  };
  float acc[8][DPT];
#pragma unroll
  for (int i = 0; i < 8; i++)
#pragma unroll
    for (int k = 0; k < DPT; k++) acc[i][k] = 0.0f;
  const int ntile = (nmax + KP_PJ - 1) / KP_PJ;
  load_tile(0);
  for (int t = 0; t < ntile; t++) {
    const int b = t & 1;
    store_tile(b);  // buffer b was last read two tiles ago, before the previous barrier
    if (t + 1 < ntile) load_tile((t + 1) * KP_PJ);
    __syncthreads();
    const float* pb = ps + b * KP_PJ * KP_PR + warp * 8;
    const float* vb = vs + b * KP_PJ * HD + lane * DPT;
#pragma unroll 4
    for (int jj = 0; jj < KP_PJ; jj++) {
      const float4 p0 = *reinterpret_cast<const float4*>(pb + jj * KP_PR);
      const float4 p1 = *reinterpret_cast<const float4*>(pb + jj * KP_PR + 4);
      const float p[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
      float v[DPT];
      if (DPT == 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(vb + jj * HD);
        v[0] = t4.x; v[1] = t4.y; v[2 % DPT] = t4.z; v[3 % DPT] = t4.w;
      } else {
        const float2 t2 = *reinterpret_cast<const float2*>(vb + jj * HD);
        v[0] = t2.x; v[1 % DPT] = t2.y;
      }
#pragma unroll
      for (int i = 0; i < 8; i++)
#pragma unroll
        for (int k = 0; k < DPT; k++) acc[i][k] = fadd(acc[i][k], fmul(p[i], v[k]));
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int R = R0 + warp * 8 + i;
    if (R >= nR) continue;
    const int tl = R / rep, hr = R - tl * rep;
    float* dst = o + (size_t)(t0 + tl) * qd + (size_t)(g * rep + hr) * HD + lane * DPT;
#pragma unroll
    for (int k = 0; k < DPT; k++) dst[k] = acc[i][k];
  }
}

// ------------------------------------------------------------------------------------------
// Router for prefill rows (model.rs:671-703): h rows are already normed (exact). One CTA per
// token. Writes sel/selw and expert token lists (entries t * 32 + rank) with per-expert counts.
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) kp_route(const float* h, int d, const float* router, const float* bias, int ne,
                                                int k, int gsig, int wnorm, float wscale, int32_t* sel, float* selw,
                                                int32_t* ecount, int32_t* elist, int list_cap) {
  __shared__ float logit_s[128], score_s[128], selsc_s[128];
  __shared__ int rank_e[MAX_TOPK];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const float* hr = h + (size_t)t * d;
  for (int e = warp; e < ne; e += nw) {
    float lg = dot_ref_warp(router + (size_t)e * d, hr, d);
    if ((threadIdx.x & 31) == 0) logit_s[e] = lg;
  }
  __syncthreads();
  if (threadIdx.x == 0 && !gsig) {
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
    float sc = gsig ? sigmoid_ref(logit_s[e]) : score_s[e];
    score_s[e] = sc;
    selsc_s[e] = fadd(sc, bias[e]);
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
  if (threadIdx.x == 0) {
    float w[MAX_TOPK];
    for (int r = 0; r < k; r++) w[r] = score_s[rank_e[r]];
    if (wnorm) {
      float s = -0.0f;
      for (int r = 0; r < k; r++) s = fadd(s, w[r]);
      s = fadd(s, 1e-9f);
      for (int r = 0; r < k; r++) w[r] = __fdiv_rn(w[r], s);
    }
    for (int r = 0; r < k; r++) {
      int e = rank_e[r];
      sel[t * k + r] = e;
      selw[t * k + r] = fmul(w[r], wscale);  // model.rs:701 stores w * expert_weights_scale
      int slot = atomicAdd(&ecount[e], 1);
      elist[(size_t)e * list_cap + slot] = t * 32 + r;
    }
  }
}

// Grouped expert tables for the routed-expert matmul launches: group e = expert e with its list
// at elist[e * list_cap] (empty experts are skipped).
__global__ void kp_expert_tables(const int32_t* ecount, int ne, int list_cap, int32_t* grp_mat, int32_t* grp_off,
                                 int32_t* grp_cnt) {
  int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= ne) return;
  int c = ecount[e];
  grp_mat[e] = c > 0 ? e : -1;
  grp_off[e] = e * list_cap;
  grp_cnt[e] = c;
}

// Output rows of the shared expert: token t writes slot k of its (k + 1)-slot group.
__global__ void kp_shared_rows(int tn, int k, int32_t* o_idx) {
  int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < tn) o_idx[t] = t * (k + 1) + k;
}

// Row indices of the grouped matmuls from the packed list entries (t * 32 + rank):
// a_idx = t (rows of the normed hidden state); o_idx = t * (k + 1) + rank (per-slot outputs).
__global__ void kp_entry_rows(const int32_t* elist, int n, int k, int32_t* a_idx, int32_t* o_idx) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int code = elist[i];
  if (code < 0) return;
  int t = code >> 5, r = code & 31;
  a_idx[i] = t;
  o_idx[i] = t * (k + 1) + r;
}

// SwiGLU: act = silu(g) * u elementwise (model.rs:721-723).
__global__ void kp_swiglu(const float* g, const float* u, float* act, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = fmul(silu_ref(g[i]), u[i]);
}

// Quantize rows of f32 (warp per 32-block).
__global__ void __launch_bounds__(256) kp_quant_rows(const float* x, long long rows, int cols, int8_t* q, float* s) {
  const int nb = cols >> 5;
  long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= rows * nb) return;
  long long r = gw / nb;
  int b = (int)(gw - r * nb);
  float dq;
  int8_t qv = quant_lane(x[r * cols + b * 32 + lane], &dq);
  q[r * cols + q8_pos(b * 32 + lane, nb)] = qv;
  if (lane == 0) s[r * q8_ss(nb) + b] = dq;
}

// MoE combine for prefill rows (model.rs:705-746) and the residual add: per token, routed expert
// outputs in ascending expert id, then the shared expert; x += out. Dense: x += y[t][0].
__global__ void kp_combine(float* x, const float* y, const int32_t* sel, const float* selw, int tn, int d, int k,
                           int moe, int n_shared) {
  const int t = blockIdx.x;
  __shared__ int ord[MAX_TOPK];
  if (threadIdx.x == 0 && moe) {
    for (int r = 0; r < k; r++) ord[r] = r;
    for (int a = 1; a < k; a++) {  // insertion sort of ranks by expert id
      int v = ord[a], b = a - 1;
      while (b >= 0 && sel[t * k + ord[b]] > sel[t * k + v]) {
        ord[b + 1] = ord[b];
        b--;
      }
      ord[b + 1] = v;
    }
  }
  __syncthreads();
  const float* yt = y + (size_t)t * (k + 1) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float o;
    if (moe) {
      o = 0.0f;
      for (int a = 0; a < k; a++) {
        int r = ord[a];
        o = fadd(o, fmul(selw[t * k + r], yt[r * d + i]));
      }
      if (n_shared > 0) o = fadd(o, yt[k * d + i]);
    } else {
      o = yt[i];
    }
    x[(size_t)t * d + i] = fadd(x[(size_t)t * d + i], o);
  }
}

__global__ void kp_embed(const float* embd, const int32_t* ids, int n, int d, int vocab, float* x, int32_t* err) {
  int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) atomicExch(err, HG_ERR_TOKEN);
    id = 0;
  }
  for (int i = threadIdx.x; i < d; i += blockDim.x) x[(size_t)t * d + i] = embd[(size_t)id * d + i];
}

// ------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------
void launch_kp_norm(float* in, const float* add, int rows, int d, const float* w, float eps, float* h_out, int8_t* q,
                    float* s, cudaStream_t st) {
  kp_norm_exact<<<(rows + 3) / 4, 128, 4 * d * sizeof(float), st>>>(in, add, rows, d, w, eps, h_out, q, s);
}
void launch_kp_matmul(const MmArgs& a, int nrows_max, int groups, cudaStream_t st) {
  // block sums from the tensor cores (tc.cu); a grouped launch indexes matrices 0..groups-1
  if (kp_tc_usable(a, nrows_max, groups) &&
      launch_kp_tc(a, nrows_max, groups, a.grp_mat ? groups : a.mat + 1, st))
    return;
  dim3 grid((a.W.rows + 63) / 64, (nrows_max + 63) / 64, groups);
  kp_matmul<<<grid, 256, 0, st>>>(a);
}
void launch_kp_qk_rope_append(const float* qkv, int rows, int base, int nh, int nkv, int hd, float eps,
                              const float* q_norm, const float* k_norm, const float* rcos, const float* rsin,
                              const int32_t* bt, float* k_pool, float* v_pool, long long page_stride, float* qo,
                              cudaStream_t st) {
  int items = rows * (nh + 2 * nkv);
  kp_qk_rope_append<<<(items + 3) / 4, 128, 4 * hd * sizeof(float), st>>>(
      qkv, rows, base, nh, nkv, hd, eps, q_norm, k_norm, rcos, rsin, bt, k_pool, v_pool, page_stride, qo);
}
void launch_kp_attention(const float* q, int qd, int t0, int tq, int base, int nfix, int nh, int nkv, int hd,
                         const int32_t* bt, const float* k_pool, const float* v_pool, long long page_stride, float* S,
                         float* inv, uint32_t* mkey, float* o, cudaStream_t st) {
  static bool smem_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !smem_set[dev]) {
    cudaFuncSetAttribute((const void*)kp_scores<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kp_scores_smem<128>());
    cudaFuncSetAttribute((const void*)kp_scores<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kp_scores_smem<64>());
    cudaFuncSetAttribute((const void*)kp_pv<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kp_pv_smem<128>());
    cudaFuncSetAttribute((const void*)kp_pv<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kp_pv_smem<64>());
    smem_set[dev] = true;
  }
  const int rep = nh / nkv;
  const int nR = tq * rep;
  const int nmax = nfix > 0 ? nfix : base + t0 + tq;
  const long long s_head = (long long)nmax * nR;  // scores of one kv head
  const dim3 gs((nR + KP_SR - 1) / KP_SR, (nmax + KP_KTILES * KP_SJ - 1) / (KP_KTILES * KP_SJ), nkv);
  cudaMemsetAsync(mkey, 0, (size_t)nkv * nR * sizeof(uint32_t), st);  // key 0 sorts below every score
  if (hd == 128)
    kp_scores<128><<<gs, 256, kp_scores_smem<128>(), st>>>(q, qd, t0, tq, base, rep, bt, k_pool, page_stride, S,
                                                           s_head, nR, nfix, mkey);
  else
    kp_scores<64><<<gs, 256, kp_scores_smem<64>(), st>>>(q, qd, t0, tq, base, rep, bt, k_pool, page_stride, S,
                                                         s_head, nR, nfix, mkey);
  kp_softmax_rows<<<dim3((nR + 31) / 32, nkv), 32, 0, st>>>(S, s_head, nR, rep, base, t0, nfix, mkey, inv);
  const dim3 gp((nR + KP_PR - 1) / KP_PR, nkv);
  if (hd == 128)
    kp_pv<128><<<gp, 256, kp_pv_smem<128>(), st>>>(S, s_head, inv, nR, rep, base, t0, nfix, bt, v_pool, page_stride,
                                                   o, qd);
  else
    kp_pv<64><<<gp, 256, kp_pv_smem<64>(), st>>>(S, s_head, inv, nR, rep, base, t0, nfix, bt, v_pool, page_stride, o,
                                                 qd);
}
void launch_kp_route(const float* h, int tn, int d, const float* router, const float* bias, int ne, int k, int gsig,
                     int wnorm, float wscale, int32_t* sel, float* selw, int32_t* ecount, int32_t* elist, int list_cap,
                     cudaStream_t st) {
  kp_route<<<tn, 256, 0, st>>>(h, d, router, bias, ne, k, gsig, wnorm, wscale, sel, selw, ecount, elist, list_cap);
}
void launch_kp_expert_tables(const int32_t* ecount, int ne, int list_cap, int32_t* grp_mat, int32_t* grp_off,
                             int32_t* grp_cnt, cudaStream_t st) {
  kp_expert_tables<<<(ne + 127) / 128, 128, 0, st>>>(ecount, ne, list_cap, grp_mat, grp_off, grp_cnt);
}
void launch_kp_shared_rows(int tn, int k, int32_t* o_idx, cudaStream_t st) {
  kp_shared_rows<<<(tn + 255) / 256, 256, 0, st>>>(tn, k, o_idx);
}
void launch_kp_entry_rows(const int32_t* elist, int n, int k, int32_t* a_idx, int32_t* o_idx, cudaStream_t st) {
  kp_entry_rows<<<(n + 255) / 256, 256, 0, st>>>(elist, n, k, a_idx, o_idx);
}
void launch_kp_swiglu(const float* g, const float* u, float* act, long long n, cudaStream_t st) {
  kp_swiglu<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, act, n);
}
void launch_kp_quant_rows(const float* x, long long rows, int cols, int8_t* q, float* s, cudaStream_t st) {
  long long warps = rows * (cols >> 5);
  kp_quant_rows<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, st>>>(x, rows, cols, q, s);
}
void launch_kp_combine(float* x, const float* y, const int32_t* sel, const float* selw, int tn, int d, int k, int moe,
                       int n_shared, cudaStream_t st) {
  kp_combine<<<tn, 256, 0, st>>>(x, y, sel, selw, tn, d, k, moe, n_shared);
}
void launch_kp_embed(const float* embd, const int32_t* ids, int n, int d, int vocab, float* x, int32_t* err,
                     cudaStream_t st) {
  kp_embed<<<n, 256, 0, st>>>(embd, ids, n, d, vocab, x, err);
}

}  // namespace hg
