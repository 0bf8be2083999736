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
#include "hg_model.cuh"

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
// Attention scores for a tile of query rows. R = (t_local, head-in-group) flattened for one kv
// head g: R = t_local * rep + hr. S[j][R] = dot(q, k_j) * scale for j < base + t + 1 (causal), or
// for j < nfix when nfix > 0: every row attends to the same nfix keys, the diffusion block's
// prefix plus the whole block (model.rs:556-565). One thread per (R, j) with the ops::dot order
// computed per SIMD lane.
// ------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(256) kp_scores(const float* q, int qd, int t0, int tq, int base, int rep, int kvh,
                                                 const int32_t* bt, const float* k_pool, long long page_stride,
                                                 float* S, int nR, int nfix) {
  __shared__ float qs[32][HD + 1];
  __shared__ float ks[32][HD + 1];
  const int R0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  const int nmax = nfix > 0 ? nfix : base + t0 + tq;  // longest row in the tile set
  if (j0 >= nmax) return;
  // rows of this R tile: token t_local = R / rep, head = kvh*rep + R%rep
  for (int i = threadIdx.x; i < 32 * HD; i += 256) {
    int rr = i / HD, dd = i - rr * HD;
    int R = R0 + rr;
    float v = 0.0f;
    if (R < nR) {
      int tl = R / rep, hr = R - tl * rep;
      v = q[(size_t)(t0 + tl) * qd + (size_t)(kvh * rep + hr) * HD + dd];
    }
    qs[rr][dd] = v;
    int j = j0 + rr;
    float kv = 0.0f;
    if (j < nmax) kv = k_pool[(long long)bt[j / PAGE] * page_stride + ((long long)kvh * PAGE + (j % PAGE)) * HD + dd];
    ks[rr][dd] = kv;
  }
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  for (int o = threadIdx.x; o < 32 * 32; o += 256) {
    int jj = o >> 5, rr = o & 31;  // consecutive threads -> consecutive R (coalesced store)
    int R = R0 + rr, j = j0 + jj;
    if (R >= nR) continue;
    int tl = R / rep;
    if (j >= (nfix > 0 ? nfix : base + t0 + tl + 1)) continue;
    const float* a = qs[rr];
    const float* b = ks[jj];
    float t8[8];
#pragma unroll
    for (int l = 0; l < 8; l++) {
      float cm[4];
#pragma unroll
      for (int m = 0; m < 4; m++) {
        float c = __fmaf_rn(a[8 * m + l], b[8 * m + l], 0.0f);
#pragma unroll
        for (int i = 32; i < HD; i += 32) c = __fmaf_rn(a[i + 8 * m + l], b[i + 8 * m + l], c);
        cm[m] = c;
      }
      t8[l] = fadd(fadd(cm[0], cm[1]), fadd(cm[2], cm[3]));
    }
    float s = fadd(fadd(fadd(t8[0], t8[4]), fadd(t8[2], t8[6])), fadd(fadd(t8[1], t8[5]), fadd(t8[3], t8[7])));
    S[(size_t)j * nR + R] = fmul(s, scale);
  }
}

// Softmax of 32 score rows (ops.rs:112-128) per CTA of 1024 threads: the row maxima in parallel
// (order does not matter for a max), then in chunks of 256 positions e = exp(s - max) is written
// back in place and staged in shared memory, where lane r of warp 0 adds row r's values in
// position order (the reference's sequential sum). inv[R] = 1 / sum. Row lengths as kp_scores.
__global__ void __launch_bounds__(1024) kp_softmax_rows(float* S, int nR, int rep, int base, int t0, int nfix,
                                                        float* inv) {
  __shared__ float ch[256][33];
  __shared__ float mred[32][33];
  __shared__ float m_s[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = blockIdx.x * 32 + lane;
  const bool valid = R < nR;
  const int n = valid ? (nfix > 0 ? nfix : base + t0 + R / rep + 1) : 0;
  const int Rl = min(blockIdx.x * 32 + 31, nR - 1);
  const int nmax = nfix > 0 ? nfix : base + t0 + Rl / rep + 1;
  float m = -INFINITY;
  for (int j = warp; j < nmax; j += 32)
    if (j < n) {
      float v = S[(size_t)j * nR + R];
      if (v > m) m = v;
    }
  mred[warp][lane] = m;
  __syncthreads();
  if (warp == 0) {
    float mm = -INFINITY;
    for (int w = 0; w < 32; w++) mm = fmaxf(mm, mred[w][lane]);
    m_s[lane] = mm;
  }
  __syncthreads();
  const float mrow = m_s[lane];
  float sum = 0.0f;
  for (int j0 = 0; j0 < nmax; j0 += 256) {
    for (int jj = warp; jj < 256; jj += 32) {
      const int j = j0 + jj;
      float e = 0.0f;
      if (j < n) {
        e = exp_cr(__fsub_rn(S[(size_t)j * nR + R], mrow));
        S[(size_t)j * nR + R] = e;
      }
      ch[jj][lane] = e;
    }
    __syncthreads();
    if (warp == 0) {  // adding the zeros past a row's end leaves its sum unchanged (sum >= +0)
#pragma unroll 8
      for (int jj = 0; jj < 256; jj++) sum = fadd(sum, ch[jj][lane]);
    }
    __syncthreads();
  }
  if (warp == 0 && valid) inv[R] = __fdiv_rn(1.0f, sum);
}

// O[t][h][dd] = sum_j (e_j * inv) * v_j[dd], sequential in j (model.rs:426-432; 573-584 for a
// diffusion block, whose prefix-then-block order is position order). Tile: 32 R x HD.
template <int HD>
__global__ void __launch_bounds__(256) kp_pv(const float* S, const float* inv, int nR, int rep, int base, int t0,
                                             int nfix, int kvh, const int32_t* bt, const float* v_pool,
                                             long long page_stride, float* o, int qd) {
  constexpr int PD = HD / 32;  // dims per thread (threads: 8 R-groups x 32 dims)
  __shared__ float ps[32][33];
  __shared__ float vs[32][HD];
  const int R0 = blockIdx.x * 32;
  const int rg = threadIdx.x >> 5, dl = threadIdx.x & 31;  // rows rg*4..rg*4+3, dims dl + 32*k
  float acc[4][PD];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int k = 0; k < PD; k++) acc[i][k] = 0.0f;
  int lim[4];
  float iv[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int R = R0 + rg * 4 + i;
    lim[i] = R < nR ? (nfix > 0 ? nfix : base + t0 + R / rep + 1) : 0;
    iv[i] = R < nR ? inv[R] : 0.0f;
  }
  int Rlast = min(R0 + 31, nR - 1);
  const int nmax = nfix > 0 ? nfix : base + t0 + Rlast / rep + 1;
  for (int j0 = 0; j0 < nmax; j0 += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * 32; i += 256) {
      int jj = i >> 5, rr = i & 31;
      int R = R0 + rr, j = j0 + jj;
      ps[rr][jj] = (R < nR && j < nmax) ? S[(size_t)j * nR + R] : 0.0f;
    }
    for (int i = threadIdx.x; i < 32 * HD; i += 256) {
      int jj = i / HD, dd = i - jj * HD;
      int j = j0 + jj;
      vs[jj][dd] = j < nmax ? v_pool[(long long)bt[j / PAGE] * page_stride + ((long long)kvh * PAGE + (j % PAGE)) * HD + dd]
                            : 0.0f;
    }
    __syncthreads();
    const int jn = min(32, nmax - j0);
    for (int jj = 0; jj < jn; jj++) {
      const int j = j0 + jj;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        if (j < lim[i]) {
          float p = fmul(ps[rg * 4 + i][jj], iv[i]);
#pragma unroll
          for (int k = 0; k < PD; k++) acc[i][k] = fadd(acc[i][k], fmul(p, vs[jj][dl + 32 * k]));
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    int R = R0 + rg * 4 + i;
    if (R >= nR) continue;
    int tl = R / rep, hr = R - tl * rep;
    float* dst = o + (size_t)(t0 + tl) * qd + (size_t)(kvh * rep + hr) * HD;
#pragma unroll
    for (int k = 0; k < PD; k++) dst[dl + 32 * k] = acc[i][k];
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
                         float* inv, float* o, cudaStream_t st) {
  const int rep = nh / nkv;
  const int nR = tq * rep;
  const int nmax = nfix > 0 ? nfix : base + t0 + tq;
  for (int g = 0; g < nkv; g++) {
    dim3 gs((nR + 31) / 32, (nmax + 31) / 32);
    if (hd == 128)
      kp_scores<128><<<gs, 256, 0, st>>>(q, qd, t0, tq, base, rep, g, bt, k_pool, page_stride, S, nR, nfix);
    else kp_scores<64><<<gs, 256, 0, st>>>(q, qd, t0, tq, base, rep, g, bt, k_pool, page_stride, S, nR, nfix);
    kp_softmax_rows<<<(nR + 31) / 32, 1024, 0, st>>>(S, nR, rep, base, t0, nfix, inv);
    dim3 gp((nR + 31) / 32);
    if (hd == 128)
      kp_pv<128><<<gp, 256, 0, st>>>(S, inv, nR, rep, base, t0, nfix, g, bt, v_pool, page_stride, o, qd);
    else kp_pv<64><<<gp, 256, 0, st>>>(S, inv, nR, rep, base, t0, nfix, g, bt, v_pool, page_stride, o, qd);
  }
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
