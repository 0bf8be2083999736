// Tensor-core (tcgen05, kind::i8) Q8 matvec for steps with many tokens.
//
// The reference dot (quant.rs:44-67) gives SIMD lane l (0..7) of block b (32 int8) the 4-element
// integer partial p[b][l] = sum_j w[32b + 4l + j] * a[32b + 4l + j], and accumulates
// acc_l = fma(sw[b] * dx[b], float(p[b][l]), acc_l) over the blocks in order, then sums the eight
// lanes in a fixed tree. The partials are exact integers, so a tensor core can produce them; the
// f32 chains stay on the CUDA cores in the reference order, so the result is bit-identical to the
// dp4a kernels'.
//
// Operands, per 128-byte lane chunk c of a row (blocks 4c..4c+3, lane l's 16 bytes at l*16, block
// q = b % 4's 4 bytes at l*16 + q*4; the packed layout of hg_device.cuh):
//   A = 128 weight rows x 128 bytes, copied verbatim into a 128-byte-swizzled K-major tile.
//   One MMA per lane pair lp (lanes 2lp, 2lp+1) with K = 32 bytes = A's bytes lp*32..lp*32+31.
//   B = the step's activations expanded so that output column n = (token t, block q, lane li)
//   keeps only the 4 bytes of lane 2lp+li in block q: B[n][k] = a[lp*32 + k] if k / 16 == li and
//   (k % 16) / 4 == q, else 0 (8 columns per token; the zero bytes are written once).
//   D[m][n] = p[b = 4c + q][l = 2lp + li] of row m and token t, an int32 in tensor memory.
// A CTA covers 128 rows x TC_TOK tokens; per chunk one thread issues the 4 MMAs (4 x 64 columns of
// tensor memory) and commits them to an mbarrier; the epilogue warps read the partials back
// (tcgen05.ld) and run the chains. Each CTA holds 256 tensor-memory columns, so two CTAs share an
// SM and one's MMAs overlap the other's epilogue; the weight chunks stream through a cp.async ring.
//
// Safety: every wait on an mbarrier is bounded (TC_SPIN_LIMIT polls); on expiry the CTA records
// HG_ERR_TIMEOUT in the step's error word, skips the remaining work, and still frees its tensor
// memory. No TMA and no multicast are used; all copies read this GPU's own memory.
#include <algorithm>
#include <cstdint>

#include "hg_launch.h"

namespace hg {

constexpr int TC_TOK = 8;             // tokens per CTA (N = 8 tokens x 8 columns per MMA)
constexpr int TC_N = TC_TOK * 8;      // MMA N
constexpr int TC_M = 128;             // rows per CTA (MMA M)
constexpr int TC_COLS = 4 * TC_N;     // tensor-memory columns per CTA: one chunk's 4 lane-pair MMAs
constexpr int TC_THREADS = 256;       // 8 warps: TMEM lane quadrant w % 4, token half w / 4
constexpr int TC_WSLOTS = 4;          // weight-chunk ring (16 KB each)
constexpr int TC_WAHEAD = 2;          // weight chunks in flight ahead of the MMAs
constexpr int TC_WCHUNK = TC_M * 128; // bytes per weight chunk
constexpr int TC_BCHUNK = 4 * TC_TOK * 256;  // bytes per expanded activation chunk (4 lane pairs)
constexpr long long TC_SPIN_LIMIT = 1ll << 26;
constexpr size_t TC_SMEM = 1024 + (size_t)TC_WSLOTS * TC_WCHUNK + 2 * TC_BCHUNK;  // + alignment slack

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// 64-bit shared-memory matrix descriptor (sm_100): start address, leading / stride byte offsets
// (all >> 4), descriptor version 1, layout (0 = no swizzle, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((addr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor of kind::i8: D s32, A and B signed 8-bit, both K-major, N and M.
constexpr uint32_t tc_idesc(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Wait for the phase with the given parity to complete; false if the bounded wait ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (long long i = 0; i < TC_SPIN_LIMIT; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void cp_async16_tc(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit_tc() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait_tc() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 32 consecutive tensor-memory columns of this warp's 32 lanes (one 32-bit value per column).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

enum { TC_EPI_STORE = 0, TC_EPI_RESID = 1, TC_EPI_LMHEAD = 2 };

// Rows r0..r0+127 of W against tokens t0..t0+TC_TOK-1 (aq/as: the step's quantized activations,
// row stride cols / ss). grid = (row tiles, token tiles).
template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 2) k_mv_tc(Dims D, DecodeBufs B, Q8M W, const int8_t* __restrict__ aq,
                                                         const float* __restrict__ as, float* out, int ostride) {
  extern __shared__ __align__(16) unsigned char tc_raw[];
  // 1024-byte aligned tiles (the 128-byte swizzle pattern repeats every 1024 bytes)
  unsigned char* base = tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023);
  unsigned char* wring = base;                                  // [TC_WSLOTS][128 rows][128 B], swizzled
  unsigned char* bbuf = base + (size_t)TC_WSLOTS * TC_WCHUNK;   // [2][4 lp][TC_TOK][2 kc][8 rows][16 B]
  __shared__ uint64_t mma_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int fail_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * TC_M, t0 = blockIdx.y * TC_TOK;
  const int cols = W.cols, nch = cols >> 7, ss = W.ss;
  const int ntok = min(TC_TOK, B.T - t0);

  // ---- set-up: tensor memory, the MMA barrier, zeroed activation expansions ----
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(&mma_bar, 1);
    fail_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < 2 * TC_BCHUNK / 16; i += TC_THREADS) reinterpret_cast<int4*>(bbuf)[i] = make_int4(0, 0, 0, 0);

  // weight chunk c into ring slot c % TC_WSLOTS: 16-byte piece j of row m at j ^ (m % 8)
  auto issue_w = [&](int c) {
    if (c < nch) {
      unsigned char* dst = wring + (size_t)(c % TC_WSLOTS) * TC_WCHUNK;
#pragma unroll
      for (int k = 0; k < TC_WCHUNK / 16 / TC_THREADS; k++) {
        const int i = tid + k * TC_THREADS, m = i >> 3, j = i & 7;
        const int r = min(r0 + m, W.rows - 1);  // rows past the end read a valid row, unused
        cp_async16_tc(dst + m * 128 + ((j ^ (m & 7)) << 4), W.qs + (long long)r * cols + c * 128 + j * 16);
      }
    }
    cp_commit_tc();
  };
#pragma unroll
  for (int c = 0; c < TC_WAHEAD; c++) issue_w(c);  // weights: older than the previous kernel
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_s;
  pdl_wait();
  pdl_trigger();

  // expanded activations of chunk c into buffer c % 2: one 4-byte word per thread
  // (lane pair lp, token tt, lane li, block q): token tt's bytes lp*32 + li*16 + q*4 .. + 3
  auto stage_b = [&](int c) {
    const int q = tid & 3, li = (tid >> 2) & 1, tt = (tid >> 3) & (TC_TOK - 1), lp = tid >> 6;
    int v = 0;
    if (tt < ntok) v = *reinterpret_cast<const int*>(aq + (size_t)(t0 + tt) * cols + c * 128 + lp * 32 + li * 16 + q * 4);
    unsigned char* dst = bbuf + (size_t)(c & 1) * TC_BCHUNK + lp * (TC_TOK * 256) + tt * 256 + li * 128 +
                         (2 * q + li) * 16 + q * 4;
    *reinterpret_cast<int*>(dst) = v;
  };
  static_assert(TC_THREADS == 4 * TC_TOK * 8, "one expansion word per thread per chunk");

  // epilogue thread: row r0 + 32 (warp % 4) + lane, tokens t0 + 4 (warp / 4) + 0..3
  const int quad = warp & 3, half = warp >> 2;
  const int row = r0 + quad * 32 + lane;
  const bool row_ok = row < W.rows;
  const float* wsc = W.sc + (long long)(row_ok ? row : 0) * ss;
  float acc[4][8];
#pragma unroll
  for (int tt = 0; tt < 4; tt++)
#pragma unroll
    for (int l = 0; l < 8; l++) acc[tt][l] = 0.0f;

  constexpr uint32_t IDESC = tc_idesc(TC_M, TC_N);
  uint32_t phase = 0;
  int fail = 0;
  stage_b(0);
  for (int c = 0; c < nch; c++) {
    issue_w(c + TC_WAHEAD);
    cp_wait_tc<TC_WAHEAD>();  // this thread's pieces of weight chunk c have landed
    fence_async_smem();       // generic-proxy writes (cp.async, the expansion) -> tensor-core reads
    tc_fence_before();
    __syncthreads();          // chunk c staged by everyone; everyone done reading chunk c-1's partials
    tc_fence_after();
    if (tid == 0 && !fail) {
      const uint32_t wa = smem_u32(wring + (size_t)(c % TC_WSLOTS) * TC_WCHUNK);
      const uint32_t ba = smem_u32(bbuf + (size_t)(c & 1) * TC_BCHUNK);
#pragma unroll
      for (int lp = 0; lp < 4; lp++) {
        const uint64_t ad = tc_desc(wa + lp * 32, 16, 1024, 2);                // 128-byte swizzled, K-major
        const uint64_t bd = tc_desc(ba + lp * (TC_TOK * 256), 128, 256, 0);    // no swizzle, K-major
        const uint32_t dt = tbase + lp * TC_N;
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(dt),
            "l"(ad), "l"(bd), "r"(IDESC), "r"(0));
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&mma_bar))
                   : "memory");
    }
    if (c + 1 < nch) stage_b(c + 1);  // the other buffer: last read by chunk c-1's MMAs (complete)
    // per-(token, block) scales of this chunk: sw[row][4c + q] * dx[t][4c + q]
    const float4 s4 = *reinterpret_cast<const float4*>(wsc + c * 4);
    float sc[4][4];
#pragma unroll
    for (int tt = 0; tt < 4; tt++) {
      const int t = min(t0 + half * 4 + tt, B.T - 1);
      const float4 d4 = *reinterpret_cast<const float4*>(as + (size_t)t * ss + c * 4);
      sc[tt][0] = fmul(s4.x, d4.x);
      sc[tt][1] = fmul(s4.y, d4.y);
      sc[tt][2] = fmul(s4.z, d4.z);
      sc[tt][3] = fmul(s4.w, d4.w);
    }
    if (!fail && !mbar_wait(&mma_bar, phase)) fail = 1;
    fail = __any_sync(0xffffffffu, fail);  // warp-uniform: tcgen05.ld below is a .sync.aligned warp op
    phase ^= 1;
    tc_fence_after();
    if (!fail) {
#pragma unroll
      for (int lp = 0; lp < 4; lp++) {
        uint32_t v[32];
        tmem_ld32(tbase + ((uint32_t)(quad * 32) << 16) + lp * TC_N + half * 32, v);
        tmem_ld_wait();
        // column tt*8 + 2q + li of this half: token tt, block 4c + q, lane 2lp + li
#pragma unroll
        for (int tt = 0; tt < 4; tt++)
#pragma unroll
          for (int q = 0; q < 4; q++)
#pragma unroll
            for (int li = 0; li < 2; li++) {
              const int l = 2 * lp + li;
              acc[tt][l] = __fmaf_rn(sc[tt][q], (float)(int)v[tt * 8 + 2 * q + li], acc[tt][l]);
            }
      }
    }
  }
  cp_wait_tc<0>();
  if (fail) fail_s = 1;  // every writer stores 1
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_COLS));
  if (fail_s) {
    if (tid == 0 && B.err) atomicExch(B.err, HG_ERR_TIMEOUT);
    return;
  }

  // ---- output: the lane tree ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)) (quant.rs:61-65) ----
#pragma unroll
  for (int tt = 0; tt < 4; tt++) {
    const int t = t0 + half * 4 + tt;
    const float* a = acc[tt];
    const float y = fadd(fadd(fadd(a[0], a[4]), fadd(a[2], a[6])), fadd(fadd(a[1], a[5]), fadd(a[3], a[7])));
    const bool ok = row_ok && t < B.T;
    if (EPI == TC_EPI_STORE) {
      if (ok) out[(size_t)t * ostride + row] = y;
    } else if (EPI == TC_EPI_RESID) {
      if (ok) {
        float* xp = B.x + (size_t)t * D.d + row;
        *xp = fadd(*xp, y);
      }
    } else {
      if (ok && out) out[(size_t)t * ostride + row] = y;
      unsigned long long key = (ok && row < D.valid) ? argmax_key(y, (uint32_t)row) : 0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
      if (lane == 0 && t < B.T && key) atomicMax(&B.amax[t], key);
    }
  }
}

// ------------------------------------------------------------------------------------------
// Grouped tensor-core matvec for the FFN (model.rs:243-255, 295-324) of steps with many tokens.
//
// Groups: the shared expert or the dense FFN (group 0, every token) and the routed experts active
// in the step (one group each, its token list from the router). A CTA covers 128 rows of the
// group's matrix and strides over the group's 8-entry tiles. The MMAs and the f32 lane chains
// are those of k_mv_tc; rows whose width is not a multiple of 128 bytes end in 1-3 tail blocks
// (the packed layout keeps a tail block's 8 lanes of 4 bytes side by side), each one extra MMA with
// one column per (entry, lane).
//   GT_UP:   gate or up rows on the ffn-normed hidden state of each entry's token, stored per
//            (token, slot) for k_swiglu_quant.
//   GT_DOWN: down rows on each (token, slot)'s quantized SwiGLU activation, stored in y[t][slot].
// ------------------------------------------------------------------------------------------
enum { GT_UP = 0, GT_DOWN = 1 };

struct GrpTc {
  Q8M W;                   // routed-expert stack [ne][rows][cols]
  Q8M W0;                  // group 0's matrix (shared expert / dense FFN); qs == null: no group 0
  const int32_t* ecount;   // [ne + 2]: entries per expert, then the active-expert count
  const int32_t* active;   // [ne]
  const int32_t* elist;    // [ne][T]: t * 32 + slot
  int T, ne, nrouted, slot0;
  const int8_t* aq;        // inputs (lane-chunked rows of `cols` bytes)
  const float* as;         // their scales (rows of ss floats)
  int in_nslot;            // GT_UP: 0 (row = token); GT_DOWN: slots per token of the input rows
  float* out;              // out[(t * out_nslot + slot) * ostride + row]
  int out_nslot, ostride;
  int nz;                  // CTAs striding over a group's entry tiles
  int32_t* err;
};

constexpr int TC_TAIL_A = 3 * 4096;                 // tail A: up to 3 blocks x 128 rows x 32 B
constexpr int TC_TAIL_B = 3 * TC_TOK * 256;         // tail B: up to 3 blocks x 8 entries x 8 lanes x 32 B
constexpr size_t GT_SMEM = TC_SMEM + TC_TAIL_B;     // (tail A shares the weight ring's slot)

template <int MODE>
__global__ void __launch_bounds__(TC_THREADS, 2) k_grp_tc(GrpTc G) {
  extern __shared__ __align__(16) unsigned char tc_raw[];
  unsigned char* base = tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023);
  unsigned char* wring = base;
  unsigned char* bbuf = base + (size_t)TC_WSLOTS * TC_WCHUNK;
  unsigned char* btail = bbuf + 2 * TC_BCHUNK;  // [3 tail blocks][8 entries][2 kc][8 lanes][16 B]
  __shared__ uint64_t mma_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int fail_s;
  __shared__ int code_s[TC_TOK];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool has0 = G.W0.qs != nullptr;
  const bool g0 = has0 && blockIdx.y == 0;
  const int ri = (int)blockIdx.y - (has0 ? 1 : 0);  // routed slot in the active list
  pdl_wait();  // the expert lists come from the router (or, for GT_DOWN, the activations from before)
  pdl_trigger();
  int expert = 0, count;
  if (g0) {
    count = G.T;
  } else {
    if (ri >= G.ecount[G.ne]) return;
    expert = G.active[ri];
    count = G.ecount[expert];
  }
  const Q8M& Wm = g0 ? G.W0 : G.W;
  const int mi = g0 ? 0 : expert;
  const int r0 = blockIdx.x * TC_M;
  if (r0 >= Wm.rows) return;
  const int ntiles = (count + TC_TOK - 1) / TC_TOK;
  if ((int)blockIdx.z >= ntiles) return;
  const int cols = Wm.cols, nb = cols >> 5, nch = nb >> 2, ntail = nb & 3, ss = Wm.ss;
  const int nsteps = nch + (ntail ? 1 : 0);
  const int8_t* wq = Wm.qs + (long long)mi * Wm.qs_mstride;
  const float* wsc_m = Wm.sc + (long long)mi * Wm.sc_mstride;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(&mma_bar, 1);
    fail_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < (2 * TC_BCHUNK + TC_TAIL_B) / 16; i += TC_THREADS)
    reinterpret_cast<int4*>(bbuf)[i] = make_int4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_s;

  const int quad = warp & 3, half = warp >> 2;
  const int row = r0 + quad * 32 + lane;
  const bool row_ok = row < Wm.rows;
  const float* wsc = wsc_m + (long long)(row_ok ? row : 0) * ss;
  constexpr uint32_t IDESC = tc_idesc(TC_M, TC_N);
  uint32_t phase = 0;
  int fail = 0;

  for (int tile = blockIdx.z; tile < ntiles; tile += G.nz) {
    const int e0 = tile * TC_TOK, ntok = min(TC_TOK, count - e0);
    __syncthreads();  // the previous tile is done with code_s
    if (tid < TC_TOK)
      code_s[tid] = tid < ntok ? (g0 ? (e0 + tid) * 32 + G.slot0 : G.elist[(size_t)expert * G.T + e0 + tid]) : -1;
    __syncthreads();
    // input row of entry tt (a valid row for padding entries)
    auto in_row = [&](int tt) {
      const int code = code_s[tt] < 0 ? code_s[0] : code_s[tt];
      const int t = code >> 5, sl = code & 31;
      return MODE == GT_UP ? t : t * G.in_nslot + sl;
    };
    auto issue_w = [&](int s) {
      if (s < nch) {
        unsigned char* dst = wring + (size_t)(s % TC_WSLOTS) * TC_WCHUNK;
#pragma unroll
        for (int k = 0; k < TC_WCHUNK / 16 / TC_THREADS; k++) {
          const int i = tid + k * TC_THREADS, m = i >> 3, j = i & 7;
          const int r = min(r0 + m, Wm.rows - 1);
          cp_async16_tc(dst + m * 128 + ((j ^ (m & 7)) << 4), wq + (long long)r * cols + s * 128 + j * 16);
        }
      } else if (s == nch && ntail) {  // tail blocks, no swizzle: 8-row x 16-byte core matrices
        unsigned char* dst = wring + (size_t)(s % TC_WSLOTS) * TC_WCHUNK;
        for (int i = tid; i < TC_M * ntail * 2; i += TC_THREADS) {
          const int m = i / (ntail * 2), rem = i - m * (ntail * 2), tb = rem >> 1, kc = rem & 1;
          const int r = min(r0 + m, Wm.rows - 1);
          cp_async16_tc(dst + tb * 4096 + (m >> 3) * 256 + kc * 128 + (m & 7) * 16,
                        wq + (long long)r * cols + nch * 128 + tb * 32 + kc * 16);
        }
      }
      cp_commit_tc();
    };
    auto stage_b = [&](int s) {
      if (s < nch) {
        const int q = tid & 3, li = (tid >> 2) & 1, tt = (tid >> 3) & (TC_TOK - 1), lp = tid >> 6;
        int v = 0;
        if (tt < ntok) v = *reinterpret_cast<const int*>(G.aq + (size_t)in_row(tt) * cols + s * 128 + lp * 32 + li * 16 + q * 4);
        *reinterpret_cast<int*>(bbuf + (size_t)(s & 1) * TC_BCHUNK + lp * (TC_TOK * 256) + tt * 256 + li * 128 +
                                (2 * q + li) * 16 + q * 4) = v;
      } else if (tid < ntail * TC_TOK * 8) {  // tail block tb, entry tt, lane l: 4 bytes
        const int l = tid & 7, tt = (tid >> 3) & (TC_TOK - 1), tb = tid >> 6;
        int v = 0;
        if (tt < ntok) v = *reinterpret_cast<const int*>(G.aq + (size_t)in_row(tt) * cols + nch * 128 + tb * 32 + l * 4);
        *reinterpret_cast<int*>(btail + tb * (TC_TOK * 256) + tt * 256 + (l >> 2) * 128 + l * 16 + (l & 3) * 4) = v;
      }
    };
    float acc[4][8];
#pragma unroll
    for (int tt = 0; tt < 4; tt++)
#pragma unroll
      for (int l = 0; l < 8; l++) acc[tt][l] = 0.0f;
#pragma unroll
    for (int s = 0; s < TC_WAHEAD; s++) issue_w(s);
    stage_b(0);
    for (int s = 0; s < nsteps; s++) {
      issue_w(s + TC_WAHEAD);
      cp_wait_tc<TC_WAHEAD>();
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      const bool tail = s == nch;
      if (tid == 0 && !fail) {
        const uint32_t wa = smem_u32(wring + (size_t)(s % TC_WSLOTS) * TC_WCHUNK);
        if (!tail) {
          const uint32_t ba = smem_u32(bbuf + (size_t)(s & 1) * TC_BCHUNK);
#pragma unroll
          for (int lp = 0; lp < 4; lp++) {
            const uint64_t ad = tc_desc(wa + lp * 32, 16, 1024, 2);
            const uint64_t bd = tc_desc(ba + lp * (TC_TOK * 256), 128, 256, 0);
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tbase + lp * TC_N),
                "l"(ad), "l"(bd), "r"(IDESC), "r"(0));
          }
        } else {
          const uint32_t ba = smem_u32(btail);
          for (int tb = 0; tb < ntail; tb++) {
            const uint64_t ad = tc_desc(wa + tb * 4096, 128, 256, 0);
            const uint64_t bd = tc_desc(ba + tb * (TC_TOK * 256), 128, 256, 0);
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tbase + tb * TC_N),
                "l"(ad), "l"(bd), "r"(IDESC), "r"(0));
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&mma_bar))
                     : "memory");
      }
      if (s + 1 < nsteps) stage_b(s + 1);
      // per-(entry, block) scales sw[row][b] * dx[entry][b] of this step's blocks
      const int b0 = s * 4;
      const float4 s4 = *reinterpret_cast<const float4*>(wsc + b0);
      float sc[4][4];
#pragma unroll
      for (int tt = 0; tt < 4; tt++) {
        const float4 d4 = *reinterpret_cast<const float4*>(G.as + (size_t)in_row(half * 4 + tt) * ss + b0);
        sc[tt][0] = fmul(s4.x, d4.x);
        sc[tt][1] = fmul(s4.y, d4.y);
        sc[tt][2] = fmul(s4.z, d4.z);
        sc[tt][3] = fmul(s4.w, d4.w);
      }
      if (!fail && !mbar_wait(&mma_bar, phase)) fail = 1;
      fail = __any_sync(0xffffffffu, fail);
      phase ^= 1;
      tc_fence_after();
      if (!fail) {
        if (!tail) {
#pragma unroll
          for (int lp = 0; lp < 4; lp++) {
            uint32_t v[32];
            tmem_ld32(tbase + ((uint32_t)(quad * 32) << 16) + lp * TC_N + half * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int tt = 0; tt < 4; tt++)
#pragma unroll
              for (int q = 0; q < 4; q++)
#pragma unroll
                for (int li = 0; li < 2; li++) {
                  const int l = 2 * lp + li;
                  acc[tt][l] = __fmaf_rn(sc[tt][q], (float)(int)v[tt * 8 + 2 * q + li], acc[tt][l]);
                }
          }
        } else {
          for (int tb = 0; tb < ntail; tb++) {  // column tt * 8 + l: entry tt, lane l of block 4 nch + tb
            uint32_t v[32];
            tmem_ld32(tbase + ((uint32_t)(quad * 32) << 16) + tb * TC_N + half * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int tt = 0; tt < 4; tt++)
#pragma unroll
              for (int l = 0; l < 8; l++)
                acc[tt][l] = __fmaf_rn(tb == 0 ? sc[tt][0] : tb == 1 ? sc[tt][1] : sc[tt][2], (float)(int)v[tt * 8 + l],
                                       acc[tt][l]);
          }
        }
      }
    }
    cp_wait_tc<0>();
    // outputs of this tile: the lane tree (quant.rs:61-65)
    if (!fail) {
#pragma unroll
      for (int tt = 0; tt < 4; tt++) {
        const int e = half * 4 + tt;
        if (e >= ntok || !row_ok) continue;
        const float* a = acc[tt];
        const float y = fadd(fadd(fadd(a[0], a[4]), fadd(a[2], a[6])), fadd(fadd(a[1], a[5]), fadd(a[3], a[7])));
        const int code = code_s[e], t = code >> 5, sl = code & 31;
        G.out[((size_t)t * G.out_nslot + sl) * G.ostride + row] = y;
      }
    }
  }
  if (fail) fail_s = 1;
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_COLS));
  if (fail_s && tid == 0 && G.err) atomicExch(G.err, HG_ERR_TIMEOUT);
}

// act = silu(g) * u (model.rs:247-248, 304, 317; silu ops.rs:80-82) of every (token, slot) row,
// quantized per 32-block (quant.rs:112-123) into the lane-chunked layout the down projection reads.
// One warp per 32-block.
__global__ void __launch_bounds__(256) k_swiglu_quant(const float* __restrict__ g, const float* __restrict__ u,
                                                      long long nrows, int fd, int8_t* q, float* sq) {
  const int nb = fd >> 5, ssq = q8_ss(nb);
  const long long blk = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_wait();
  pdl_trigger();
  if (blk >= nrows * nb) return;
  const long long r = blk / nb;
  const int b = (int)(blk - r * nb), lane = threadIdx.x & 31;
  const size_t i = (size_t)r * fd + b * 32 + lane;
  const float a = fmul(silu_ref(g[i]), u[i]);
  float d;
  const int8_t qv = quant_lane(a, &d);
  q[(size_t)r * fd + q8_pos(b * 32 + lane, nb)] = qv;
  if (lane == 0) sq[(size_t)r * ssq + b] = d;
}

static bool g_tc_ready[64];

template <int EPI>
static cudaError_t prepare_tc_t() {
  return cudaFuncSetAttribute((const void*)k_mv_tc<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
}
template <int MODE>
static cudaError_t prepare_grp_t() {
  return cudaFuncSetAttribute((const void*)k_grp_tc<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GT_SMEM);
}

cudaError_t prepare_tc() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = prepare_tc_t<TC_EPI_STORE>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<TC_EPI_RESID>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<TC_EPI_LMHEAD>()) != cudaSuccess) return e;
  if ((e = prepare_grp_t<GT_UP>()) != cudaSuccess) return e;
  if ((e = prepare_grp_t<GT_DOWN>()) != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) g_tc_ready[dev] = true;
  return cudaSuccess;
}

bool tc_usable(const Q8M& W, int T) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_tc_ready[dev]) return false;
  return T >= TC_MIN_T && W.cols % 128 == 0 && W.cols >= 128 && W.ss % 4 == 0;
}

void launch_mv_tc(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* out,
                  int ostride, int epi, cudaStream_t st) {
  const dim3 grid((W.rows + TC_M - 1) / TC_M, (B.T + TC_TOK - 1) / TC_TOK);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = B.T <= 64 ? 1 : 0;
  if (epi == TC_EPI_STORE) cudaLaunchKernelEx(&cfg, k_mv_tc<TC_EPI_STORE>, D, B, W, aq, as, out, ostride);
  else if (epi == TC_EPI_RESID) cudaLaunchKernelEx(&cfg, k_mv_tc<TC_EPI_RESID>, D, B, W, aq, as, out, ostride);
  else cudaLaunchKernelEx(&cfg, k_mv_tc<TC_EPI_LMHEAD>, D, B, W, aq, as, out, ostride);
}

bool ffn_tc_usable(const Dims& D, const DecodeBufs& B, const LayerDev& L) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_tc_ready[dev]) return false;
  return B.T >= TC_MIN_T && B.ubuf && B.qact && B.sact && D.d % 128 == 0 && (L.moe ? D.f : D.df) % 32 == 0;
}

// The FFN of one layer for a step of many tokens: gate and up on the tensor cores, SwiGLU and the
// quantization of the activations, down on the tensor cores. Same results as launch_ffn.
void launch_ffn_tc(const Dims& D, const DecodeBufs& B, const LayerDev& L, cudaStream_t st) {
  const bool moe = L.moe != 0;
  const int fd = moe ? D.f : D.df, bslot = moe ? D.k + 1 : 1;
  const int nrouted = moe ? std::min(D.ne, B.T * D.k) : 0;
  const bool shared = moe ? D.nsh > 0 : true;
  GrpTc G{};
  G.T = B.T;
  G.ne = D.ne;
  G.nrouted = nrouted;
  G.ecount = B.ecount;
  G.active = B.active;
  G.elist = B.elist;
  G.err = B.err;
  G.slot0 = moe ? D.k : 0;
  G.nz = std::min((B.T + TC_TOK - 1) / TC_TOK, 16);
  const int groups = (shared ? 1 : 0) + nrouted;
  if (groups == 0) return;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = GT_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = B.T <= 64 ? 1 : 0;
  auto up = [&](const Q8M& routed, const Q8M& grp0, float* out) {
    G.W = moe ? routed : Q8M{};
    G.W0 = shared ? grp0 : Q8M{};
    G.aq = B.qh;
    G.as = B.sh;
    G.in_nslot = 0;
    G.out = out;
    G.out_nslot = bslot;
    G.ostride = fd;
    cfg.gridDim = dim3((fd + TC_M - 1) / TC_M, groups, G.nz);
    cudaLaunchKernelEx(&cfg, k_grp_tc<GT_UP>, G);
  };
  up(L.gate, moe ? L.sgate : L.gate, B.act);
  up(L.up, moe ? L.sup : L.up, B.ubuf);
  const long long nrows = (long long)B.T * bslot, nblk = nrows * (fd >> 5);
  {
    cudaLaunchConfig_t c2 = cfg;
    c2.gridDim = dim3((unsigned)((nblk + 7) / 8));
    c2.blockDim = dim3(256);
    c2.dynamicSmemBytes = 0;
    cudaLaunchKernelEx(&c2, k_swiglu_quant, (const float*)B.act, (const float*)B.ubuf, nrows, fd, B.qact, B.sact);
  }
  G.W = moe ? L.down : Q8M{};
  G.W0 = shared ? (moe ? L.sdown : L.down) : Q8M{};
  G.aq = B.qact;
  G.as = B.sact;
  G.in_nslot = bslot;
  G.out = B.y;
  G.out_nslot = D.k + 1;
  G.ostride = D.d;
  cfg.gridDim = dim3((D.d + TC_M - 1) / TC_M, groups, G.nz);
  cudaLaunchKernelEx(&cfg, k_grp_tc<GT_DOWN>, G);
}

}  // namespace hg
