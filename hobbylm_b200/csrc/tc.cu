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
//   B = the step's activations expanded so that output column n = (entry e, block q, lane li)
//   keeps only the 4 bytes of lane 2lp+li in block q: B[n][k] = a[lp*32 + k] if k / 16 == li and
//   (k % 16) / 4 == q, else 0 (8 columns per entry; the zero bytes are written once).
//   D[m][n] = p[b = 4c + q][l = 2lp + li] of row m and entry e, an int32 in tensor memory.
// Rows whose width is not a multiple of 128 bytes end in 1-3 tail blocks (the packed layout keeps
// a tail block's 8 lanes of 4 bytes side by side): one MMA per tail block with one column per
// (entry, lane).
//
// Pipeline: one CTA per SM (512 threads) owns all 512 tensor-memory columns as two 256-column
// buffers. A CTA walks a stream of steps (its entry tiles x the chunks of a row); in step g one
// thread issues the MMAs of step g + 1 into the other buffer while all 16 warps run the f32
// chains of step g out of tensor memory. Weight chunks stream through a 6-slot cp.async ring four
// steps ahead; the activation words and the scales of the next steps are loaded into registers a
// step ahead, so no global-memory latency sits between two steps.
//
// Safety: every wait on an mbarrier is bounded (TC_SPIN_LIMIT polls); on expiry the CTA records
// HG_ERR_TIMEOUT in the step's error word, stops issuing, waits (bounded) for its last MMAs and
// copies, and still frees its tensor memory. No TMA and no multicast are used; all copies read
// this GPU's own memory.
#include <algorithm>
#include <cstdint>

#include "hg_launch.h"

namespace hg {

constexpr int TC_TOK = 8;             // entries per tile (N = 8 entries x 8 columns per MMA)
constexpr int TC_N = TC_TOK * 8;      // MMA N
constexpr int TC_M = 128;             // rows per CTA (MMA M)
constexpr int TC_BUFCOLS = 4 * TC_N;  // tensor-memory columns of one step: 4 lane-pair MMAs
constexpr int TC_COLS = 2 * TC_BUFCOLS;  // two step buffers: all 512 columns of the SM
constexpr int TC_THREADS = 512;       // 16 warps: TMEM lane quadrant w % 4, entry pair w / 4
constexpr int TC_WSLOTS = 6;          // weight-chunk ring (16 KB each)
constexpr int TC_WAHEAD = 4;          // weight chunks in flight ahead of the step being reduced
constexpr int TC_WCHUNK = TC_M * 128; // bytes per weight chunk
constexpr int TC_BCHUNK = 4 * TC_TOK * 256;  // bytes per expanded activation chunk (4 lane pairs)
constexpr int TC_TAIL_B = 3 * TC_TOK * 256;  // expanded tail blocks: up to 3 x 8 entries x 8 lanes x 32 B
constexpr long long TC_SPIN_LIMIT = 1ll << 26;
// + alignment slack, the weight ring (a tail step's A tiles use a ring slot), two expanded
// activation chunks and two expanded tail chunks
constexpr size_t TC_SMEM = 1024 + (size_t)TC_WSLOTS * TC_WCHUNK + 2 * TC_BCHUNK + 2 * TC_TAIL_B;
static_assert(TC_COLS == 512, "tensor memory holds 512 columns per SM");

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

// 16 consecutive tensor-memory columns of this warp's 32 lanes (one 32-bit value per column).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same 32-bit value into 16 consecutive columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_st16_same(uint32_t taddr, uint32_t x) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr),
      "r"(x)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// The accumulators start at TC_BIAS, the bit pattern of 1.5 * 2^23: the MMAs add the exact partial
// p (|p| <= 4 * 128 * 128 < 2^22) in int32, so the result read back is the float 1.5 * 2^23 + p
// (every integer in [2^23, 2^24) is representable), and subtracting 1.5 * 2^23 gives float(p)
// exactly -- one full-rate add instead of an int-to-float conversion.
constexpr uint32_t TC_BIAS = 0x4B400000u;
constexpr float TC_BIAS_F = 12582912.0f;
__device__ __forceinline__ float tc_partial(uint32_t v) { return __fsub_rn(__uint_as_float(v), TC_BIAS_F); }

// Output of a finished row tile x entry tile.
//   TC_OUT_STORE:  out[(t * out_nslot + slot) * ostride + row] = y
//   TC_OUT_RESID:  x[t * d + row] += y (the residual add of the attention / dense output)
//   TC_OUT_LMHEAD: out[t * ostride + row] = y when out is set; argmax key of rows < valid into amax[t]
enum { TC_OUT_STORE = 0, TC_OUT_RESID = 1, TC_OUT_LMHEAD = 2 };

// One launch covers the rows of group 0's matrix (every token, or the shared expert / dense FFN)
// and, for the FFN, of the routed experts active in the step (one group each, its entries from
// the router). Entries are codes t * 32 + slot; a unit is one 128-row tile x 8 consecutive entries
// of a group, ordered group by group, row tile by row tile, entry tile fastest. Every unit has the
// same number of steps, so CTA c of the 1-D grid takes the contiguous run of units
// [c * U / grid, (c + 1) * U / grid) and the CTAs finish together.
struct TcArgs {
  Q8M W;                   // routed-expert stack [ne][rows][cols]
  Q8M W0;                  // group 0's matrix (same shape); qs == null: no group 0
  const int32_t* ecount;   // [ne + 2]: entries per expert, then the active-expert count
  const int32_t* active;   // [ne]
  const int32_t* elist;    // [ne][T]: t * 32 + slot
  int T, ne, nrouted, slot0;  // nrouted: routed group slots; group 0's entries are t * 32 + slot0
  const int8_t* aq;        // inputs (lane-chunked rows of `cols` bytes)
  const float* as;         // their scales (rows of ss floats)
  int in_nslot;            // 0: input row = t; else input row = t * in_nslot + slot
  float* out;
  int out_nslot, ostride;
  float* x;                // TC_OUT_RESID: the residual stream [T][d]
  int d, valid;            // TC_OUT_LMHEAD: rows below `valid` compete for the argmax
  unsigned long long* amax;
  int32_t* err;
};

constexpr int TC_MAX_GROUPS = 72;   // group 0 + up to 71 routed experts
constexpr int TC_MAX_UNITS = 128;   // units per CTA (the host sizes the grid so that runs fit)

template <int OUT>
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc(TcArgs G) {
  extern __shared__ __align__(16) unsigned char tc_raw[];
  // 1024-byte aligned tiles (the 128-byte swizzle pattern repeats every 1024 bytes)
  unsigned char* base = tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023);
  unsigned char* wring = base;                                 // [TC_WSLOTS][128 rows][128 B], swizzled
  unsigned char* bbuf = base + (size_t)TC_WSLOTS * TC_WCHUNK;  // [2][4 lp][TC_TOK][2 kc][8 rows][16 B]
  unsigned char* btail = bbuf + 2 * TC_BCHUNK;                 // [2][3 tail blocks][TC_TOK][2 kc][8][16 B]
  __shared__ uint64_t mma_bar[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ int fail_s, run_s[2];
  __shared__ int g_start[TC_MAX_GROUPS + 1], g_tiles[TC_MAX_GROUPS], g_count[TC_MAX_GROUPS], g_exp[TC_MAX_GROUPS];
  __shared__ int u_gi[TC_MAX_UNITS], u_r0[TC_MAX_UNITS];
  __shared__ int u_code[TC_MAX_UNITS][TC_TOK];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool has0 = G.W0.qs != nullptr;
  const Q8M& W1 = has0 ? G.W0 : G.W;  // shape of every group's matrix
  const int rows = W1.rows, cols = W1.cols, nb = cols >> 5, nch = nb >> 2, ntail = nb & 3, ss = W1.ss;
  const int nst = nch + (ntail ? 1 : 0);
  const int rt = (rows + TC_M - 1) / TC_M;
  const int ng = (has0 ? 1 : 0) + G.nrouted;
  if (G.nrouted > 0) pdl_wait();  // the expert lists come from the router

  // ---- the groups, this CTA's run of units, and the units' entry codes ----
  if (warp == 0) {
    const int nact = G.nrouted > 0 ? G.ecount[G.ne] : 0;
    for (int gi = lane; gi < ng; gi += 32) {
      int cnt = G.T, ex = 0;
      if (!(has0 && gi == 0)) {
        const int ri = gi - (has0 ? 1 : 0);
        ex = ri < nact ? G.active[ri] : 0;
        cnt = ri < nact ? G.ecount[ex] : 0;
      }
      g_count[gi] = cnt;
      g_exp[gi] = ex;
      g_tiles[gi] = (cnt + TC_TOK - 1) / TC_TOK;
    }
    __syncwarp();
    if (lane == 0) {
      int acc = 0;
      for (int gi = 0; gi < ng; gi++) {
        g_start[gi] = acc;
        acc += rt * g_tiles[gi];
      }
      g_start[ng] = acc;
      const long long U = acc, nc = gridDim.x;
      const int ub = (int)(U * blockIdx.x / nc), ue = (int)(U * (blockIdx.x + 1) / nc);
      run_s[0] = ub;
      run_s[1] = min(ue - ub, TC_MAX_UNITS);
      if (ue - ub > TC_MAX_UNITS && G.err) atomicExch(G.err, HG_ERR_INVALID);  // host sizing bug: loud
    }
  }
  __syncthreads();
  const int ub = run_s[0], nun = run_s[1];
  if (nun <= 0) return;
  for (int i = tid; i < nun * TC_TOK; i += TC_THREADS) {
    const int ui = i / TC_TOK, e = i - ui * TC_TOK, u = ub + ui;
    int lo = 0, hi = ng - 1;  // the group gi with g_start[gi] <= u < g_start[gi + 1]
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (g_start[mid] <= u) lo = mid;
      else hi = mid - 1;
    }
    const int gi = lo, tl = g_tiles[gi], ul = u - g_start[gi], rtile = ul / tl, tile = ul - rtile * tl;
    const int idx = tile * TC_TOK + e;
    int code = -1;
    if (idx < g_count[gi]) code = (has0 && gi == 0) ? idx * 32 + G.slot0 : G.elist[(size_t)g_exp[gi] * G.T + idx];
    u_code[ui][e] = code;
    if (e == 0) {
      u_gi[ui] = gi;
      u_r0[ui] = rtile * TC_M;
    }
  }
  const int S = nun * nst;

  // ---- set-up: tensor memory, the MMA barriers, zeroed activation expansions ----
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(&mma_bar[0], 1);
    mbar_init(&mma_bar[1], 1);
    fail_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < (2 * TC_BCHUNK + 2 * TC_TAIL_B) / 16; i += TC_THREADS)
    reinterpret_cast<int4*>(bbuf)[i] = make_int4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_s;

  // matrix of unit ui: its quantized rows and scales
  auto unit_q = [&](int ui) -> const int8_t* {
    const int gi = u_gi[ui];
    return (has0 && gi == 0) ? G.W0.qs : G.W.qs + (long long)g_exp[gi] * G.W.qs_mstride;
  };
  auto unit_s = [&](int ui) -> const float* {
    const int gi = u_gi[ui];
    return (has0 && gi == 0) ? G.W0.sc : G.W.sc + (long long)g_exp[gi] * G.W.sc_mstride;
  };
  auto in_row = [&](int code) -> int {
    return G.in_nslot ? (code >> 5) * G.in_nslot + (code & 31) : (code >> 5);
  };

  // Steps g = 0..S-1: step g is chunk s = g % nst of unit g / nst, ring slot g % TC_WSLOTS,
  // buffers g % 2. Four running positions: the weight copies (g + TC_WAHEAD), the activation
  // words (g + 2), the scales (g + 1) and the chains (g), each with the pointers of its unit.
  // ---- weight copies: 16-byte pieces (rows wm0 and wm0 + 64, piece wj) of each chunk ----
  const int wj = tid & 7, wm0 = tid >> 3;
  const int wdst = wm0 * 128 + ((wj ^ (wm0 & 7)) << 4);  // same swizzle phase for row wm0 + 64
  int uw = 0, sw = 0, rw = 0;                            // unit, chunk and ring slot of step g + TC_WAHEAD
  const int8_t* wsrc0 = nullptr;
  const int8_t* wsrc1 = nullptr;
  auto w_unit = [&](int ui) {
    const int8_t* q = unit_q(ui) + wj * 16;
    const int r0 = u_r0[ui];
    wsrc0 = q + (long long)min(r0 + wm0, rows - 1) * cols;
    wsrc1 = q + (long long)min(r0 + wm0 + 64, rows - 1) * cols;
  };
  auto issue_w = [&](bool live) {  // one commit group per call
    if (live) {
      unsigned char* dst = wring + (size_t)rw * TC_WCHUNK;
      if (sw < nch) {
        cp_async16_tc(dst + wdst, wsrc0 + sw * 128);
        cp_async16_tc(dst + wdst + 64 * 128, wsrc1 + sw * 128);
      } else {  // tail blocks, no swizzle: 8-row x 16-byte core matrices
        const int8_t* q = unit_q(uw);
        const int r0 = u_r0[uw];
        for (int i = tid; i < TC_M * ntail * 2; i += TC_THREADS) {
          const int m = i / (ntail * 2), rem = i - m * (ntail * 2), tb = rem >> 1, kc = rem & 1;
          cp_async16_tc(dst + tb * 4096 + (m >> 3) * 256 + kc * 128 + (m & 7) * 16,
                        q + (long long)min(r0 + m, rows - 1) * cols + nch * 128 + tb * 32 + kc * 16);
        }
      }
    }
    cp_commit_tc();
  };
  auto w_next = [&]() {
    if (++rw == TC_WSLOTS) rw = 0;
    if (++sw == nst) {
      sw = 0;
      if (++uw < nun) w_unit(uw);
    }
  };

  // ---- activation words: thread tid < 256 = (lane pair lp, entry eb, lane li, block q) holds
  // the entry's bytes lp*32 + li*16 + q*4 .. + 3; tail: tid < ntail * 64 = (tail block, entry, lane)
  const int eb = (tid >> 3) & (TC_TOK - 1);
  const int sq = tid & 3, sli = (tid >> 2) & 1, slp = tid >> 6, stl = tid & 7, stb = tid >> 6;
  const bool smain = tid < 4 * TC_TOK * 8, stail = tid < ntail * TC_TOK * 8;
  const int aoff = slp * 32 + sli * 16 + sq * 4, atoff = nch * 128 + stb * 32 + stl * 4;
  const int boff = slp * (TC_TOK * 256) + eb * 256 + sli * 128 + (2 * sq + sli) * 16 + sq * 4;
  const int btoff = stb * (TC_TOK * 256) + eb * 256 + (stl >> 2) * 128 + stl * 16 + (stl & 3) * 4;
  int ua = 0, sa = 0;  // unit and chunk of the next word to load
  const int8_t* arow = nullptr;
  auto a_unit = [&](int ui) {
    const int code = u_code[ui][eb];
    arow = code >= 0 ? G.aq + (size_t)in_row(code) * cols : nullptr;
  };
  auto load_word = [&]() -> int {
    if (!arow) return 0;
    if (sa < nch) return smain ? *reinterpret_cast<const int*>(arow + sa * 128 + aoff) : 0;
    return stail ? *reinterpret_cast<const int*>(arow + atoff) : 0;
  };
  auto a_next = [&]() {
    if (++sa == nst) {
      sa = 0;
      if (++ua < nun) a_unit(ua);
    }
  };
  auto store_word = [&](int b, int s, int v) {
    if (s < nch) {
      if (smain) *reinterpret_cast<int*>(bbuf + (size_t)b * TC_BCHUNK + boff) = v;
    } else if (stail) {
      *reinterpret_cast<int*>(btail + (size_t)b * TC_TAIL_B + btoff) = v;
    }
  };

  // ---- chains: row r0 + 32 (warp % 4) + lane of the unit, entries 2 (warp / 4) + 0..1 ----
  const int quad = warp & 3, pr = warp >> 2;
  int u1 = 0, s1 = 0;  // unit and chunk of the next scales to load
  const float* wsc = nullptr;
  const float* dsc0 = nullptr;
  const float* dsc1 = nullptr;
  auto c_unit = [&](int ui) {
    wsc = unit_s(ui) + (long long)min(u_r0[ui] + quad * 32 + lane, rows - 1) * ss;
    const int c0 = u_code[ui][2 * pr], c1 = u_code[ui][2 * pr + 1];
    dsc0 = G.as + (size_t)(c0 >= 0 ? in_row(c0) : 0) * ss;  // padding entries read row 0, unused
    dsc1 = G.as + (size_t)(c1 >= 0 ? in_row(c1) : 0) * ss;
  };
  auto load_scales = [&](float4& s4, float4& d0, float4& d1) {
    s4 = __ldg(reinterpret_cast<const float4*>(wsc + 4 * s1));
    d0 = *reinterpret_cast<const float4*>(dsc0 + 4 * s1);
    d1 = *reinterpret_cast<const float4*>(dsc1 + 4 * s1);
  };
  auto c_next = [&]() {
    if (++s1 == nst) {
      s1 = 0;
      if (++u1 < nun) c_unit(u1);
    }
  };

  constexpr uint32_t IDESC = tc_idesc(TC_M, TC_N);
  // the MMAs of a step (chunk s, ring slot) into tensor-memory buffer b, committed to mma_bar[b]
  auto issue_mma = [&](int b, int s, int slot) {
    const uint32_t wa = smem_u32(wring + (size_t)slot * TC_WCHUNK);
    const uint32_t dt = tbase + b * TC_BUFCOLS;
    if (s < nch) {
      const uint32_t ba = smem_u32(bbuf + (size_t)b * TC_BCHUNK);
#pragma unroll
      for (int lp = 0; lp < 4; lp++) {
        const uint64_t ad = tc_desc(wa + lp * 32, 16, 1024, 2);              // 128-byte swizzled, K-major
        const uint64_t bd = tc_desc(ba + lp * (TC_TOK * 256), 128, 256, 0);  // no swizzle, K-major
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(dt + lp * TC_N),
            "l"(ad), "l"(bd), "r"(IDESC), "r"(1));  // D += A * B onto the bias
      }
    } else {
      const uint32_t ba = smem_u32(btail + (size_t)b * TC_TAIL_B);
      for (int tb = 0; tb < ntail; tb++) {
        const uint64_t ad = tc_desc(wa + tb * 4096, 128, 256, 0);
        const uint64_t bd = tc_desc(ba + tb * (TC_TOK * 256), 128, 256, 0);
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(dt + tb * TC_N),
            "l"(ad), "l"(bd), "r"(IDESC), "r"(1));
      }
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(&mma_bar[b]))
                 : "memory");
  };

  // ---- prologue: weights of steps 0..TC_WAHEAD-1 (constant data: before the dependency wait for
  // a launch without routed groups), step 0 staged and issued, step 1's word and step 0's scales
  // in registers ----
  w_unit(0);
#pragma unroll
  for (int g = 0; g < TC_WAHEAD; g++) {
    issue_w(g < S);
    w_next();
  }
  if (G.nrouted == 0) pdl_wait();
  pdl_trigger();
  a_unit(0);
  c_unit(0);
  store_word(0, 0, load_word());
  a_next();
  int wnext = 0;
  if (S > 1) {
    wnext = load_word();
    a_next();
  }
  float4 s4, d0, d1;
  load_scales(s4, d0, d1);
  c_next();
  cp_wait_tc<TC_WAHEAD - 1>();  // this thread's pieces of step 0's weights
  fence_async_smem();           // generic-proxy writes (cp.async, the expansion) -> tensor-core reads
  // this warp's accumulator columns of both buffers start at the bias
  const uint32_t tw = tbase + ((uint32_t)(quad * 32) << 16) + pr * 16;
#pragma unroll
  for (int b = 0; b < 2; b++)
#pragma unroll
    for (int lp = 0; lp < 4; lp++) tmem_st16_same(tw + b * TC_BUFCOLS + lp * TC_N, TC_BIAS);
  tmem_st_wait();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  int issued = 0;  // steps whose MMAs were issued (thread 0)
  if (tid == 0) {
    issue_mma(0, 0, 0);
    issued = 1;
  }

  float acc[2][8];
#pragma unroll
  for (int e = 0; e < 2; e++)
#pragma unroll
    for (int l = 0; l < 8; l++) acc[e][l] = 0.0f;
  int u0 = 0, s0 = 0, r1 = 1;  // unit and chunk of step g; ring slot of step g + 1
  int fail = 0;
  for (int g = 0; g < S; g++) {
    issue_w(g + TC_WAHEAD < S);  // ring slot of step g - 2, whose MMAs this thread saw complete
    w_next();
    int s_next = s0 + 1 == nst ? 0 : s0 + 1;  // chunk of step g + 1
    if (g + 1 < S) {
      store_word((g + 1) & 1, s_next, wnext);  // buffer (g + 1) % 2: last read by step g - 1's MMAs
      if (g + 2 < S) {
        wnext = load_word();
        a_next();
      }
    }
    cp_wait_tc<TC_WAHEAD - 1>();  // this thread's pieces of step g + 1's weights have landed
    fence_async_smem();
    if (fail && lane == 0) fail_s = 1;
    tc_fence_before();
    __syncthreads();  // step g + 1 staged; everyone done reading step g - 1's partials
    tc_fence_after();
    fail = fail_s;
    if (tid == 0 && !fail && g + 1 < S) {
      issue_mma((g + 1) & 1, s_next, r1);
      issued = g + 2;
    }
    if (++r1 == TC_WSLOTS) r1 = 0;
    float sc0[4], sc1[4];
    sc0[0] = fmul(s4.x, d0.x); sc0[1] = fmul(s4.y, d0.y); sc0[2] = fmul(s4.z, d0.z); sc0[3] = fmul(s4.w, d0.w);
    sc1[0] = fmul(s4.x, d1.x); sc1[1] = fmul(s4.y, d1.y); sc1[2] = fmul(s4.z, d1.z); sc1[3] = fmul(s4.w, d1.w);
    if (g + 1 < S) {
      load_scales(s4, d0, d1);
      c_next();
    }
    if (!fail && !mbar_wait(&mma_bar[g & 1], (g >> 1) & 1)) fail = 1;
    fail = __any_sync(0xffffffffu, fail);  // warp-uniform: tcgen05.ld below is a .sync.aligned warp op
    tc_fence_after();
    if (!fail) {
      const uint32_t ta = tw + (g & 1) * TC_BUFCOLS;
      uint32_t v[16];
      if (s0 < nch) {
        // column e*8 + 2q + li of lane pair lp: entry 2pr + e, block 4c + q, lane 2lp + li
#pragma unroll
        for (int lp = 0; lp < 4; lp++) {  // one lane pair per tensor-memory round trip
          tmem_ld16(ta + lp * TC_N, v);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 4; q++)
#pragma unroll
            for (int li = 0; li < 2; li++) {
              const int l = 2 * lp + li;
              acc[0][l] = __fmaf_rn(sc0[q], tc_partial(v[2 * q + li]), acc[0][l]);
              acc[1][l] = __fmaf_rn(sc1[q], tc_partial(v[8 + 2 * q + li]), acc[1][l]);
            }
        }
      } else {
        // column e*8 + l of tail block tb: entry 2pr + e, lane l of block 4 nch + tb
#pragma unroll
        for (int tb = 0; tb < 3; tb++)
          if (tb < ntail) {
            tmem_ld16(ta + tb * TC_N, v);
            tmem_ld_wait();
#pragma unroll
            for (int l = 0; l < 8; l++) {
              acc[0][l] = __fmaf_rn(sc0[tb], tc_partial(v[l]), acc[0][l]);
              acc[1][l] = __fmaf_rn(sc1[tb], tc_partial(v[8 + l]), acc[1][l]);
            }
          }
      }
      // back to the bias for step g + 2's MMAs (issued after the next barrier)
#pragma unroll
      for (int lp = 0; lp < 4; lp++) tmem_st16_same(ta + lp * TC_N, TC_BIAS);
      tmem_st_wait();
    }
    if (++s0 == nst) {
      // ---- unit u0 done: the lane tree ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)) (quant.rs:61-65) ----
      s0 = 0;
      if (!fail) {
        const int row = u_r0[u0] + quad * 32 + lane;
        const bool row_ok = row < rows;
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const int code = u_code[u0][2 * pr + e];  // warp-uniform
          const float* a = acc[e];
          const float yv = fadd(fadd(fadd(a[0], a[4]), fadd(a[2], a[6])), fadd(fadd(a[1], a[5]), fadd(a[3], a[7])));
          const bool ok = row_ok && code >= 0;
          const int t = code >> 5, sl = code & 31;
          if (OUT == TC_OUT_STORE) {
            if (ok) G.out[((size_t)t * G.out_nslot + sl) * G.ostride + row] = yv;
          } else if (OUT == TC_OUT_RESID) {
            if (ok) {
              float* xp = G.x + (size_t)t * G.d + row;
              *xp = fadd(*xp, yv);
            }
          } else {
            if (ok && G.out) G.out[(size_t)t * G.ostride + row] = yv;
            unsigned long long key = (ok && row < G.valid) ? argmax_key(yv, (uint32_t)row) : 0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
            if (lane == 0 && code >= 0 && key) atomicMax(&G.amax[t], key);
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 2; e++)
#pragma unroll
        for (int l = 0; l < 8; l++) acc[e][l] = 0.0f;
      u0++;
    }
  }
  cp_wait_tc<0>();
  if (fail && lane == 0) fail_s = 1;
  __syncthreads();
  if (fail_s && tid == 0 && issued > 0) {
    // stopped early: let the last issued MMAs finish (bounded) before the columns are freed
    const int last = issued - 1;
    mbar_wait(&mma_bar[last & 1], (last >> 1) & 1);
  }
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
static int g_tc_sms[64];

template <int OUT>
static cudaError_t prepare_tc_t() {
  return cudaFuncSetAttribute((const void*)k_tc<OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM);
}

cudaError_t prepare_tc() {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = prepare_tc_t<TC_OUT_STORE>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<TC_OUT_RESID>()) != cudaSuccess) return e;
  if ((e = prepare_tc_t<TC_OUT_LMHEAD>()) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) {
    g_tc_sms[dev] = sms;
    g_tc_ready[dev] = true;
  }
  return cudaSuccess;
}

static bool tc_ready_here(int* sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || !g_tc_ready[dev]) return false;
  if (sms) *sms = g_tc_sms[dev] > 0 ? g_tc_sms[dev] : 148;
  return true;
}

bool tc_usable(const Q8M& W, int T) {
  return tc_ready_here(nullptr) && T >= TC_MIN_T && W.cols % 128 == 0 && W.cols >= 128 && W.ss % 4 == 0;
}

// CTAs of a launch of at most `units` units: one per SM (the runs balance the work), more when a
// run would exceed TC_MAX_UNITS, fewer when there are fewer units than SMs.
static int tc_ctas(long long units, int sms) {
  long long nc = std::max<long long>(sms, (units + TC_MAX_UNITS - 1) / TC_MAX_UNITS);
  nc = std::min<long long>(nc, std::max<long long>(units, 1));
  return (int)nc;
}


static void tc_launch(int out, const TcArgs& G, int nc, int T, cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(nc);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TC_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = T <= 64 ? 1 : 0;
  if (out == TC_OUT_STORE) cudaLaunchKernelEx(&cfg, k_tc<TC_OUT_STORE>, G);
  else if (out == TC_OUT_RESID) cudaLaunchKernelEx(&cfg, k_tc<TC_OUT_RESID>, G);
  else cudaLaunchKernelEx(&cfg, k_tc<TC_OUT_LMHEAD>, G);
}

// epi: 0 store (out[t * ostride + row]), 1 residual add into B.x, 2 lm_head (logits to out when
// set, argmax keys into B.amax) -- the EPI codes of the dp4a kernels in decode.cu.
void launch_mv_tc(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* out,
                  int ostride, int epi, cudaStream_t st) {
  int sms = 148;
  tc_ready_here(&sms);
  TcArgs G{};
  G.W0 = W;
  G.T = B.T;
  G.ne = 0;
  G.nrouted = 0;
  G.slot0 = 0;
  G.aq = aq;
  G.as = as;
  G.in_nslot = 0;
  G.out = out;
  G.out_nslot = 1;
  G.ostride = ostride;
  G.x = B.x;
  G.d = D.d;
  G.valid = D.valid;
  G.amax = B.amax;
  G.err = B.err;
  const long long units = (long long)((W.rows + TC_M - 1) / TC_M) * ((B.T + TC_TOK - 1) / TC_TOK);
  const int out_mode = epi == 1 ? TC_OUT_RESID : epi == 2 ? TC_OUT_LMHEAD : TC_OUT_STORE;
  tc_launch(out_mode, G, tc_ctas(units, sms), B.T, st);
}

bool ffn_tc_usable(const Dims& D, const DecodeBufs& B, const LayerDev& L) {
  return tc_ready_here(nullptr) && B.T >= TC_MIN_T && B.ubuf && B.qact && B.sact && D.d % 128 == 0 &&
         (L.moe ? D.f : D.df) % 32 == 0 && (!L.moe || D.ne + 1 <= TC_MAX_GROUPS);
}

// The FFN of one layer for a step of many tokens: gate and up on the tensor cores, SwiGLU and the
// quantization of the activations, down on the tensor cores. Same results as launch_ffn.
void launch_ffn_tc(const Dims& D, const DecodeBufs& B, const LayerDev& L, cudaStream_t st) {
  int sms = 148;
  tc_ready_here(&sms);
  const bool moe = L.moe != 0;
  const int fd = moe ? D.f : D.df, bslot = moe ? D.k + 1 : 1;
  const int nrouted = moe ? std::min(D.ne, B.T * D.k) : 0;
  const bool shared = moe ? D.nsh > 0 : true;
  if (!shared && nrouted == 0) return;
  // units per row tile: group 0's tiles and at most T * k / 8 + nrouted routed tiles (each active
  // expert's last tile may be partial)
  const long long tiles = (shared ? (B.T + TC_TOK - 1) / TC_TOK : 0) +
                          (moe ? ((long long)B.T * D.k + TC_TOK - 1) / TC_TOK + nrouted : 0);
  TcArgs G{};
  G.T = B.T;
  G.ne = D.ne;
  G.ecount = B.ecount;
  G.active = B.active;
  G.elist = B.elist;
  G.err = B.err;
  G.nrouted = nrouted;
  G.slot0 = moe ? D.k : 0;
  auto up = [&](const Q8M& routed, const Q8M& grp0, float* out) {
    G.W = moe ? routed : Q8M{};
    G.W0 = shared ? grp0 : Q8M{};
    G.aq = B.qh;
    G.as = B.sh;
    G.in_nslot = 0;
    G.out = out;
    G.out_nslot = bslot;
    G.ostride = fd;
    tc_launch(TC_OUT_STORE, G, tc_ctas(tiles * ((fd + TC_M - 1) / TC_M), sms), B.T, st);
  };
  up(L.gate, moe ? L.sgate : L.gate, B.act);
  up(L.up, moe ? L.sup : L.up, B.ubuf);
  const long long nrows = (long long)B.T * bslot, nblk = nrows * (fd >> 5);
  {
    cudaLaunchConfig_t c2{};
    c2.gridDim = dim3((unsigned)((nblk + 7) / 8));
    c2.blockDim = dim3(256);
    c2.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c2.attrs = at;
    c2.numAttrs = B.T <= 64 ? 1 : 0;
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
  tc_launch(TC_OUT_STORE, G, tc_ctas(tiles * ((D.d + TC_M - 1) / TC_M), sms), B.T, st);
}

}  // namespace hg
