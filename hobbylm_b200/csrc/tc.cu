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
// Pipeline: one CTA per SM owns all 512 tensor-memory columns as two 256-column buffers and walks
// a balanced run of units (a 128-row tile x 8 entries of one matrix; the steps of a unit are its
// 128-byte chunks). Roles: two copy warps fill a 6-slot ring (the weight tile by one TMA copy with
// the 128-byte swizzle, the activation words by 4-byte cp.async), one thread issues each step's
// MMAs into the free buffer, and 16 chain warps read the partials back and run the f32 chains;
// they hand off through mbarriers (slot full / empty, buffer full / empty), not CTA barriers.
//
// Safety: every wait on an mbarrier is bounded (TC_SPIN_LIMIT polls); on expiry the CTA records
// HG_ERR_TIMEOUT in the step's error word, its roles stop waiting, it waits (bounded) for its last
// MMAs and copies, and still frees its tensor memory. TMA loads carry no multicast and read only
// this GPU's own memory; their x coordinates are multiples of 16 bytes.
#include <cuda.h>  // CUtensorMap (the encoder is fetched through the runtime; no driver library link)

#include <algorithm>
#include <cstdint>

#include "hg_launch.h"

namespace hg {

constexpr int TC_TOK = 8;             // entries per tile (N = 8 entries x 8 columns per MMA)
constexpr int TC_N = TC_TOK * 8;      // MMA N
constexpr int TC_M = 128;             // rows per CTA (MMA M)
constexpr int TC_BUFCOLS = 4 * TC_N;  // tensor-memory columns of one step: 4 lane-pair MMAs
constexpr int TC_COLS = 2 * TC_BUFCOLS;  // two step buffers: all 512 columns of the SM
// roles: 16 chain warps (TMEM lane quadrant w % 4, entry pair w / 4), 2 copy warps, 1 MMA warp
constexpr int TC_EPI_WARPS = 16;
constexpr int TC_PROD_WARPS = 2;
constexpr int TC_MMA_WARP = TC_EPI_WARPS + TC_PROD_WARPS;
constexpr int TC_THREADS = 32 * (TC_MMA_WARP + 1);
constexpr int TC_PROD0 = 32 * TC_EPI_WARPS;   // first copy thread
constexpr int TC_NPROD = 32 * TC_PROD_WARPS;  // copy threads
constexpr int TC_SLOTS = 6;                   // ring slots, each one step's operands
constexpr int TC_WCHUNK = TC_M * 128;         // bytes of a step's weights
constexpr int TC_BCHUNK = 4 * TC_TOK * 256;   // bytes of an expanded activation chunk (4 lane pairs)
constexpr int TC_TAIL_B = 3 * TC_TOK * 256;   // expanded tail blocks: up to 3 x 8 entries x 8 lanes x 32 B
constexpr int TC_SLOT_BYTES = TC_WCHUNK + TC_BCHUNK + TC_TAIL_B;  // a multiple of 1024
constexpr long long TC_SPIN_LIMIT = 1ll << 26;
constexpr size_t TC_SMEM = 1024 + (size_t)TC_SLOTS * TC_SLOT_BYTES;  // + alignment slack
static_assert(TC_SLOT_BYTES % 1024 == 0, "slots keep the 1024-byte alignment of the swizzled tiles");
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
__device__ __forceinline__ void cp_async4_tc(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// D (tensor memory) = A * B (+ D when acc), kind::i8, one thread
__device__ __forceinline__ void tc_mma_acc(uint32_t dt, uint64_t ad, uint64_t bd, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(dt),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc ? 1 : 0));
}
// the mbarrier completes a phase once every MMA this thread issued before has completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// the barrier's current phase also waits for `bytes` more bytes of bulk copies (no arrival)
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// One box of a 3-D tensor map (this GPU's own memory; no multicast) into shared memory; the bytes
// complete on the mbarrier. x (bytes of an 8-bit tensor) is a multiple of 16.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 16 consecutive tensor-memory columns of this warp's 32 lanes (one 32-bit value per column).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// float(v) of an int32 |v| < 2^22 (a lane partial or a block sum), exactly: 1.5 * 2^23 added in
// integer arithmetic makes the bit pattern of the float 1.5 * 2^23 + v (every integer in
// [2^23, 2^24) is representable), and subtracting 1.5 * 2^23 as a float leaves v -- an integer add
// and a full-rate float add instead of an int-to-float conversion.
constexpr uint32_t TC_BIAS = 0x4B400000u;
constexpr float TC_BIAS_F = 12582912.0f;
__device__ __forceinline__ float tc_isum(uint32_t v) { return __fsub_rn(__uint_as_float(v + TC_BIAS), TC_BIAS_F); }

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
// Tensor maps of a Q8 matrix stack (x = byte of the row, y = row, z = matrix): `main` boxes a
// chunk of 128 rows x 128 bytes with the 128-byte swizzle (the MMA's A tile as is); `tail` boxes
// 128 rows x 16 bytes (half of a tail block, 8-row x 16-byte core matrices).
struct TcMaps {
  CUtensorMap main, tail;
};

struct TcArgs {
  TcMaps m0, m1;           // maps of W0 and W (64-byte aligned members first)
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
__global__ void __launch_bounds__(TC_THREADS, 1) k_tc(const __grid_constant__ TcArgs G) {
  extern __shared__ __align__(16) unsigned char tc_raw[];
  // slots of 1024-byte aligned tiles (the 128-byte swizzle pattern repeats every 1024 bytes):
  // [weights 128 rows x 128 B, swizzled][expanded chunk: 4 lp x TC_TOK x 256 B][expanded tail]
  unsigned char* ring = tc_raw + ((1024 - (smem_u32(tc_raw) & 1023)) & 1023);
  __shared__ uint64_t full_bar[TC_SLOTS], empty_bar[TC_SLOTS], tfull_bar[2], tempty_bar[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ int fail_s, run_s[2], mma_last_s;
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
  pdl_wait();  // activations (and, for the FFN, the expert lists) come from the previous kernels

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
  pdl_trigger();
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

  // ---- set-up: tensor memory, barriers, zeroed activation expansions, biased accumulators ----
  if (warp == TC_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int k = 0; k < TC_SLOTS; k++) {
      mbar_init(&full_bar[k], TC_NPROD);  // every copy thread, after its copies of the slot landed
      mbar_init(&empty_bar[k], 1);        // the MMAs that read the slot (commit)
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull_bar[b], 1);              // the MMAs that wrote the buffer (commit)
      mbar_init(&tempty_bar[b], TC_EPI_WARPS);  // every chain warp, after reading the buffer
    }
    fail_s = 0;
    mma_last_s = -1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < TC_SLOTS * (TC_BCHUNK + TC_TAIL_B) / 16; i += TC_THREADS) {
    const int k = i / ((TC_BCHUNK + TC_TAIL_B) / 16), r = i - k * ((TC_BCHUNK + TC_TAIL_B) / 16);
    reinterpret_cast<int4*>(ring + (size_t)k * TC_SLOT_BYTES + TC_WCHUNK)[r] = make_int4(0, 0, 0, 0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_s;
  const int quad = warp & 3, pr = (warp >> 2) & 3;
  const uint32_t tw = tbase + ((uint32_t)(quad * 32) << 16) + pr * 16;  // chain warps' columns
  fence_async_smem();  // the zeroed expansions -> tensor-core reads
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  auto in_row = [&](int code) -> int {
    return G.in_nslot ? (code >> 5) * G.in_nslot + (code & 31) : (code >> 5);
  };
  auto failed = [&]() -> bool { return *reinterpret_cast<volatile int*>(&fail_s) != 0; };
  auto give_up = [&]() { *reinterpret_cast<volatile int*>(&fail_s) = 1; };

  if (warp >= TC_EPI_WARPS && warp < TC_MMA_WARP) {
    // =================== copy warps: weights and activation words of every step ===================
    const int p = tid - TC_PROD0;  // 0..TC_NPROD-1
    constexpr int APT = 4 * TC_TOK * 8 / TC_NPROD;  // activation words per thread
    // weights: one bulk tensor copy per step by thread 0 (rows past the matrix read as zeros);
    // activation words: w = p + TC_NPROD i (i < APT) = (lane pair lp, entry e, lane li, block q)
    const TcMaps* wmap = nullptr;
    int r0 = 0, wz = 0;
    const int8_t* arow[APT];
    int aoff[APT], boff[APT];
#pragma unroll
    for (int i = 0; i < APT; i++) {
      const int w = p + TC_NPROD * i, q = w & 3, li = (w >> 2) & 1, e = (w >> 3) & (TC_TOK - 1), lp = w >> 6;
      aoff[i] = lp * 32 + li * 16 + q * 4;
      boff[i] = lp * (TC_TOK * 256) + e * 256 + li * 128 + (2 * q + li) * 16 + q * 4;
      arow[i] = nullptr;
    }
    int ui = -1;
    auto set_unit = [&](int u) {
      ui = u;
      const int gi = u_gi[u];
      wmap = (has0 && gi == 0) ? &G.m0 : &G.m1;
      wz = (has0 && gi == 0) ? 0 : g_exp[gi];
      r0 = u_r0[u];
#pragma unroll
      for (int i = 0; i < APT; i++) {
        const int e = ((p + TC_NPROD * i) >> 3) & (TC_TOK - 1), code = u_code[u][e];
        arow[i] = code >= 0 ? G.aq + (size_t)in_row(code) * cols : nullptr;
      }
    };
    constexpr int PD = 3;  // copy groups in flight per thread before a slot is signalled
    int s = 0, u = 0;
    set_unit(0);
    int sig = 0;  // next step to signal
    for (int g = 0; g < S; g++) {
      const int k = g % TC_SLOTS, n = g / TC_SLOTS;
      if (n >= 1 && !failed() && !mbar_wait(&empty_bar[k], (n - 1) & 1)) give_up();
      if (!failed()) {
        unsigned char* slot = ring + (size_t)k * TC_SLOT_BYTES;
        if (s < nch) {
          if (p == 0) {  // the A tile: 128 rows x 128 bytes, swizzled by the copy engine
            mbar_expect_tx(&full_bar[k], TC_WCHUNK);
            tma_load_3d(slot, &wmap->main, s * 128, r0, wz, &full_bar[k]);
          }
#pragma unroll
          for (int i = 0; i < APT; i++)
            if (arow[i]) cp_async4_tc(slot + TC_WCHUNK + boff[i], arow[i] + s * 128 + aoff[i]);
        } else {
          if (p == 0) {  // tail block tb, half kc: 128 rows x 16 bytes at tb * 4096 + kc * 2048
            mbar_expect_tx(&full_bar[k], ntail * 4096);
            for (int tb = 0; tb < ntail; tb++)
              for (int kc = 0; kc < 2; kc++)
                tma_load_3d(slot + tb * 4096 + kc * 2048, &wmap->tail, nch * 128 + tb * 32 + kc * 16, r0, wz,
                            &full_bar[k]);
          }
          for (int w = p; w < ntail * TC_TOK * 8; w += TC_NPROD) {  // (tail block tb, entry e, lane l)
            const int l = w & 7, e = (w >> 3) & (TC_TOK - 1), tb = w >> 6, code = u_code[ui][e];
            if (code >= 0)
              cp_async4_tc(slot + TC_WCHUNK + TC_BCHUNK + tb * (TC_TOK * 256) + e * 256 + (l >> 2) * 128 + l * 16 +
                               (l & 3) * 4,
                           G.aq + (size_t)in_row(code) * cols + nch * 128 + tb * 32 + l * 4);
          }
        }
      }
      cp_commit_tc();
      if (++s == nst) {
        s = 0;
        if (++u < nun) set_unit(u);
      }
      if (g - sig == PD - 1) {  // step sig's copies landed: publish them to the tensor cores
        cp_wait_tc<PD - 1>();
        fence_async_smem();
        mbar_arrive(&full_bar[sig % TC_SLOTS]);
        sig++;
      }
    }
    cp_wait_tc<0>();
    fence_async_smem();
    for (; sig < S; sig++) mbar_arrive(&full_bar[sig % TC_SLOTS]);
  } else if (warp == TC_MMA_WARP) {
    // =================== MMA warp: one thread issues every step's MMAs ===================
    if (lane == 0) {
      constexpr uint32_t IDESC = tc_idesc(TC_M, TC_N);
      int s = 0;
      for (int g = 0; g < S && !failed(); g++) {
        const int k = g % TC_SLOTS, b = g & 1;
        if (!mbar_wait(&full_bar[k], (g / TC_SLOTS) & 1)) { give_up(); break; }
        if (g >= 2 && !mbar_wait(&tempty_bar[b], ((g >> 1) - 1) & 1)) { give_up(); break; }
        tc_fence_after();
        unsigned char* slot = ring + (size_t)k * TC_SLOT_BYTES;
        const uint32_t wa = smem_u32(slot), dt = tbase + b * TC_BUFCOLS;
        if (s < nch) {
          const uint32_t ba = smem_u32(slot + TC_WCHUNK);
#pragma unroll
          for (int lp = 0; lp < 4; lp++) {
            const uint64_t ad = tc_desc(wa + lp * 32, 16, 1024, 2);              // 128-byte swizzled, K-major
            const uint64_t bd = tc_desc(ba + lp * (TC_TOK * 256), 128, 256, 0);  // no swizzle, K-major
            tc_mma_acc(dt + lp * TC_N, ad, bd, IDESC, false);  // every lane pair has its own columns
          }
        } else {
          const uint32_t ba = smem_u32(slot + TC_WCHUNK + TC_BCHUNK);
          for (int tb = 0; tb < ntail; tb++)
            tc_mma_acc(dt + tb * TC_N, tc_desc(wa + tb * 4096, 2048, 128, 0),
                       tc_desc(ba + tb * (TC_TOK * 256), 128, 256, 0), IDESC, false);
        }
        tc_commit(&tfull_bar[b]);   // the chain warps may read buffer b
        tc_commit(&empty_bar[k]);   // the copy warps may refill slot k
        mma_last_s = g;
        if (++s == nst) s = 0;
      }
    }
    __syncwarp();
  } else {
    // =================== chain warps: row r0 + 32 (warp % 4) + lane, entries 2 (warp / 4) + 0..1 =====
    int u1 = 0, s1 = 0;  // unit and chunk of the next scales to load
    const float* wsc = nullptr;
    const float* dsc0 = nullptr;
    const float* dsc1 = nullptr;
    auto c_unit = [&](int ui) {
      const int gi = u_gi[ui];
      const float* sc = (has0 && gi == 0) ? G.W0.sc : G.W.sc + (long long)g_exp[gi] * G.W.sc_mstride;
      wsc = sc + (long long)min(u_r0[ui] + quad * 32 + lane, rows - 1) * ss;
      const int c0 = u_code[ui][2 * pr], c1 = u_code[ui][2 * pr + 1];
      dsc0 = G.as + (size_t)(c0 >= 0 ? in_row(c0) : 0) * ss;  // padding entries read row 0, unused
      dsc1 = G.as + (size_t)(c1 >= 0 ? in_row(c1) : 0) * ss;
    };
    float4 s4, d0, d1;
    auto load_scales = [&]() {
      s4 = __ldg(reinterpret_cast<const float4*>(wsc + 4 * s1));
      d0 = *reinterpret_cast<const float4*>(dsc0 + 4 * s1);
      d1 = *reinterpret_cast<const float4*>(dsc1 + 4 * s1);
      if (++s1 == nst) {
        s1 = 0;
        if (++u1 < nun) c_unit(u1);
      }
    };
    c_unit(0);
    load_scales();
    float acc[2][8];
#pragma unroll
    for (int e = 0; e < 2; e++)
#pragma unroll
      for (int l = 0; l < 8; l++) acc[e][l] = 0.0f;
    int u0 = 0, s0 = 0, fail = 0;
    for (int g = 0; g < S; g++) {
      const int b = g & 1;
      float sc0[4], sc1[4];
      sc0[0] = fmul(s4.x, d0.x); sc0[1] = fmul(s4.y, d0.y); sc0[2] = fmul(s4.z, d0.z); sc0[3] = fmul(s4.w, d0.w);
      sc1[0] = fmul(s4.x, d1.x); sc1[1] = fmul(s4.y, d1.y); sc1[2] = fmul(s4.z, d1.z); sc1[3] = fmul(s4.w, d1.w);
      if (g + 1 < S) load_scales();
      if (!fail) {
        if (failed() || !mbar_wait(&tfull_bar[b], (g >> 1) & 1)) fail = 1;
        fail = __any_sync(0xffffffffu, fail);  // warp-uniform: tcgen05.ld below is a .sync.aligned warp op
        if (fail) give_up();
      }
      tc_fence_after();
      if (!fail) {
        const uint32_t ta = tw + b * TC_BUFCOLS;
        uint32_t v[16];
        if (s0 < nch) {
          // column e*8 + 2q + li of lane pair lp: entry 2pr + e, block 4c + q, lane 2lp + li
#pragma unroll
          for (int h = 0; h < 2; h++) {  // two lane pairs per tensor-memory round trip
            uint32_t w[16];
            tmem_ld16(ta + (2 * h) * TC_N, v);
            tmem_ld16(ta + (2 * h + 1) * TC_N, w);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 4; q++)
#pragma unroll
              for (int li = 0; li < 2; li++) {
                const int l = 4 * h + li, l2 = 4 * h + 2 + li;  // lanes of pairs 2h and 2h + 1
                acc[0][l] = __fmaf_rn(sc0[q], tc_isum(v[2 * q + li]), acc[0][l]);
                acc[1][l] = __fmaf_rn(sc1[q], tc_isum(v[8 + 2 * q + li]), acc[1][l]);
                acc[0][l2] = __fmaf_rn(sc0[q], tc_isum(w[2 * q + li]), acc[0][l2]);
                acc[1][l2] = __fmaf_rn(sc1[q], tc_isum(w[8 + 2 * q + li]), acc[1][l2]);
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
                acc[0][l] = __fmaf_rn(sc0[tb], tc_isum(v[l]), acc[0][l]);
                acc[1][l] = __fmaf_rn(sc1[tb], tc_isum(v[8 + l]), acc[1][l]);
              }
            }
        }
        // hand the buffer back to the MMAs of step g + 2
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[b]);
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
            const float yv =
                fadd(fadd(fadd(a[0], a[4]), fadd(a[2], a[6])), fadd(fadd(a[1], a[5]), fadd(a[3], a[7])));
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
  }
  // ---- wind-down: every MMA complete before the columns are freed ----
  __syncthreads();
  if (tid == TC_MMA_WARP * 32 && failed() && mma_last_s >= 0) {
    // stopped early: the last commit covers every MMA issued before it (bounded wait)
    const int last = mma_last_s;
    mbar_wait(&tfull_bar[last & 1], (last >> 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TC_MMA_WARP)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_COLS));
  if (failed() && tid == 0 && G.err) atomicExch(G.err, HG_ERR_TIMEOUT);
}

// ------------------------------------------------------------------------------------------
// Prefill-order Q8 matmul on the tensor cores (quant.rs:144-193): per output (row o, activation
// row t) acc = fadd(acc, fmul(fmul(sw[o][b], sx[t][b]), float(isum[o][t][b]))) over the blocks b
// in order, isum the exact int32 dot of one 32-element block. An MMA of kind::i8 gives the block
// sums: for lane pair lp of a 128-byte chunk, B row n = 4 t + q holds activation row t's bytes of
// block q (its 8 bytes in the lane pair, zeros elsewhere), so the four lane-pair MMAs accumulate
// D[o][4 t + q] = isum of block 4c + q. Tail blocks (rows whose width is not a multiple of 128
// bytes) are contiguous 32 bytes: one MMA per tail block with B row t = activation row t.
// A unit is 128 weight rows x 64 activation rows of one group (a matrix of the stack and its
// entry range, MmArgs grp tables); CTAs take balanced runs of units; the roles and the pipeline
// are those of k_tc (copy warps, one MMA thread, chain warps) with a 3-slot ring.
// ------------------------------------------------------------------------------------------
constexpr int KT_TOK = 64;                              // activation rows per unit
constexpr int KT_N = 4 * KT_TOK;                        // MMA N of a chunk step
constexpr int KT_BMAIN = 4 * KT_N * 32;                 // expanded chunk: 4 lp x 256 rows x 32 B
constexpr int KT_BTAIL = 3 * KT_TOK * 32;               // tail blocks: 3 x 64 rows x 32 B
constexpr int KT_SX = KT_TOK * 16;                      // the rows' 4 block scales of the step
constexpr int KT_SLOT_BYTES = ((TC_WCHUNK + KT_BMAIN + KT_BTAIL + KT_SX + 1023) / 1024) * 1024;
constexpr int KT_SLOTS = 3;
constexpr int KT_PROD_WARPS = 2;
constexpr int KT_NPROD = 32 * KT_PROD_WARPS;            // == KT_TOK: copy thread p serves activation row p
constexpr int KT_MMA_WARP = TC_EPI_WARPS + KT_PROD_WARPS;
constexpr int KT_THREADS = 32 * (KT_MMA_WARP + 1);
constexpr size_t KT_SMEM = 1024 + (size_t)KT_SLOTS * KT_SLOT_BYTES;
static_assert(KT_NPROD == KT_TOK, "one copy thread per activation row");

struct KtArgs {
  TcMaps m;     // maps of the stack W
  MmArgs a;
  int ngroups;
};

__global__ void __launch_bounds__(KT_THREADS, 1) kp_tc(const __grid_constant__ KtArgs K) {
  const MmArgs& a = K.a;
  const int ngroups = K.ngroups;
  extern __shared__ __align__(16) unsigned char kt_raw[];
  unsigned char* ring = kt_raw + ((1024 - (smem_u32(kt_raw) & 1023)) & 1023);
  __shared__ uint64_t full_bar[KT_SLOTS], empty_bar[KT_SLOTS], sxfree_bar[KT_SLOTS], tfull_bar[2], tempty_bar[2];
  __shared__ uint32_t tmem_base_s;
  __shared__ int fail_s, run_s[2], mma_last_s;
  __shared__ int g_start[TC_MAX_GROUPS + 1], g_tiles[TC_MAX_GROUPS], g_count[TC_MAX_GROUPS], g_mat[TC_MAX_GROUPS],
      g_off[TC_MAX_GROUPS];
  __shared__ int u_gi[TC_MAX_UNITS], u_r0[TC_MAX_UNITS], u_a0[TC_MAX_UNITS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Q8M& W = a.W;
  const int rows = W.rows, cols = W.cols, nb = cols >> 5, nch = nb >> 2, ntail = nb & 3, ss = W.ss;
  const int nst = nch + (ntail ? 1 : 0);
  const int rt = (rows + TC_M - 1) / TC_M;

  // ---- groups (one, or the grp tables of an expert launch), this CTA's run of units ----
  if (warp == 0) {
    for (int gi = lane; gi < ngroups; gi += 32) {
      int mat = a.mat, off = 0, cnt = a.nrows;
      if (a.grp_mat) {
        mat = a.grp_mat[gi];
        off = a.grp_off[gi];
        cnt = mat < 0 ? 0 : a.grp_cnt[gi];
      }
      g_mat[gi] = mat;
      g_off[gi] = off;
      g_count[gi] = cnt;
      g_tiles[gi] = (cnt + KT_TOK - 1) / KT_TOK;
    }
    __syncwarp();
    if (lane == 0) {
      int acc = 0;
      for (int gi = 0; gi < ngroups; gi++) {
        g_start[gi] = acc;
        acc += rt * g_tiles[gi];
      }
      g_start[ngroups] = acc;
      const long long U = acc, nc = gridDim.x;
      const int ub = (int)(U * blockIdx.x / nc), ue = (int)(U * (blockIdx.x + 1) / nc);
      run_s[0] = ub;
      run_s[1] = min(ue - ub, TC_MAX_UNITS);
      if (ue - ub > TC_MAX_UNITS && a.err) atomicExch(a.err, HG_ERR_INVALID);  // host sizing bug: loud
    }
  }
  __syncthreads();
  const int ub = run_s[0], nun = run_s[1];
  if (nun <= 0) return;
  for (int ui = tid; ui < nun; ui += KT_THREADS) {
    const int u = ub + ui;
    int lo = 0, hi = ngroups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (g_start[mid] <= u) lo = mid;
      else hi = mid - 1;
    }
    const int tl = g_tiles[lo], ul = u - g_start[lo], rtile = ul / tl;
    u_gi[ui] = lo;
    u_r0[ui] = rtile * TC_M;
    u_a0[ui] = (ul - rtile * tl) * KT_TOK;
  }
  const int S = nun * nst;

  if (warp == KT_MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(TC_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int k = 0; k < KT_SLOTS; k++) {
      mbar_init(&full_bar[k], KT_NPROD);
      mbar_init(&empty_bar[k], 1);
      mbar_init(&sxfree_bar[k], TC_EPI_WARPS);  // every chain warp, after reading the slot's scales
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], TC_EPI_WARPS);
    }
    fail_s = 0;
    mma_last_s = -1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int i = tid; i < KT_SLOTS * (KT_BMAIN / 16); i += KT_THREADS) {  // the expansions' zeros, once
    const int k = i / (KT_BMAIN / 16), r = i - k * (KT_BMAIN / 16);
    reinterpret_cast<int4*>(ring + (size_t)k * KT_SLOT_BYTES + TC_WCHUNK)[r] = make_int4(0, 0, 0, 0);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base_s;
  auto failed = [&]() -> bool { return *reinterpret_cast<volatile int*>(&fail_s) != 0; };
  auto give_up = [&]() { *reinterpret_cast<volatile int*>(&fail_s) = 1; };
  auto arow_of = [&](int ui, int i) -> long long {  // activation row of entry i of unit ui, or -1
    const int gi = u_gi[ui], e = u_a0[ui] + i;
    if (e >= g_count[gi]) return -1;
    const int idx = g_off[gi] + e;
    return a.a_idx ? (long long)a.a_idx[idx] : (long long)idx;
  };

  if (warp >= TC_EPI_WARPS && warp < KT_MMA_WARP) {
    // =================== copy warps: thread p = activation row p of the unit ===================
    const int p = tid - TC_EPI_WARPS * 32;
    int r0 = 0, wz = 0;
    const int8_t* xrow = nullptr;  // activation row p of the unit (null past the group's rows)
    const float* xsc = nullptr;
    int ui = 0;
    auto set_unit = [&](int u) {
      ui = u;
      const int mat = g_mat[u_gi[u]];
      wz = mat < 0 ? 0 : mat;
      r0 = u_r0[u];
      const long long ar = arow_of(u, p);
      xrow = ar >= 0 ? a.aq + ar * cols : nullptr;
      xsc = ar >= 0 ? a.as + ar * ss : nullptr;
    };
    constexpr int PD = 2;
    int s = 0, u = 0, sig = 0;
    set_unit(0);
    for (int g = 0; g < S; g++) {
      const int k = g % KT_SLOTS, n = g / KT_SLOTS;
      if (n >= 1 && !failed() &&
          (!mbar_wait(&empty_bar[k], (n - 1) & 1) || !mbar_wait(&sxfree_bar[k], (n - 1) & 1)))
        give_up();
      if (!failed()) {
        unsigned char* slot = ring + (size_t)k * KT_SLOT_BYTES;
        float* sxd = reinterpret_cast<float*>(slot + TC_WCHUNK + KT_BMAIN + KT_BTAIL) + p * 4;
        if (s < nch) {
          if (p == 0) {  // the A tile: 128 rows x 128 bytes, swizzled by the copy engine
            mbar_expect_tx(&full_bar[k], TC_WCHUNK);
            tma_load_3d(slot, &K.m.main, s * 128, r0, wz, &full_bar[k]);
          }
          if (xrow) {
            // byte lp*32 + li*16 + q*4 .. + 3 of the chunk -> B row n = 4 p + q of lane pair lp, K
            // bytes li*16 + q*4 .. + 3 (8-row x 16-byte core matrices, rows 16 B apart)
            unsigned char* bb = slot + TC_WCHUNK;
            const int8_t* src = xrow + s * 128;
#pragma unroll
            for (int lp = 0; lp < 4; lp++)
#pragma unroll
              for (int li = 0; li < 2; li++)
#pragma unroll
                for (int q = 0; q < 4; q++) {
                  const int nrow = 4 * p + q;
                  cp_async4_tc(bb + lp * (KT_N * 32) + (nrow >> 3) * 256 + li * 128 + (nrow & 7) * 16 + q * 4,
                               src + lp * 32 + li * 16 + q * 4);
                }
            cp_async16_tc(sxd, xsc + 4 * s);
          }
        } else {
          if (p == 0) {  // tail block tb, half kc: 128 rows x 16 bytes at tb * 4096 + kc * 2048
            mbar_expect_tx(&full_bar[k], ntail * 4096);
            for (int tb = 0; tb < ntail; tb++)
              for (int kc = 0; kc < 2; kc++)
                tma_load_3d(slot + tb * 4096 + kc * 2048, &K.m.tail, nch * 128 + tb * 32 + kc * 16, r0, wz,
                            &full_bar[k]);
          }
          if (xrow) {
            unsigned char* bt = slot + TC_WCHUNK + KT_BMAIN;
            for (int tb = 0; tb < ntail; tb++)
#pragma unroll
              for (int kc = 0; kc < 2; kc++)
                cp_async16_tc(bt + tb * (KT_TOK * 32) + (p >> 3) * 256 + kc * 128 + (p & 7) * 16,
                              xrow + nch * 128 + tb * 32 + kc * 16);
            cp_async16_tc(sxd, xsc + 4 * s);
          }
        }
      }
      cp_commit_tc();
      if (++s == nst) {
        s = 0;
        if (++u < nun) set_unit(u);
      }
      if (g - sig == PD - 1) {
        cp_wait_tc<PD - 1>();
        fence_async_smem();
        mbar_arrive(&full_bar[sig % KT_SLOTS]);
        sig++;
      }
    }
    cp_wait_tc<0>();
    fence_async_smem();
    for (; sig < S; sig++) mbar_arrive(&full_bar[sig % KT_SLOTS]);
  } else if (warp == KT_MMA_WARP) {
    // =================== MMA thread ===================
    if (lane == 0) {
      constexpr uint32_t IDESC = tc_idesc(TC_M, KT_N), IDESC_T = tc_idesc(TC_M, KT_TOK);
      int s = 0;
      for (int g = 0; g < S && !failed(); g++) {
        const int k = g % KT_SLOTS, b = g & 1;
        if (!mbar_wait(&full_bar[k], (g / KT_SLOTS) & 1)) { give_up(); break; }
        if (g >= 2 && !mbar_wait(&tempty_bar[b], ((g >> 1) - 1) & 1)) { give_up(); break; }
        tc_fence_after();
        unsigned char* slot = ring + (size_t)k * KT_SLOT_BYTES;
        const uint32_t wa = smem_u32(slot), dt = tbase + b * (TC_COLS / 2);
        if (s < nch) {
          const uint32_t ba = smem_u32(slot + TC_WCHUNK);
#pragma unroll
          for (int lp = 0; lp < 4; lp++)  // the four lane pairs accumulate into the same block sums
            tc_mma_acc(dt, tc_desc(wa + lp * 32, 16, 1024, 2), tc_desc(ba + lp * (KT_N * 32), 128, 256, 0), IDESC,
                       lp > 0);
        } else {
          const uint32_t ba = smem_u32(slot + TC_WCHUNK + KT_BMAIN);
          for (int tb = 0; tb < ntail; tb++)
            tc_mma_acc(dt + tb * KT_TOK, tc_desc(wa + tb * 4096, 2048, 128, 0),
                       tc_desc(ba + tb * (KT_TOK * 32), 128, 256, 0), IDESC_T, false);
        }
        tc_commit(&tfull_bar[b]);
        tc_commit(&empty_bar[k]);
        mma_last_s = g;
        if (++s == nst) s = 0;
      }
    }
    __syncwarp();
  } else {
    // =================== chain warps: row 32 (warp % 4) + lane, activation rows 16 (warp / 4) + 0..15
    const int quad = warp & 3, grp = warp >> 2;
    const uint32_t tw = tbase + ((uint32_t)(quad * 32) << 16);
    int u1 = 0, s1 = 0;
    const float* wsc = nullptr;
    auto c_unit = [&](int ui) {
      const int mat = g_mat[u_gi[ui]];
      wsc = W.sc + (long long)(mat < 0 ? 0 : mat) * W.sc_mstride +
            (long long)min(u_r0[ui] + quad * 32 + lane, rows - 1) * ss;
    };
    float4 sw4;
    auto load_scales = [&]() {
      sw4 = __ldg(reinterpret_cast<const float4*>(wsc + 4 * s1));
      if (++s1 == nst) {
        s1 = 0;
        if (++u1 < nun) c_unit(u1);
      }
    };
    c_unit(0);
    load_scales();
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; i++) acc[i] = 0.0f;
    int u0 = 0, s0 = 0, fail = 0;
    for (int g = 0; g < S; g++) {
      const int b = g & 1, k = g % KT_SLOTS;
      const float sw[4] = {sw4.x, sw4.y, sw4.z, sw4.w};
      if (g + 1 < S) load_scales();
      if (!fail) {
        if (failed() || !mbar_wait(&tfull_bar[b], (g >> 1) & 1)) fail = 1;
        fail = __any_sync(0xffffffffu, fail);
        if (fail) give_up();
      }
      tc_fence_after();
      if (!fail) {
        // the rows' block scales, staged with the step's operands (the slot is refilled only after
        // every chain warp released it on sxfree_bar)
        const float4* sx = reinterpret_cast<const float4*>(ring + (size_t)k * KT_SLOT_BYTES + TC_WCHUNK + KT_BMAIN +
                                                           KT_BTAIL) + grp * 16;
        const uint32_t ta = tw + b * (TC_COLS / 2);
        uint32_t v[16];
        if (s0 < nch) {
#pragma unroll
          for (int j = 0; j < 4; j++) {  // rows 16 grp + 4 j .. + 3: columns (4 rows x 4 blocks)
            tmem_ld16(ta + grp * 64 + j * 16, v);
            tmem_ld_wait();
#pragma unroll
            for (int r = 0; r < 4; r++) {
              const float4 x4 = sx[4 * j + r];
              const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
              for (int q = 0; q < 4; q++)
                acc[4 * j + r] = fadd(acc[4 * j + r], fmul(fmul(sw[q], xs[q]), tc_isum(v[4 * r + q])));
            }
          }
        } else {
#pragma unroll
          for (int tb = 0; tb < 3; tb++)
            if (tb < ntail) {
              tmem_ld16(ta + tb * KT_TOK + grp * 16, v);
              tmem_ld_wait();
#pragma unroll
              for (int r = 0; r < 16; r++) {
                const float4 x4 = sx[r];
                const float xq = tb == 0 ? x4.x : tb == 1 ? x4.y : x4.z;
                acc[r] = fadd(acc[r], fmul(fmul(sw[tb], xq), tc_isum(v[r])));
              }
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty_bar[b]);
          mbar_arrive(&sxfree_bar[k]);
        }
      }
      if (++s0 == nst) {
        s0 = 0;
        if (!fail) {
          const int row = u_r0[u0] + quad * 32 + lane;
          if (row < rows) {
            const int gi = u_gi[u0];
#pragma unroll
            for (int r = 0; r < 16; r++) {
              const int e = u_a0[u0] + grp * 16 + r;
              if (e < g_count[gi]) {
                const int idx = g_off[gi] + e;
                const long long orow = a.o_idx ? (long long)a.o_idx[idx] : (long long)idx;
                float* po = a.out + orow * a.ostride + row;
                *po = a.mode == 1 ? fadd(*po, acc[r]) : acc[r];
              }
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 16; i++) acc[i] = 0.0f;
        u0++;
      }
    }
  }
  __syncthreads();
  if (tid == KT_MMA_WARP * 32 && failed() && mma_last_s >= 0) {
    const int last = mma_last_s;
    mbar_wait(&tfull_bar[last & 1], (last >> 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == KT_MMA_WARP)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(TC_COLS));
  if (failed() && tid == 0 && a.err) atomicExch(a.err, HG_ERR_TIMEOUT);
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

// cuTensorMapEncodeTiled, fetched through the runtime once (no link against the driver library)
typedef CUresult (*TmapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static TmapEncodeFn g_tmap_encode = nullptr;

static bool tmap_init() {
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_tmap_encode = reinterpret_cast<TmapEncodeFn>(fn);
  }
  return g_tmap_encode != nullptr;
}

// the layout a tensor map can describe: 16-byte aligned base, rows and matrices 16-byte strided
static bool tc_mappable(const Q8M& W, int count) {
  const unsigned long long ms = count > 1 ? (unsigned long long)W.qs_mstride : (unsigned long long)W.rows * W.cols;
  return W.qs && reinterpret_cast<uintptr_t>(W.qs) % 16 == 0 && W.cols % 16 == 0 && ms % 16 == 0;
}

// maps of a stack of `count` matrices (count 1: one matrix)
static bool tc_maps(const Q8M& W, int count, TcMaps* m) {
  if (!g_tmap_encode || !tc_mappable(W, count)) return false;
  const cuuint64_t ms = count > 1 ? (cuuint64_t)W.qs_mstride : (cuuint64_t)W.rows * W.cols;
  const cuuint64_t dims[3] = {(cuuint64_t)W.cols, (cuuint64_t)W.rows, (cuuint64_t)count};
  const cuuint64_t strides[2] = {(cuuint64_t)W.cols, ms};
  const cuuint32_t box_main[3] = {128, TC_M, 1}, box_tail[3] = {16, TC_M, 1}, es[3] = {1, 1, 1};
  *m = TcMaps{};
  if (W.cols >= 128 &&
      g_tmap_encode(&m->main, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(W.qs), dims, strides, box_main,
                    es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  return g_tmap_encode(&m->tail, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(W.qs), dims, strides, box_tail,
                       es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

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
  if ((e = cudaFuncSetAttribute((const void*)kp_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KT_SMEM)) !=
      cudaSuccess)
    return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if (!tmap_init()) return cudaSuccess;  // no tensor-map encoder: the dp4a kernels serve every step
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
  return tc_ready_here(nullptr) && T >= TC_MIN_T && W.cols % 128 == 0 && W.cols >= 128 && W.ss % 4 == 0 &&
         tc_mappable(W, 1);
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
bool launch_mv_tc(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* out,
                  int ostride, int epi, cudaStream_t st) {
  int sms = 148;
  tc_ready_here(&sms);
  TcArgs G{};
  if (!tc_maps(W, 1, &G.m0)) return false;
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
  return true;
}

bool ffn_tc_usable(const Dims& D, const DecodeBufs& B, const LayerDev& L) {
  if (!(tc_ready_here(nullptr) && B.T >= TC_MIN_T && B.ubuf && B.qact && B.sact && D.d % 128 == 0 &&
        (L.moe ? D.f : D.df) % 32 == 0 && (!L.moe || D.ne + 1 <= TC_MAX_GROUPS)))
    return false;
  const bool moe = L.moe != 0;
  if (moe) {
    if (!tc_mappable(L.gate, D.ne) || !tc_mappable(L.up, D.ne) || !tc_mappable(L.down, D.ne)) return false;
    if (D.nsh > 0 && (!tc_mappable(L.sgate, 1) || !tc_mappable(L.sup, 1) || !tc_mappable(L.sdown, 1))) return false;
    return true;
  }
  return tc_mappable(L.gate, 1) && tc_mappable(L.up, 1) && tc_mappable(L.down, 1);
}

// The FFN of one layer for a step of many tokens: gate and up on the tensor cores, SwiGLU and the
// quantization of the activations, down on the tensor cores. Same results as launch_ffn.
bool launch_ffn_tc(const Dims& D, const DecodeBufs& B, const LayerDev& L, cudaStream_t st) {
  int sms = 148;
  tc_ready_here(&sms);
  const bool moe = L.moe != 0;
  const int fd = moe ? D.f : D.df, bslot = moe ? D.k + 1 : 1;
  const int nrouted = moe ? std::min(D.ne, B.T * D.k) : 0;
  const bool shared = moe ? D.nsh > 0 : true;
  if (!shared && nrouted == 0) return true;
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
  // the maps of all three projections first: a failure leaves the step to the dp4a kernels
  TcMaps mg0{}, mg1{}, mu0{}, mu1{}, md0{}, md1{};
  if (shared && (!tc_maps(moe ? L.sgate : L.gate, 1, &mg0) || !tc_maps(moe ? L.sup : L.up, 1, &mu0) ||
                 !tc_maps(moe ? L.sdown : L.down, 1, &md0)))
    return false;
  if (moe && (!tc_maps(L.gate, D.ne, &mg1) || !tc_maps(L.up, D.ne, &mu1) || !tc_maps(L.down, D.ne, &md1)))
    return false;
  auto up = [&](const Q8M& routed, const Q8M& grp0, const TcMaps& m0, const TcMaps& m1, float* out) {
    G.m0 = m0;
    G.m1 = m1;
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
  up(L.gate, moe ? L.sgate : L.gate, mg0, mg1, B.act);
  up(L.up, moe ? L.sup : L.up, mu0, mu1, B.ubuf);
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
  G.m0 = md0;
  G.m1 = md1;
  G.W = moe ? L.down : Q8M{};
  G.W0 = shared ? (moe ? L.sdown : L.down) : Q8M{};
  G.aq = B.qact;
  G.as = B.sact;
  G.in_nslot = bslot;
  G.out = B.y;
  G.out_nslot = D.k + 1;
  G.ostride = D.d;
  tc_launch(TC_OUT_STORE, G, tc_ctas(tiles * ((D.d + TC_M - 1) / TC_M), sms), B.T, st);
  return true;
}

bool kp_tc_usable(const MmArgs& a, int nrows_max, int groups) {
  return tc_ready_here(nullptr) && nrows_max >= TC_MIN_T && groups >= 1 && groups <= TC_MAX_GROUPS &&
         a.W.cols % 32 == 0 && a.W.cols >= 32 && a.W.ss % 4 == 0;
}

// the stacked matrices a launch may index: the grp tables' (up to `groups`) or a.mat
bool launch_kp_tc(const MmArgs& a, int nrows_max, int groups, int count, cudaStream_t st) {
  int sms = 148;
  tc_ready_here(&sms);
  KtArgs K{};
  if (!tc_maps(a.W, count, &K.m)) return false;
  K.a = a;
  K.ngroups = groups;
  const long long units = (long long)((a.W.rows + TC_M - 1) / TC_M) * groups * ((nrows_max + KT_TOK - 1) / KT_TOK);
  kp_tc<<<tc_ctas(units, sms), KT_THREADS, KT_SMEM, st>>>(K);
  return true;
}

}  // namespace hg
