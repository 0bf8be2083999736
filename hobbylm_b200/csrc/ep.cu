// Expert parallelism over NCCL (hg_ep.h).
//
// Placement: with E routed experts and W ranks, rank q owns experts [q E/W, (q+1) E/W). Every rank
// holds all weights (prefill runs locally) but a decode step computes only its own experts.
//
// Per MoE layer, after the router has chosen each local token's top-k:
//   k_ep_pack      each (token t, rank r) row -- the quantized ffn-normed hidden state the expert
//                  kernels read (d int8 + its per-32 scales) and the expert id -- goes to its
//                  owner's block of the send buffer; (t, r) is remembered per sent slot.
//   shared expert  computed locally into y[t][k] (launch_ffn_ex, group 0 only).
//   dispatch       one NCCL group of send/recv pairs, one fixed-size block per peer (the block's
//                  first word holds its row count), so the step stays one CUDA graph.
//   k_ep_unpack    received rows become "tokens" of an expert view of the step: their activations
//                  are copied into place and each row is entered in its expert's list.
//   experts        the owner's routed experts over all received rows (launch_ffn_ex, routed
//                  groups only), one output row per received row.
//   combine        the output rows travel back in the same slots.
//   k_ep_return    each returned row lands in y[t][r] of the token that sent it.
// The next layer's residual update then sums y[t][0..k-1] in rank order and adds y[t][k], as on one
// GPU, so expert parallelism changes no result: every row is computed by the same kernels with the
// same inputs.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "hg_ep.h"
#include "hg_host.h"
#include "hg_launch.h"

namespace hg {

namespace {

// NCCL is resolved at run time (the library torch loaded, else the system's), so the engine
// library needs no NCCL at load time and runs without it when expert parallelism is not used.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  static std::string why;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      why = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    auto sym = [&](const char* n) {
      void* p = dlsym(h, n);
      if (!p && why.empty()) why = std::string("libnccl.so.2 lacks ") + n;
      return p;
    };
    api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(sym("ncclGetUniqueId"));
    api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(sym("ncclCommInitRank"));
    api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(sym("ncclCommDestroy"));
    api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(sym("ncclGroupStart"));
    api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(sym("ncclGroupEnd"));
    api.Send = reinterpret_cast<decltype(api.Send)>(sym("ncclSend"));
    api.Recv = reinterpret_cast<decltype(api.Recv)>(sym("ncclRecv"));
    api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(sym("ncclGetErrorString"));
  });
  if (!why.empty()) throw Error(HG_ERR_CUDA, why);
  return api;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess)
    throw Error(HG_ERR_CUDA, std::string(what) + ": " + (nccl().GetErrorString ? nccl().GetErrorString(r) : "error"));
}

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error(HG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

constexpr int EP_HDR = 16;  // bytes before a peer block's rows: the row count

}  // namespace

struct EpCtx {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1, epr = 0, cap = 0, device = 0;
  size_t rb = 0;   // bytes per dispatched row: d int8, ss f32 scales, the expert id
  size_t blk = 0;  // bytes per peer block: header + cap rows
  unsigned char* send = nullptr;  // [world][blk]
  unsigned char* recv = nullptr;  // [world][blk]
  int32_t* cnt = nullptr;         // [world] rows sent to each peer in the current layer
  int32_t* sent = nullptr;        // [world][cap] t * 32 + r of each sent row
  int8_t* qh = nullptr;           // [world * cap][d] received activations
  float* sh = nullptr;            // [world * cap][ss]
  int32_t* ecount = nullptr;      // [ne + 2] entries per expert, then the active-expert count
  int32_t* active = nullptr;      // [ne]
  int32_t* elist = nullptr;       // [ne][world * cap]
  float* act = nullptr;           // [world * cap][f]
  float* y = nullptr;             // [world * cap][d] expert outputs of the received rows
  float* ret = nullptr;           // [world * cap][d] outputs of this rank's rows, returned
};

struct EpArgs {
  int epr, cap, world, ss;
  size_t rb, blk;
  unsigned char* send;
  const unsigned char* recv;
  int32_t* cnt;
  int32_t* sent;
  int8_t* qh;
  float* sh;
  int32_t* ecount;
  int32_t* active;
  int32_t* elist;
  const float* ret;
};

// one CTA per (token, rank) pair
__global__ void k_ep_pack(Dims D, DecodeBufs B, EpArgs E) {
  __shared__ int slot_s, peer_s;
  const int t = blockIdx.x / D.k, r = blockIdx.x - t * D.k;
  const int e = B.sel[t * D.k + r];
  if (threadIdx.x == 0) {
    const int p = e / E.epr;
    const int slot = atomicAdd(&E.cnt[p], 1);
    E.sent[p * E.cap + slot] = t * 32 + r;
    peer_s = p;
    slot_s = slot;
  }
  __syncthreads();
  unsigned char* row = E.send + (size_t)peer_s * E.blk + EP_HDR + (size_t)slot_s * E.rb;
  const int nq = D.d / 16, ns = E.ss / 4;
  for (int i = threadIdx.x; i < nq; i += blockDim.x)
    reinterpret_cast<int4*>(row)[i] = reinterpret_cast<const int4*>(B.qh + (size_t)t * D.d)[i];
  for (int i = threadIdx.x; i < ns; i += blockDim.x)
    reinterpret_cast<float4*>(row + D.d)[i] = reinterpret_cast<const float4*>(B.sh + (size_t)t * E.ss)[i];
  if (threadIdx.x == 0) *reinterpret_cast<int*>(row + D.d + E.ss * 4) = e;
}

// row counts into the block headers; the expert view's lists start empty
__global__ void k_ep_headers(Dims D, EpArgs E) {
  for (int p = threadIdx.x; p < E.world; p += blockDim.x) *reinterpret_cast<int*>(E.send + (size_t)p * E.blk) = E.cnt[p];
  for (int i = threadIdx.x; i < D.ne + 2; i += blockDim.x) E.ecount[i] = 0;
}

// one CTA per receive slot (peer p, row i)
__global__ void k_ep_unpack(Dims D, EpArgs E) {
  const int p = blockIdx.x / E.cap, i = blockIdx.x - p * E.cap;
  const unsigned char* blk = E.recv + (size_t)p * E.blk;
  if (i >= *reinterpret_cast<const int*>(blk)) return;
  const unsigned char* row = blk + EP_HDR + (size_t)i * E.rb;
  const int R = blockIdx.x;  // row index of the expert view
  const int nq = D.d / 16, ns = E.ss / 4;
  for (int j = threadIdx.x; j < nq; j += blockDim.x)
    reinterpret_cast<int4*>(E.qh + (size_t)R * D.d)[j] = reinterpret_cast<const int4*>(row)[j];
  for (int j = threadIdx.x; j < ns; j += blockDim.x)
    reinterpret_cast<float4*>(E.sh + (size_t)R * E.ss)[j] = reinterpret_cast<const float4*>(row + D.d)[j];
  if (threadIdx.x == 0) {
    const int e = *reinterpret_cast<const int*>(row + D.d + E.ss * 4);
    const int slot = atomicAdd(&E.ecount[e], 1);
    if (slot == 0) E.active[atomicAdd(&E.ecount[D.ne], 1)] = e;
    E.elist[(size_t)e * E.world * E.cap + slot] = R * 32;
  }
}

// one CTA per send slot (peer p, row i): the returned output into y[t][r]
__global__ void k_ep_return(Dims D, DecodeBufs B, EpArgs E) {
  const int p = blockIdx.x / E.cap, i = blockIdx.x - p * E.cap;
  if (i >= E.cnt[p]) return;
  const int code = E.sent[p * E.cap + i], t = code >> 5, r = code & 31;
  const float4* src = reinterpret_cast<const float4*>(E.ret + (size_t)blockIdx.x * D.d);
  float4* dst = reinterpret_cast<float4*>(B.y + ((size_t)t * (D.k + 1) + r) * D.d);
  for (int j = threadIdx.x; j < D.d / 4; j += blockDim.x) dst[j] = src[j];
}

void ep_unique_id(void* out) {
  ncclUniqueId id;
  nccl_check(nccl().GetUniqueId(&id), "ncclGetUniqueId");
  static_assert(sizeof(id) == 128, "NCCL unique ids are 128 bytes");
  std::memcpy(out, &id, sizeof(id));
}

EpCtx* ep_create(const Dims& D, int max_batch, int device, const void* nccl_id, int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world) throw Error(HG_ERR_INVALID, "bad rank / world");
  if (D.ne <= 0 || D.ne % world != 0) throw Error(HG_ERR_INVALID, "n_experts must be a multiple of the world size");
  if (D.d % 16 != 0) throw Error(HG_ERR_INVALID, "d_model must be a multiple of 16");
  const NcclApi& api = nccl();
  EpCtx* ep = new EpCtx();
  try {
    ep->rank = rank;
    ep->world = world;
    ep->epr = D.ne / world;
    ep->cap = max_batch * D.k;  // a step's (token, rank) pairs, the most any one peer can receive
    ep->device = device;
    const int ss = host_q8_ss(D.d), rows = world * ep->cap;
    ep->rb = ((size_t)D.d + (size_t)ss * 4 + 4 + 15) & ~size_t(15);
    ep->blk = ((EP_HDR + (size_t)ep->cap * ep->rb) + 255) & ~size_t(255);
    cuda_check(cudaSetDevice(device), "cudaSetDevice");
    auto alloc = [&](auto*& ptr, size_t bytes) { cuda_check(cudaMalloc((void**)&ptr, bytes), "cudaMalloc (expert parallel)"); };
    alloc(ep->send, world * ep->blk);
    alloc(ep->recv, world * ep->blk);
    alloc(ep->cnt, (size_t)world * 4);
    alloc(ep->sent, (size_t)rows * 4);
    alloc(ep->qh, (size_t)rows * D.d);
    alloc(ep->sh, (size_t)rows * ss * 4);
    alloc(ep->ecount, (size_t)(D.ne + 2) * 4);
    alloc(ep->active, (size_t)D.ne * 4);
    alloc(ep->elist, (size_t)D.ne * rows * 4);
    alloc(ep->act, (size_t)rows * D.f * 4);
    alloc(ep->y, (size_t)rows * D.d * 4);
    alloc(ep->ret, (size_t)rows * D.d * 4);
    cuda_check(cudaMemset(ep->send, 0, world * ep->blk), "cudaMemset");
    cuda_check(cudaMemset(ep->recv, 0, world * ep->blk), "cudaMemset");
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof(id));
    nccl_check(api.CommInitRank(&ep->comm, world, id, rank), "ncclCommInitRank");
  } catch (...) {
    ep_destroy(ep);
    throw;
  }
  return ep;
}

void ep_destroy(EpCtx* ep) {
  if (!ep) return;
  cudaSetDevice(ep->device);
  if (ep->comm) nccl().CommDestroy(ep->comm);
  for (void* p : {(void*)ep->send, (void*)ep->recv, (void*)ep->cnt, (void*)ep->sent, (void*)ep->qh, (void*)ep->sh,
                  (void*)ep->ecount, (void*)ep->active, (void*)ep->elist, (void*)ep->act, (void*)ep->y, (void*)ep->ret})
    if (p) cudaFree(p);
  delete ep;
}

int ep_rank(const EpCtx* ep) { return ep ? ep->rank : 0; }
int ep_world(const EpCtx* ep) { return ep ? ep->world : 1; }

void ep_record_moe(EpCtx* ep, const Dims& D, const DecodeBufs& B, const LayerDev& Ld, cudaStream_t st) {
  const NcclApi& api = nccl();
  EpArgs E{};
  E.epr = ep->epr;
  E.cap = ep->cap;
  E.world = ep->world;
  E.ss = host_q8_ss(D.d);
  E.rb = ep->rb;
  E.blk = ep->blk;
  E.send = ep->send;
  E.recv = ep->recv;
  E.cnt = ep->cnt;
  E.sent = ep->sent;
  E.qh = ep->qh;
  E.sh = ep->sh;
  E.ecount = ep->ecount;
  E.active = ep->active;
  E.elist = ep->elist;
  E.ret = ep->ret;
  // the shared expert of the local tokens (y[t][k])
  launch_ffn_ex(D, B, Ld, true, 0, st);
  // dispatch
  cuda_check(cudaMemsetAsync(ep->cnt, 0, (size_t)ep->world * 4, st), "cudaMemsetAsync");
  k_ep_pack<<<B.T * D.k, 64, 0, st>>>(D, B, E);
  k_ep_headers<<<1, 64, 0, st>>>(D, E);
  nccl_check(api.GroupStart(), "ncclGroupStart");
  for (int p = 0; p < ep->world; p++) {
    nccl_check(api.Send(ep->send + p * ep->blk, ep->blk, ncclInt8, p, ep->comm, st), "ncclSend");
    nccl_check(api.Recv(ep->recv + p * ep->blk, ep->blk, ncclInt8, p, ep->comm, st), "ncclRecv");
  }
  nccl_check(api.GroupEnd(), "ncclGroupEnd");
  const int rows = ep->world * ep->cap;
  k_ep_unpack<<<rows, 64, 0, st>>>(D, E);
  // this rank's routed experts over every received row: an expert view of the step in which each
  // received row is a token with one slot (k = 0) and no shared expert
  Dims De = D;
  De.k = 0;
  De.nsh = 0;
  DecodeBufs Be = B;
  Be.T = rows;
  Be.qh = ep->qh;
  Be.sh = ep->sh;
  Be.ecount = ep->ecount;
  Be.active = ep->active;
  Be.elist = ep->elist;
  Be.act = ep->act;
  Be.act_stride = D.f;
  Be.y = ep->y;
  launch_ffn_ex(De, Be, Ld, false, ep->epr, st);
  // combine: each peer's output rows go back in the slots they came in
  nccl_check(api.GroupStart(), "ncclGroupStart");
  for (int p = 0; p < ep->world; p++) {
    const size_t off = (size_t)p * ep->cap * D.d;
    nccl_check(api.Send(ep->y + off, (size_t)ep->cap * D.d, ncclFloat32, p, ep->comm, st), "ncclSend");
    nccl_check(api.Recv(ep->ret + off, (size_t)ep->cap * D.d, ncclFloat32, p, ep->comm, st), "ncclRecv");
  }
  nccl_check(api.GroupEnd(), "ncclGroupEnd");
  k_ep_return<<<rows, 128, 0, st>>>(D, B, E);
}

}  // namespace hg
