// Expert parallelism for the decode step (ep.cu): the routed experts of every MoE layer are split
// across the ranks of an NCCL communicator; each rank decodes its own sequences and sends each
// (token, selected expert) row to the expert's owner and back (model.rs:295-324 semantics kept:
// the returned rows land in the token's rank slots and the rank-order combine runs unchanged).
#pragma once
#include <cuda_runtime.h>

#include "hg_model.cuh"

namespace hg {

struct EpCtx;

// Creates the communicator (rank of world; nccl_id: the 128-byte unique id every rank received
// from rank 0; every rank must call this, the call returns once all have joined) and the
// exchange buffers for steps of up to max_batch tokens. Throws Error(HG_ERR_INVALID) when
// n_experts is not a multiple of world, Error(HG_ERR_CUDA) when NCCL cannot be loaded or fails.
EpCtx* ep_create(const Dims& D, int max_batch, int device, const void* nccl_id, int rank, int world);
void ep_destroy(EpCtx* ep);
int ep_rank(const EpCtx* ep);
int ep_world(const EpCtx* ep);

// One MoE layer's FFN for the step's tokens (after the router): the shared expert locally, the
// routed experts through the two all-to-alls. Leaves B.y[t][0..k] exactly as launch_ffn does.
void ep_record_moe(EpCtx* ep, const Dims& D, const DecodeBufs& B, const LayerDev& Ld, cudaStream_t st);

// Fills out[128] with a new NCCL unique id (rank 0 calls this and shares the bytes).
void ep_unique_id(void* out);

}  // namespace hg
