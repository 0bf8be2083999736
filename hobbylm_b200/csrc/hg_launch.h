// Host-callable kernel launchers (decode.cu, prefill.cu).
#pragma once
#include <cuda_runtime.h>

#include "hg_model.cuh"

namespace hg {

// decode.cu
void launch_mv_store(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* out,
                     int ostride, cudaStream_t st);
void launch_mv_resid(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as,
                     cudaStream_t st);
void launch_lmhead(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* logits,
                   cudaStream_t st);
void launch_pre_norm(const Dims& D, const DecodeBufs& B, int mode, const float* embd, const float* norm_w,
                     int8_t* q_out, float* s_out, float* h_out, int reset_moe, int reset_amax, cudaStream_t st);
void launch_route(const Dims& D, const DecodeBufs& B, const LayerDev& L, int layer, int prenormed, cudaStream_t st);
void launch_ffn(const Dims& D, const DecodeBufs& B, const LayerDev& L, cudaStream_t st);
// group0: run the shared expert / dense FFN group; nrouted: routed-expert groups (slots of the
// active-expert list B.active, counted in B.ecount[D.ne])
void launch_ffn_ex(const Dims& D, const DecodeBufs& B, const LayerDev& L, bool group0, int nrouted, cudaStream_t st);
void launch_moe_combine(const Dims& D, const DecodeBufs& B, float* y_out, cudaStream_t st);
void launch_quant_rows(const float* x, int rows, int cols, int8_t* q, float* s, cudaStream_t st);
cudaError_t launch_attn_args(const AttnArgs& A, cudaStream_t st);
cudaError_t prepare_attn(int hd, int rep);
cudaError_t launch_attn_scores_only(const AttnArgs& A, cudaStream_t st);
cudaError_t launch_attn_out_only(const AttnArgs& A, cudaStream_t st);
void launch_feedback(const DecodeBufs& B, int32_t* tok, int32_t* pos, int32_t* gen, int gen_cap, int32_t* step,
                     cudaStream_t st);

// tc.cu: the tcgen05 Q8 matvec for steps of at least TC_MIN_T tokens (rows of 128-byte lane chunks)
constexpr int TC_MIN_T = 32;
cudaError_t prepare_tc();
bool tc_usable(const Q8M& W, int T);
// false (nothing launched) when the weights cannot be described by a tensor map
bool launch_mv_tc(const Dims& D, const DecodeBufs& B, const Q8M& W, const int8_t* aq, const float* as, float* out,
                  int ostride, int epi, cudaStream_t st);
// the FFN of a layer on the tensor cores (gate, up, SwiGLU + quantization, down); needs B.ubuf,
// B.qact and B.sact
bool ffn_tc_usable(const Dims& D, const DecodeBufs& B, const LayerDev& L);
bool launch_ffn_tc(const Dims& D, const DecodeBufs& B, const LayerDev& L, cudaStream_t st);
// the prefill-order matmul (MmArgs) on the tensor cores, for at least TC_MIN_T activation rows
bool kp_tc_usable(const MmArgs& a, int nrows_max, int groups);
// count: matrices of the stack a.W the launch may index (tensor-map extent)
bool launch_kp_tc(const MmArgs& a, int nrows_max, int groups, int count, cudaStream_t st);

// sample.cu: Engine::generate's sampled tokens on the GPU (temperature, top-p, repetition penalty,
// xorshift64*), bit-identical to the host sampler; the scratch keeps the history counts and the
// RNG state between calls of one generate
bool sample_usable(int V);
size_t sample_scratch_bytes(int V);
void sample_reset(void* scratch, int V, unsigned long long seed, cudaStream_t st, unsigned long long* h_state);
void launch_sample(const float* logits, int V, int valid, float temp, float top_p, float rep_penalty, void* scratch,
                   cudaStream_t st);
uint32_t* sample_next_ptr(void* scratch);

// prefill.cu
void launch_kp_norm(float* in, const float* add, int rows, int d, const float* w, float eps, float* h_out, int8_t* q,
                    float* s, cudaStream_t st);
void launch_kp_matmul(const MmArgs& a, int nrows_max, int groups, cudaStream_t st);
void launch_kp_qk_rope_append(const float* qkv, int rows, int base, int nh, int nkv, int hd, float eps,
                              const float* q_norm, const float* k_norm, const float* rcos, const float* rsin,
                              const int32_t* bt, float* k_pool, float* v_pool, long long page_stride, float* qo,
                              cudaStream_t st);
// nfix = 0: causal rows (query t sees keys 0..base+t); nfix > 0: every row sees keys 0..nfix-1.
void launch_kp_attention(const float* q, int qd, int t0, int tq, int base, int nfix, int nh, int nkv, int hd,
                         const int32_t* bt, const float* k_pool, const float* v_pool, long long page_stride, float* S,
                         float* inv, uint32_t* mkey, float* o, cudaStream_t st);
void launch_kp_route(const float* h, int tn, int d, const float* router, const float* bias, int ne, int k, int gsig,
                     int wnorm, float wscale, int32_t* sel, float* selw, int32_t* ecount, int32_t* elist, int list_cap,
                     cudaStream_t st);
void launch_kp_expert_tables(const int32_t* ecount, int ne, int list_cap, int32_t* grp_mat, int32_t* grp_off,
                             int32_t* grp_cnt, cudaStream_t st);
void launch_kp_shared_rows(int tn, int k, int32_t* o_idx, cudaStream_t st);
void launch_kp_entry_rows(const int32_t* elist, int n, int k, int32_t* a_idx, int32_t* o_idx, cudaStream_t st);
void launch_kp_swiglu(const float* g, const float* u, float* act, long long n, cudaStream_t st);
void launch_kp_quant_rows(const float* x, long long rows, int cols, int8_t* q, float* s, cudaStream_t st);
void launch_kp_combine(float* x, const float* y, const int32_t* sel, const float* selw, int tn, int d, int k, int moe,
                       int n_shared, cudaStream_t st);
void launch_kp_embed(const float* embd, const int32_t* ids, int n, int d, int vocab, float* x, int32_t* err,
                     cudaStream_t st);

inline MmArgs mm_args(const Q8M& W, const int8_t* aq, const float* as, int n, float* out, int ostride, int mode) {
  MmArgs a{};
  a.W = W;
  a.mat = 0;
  a.aq = aq;
  a.as = as;
  a.nrows = n;
  a.out = out;
  a.ostride = ostride;
  a.mode = mode;
  return a;
}

}  // namespace hg
