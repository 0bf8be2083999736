/*
 * hobbygpu — B200 (sm_100a) decode engine for hobbylm GGUF models (the hobby-rs decode path).
 *
 * C ABI. Conventions:
 *   - every function returning int returns HG_OK (0) or a negative HG_ERR_* code; the message of
 *     the last failure on the calling thread is hg_last_error();
 *   - the caller owns every host buffer it passes; the engine owns all device memory it allocates;
 *   - one CUDA stream per engine: calls on one engine must be serialized by the caller (distinct
 *     hg_seq objects may be used from different threads as long as calls do not overlap);
 *   - "_op_" functions are the kernel-level seams: they take DEVICE pointers and a cudaStream_t
 *     passed as void* (NULL = legacy default stream) and do not synchronize.
 *
 * The reference (harishsg993010/HobbyLM, hobby-rs) is a Rust crate with no FFI; each entry point
 * below names the Rust item (file:line) whose behaviour it takes over. A Rust caller binds them
 * with an `extern "C"` block.
 */
#ifndef HOBBYGPU_H
#define HOBBYGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  HG_OK = 0,
  HG_ERR_INVALID = -1,        /* bad argument (null pointer, size out of range) */
  HG_ERR_IO = -2,             /* cannot open / map the GGUF file */
  HG_ERR_FORMAT = -3,         /* bad magic, unsupported version, truncated file, bad tensor */
  HG_ERR_MISSING = -4,        /* missing tensor or required metadata key */
  HG_ERR_CUDA = -5,           /* CUDA runtime error */
  HG_ERR_POOL_EXHAUSTED = -6, /* KV page pool has no free pages */
  HG_ERR_CONTEXT = -7,        /* position would reach the sequence's max context */
  HG_ERR_TOKEN = -8,          /* token id >= vocab size */
  HG_ERR_TIMEOUT = -9         /* a device-side bounded wait gave up */
};

typedef struct hg_engine hg_engine;
typedef struct hg_seq hg_seq;

/* Model hyper-parameters read from GGUF metadata, same keys and defaults as
 * Config::from_gguf (hobby-rs/src/config.rs:35-98). */
typedef struct {
  int32_t d_model, n_layers, n_dense, n_heads, n_kv_heads, head_dim, dense_ffn, expert_ffn;
  int32_t n_experts, top_k, n_shared, vocab_size, context_length;
  int32_t expert_weights_norm, gating_sigmoid, eos_token;
  float rms_eps, rope_theta, expert_weights_scale;
  /* diffusion.enabled (default 0), diffusion.mask_token_id (50257), diffusion.block_size (32):
   * config.rs:92-94, keys without the architecture prefix */
  int32_t diffusion, mask_token_id, block_size;
} hg_config;

/* Engine options (zero-initialised = defaults). */
typedef struct {
  int32_t device;              /* CUDA device ordinal */
  int32_t max_batch;           /* largest hg_decode_batch size (default 1) */
  int64_t kv_pool_tokens;      /* KV page pool capacity in tokens (default 2 * context_length) */
  uint64_t kv_page_shuffle;    /* nonzero: hand out pool pages in a seeded random order */
} hg_engine_opts;

/* Generation options, GenOpts (hobby-rs/src/lib.rs:29-41). temp <= 0 is greedy. */
typedef struct {
  int32_t max_new;
  float temp, top_p;
  uint64_t seed;
  float rep_penalty;
} hg_gen_opts;

/* Streaming callback: receives each generated token id; return 0 to stop (lib.rs:152). */
typedef int (*hg_token_cb)(uint32_t token, void* user);

/* Diffusion decode options, DiffOpts (lib.rs:43-63); NULL = DiffOpts::default(). block <= 0 takes
 * the model's diffusion.block_size (main.rs:174). threshold > 0 selects the confidence-threshold
 * schedule of the cached path; otherwise `steps` passes spread over gen_len (lib.rs:304-354). */
typedef struct {
  int32_t gen_len, block, steps;
  float temp, rep_penalty;
  int32_t remask_steps;
  float remask_frac;
  uint64_t seed;
  int32_t cached;
  float threshold;
} hg_diff_opts;

/* Diffusion streaming callback, called once per finished block with the ids it adds before the
 * first eos (lib.rs:393-405, in ids instead of text; n may be 0); return 0 to stop. */
typedef int (*hg_block_cb)(const uint32_t* ids, int n, void* user);

const char* hg_last_error(void);

/* Engine::load (hobby-rs/src/lib.rs:85-92) with quant = true: parses the GGUF, re-quantizes every
 * weight matrix to int8 + f32 per-32 scales exactly as Model::load / Q8Tensor::quantize
 * (model.rs:79-131, quant.rs:78-102) and uploads it to HBM once. */
int hg_engine_load(const char* gguf_path, int device, hg_engine** out);
int hg_engine_load_ex(const char* gguf_path, const hg_engine_opts* opts, hg_engine** out);
void hg_engine_free(hg_engine* e);
int hg_engine_config(const hg_engine* e, hg_config* out);
/* Config::from_gguf alone: parse a GGUF file's header + metadata (no GPU needed). */
int hg_gguf_config(const char* gguf_path, hg_config* out);
/* Gguf::load (gguf.rs:250-269): tensor `name` of a GGUF file as f32 on the host (F32 copied; F16,
 * Q5_0, Q8_0, Q4_K and Q6_K dequantized as gguf.rs:329-468 does). n is the element count of out
 * and must equal the tensor's (HG_ERR_INVALID otherwise); a missing tensor is HG_ERR_MISSING and
 * an unsupported type HG_ERR_FORMAT. No GPU work. */
int hg_gguf_tensor_f32(const char* gguf_path, const char* name, float* out, int64_t n);
/* Engine::weight_bytes (lib.rs:100-102): bytes of all re-quantized matmul weights (int8 + f32 scales). */
uint64_t hg_engine_weight_bytes(const hg_engine* e);
/* Engine::eos (lib.rs:94-96). */
uint32_t hg_engine_eos(const hg_engine* e);
/* Device bytes held by the engine (weights, KV pool, work buffers). */
uint64_t hg_engine_device_bytes(const hg_engine* e);

/* KvCache::new (model.rs:66-75): a sequence with room for max_ctx positions (<= context_length),
 * backed by pages of the engine's pool. */
int hg_seq_create(hg_engine* e, int max_ctx, hg_seq** out);
/* Returns the sequence's pages to its engine. A sequence still open when its engine is freed loses
 * its pages with the engine; hg_seq_free is then the only call it may still be passed to. */
void hg_seq_free(hg_seq* s);
int hg_seq_len(const hg_seq* s);

/* Model::prefill (model.rs:340-370) on token ids: embeds, runs all positions with the prefill
 * arithmetic, appends K/V and writes the last position's vocab logits (may be NULL). */
int hg_prefill(hg_engine* e, hg_seq* s, const uint32_t* ids, int n, float* logits_or_null);
/* Model::prefill (model.rs:340-370) on caller rows: n initial residual vectors of d_model floats
 * (host memory, row-major), e.g. modality embeddings spliced before a prompt's token embeddings
 * (lib.rs:118-121: prefill the embeddings, then the prompt ids with hg_prefill on the same
 * sequence; chunked prefill equals one prefill over all rows). logits as for hg_prefill. */
int hg_prefill_embeds(hg_engine* e, hg_seq* s, const float* embeds, int n, float* logits_or_null);

/* Model::forward (model.rs:152-184): one decode step of `token` at position hg_seq_len(s).
 * logits_or_null receives the raw vocab logits; argmax_or_null the greedy pick with ids >= 50257
 * masked (lib.rs:127-134, sample.rs:53-64). */
int hg_forward(hg_engine* e, hg_seq* s, uint32_t token, float* logits_or_null, uint32_t* argmax_or_null);
/* Model::forward_x (model.rs:160-184): one decode step from a caller row of d_model floats (host
 * memory) in place of a token embedding, e.g. a modality vector fed during decode. logits and
 * argmax as for hg_forward. */
int hg_forward_x(hg_engine* e, hg_seq* s, const float* row, float* logits_or_null, uint32_t* argmax_or_null);

/* One batched decode step: seqs[i] consumes tokens[i]; next_ids[i] gets its greedy pick.
 * Per sequence the result equals hg_forward. n <= max_batch. */
int hg_decode_batch(hg_engine* e, hg_seq** seqs, int n, const uint32_t* tokens, uint32_t* next_ids,
                    float* logits_or_null);

/* `steps` greedy decode steps for n sequences driven on the device: each step's masked argmax is
 * fed back as the sequence's next token without a host round trip (the multi-token form of the
 * lib.rs:131-160 loop with temp = 0, without the EOS stop). tokens: the first step's inputs;
 * out_ids (may be NULL): [steps][n] generated ids. */
int hg_decode_greedy(hg_engine* e, hg_seq** seqs, int n, const uint32_t* tokens, int steps, uint32_t* out_ids);

/* The engine's CUDA stream (a cudaStream_t), for callers that order or time work around it. */
void* hg_engine_stream(const hg_engine* e);

/* No counterpart in the reference (hobby-rs runs every expert in one process). Expert
 * parallelism for batched decode on several GPUs: each rank (one process, one engine per GPU)
 * decodes its own sequences, and the routed experts of every MoE layer are split evenly across the
 * ranks (rank q owns experts [q E/W, (q+1) E/W)). A step sends each (token, selected expert) row to
 * the expert's owner and the expert's output back over NCCL (two grouped send/recv exchanges per
 * MoE layer, inside the step's CUDA graph); the shared expert and attention stay local. Results
 * equal the one-GPU engine's bit for bit. hg_ep_unique_id fills out[128] with a new NCCL unique
 * id; rank 0 makes one and gives the bytes to every rank (e.g. over torch.distributed), and each
 * rank calls hg_engine_ep_init once, before its first decode step; the call returns when all
 * `world` ranks have joined. Afterwards every rank must take its decode steps (hg_decode_batch /
 * hg_decode_greedy / hg_forward) in lockstep: each step's exchanges pair up across ranks. n_experts
 * must be a multiple of world (HG_ERR_INVALID otherwise); HG_ERR_CUDA if NCCL cannot be loaded. */
int hg_ep_unique_id(void* out);
int hg_engine_ep_init(hg_engine* e, const void* nccl_id, int rank, int world);

/* Kernels one decode step of batch size n launches (kernel nodes of its CUDA graph), or < 0. */
int hg_decode_kernel_count(hg_engine* e, int n);

/* Device time in ms (CUDA events on the engine stream, mean over iters) of the attention kernels
 * of one decode step of the last layer for these sequences, re-run on their current state (each
 * must have decoded at least one step; the K/V append rewrites the same row): ms_scores covers the
 * q/k preparation and the scores, ms_out the softmax and the value sums. */
int hg_debug_time_attention(hg_engine* e, hg_seq** seqs, int n, int iters, float* ms_scores, float* ms_out);

/* Engine::generate (lib.rs:107-162) on token ids: prefill, then per step mask ids >= 50257,
 * sample (greedy when temp <= 0), stop on EOS, stream the id, stop at context_length.
 * The sample is drawn on the GPU from the step's logits (temperature, top-p, repetition penalty,
 * the xorshift64* state of opts->seed kept on the device) with the same ids as sample.rs; only
 * the id is read back per step. out_ids (may be NULL) receives up to opts->max_new ids. Returns
 * the count (>= 0) or an error. */
int hg_generate(hg_engine* e, const uint32_t* ids, int n, const hg_gen_opts* opts, hg_token_cb cb, void* user,
                uint32_t* out_ids);
/* Engine::generate (lib.rs:107-162) with `embeds`: n_embeds caller rows of d_model floats (host
 * memory, e.g. modality vectors) precede the prompt ids' embeddings in the prefill
 * (lib.rs:118-121); either part may be empty. Otherwise as hg_generate. */
int hg_generate_embeds(hg_engine* e, const float* embeds, int n_embeds, const uint32_t* ids, int n,
                       const hg_gen_opts* opts, hg_token_cb cb, void* user, uint32_t* out_ids);

/* Model::run_block (model.rs:472-510): n token ids at positions hg_seq_len(s).. attend to the
 * sequence's prefix and to every one of the n rows (bidirectional within the block), with the
 * prefill arithmetic. The block's K/V rows are written past the sequence's length; commit != 0
 * appends them to it (lib.rs:386-391), otherwise the length is unchanged and the next call at the
 * same position overwrites them. logits_or_null: [n_logits][vocab] of the last n_logits rows
 * (0 <= n_logits <= n) through the lm_head matmul (model.rs:505-508). On a sequence of length 0
 * the logits are those of Model::forward_bidir (model.rs:441-470). n <= 1024 per call. */
int hg_run_block(hg_engine* e, hg_seq* s, const uint32_t* ids, int n, int n_logits, int commit,
                 float* logits_or_null);

/* Engine::generate_diffusion (lib.rs:211-495) on token ids: the prefix-cached path (the prompt
 * encoded bidirectionally, each denoising pass re-running only the active block) or, with
 * cached = 0, the uncached path (every pass re-runs the canvas). The [MASK] id is the model's
 * diffusion.mask_token_id; ids >= 50257 are never emitted. out_ids (may be NULL) receives up to
 * gen_len ids. Returns the generated count (>= 0) or an error. The prompt (cached) or the canvas
 * (uncached) holds at most 1024 positions. */
int hg_generate_diffusion(hg_engine* e, const uint32_t* ids, int n, const hg_diff_opts* opts, hg_block_cb cb,
                          void* user, uint32_t* out_ids);

/* Debug: expert ids selected at every MoE layer by the last decode step of sequence slot `slot`
 * of the last hg_forward / hg_decode_batch ([n_layers][top_k], -1 for dense layers). */
int hg_debug_last_routing(hg_engine* e, int slot, int32_t* sel);

/* ---- host-side weight packing (the load-time re-quantization, usable without a GPU) ---- */

/* Q8Tensor::quantize (quant.rs:78-102) of a row-major f32 [rows][cols] matrix into the device
 * layout: qs_out [rows][cols] int8 in the lane-chunked order (for 32-blocks 4c..4c+3 of a row, byte
 * c*128 + l*16 + (b%4)*4 + j holds element 32b + 4l + j; the blocks b >= 4nc, nc = cols / 128,
 * follow as nc*128 + (b-4nc)*32 + l*4 + j), scales_out [rows][scale_stride] f32 with scale_stride = hg_q8_scale_stride(cols). */
int hg_q8_pack(const float* w, int64_t rows, int64_t cols, int8_t* qs_out, float* scales_out);
int hg_q8_scale_stride(int64_t cols);
/* Inverse of the lane-chunked byte permutation (for tests): packed row bytes -> reference order. */
int hg_q8_unpack_qs(const int8_t* packed, int64_t rows, int64_t cols, int8_t* qs_out);

/* ---- host-side token selection over logits in host memory (no GPU work) ---- */

/* sample.rs:66-112 over n logits (temp <= 0: the first-max argmax, sample.rs:53-64): softmax of
 * logits / temp, the top-p prefix (probabilities descending, ties by id) when 0 < top_p < 1, one
 * draw. *rng_state is the xorshift64* state (sample.rs:3-22; start it at the seed) and is advanced. */
int hg_host_sample(const float* logits, int n, float temp, float top_p, uint64_t* rng_state, uint32_t* out);
/* The diffusion block scoring of lib.rs:221-263 over blk_len rows of vocab logits: ids >= 50257
 * banned, the presence penalty over the committed ids and the block's non-mask ids, the pick
 * (Gumbel-max at temp > 0, sample.rs:29-47, drawing from *rng_state row after row) and the
 * softmax probabilities of the pick (pconf) and of the row's current id (cconf). */
int hg_host_score_block(const float* logits, int vocab, const uint32_t* blk, int blk_len, const uint32_t* committed,
                        int n_committed, uint32_t mask, float rep_penalty, float temp, uint64_t* rng_state,
                        uint32_t* pred, float* pconf, float* cconf);

/* ---- kernel-level ops (device pointers) ---- */

/* Q8Tensor::matvec (quant.rs:106-136) for ntok activation rows: y[t][r] = row r of the packed
 * matrix . x[t] with x[t] quantized per 32-block (quant.rs:112-123) and the AVX2 lane order
 * (quant.rs:44-67). x: [ntok][cols] f32, y: [ntok][rows] f32. */
int hg_op_q8_matvec(const int8_t* qs, const float* scales, int64_t rows, int64_t cols, const float* x, float* y,
                    int ntok, void* stream);

/* No counterpart in the reference. The same computation as hg_op_q8_matvec, for callers that
 * cannot allocate device memory: for example a host framework that has already handed all free
 * device memory to its own pool, or a serving thread that must not block on the driver's
 * allocation calls. hg_op_q8_matvec allocates its activation scratch on the stream; this variant
 * uses a fixed HG_NOALLOC_SCRATCH_BYTES device array compiled into the library instead (every GPU
 * that loads the library holds it until the process exits) and makes no allocation call. Sizes
 * whose scratch (ntok * cols bytes + ntok * hg_q8_scale_stride(cols) * 4, rounded up) exceed it
 * are rejected with HG_ERR_INVALID. All calls share the array: calls that overlap on the GPU
 * race and must be ordered by the caller. The first call on a device looks up the array's device
 * address with that device current; make that first call before any stream capture. The address
 * is cached for the device's primary context: do not call this after cudaDeviceReset on a device
 * that has already used it. rows and cols above INT_MAX are rejected with HG_ERR_INVALID. */
#define HG_NOALLOC_SCRATCH_BYTES (4u << 20)
int hg_op_q8_matvec_noalloc(const int8_t* qs, const float* scales, int64_t rows, int64_t cols, const float* x,
                            float* y, int ntok, void* stream);

/* Q8Tensor::matmul (quant.rs:144-193): the prefill arithmetic (block-sequential mul-add). */
int hg_op_q8_matmul(const int8_t* qs, const float* scales, int64_t rows, int64_t cols, const float* x, float* y,
                    int ntok, void* stream);

/* Ffn::Moe of one layer (model.rs:256-324) for ntok tokens, decode arithmetic per token:
 * f32 router (ops::dot order), sigmoid, +bias, top-k by descending score, routed SwiGLU experts
 * combined in rank order, then the shared expert. Packed expert stacks are [E][rows][...]. */
typedef struct {
  int32_t d_model, expert_ffn, n_experts, top_k, n_shared, gating_sigmoid, weights_norm;
  float weights_scale;
  const float* router;       /* [n_experts][d_model] f32 */
  const float* bias;         /* [n_experts] f32 */
  const int8_t* gate_qs;     /* [E][f][d] packed */
  const float* gate_sc;      /* [E][f][scale_stride(d)] */
  const int8_t* up_qs;
  const float* up_sc;
  const int8_t* down_qs;     /* [E][d][f] packed */
  const float* down_sc;      /* [E][d][scale_stride(f)] */
  const int8_t* sh_gate_qs;  /* shared expert (ignored when n_shared == 0) */
  const float* sh_gate_sc;
  const int8_t* sh_up_qs;
  const float* sh_up_sc;
  const int8_t* sh_down_qs;
  const float* sh_down_sc;
} hg_moe_weights;

/* x: [ntok][d] f32 (the normed hidden state), y: [ntok][d] f32, sel_out (may be NULL): [ntok][top_k]
 * int32 expert ids in rank order. scratch: device buffer of hg_op_moe_scratch_bytes() bytes. */
size_t hg_op_moe_scratch_bytes(const hg_moe_weights* w, int ntok);
int hg_op_moe_ffn(const hg_moe_weights* w, const float* x, int ntok, float* y, int32_t* sel_out, void* scratch,
                  void* stream);

/* KV append + GQA decode attention for one layer (model.rs:199-233) over a paged f32 pool.
 * Pages hold 16 positions; page p of a sequence's block table stores K at
 * k_pool + page * page_stride + kvh * 16 * head_dim (16 rows of head_dim floats) and V likewise at
 * v_pool. qkv: [n_seqs][q_dim + 2 kv_dim] pre-norm projections of the new token at pos[i].
 * The new K/V are QK-normed, roped, appended; out: [n_seqs][q_dim] attention outputs. */
typedef struct {
  int32_t n_seqs, n_heads, n_kv_heads, head_dim, max_pos;
  float eps;
  const float* qkv;
  const float* q_norm;       /* [head_dim] */
  const float* k_norm;       /* [head_dim] */
  const float* rope_cos;     /* [max_pos][head_dim/2] (Rope::new tables) */
  const float* rope_sin;
  const int32_t* pos;        /* [n_seqs] */
  const int32_t* block_table;/* [n_seqs][bt_stride] page ids */
  int32_t bt_stride;
  float* k_pool;
  float* v_pool;
  int64_t page_stride;       /* floats between consecutive pages */
  float* out;
} hg_kv_attn_args;

size_t hg_op_kv_attn_scratch_bytes(const hg_kv_attn_args* a);
int hg_op_kv_attn(const hg_kv_attn_args* a, void* scratch, void* stream);

/* Rope::new tables (ops.rs:139-154), computed on the host in f64: cos/sin [max_pos][head_dim/2]. */
int hg_rope_tables(int head_dim, int max_pos, float theta, float* cos_out, float* sin_out);

#ifdef __cplusplus
}
#endif
#endif /* HOBBYGPU_H */
