/*
 * b2engine.h -- C-ABI boundary of the B200-native (sm_100a) per-token forward
 * path.  Every entry point takes plain device pointers, sizes and a CUDA
 * stream (as void*), never allocates or synchronises unless its comment says
 * so, and returns a status: 0 on success, a cudaError_t value (> 0) when CUDA
 * reported an error, or one of the negative B2_ERR_* codes below.
 *
 * Each entry point names the reference interface it replaces
 * (XVX-016/serving-engine, paths relative to that project).  The reference's
 * C++ signatures (namespace engine::cuda, void returns, exceptions on error)
 * are kept as inline wrappers over this layer in serving-engine_b200/compat
 * (src/cuda/kernels.h, src/cuda/kv_view.h, src/runtime/sampler.h,
 * src/runtime/kv_cache.h) so that its callers build unchanged.
 *
 * Element types: "half" is IEEE fp16, "bf16" is bfloat16, "float" is fp32.
 */
#ifndef B2ENGINE_H
#define B2ENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    B2_OK = 0,
    B2_ERR_INVALID = -1,     /* bad argument (null pointer, non-positive size, ...) */
    B2_ERR_UNSUPPORTED = -2, /* shape or alignment this build does not handle */
    B2_ERR_WORKSPACE = -3,   /* caller-provided scratch too small */
    B2_ERR_NCCL = -4,        /* NCCL call failed */
    B2_ERR_STATE = -5,       /* object used in the wrong state */
    B2_ERR_TIMEOUT = -6      /* a bounded device-side wait gave up */
};

/* Human-readable text for a status value (static storage). */
const char* b2_status_string(int status);
/* Detail text of the last failure a call on this host thread recorded (for
 * instance NCCL's own message when B2_ERR_NCCL is returned); "" if none. */
const char* b2_last_error(void);
/* Build identification, e.g. "b2engine 0.1 sm_100a". */
const char* b2_version(void);

/* Synchronises the current device and reports whether a bounded device-side
 * wait of a tensor-core kernel gave up since the last clear: B2_OK, or
 * B2_ERR_TIMEOUT (its pipeline stalled; the kernel skipped its remaining work
 * and exited).  clear != 0 resets the record.  No reference counterpart: the
 * reference's kernels have no device-side waits. */
int b2_device_status(int clear);

/* Strided view over a K or V cache: element (b, h, s, d) lives at
 * data + b*stride_b + h*stride_h + s*stride_s + d*stride_d (elements of half).
 * Replaces engine::cuda::KVView (src/cuda/kv_view.h:17-31). stride_d must be 1. */
typedef struct b2_kv_view {
    const void* data;
    int64_t stride_b;
    int64_t stride_h;
    int64_t stride_s;
    int64_t stride_d;
} b2_kv_view;

/* ---------------------------------------------------------------------------
 * Operator API (one entry per engine::cuda function, src/cuda/kernels.h)
 * ------------------------------------------------------------------------- */

/* out[i,:] = table[ids[i],:]; ids int64 [seq_len], table/out half.
 * Replaces engine::cuda::embedding_lookup (src/cuda/kernels.h:14-21). */
int b2_embedding_lookup(const int64_t* token_ids, const void* table, void* out,
                        int64_t seq_len, int64_t hidden_size, void* stream);

/* out = x * rsqrt(mean(x^2) + eps) * weight, fp32 accumulation; half [rows,dim].
 * Replaces engine::cuda::rmsnorm (src/cuda/kernels.h:26-34). */
int b2_rmsnorm(const void* x, const void* weight, void* out, int64_t rows, int64_t dim,
               float eps, void* stream);

/* out[i,j] = x[i,j] + bias[j]; half. Replaces engine::cuda::bias_add (src/cuda/kernels.h:38-45). */
int b2_bias_add(const void* x, const void* bias, void* out, int64_t M, int64_t N, void* stream);

/* out = a + b; half. Replaces engine::cuda::residual_add (src/cuda/kernels.h:48-54). */
int b2_residual_add(const void* a, const void* b, void* out, int64_t count, void* stream);

/* Rotate-half RoPE in place on q [S,nq,D] and k [S,nkv,D] at positions
 * start_pos + s.  Replaces engine::cuda::apply_rope (src/cuda/kernels.h:59-69). */
int b2_apply_rope(void* q, void* k, int64_t seq_len, int64_t num_q_heads, int64_t num_kv_heads,
                  int64_t head_dim, int64_t start_pos, float rope_theta, void* stream);

/* Causal GQA attention, q/out [S,nq,D], k/v [S,nkv,D], half, scale 1/sqrt(D).
 * Replaces engine::cuda::causal_gqa (src/cuda/kernels.h:77-87). */
int b2_causal_gqa(const void* q, const void* k, const void* v, void* out, int64_t seq_len,
                  int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, void* stream);

/* Row softmax over the last dimension, half in/out, fp32 math.
 * Replaces engine::cuda::softmax (src/cuda/kernels.h:91-97). */
int b2_softmax(const void* x, void* out, int64_t rows, int64_t cols, void* stream);

/* Single-token attention over a head-major cache [nkv, max_seq, D] for one
 * sequence of total_seq_len tokens. q/out [nq, D].
 * Replaces engine::cuda::decode_gqa (src/cuda/kernels.h:104-115). */
int b2_decode_gqa(const void* q, const void* k_cache, const void* v_cache, void* out,
                  int total_seq_len, int num_q_heads, int num_kv_heads, int max_seq, int head_dim,
                  void* stream);

/* Split-KV GQA decode attention: one query token per sequence, q/out
 * [B, nq, D] half, seq_lens int32 [B] on the device (read by the kernel, so
 * the call is graph-capturable across steps), K/V through strided views.
 * The positions of each (sequence, kv head) are cut into up to 8 splits
 * that form one thread-block cluster; K/V tiles arrive by TMA and the splits
 * are merged through distributed shared memory in the same kernel, so
 * split_buffer is not used (head_dim 32/64/128/256 with 8-element-aligned
 * view strides).  Other shapes take the global-merge kernel: splits of at
 * least one kernel iteration (16 to 64 positions), as many as split_buffer
 * holds (about split_buffer_floats / (B*nq*(D+2)); a few floats hold
 * per-(sequence, kv head) counters), each writing a partial output and its
 * (max, sum) pair that the last split to finish merges; split_buffer may be
 * NULL there (one split per (sequence, kv head)).  max_seq_len bounds
 * seq_lens, sizes the split count, and the views must cover max_seq_len
 * positions of every (sequence, kv head).
 * Replaces engine::cuda::decode_gqa_split (src/cuda/kernels.h:120-133,
 * src/cuda/decode_attention_split.cu:183-214). */
int b2_decode_gqa_split(const void* q, b2_kv_view k_view, b2_kv_view v_view, const int* seq_lens,
                        void* out, int batch_size, int num_q_heads, int num_kv_heads, int head_dim,
                        int max_seq_len, float* split_buffer, size_t split_buffer_floats,
                        void* stream);

/* b2_decode_gqa_split for callers that cannot allocate device memory (code
 * running inside an allocator or memory-pool callback, plugin hosts that own
 * every device byte, hot paths that must avoid allocator locks).  It has no
 * counterpart in the reference.  Same arguments and result as
 * b2_decode_gqa_split minus the scratch buffer, and the call allocates
 * nothing.  Shapes the cluster-merged kernels take need no scratch and run
 * exactly as in b2_decode_gqa_split.  The others run the global-merge kernel,
 * whose partial results live in a fixed 4 MiB array inside the library's
 * device image (every GPU that loads the library keeps it until the process
 * exits): the split count is the one the shape prefers, lowered until the
 * partials fit 4 MiB (one split needs none), so the array limits the speed of
 * very large batch x head x context problems, not which shapes run.  The
 * first call on a device that uses the array looks up its device address
 * (with that device current) and caches it for the life of the process: make
 * that first call before any stream capture, and not across a
 * cudaDeviceReset (the cached address would be stale).  All calls on one
 * device share the array, so calls that overlap on the GPU race; the arrival
 * counters in it are cleared by each call. */
int b2_decode_gqa_split_noalloc(const void* q, b2_kv_view k_view, b2_kv_view v_view, const int* seq_lens,
                                void* out, int batch_size, int num_q_heads, int num_kv_heads, int head_dim,
                                int max_seq_len, void* stream);

/* Causal GQA prefill attention, q/out [B,S,nq,D], k/v [B,S,nkv,D], half,
 * scale 1/sqrt(D).  head_dim 64 and 128 run on the tcgen05 tensor cores
 * (fp32 accumulation in TMEM); other head dims through the split-KV kernel.
 * Replaces engine::cuda::flash_prefill_gqa (src/cuda/kernels.h:136-147). */
int b2_flash_prefill_gqa(const void* q, const void* k, const void* v, void* out, int64_t seq_len,
                         int num_q_heads, int num_kv_heads, int head_dim, int batch_size, void* stream);

/* b2_flash_prefill_gqa with a choice of element type (bf16 != 0: bf16
 * q/k/v/out, else half) and rotate-half RoPE at positions start_pos + s when
 * rope_theta > 0: q and k rotated once by a pre-pass kernel of the same
 * call into per-device scratch copies (batch*S*(nq+nkv)*head_dim*2 bytes,
 * allocated on first use and grown as needed; RoPE calls on one device
 * must not overlap in time; see
 * b2_flash_prefill_gqa_ws for the form that allocates nothing).  q, k in
 * memory are left unrotated.  head_dim 64 or 128 only.  New API (the
 * reference applies RoPE as a separate apply_rope launch,
 * src/model/forward_gpu.cu:419-421). */
int b2_flash_prefill_gqa_ex(const void* q, const void* k, const void* v, void* out, int64_t seq_len,
                            int num_q_heads, int num_kv_heads, int head_dim, int batch_size, int bf16,
                            float rope_theta, int64_t start_pos, void* stream);

/* Device scratch owned by the caller and lent to the entry points that take
 * one, so that those never allocate (no counterpart in the reference, whose
 * only internal workspaces are the sampler's).  b2_workspace_create
 * allocates `bytes` of device memory on the current device; the handle may
 * be reused by any number of calls on that device that do not overlap in
 * time. */
typedef struct b2_workspace b2_workspace;
int b2_workspace_create(size_t bytes, b2_workspace** out);
int b2_workspace_destroy(b2_workspace* ws);
size_t b2_workspace_bytes(const b2_workspace* ws);

/* Workspace bytes b2_flash_prefill_gqa_ws needs for the RoPE form:
 * batch * S * (num_q_heads + num_kv_heads) * head_dim * 2 (the rotated q
 * and k copies). */
size_t b2_flash_prefill_workspace_bytes(int64_t seq_len, int num_q_heads, int num_kv_heads, int head_dim,
                                        int batch_size);

/* b2_flash_prefill_gqa_ex with the rotated q / k scratch taken from `ws`
 * (B2_ERR_WORKSPACE when it is smaller than
 * b2_flash_prefill_workspace_bytes): allocates nothing, so it is
 * graph-capturable from its first call.  ws == NULL behaves as _ex.  New API
 * (see b2_flash_prefill_gqa_ex). */
int b2_flash_prefill_gqa_ws(const void* q, const void* k, const void* v, void* out, int64_t seq_len,
                            int num_q_heads, int num_kv_heads, int head_dim, int batch_size, int bf16,
                            float rope_theta, int64_t start_pos, b2_workspace* ws, void* stream);

/* out = silu(gate) * up, half. Replaces engine::cuda::swiglu (src/cuda/kernels.h:151-157). */
int b2_swiglu(const void* gate, const void* up, void* out, int64_t count, void* stream);

/* C[M,N] = A[M,K] * B[N,K]^T, half in, fp32 accumulate, half out.
 * Replaces engine::cuda::matmul_transB (src/cuda/kernels.h:164-172). */
int b2_matmul_transB(const void* A, const void* B, void* C, int M, int K, int N, void* stream);

/* As b2_matmul_transB with fp32 output.
 * Replaces engine::cuda::matmul_transB_f32 (src/cuda/kernels.h:177-185). */
int b2_matmul_transB_f32(const void* A, const void* B, float* C, int M, int K, int N, void* stream);

/* y[n] = dot(W[n,:], x), W [N,K] half row-major, fp32 accumulate, half out.
 * Replaces engine::cuda::gemv (src/cuda/kernels.h:189-196). */
int b2_gemv(const void* W, const void* x, void* y, int N, int K, void* stream);

/* y[n] = dot(W[n,:], x) + b[n]. Replaces engine::cuda::gemv_bias (src/cuda/kernels.h:199-207). */
int b2_gemv_bias(const void* W, const void* x, const void* b, void* y, int N, int K, void* stream);

/* y[n] = dot(W[n,:], x) + r[n]. Replaces engine::cuda::gemv_residual (src/cuda/kernels.h:211-219). */
int b2_gemv_residual(const void* W, const void* x, const void* r, void* y, int N, int K, void* stream);

/* Batched decode GEMV (new API; the reference GEMV is M=1 only):
 * y[b,n] = dot(W[n,:], x[b,:]) (+ extra), x [B,K] half, y [B,N].
 * epilogue: 0 none, 1 bias extra[n] (half), 2 residual extra[b,n] (half).
 * out_f32 != 0 writes fp32 y instead of half (the lm_head form). */
int b2_gemv_batched(const void* W, const void* x, const void* extra, void* y, int B, int N, int K,
                    int epilogue, int out_f32, void* stream);

/* FP8 weights (OCP E4M3) for the decode GEMVs: per row r of w [rows, K]
 * (half), scales[r] = max|w[r,:]| / 448 (1 for an all-zero row) and
 * q[r,k] = E4M3(w[r,k] / scales[r]), round to nearest even, saturating.
 * q: rows * K bytes.  New API (the reference plans INT8/INT4 weights,
 * RESULTS.md:39). */
int b2_quantize_fp8_rows(const void* w, int64_t rows, int K, void* q, float* scales, void* stream);

/* y[b,n] = scales[n] * dot(E4M3 Wq[n,:], x[b,:]), x [B,K] half, fp32
 * accumulate, y [B,N] half (out_f32 != 0: fp32).  K % 16 == 0, 16-byte
 * aligned Wq and x.  The decode GEMV of a quantised model.  New API. */
int b2_gemv_fp8(const void* Wq, const float* scales, const void* x, void* y, int B, int N, int K, int out_f32,
                void* stream);

/* 4-bit weights for the decode GEMVs: per group of 128 consecutive weights
 * of a row of w [rows, K] (half), scales[r, g] = max|w| / 7 (fp32 division;
 * 0 for an all-zero group) and q = rint(w / scale) in [-7, 7], stored as
 * q + 8 in 4 bits: q [rows, K/2] bytes, each 32-bit word holding 8
 * consecutive weights, weight j of the word at bit 16*(j & 1) + 4*(j >> 1);
 * scales [rows, K/128] fp32.  K % 128 == 0, 16-byte aligned w and q.  New
 * API (the reference plans INT4 weights, RESULTS.md:39). */
int b2_quantize_int4_rows(const void* w, int64_t rows, int K, void* q, float* scales, void* stream);

/* y[b,n] = sum over groups g of scales[n,g] * dot(q[n, group g], x[b, group
 * g]), x [B,K] half, fp32 accumulate, y [B,N] half (out_f32 != 0: fp32).
 * K % 128 == 0, 16-byte aligned Wq and x.  The batch-1/2 decode GEMV of a
 * 4-bit model (any B: run two sequences at a time).  New API. */
int b2_gemv_int4(const void* Wq, const float* scales, const void* x, void* y, int B, int N, int K, int out_f32,
                 void* stream);

/* Copy K/V rows [num_tokens, nkv, D] into head-major caches [nkv, max_seq, D]
 * at positions start_pos..start_pos+num_tokens-1 (positions >= max_seq are
 * skipped).  Replaces engine::cuda::append_kv_cache (src/runtime/kv_cache.h:80-91). */
int b2_append_kv_cache(const void* src_k, const void* src_v, void* dst_k, void* dst_v,
                       int num_tokens, int start_pos, int num_kv_heads, int max_seq, int head_dim,
                       void* stream);

/* ---------------------------------------------------------------------------
 * Sampler  (replaces engine::SamplerGPU, src/runtime/sampler.h:10-65)
 * ------------------------------------------------------------------------- */

typedef struct b2_sampler_config {
    float temperature;        /* <= 1e-6: greedy argmax */
    int top_k;                /* <= 0 or > max_top_k: min(max_top_k, 64) */
    float top_p;              /* >= 1: disabled */
    float repetition_penalty; /* 1: disabled */
    uint64_t seed;            /* reseed iff seed != 0 and seed != current state */
} b2_sampler_config;

typedef struct b2_sampler b2_sampler;

/* Allocates the sampler's device workspace (this call allocates). */
int b2_sampler_create(int vocab_size, int max_top_k, b2_sampler** out);
int b2_sampler_destroy(b2_sampler* s);
/* Penalty, argmax or top-k/top-p selection and the seeded draw run on the
 * device; the chosen id is copied back (this call synchronises `stream`).
 * d_logits: float [vocab] on the device, left unmodified.  history: host ids.
 * Replaces SamplerGPU::sample (src/runtime/sampler.h:28-33, sampler.cu:202-340). */
int b2_sampler_sample(b2_sampler* s, const float* d_logits, const int64_t* history, int history_len,
                      const b2_sampler_config* cfg, void* stream, int* token_out);
/* b2_sampler_sample without a host round trip: history is a device int64
 * array, the chosen id is written to d_token (device int) on `stream`, and
 * nothing is allocated or synchronised (the LCG state, kept on the host, is
 * advanced at enqueue time, so draws follow the order of the calls).  Same
 * selection, semantics and bit-exact ids as b2_sampler_sample.  New API (the
 * reference copies the logits to the host, src/runtime/sampler.cu:253-256). */
int b2_sampler_sample_async(b2_sampler* s, const float* d_logits, const int64_t* d_history, int history_len,
                            const b2_sampler_config* cfg, void* stream, int* d_token);
/* Current LCG state (for tests) and explicit set. */
uint64_t b2_sampler_rng_state(const b2_sampler* s);
int b2_sampler_set_rng_state(b2_sampler* s, uint64_t state);

/* ---------------------------------------------------------------------------
 * Model runtime  (replaces ModelWeightsGPU / ActivationBuffersGPU /
 * prefill_gpu / decode_step_gpu, src/model/forward_gpu.h:15-113, and the
 * KVCache layout of src/runtime/kv_cache.h:12-73)
 * ------------------------------------------------------------------------- */

typedef struct b2_model_config {
    int vocab_size;
    int hidden_size;
    int intermediate_size;
    int num_layers;
    int num_q_heads;
    int num_kv_heads;
    int head_dim;
    float rms_norm_eps;
    float rope_theta;
    int tie_word_embeddings; /* 1: lm_head is the embedding table */
    int has_qkv_bias;        /* 1: q/k/v biases (Qwen2); 0: Llama */
    int max_batch;           /* sequences decoded together */
    int max_seq;             /* KV capacity per sequence */
} b2_model_config;

typedef struct b2_model b2_model;

/* Writes a fresh 128-byte ncclUniqueId (rank 0 calls it and shares the bytes
 * with the other ranks).  B2_ERR_NCCL when NCCL cannot be loaded. */
int b2_nccl_unique_id(void* out128);

/* Creates a model shard on the current CUDA device (allocates all weights,
 * the KV cache and activations).  tp_size > 1 shards heads / FFN rows /
 * vocabulary Megatron-style across ranks; nccl_id is the 128-byte
 * ncclUniqueId shared by all ranks (NULL when tp_size == 1). */
int b2_model_create(const b2_model_config* cfg, int tp_rank, int tp_size, const void* nccl_id,
                    b2_model** out);
int b2_model_destroy(b2_model* m);

/* A model shard whose KV cache is a paged block pool instead of one
 * max_seq slab per sequence: per layer, K and V pools
 * [num_blocks][block_size][kv heads of this rank][head_dim] half -- the
 * physical block pool of the reference's paged runner contract
 * (docs/runner_interface.md:18-84, block size 16 there) -- read through
 * per-sequence block tables of physical block ids that the caller (the
 * scheduler, sole owner of block allocation) passes with every call.
 * head_dim 128 only (the tensor-core decode attention reads the pool; a
 * 128-position tile is 128/block_size block boxes), block_size a multiple
 * of 8 dividing 128.  A paged model takes b2_model_prefill_paged and
 * b2_model_decode_step_paged; b2_model_prefill / _decode_step /
 * _decode_enqueue / _forward_logits / _kv_layout return B2_ERR_STATE on it.
 * cfg->max_seq bounds sequence lengths (block-table width
 * ceil(max_seq / block_size)), cfg->max_batch the decode batch.  Allocates
 * like b2_model_create.  New API (the reference runner is Python and not
 * part of its C++ tree). */
int b2_model_create_paged(const b2_model_config* cfg, int num_blocks, int block_size, int tp_rank, int tp_size,
                          const void* nccl_id, b2_model** out);

/* Tensor-parallel exchange over peer memory (one node, tp_size > 1).  Each
 * rank exports the 64-byte CUDA IPC handle of its exchange buffer; the
 * caller all-gathers the tp handles (rank order) with its own launcher and
 * passes them to b2_model_p2p_open on every rank.  From then on the decode
 * step runs without NCCL: the o and down GEMVs store their fp32 partial rows
 * into every rank's receive slots over NVLink as 8-byte words tagged with
 * the exchange's epoch, and the next GEMV's RMSNorm prologue polls (bounded,
 * about a second) until the words it needs carry the epoch, then sums the
 * slots in rank order; the lm_head's argmax is exchanged with one flag per
 * rank.  Without b2_model_p2p_open the step uses NCCL
 * all-reduces.  New API (the reference has no parallelism). */
int b2_model_p2p_handle(b2_model* m, void* out64);
int b2_model_p2p_open(b2_model* m, const void* handles);

/* Fills every weight from the seeded generator (identical global tensors at
 * any tp_size; norm weights 1.0).  Synchronises. */
int b2_model_init_random(b2_model* m, uint64_t seed, float stddev);

/* Uploads one global tensor given in host fp16 [rows, cols] (the rank keeps
 * its shard).  Names: "embed", "lm_head", "final_norm", and per layer l
 * "l.ln1", "l.ln2", "l.wq", "l.wk", "l.wv", "l.bq", "l.bk", "l.bv", "l.wo",
 * "l.wg", "l.wu", "l.wd".  Synchronises. */
int b2_model_set_tensor(b2_model* m, const char* name, const uint16_t* host_f16, int64_t rows,
                        int64_t cols);

/* b2_model_set_tensor for a bf16 checkpoint tensor (host bf16 [rows, cols],
 * e.g. straight from a memory-mapped safetensors file): the rank's block is
 * copied to the device and converted there to fp16 by the loader's rule
 * (exponent rebased; values below the fp16 normal range become signed zero,
 * values above it signed infinity; the mantissa bits carry over exactly).
 * Synchronises.  Replaces the host-side conversion of
 * ModelWeightsGPU::init_from_weights (src/model/forward_gpu.cu:18-28,
 * src/loader/safetensors.cpp:307-328). */
int b2_model_set_tensor_bf16(b2_model* m, const char* name, const uint16_t* host_bf16, int64_t rows,
                             int64_t cols);

/* How the model picks each next token from here on (prefill, decode steps
 * and the device-resident loop): cfg->temperature <= 1e-6 is greedy argmax
 * (the default); otherwise every sequence draws from top-k / temperature /
 * top-p inside the captured step -- the selection of b2_sampler_sample, with
 * one LCG state per sequence, reset by this call to a fresh sampler's state
 * (13374269) -- so a sampled decode keeps its logits on the device.  The
 * configuration lives in device memory: changing temperature / top-k /
 * top-p / seed needs no recapture (switching greedy <-> sampling recaptures
 * the step).  B2_ERR_UNSUPPORTED for a repetition penalty != 1 or tp_size >
 * 1 when sampling.  Synchronises.  New API (the reference samples on the
 * host, src/runtime/sampler.cu:253-339, apps/generate.cpp:884-898). */
int b2_model_set_sampling(b2_model* m, const b2_sampler_config* cfg);

/* Weight format of the decode steps.  B2_WEIGHTS_FP8_E4M3 quantises every
 * projection and the lm_head per output row (b2_quantize_fp8_rows) from the
 * fp16 weights the model holds now, on the device, into copies allocated on
 * first use; decode steps of 1-2 sequences (the GEMVs) and of more than 4
 * (the tensor-core step, up to 128) then stream the 1-byte copies -- half
 * the bytes of a step.  Batches of 3-4 (GEMVs bound by arithmetic, not
 * bytes) and prefill keep the fp16 weights.  Call again after changing
 * weights; B2_WEIGHTS_FP16 returns to fp16 everywhere (the copies are kept).
 * B2_WEIGHTS_INT4 makes 4-bit copies (b2_quantize_int4_rows: a scale per 128
 * weights) read by the decode GEMVs at 1-2 sequences -- about a quarter of
 * the bytes; every other step and prefill keep the fp16 weights.  Hidden,
 * head and FFN widths must be multiples of 128.  Synchronises.  New API
 * (the reference plans quantised weights as P8, RESULTS.md:39). */
enum { B2_WEIGHTS_FP16 = 0, B2_WEIGHTS_FP8_E4M3 = 1, B2_WEIGHTS_INT4 = 2 };
int b2_model_quantize_weights(b2_model* m, int format);

/* Clears the KV cache positions of all sequences (sets lengths to 0). */
int b2_model_reset(b2_model* m);

/* Processes `seq_len` prompt tokens of each of `batch` sequences
 * (host ids [batch, seq_len]) starting at position 0, filling the KV cache.
 * If host_logits != NULL the fp32 logits of the last position are copied to
 * it ([batch, vocab]).  Synchronises. */
int b2_model_prefill(b2_model* m, const int64_t* host_ids, int batch, int seq_len, float* host_logits);

/* One decode step for `batch` sequences: host tokens [batch] at host
 * positions [batch]; appends K/V and produces logits.  host_logits
 * ([batch, vocab] fp32) and/or host_next (greedy ids [batch]) may be NULL;
 * host_logits must hold batch * vocab floats.  When its first and last bytes
 * are page-locked (cudaMallocHost / cudaHostRegister memory covering the
 * whole [batch, vocab] range) the copy engine writes it directly, otherwise
 * the logits go through a staging buffer.  Synchronises.  The step runs as a captured CUDA graph after its
 * first call. */
int b2_model_decode_step(b2_model* m, const int64_t* host_tokens, const int* host_positions, int batch,
                         float* host_logits, int64_t* host_next);

/* Paged prefill of one sequence (the runner's prefill(seq)): all seq_len
 * prompt tokens at once; K/V of position p land in block
 * host_block_table[p / block_size] (n_blocks entries, host int32), except
 * positions below skip_blocks * block_size, whose blocks are shared and kept
 * (prefix "share" mode: the prompt is recomputed, shared blocks are not
 * overwritten).  first_token (may be NULL) receives the argmax of the last
 * position, host_logits (may be NULL) its fp32 logits [vocab].  Synchronises.
 * New API (docs/runner_interface.md:33-46). */
int b2_model_prefill_paged(b2_model* m, const int64_t* host_ids, int seq_len, const int* host_block_table,
                           int n_blocks, int skip_blocks, float* host_logits, int64_t* first_token);

/* Paged decode step of `batch` sequences (the runner's decode_step(seqs)):
 * sequence b consumes host_tokens[b] at position host_seq_lens[b] - 1 (the
 * runner has already bumped its length to include this token), its K/V row
 * goes to block host_block_tables[b * max_blocks + pos / block_size], and it
 * attends over all host_seq_lens[b] positions through its table row (int32,
 * unused slots padded with any valid id, e.g. 0).  host_logits ([batch,
 * vocab]) and host_next (argmax ids) may be NULL.  The step runs as the
 * captured graph of the batch size; the tables travel with each call, so
 * sequences may join, leave and change blocks between steps.
 * Synchronises.  New API (docs/runner_interface.md:48-72). */
int b2_model_decode_step_paged(b2_model* m, const int64_t* host_tokens, const int* host_seq_lens,
                               const int* host_block_tables, int max_blocks, int batch, float* host_logits,
                               int64_t* host_next);

/* Full forward over one sequence of `seq_len` host ids: fp32 logits of every
 * position into host_logits ([seq_len, vocab]).  Runs the batched prefill
 * (tensor-core projections and flash prefill), then the final RMSNorm and the
 * lm_head over all positions as one tensor-core GEMM; sequence 0's KV cache
 * holds the sequence afterwards.  Allocates its logits workspace on first use
 * (grown as needed); synchronises; tp_size 1 only.
 * Replaces forward_gpu (src/model/forward_gpu.h:76-84). */
int b2_model_forward_logits(b2_model* m, const int64_t* host_ids, int seq_len, float* host_logits);

/* b2_model_decode_step without synchronising: the host tokens and positions
 * go to the device as launch parameters (the host arrays are free once the
 * call returns), the step's graph is launched on the model's stream, and
 * when d_logits is not NULL the fp32 logits [batch, vocab] are copied to that
 * device buffer on the same stream (tp_size 1 only).  Order other work
 * against it through b2_model_stream.  Replaces decode_step_gpu's
 * d_last_logits form, which skips the host copy for an asynchronous
 * pipeline (src/model/forward_gpu.h:98-113, forward_gpu.cu:694-707). */
int b2_model_decode_enqueue(b2_model* m, const int64_t* host_tokens, const int* host_positions, int batch,
                            float* d_logits);

/* Device-resident generation: `steps` decode steps replayed back to back
 * without host round trips, each consuming the token the previous one chose
 * (the argmax, or the draw of b2_model_set_sampling's configuration).  It continues from the last prefill / decode step: the first step
 * consumes that step's argmax.  host_tokens_out ([steps, batch]) receives the
 * token each step consumed (so row 0 is the argmax of the last processed
 * position); when it is NULL the call only enqueues the steps on the model's
 * stream (see b2_model_sync), otherwise it synchronises. */
int b2_model_generate_greedy(b2_model* m, int steps, int64_t* host_tokens_out);
int b2_model_sync(b2_model* m);

/* The model's CUDA stream (cudaStream_t). */
void* b2_model_stream(b2_model* m);

/* Device pointers for tests and tools: "logits" (float [max_batch, vocab]),
 * "hidden" (float [max_batch, hidden]), "kv" (half, the whole cache),
 * "tokens" (int64 [max_batch]), "positions" (int32 [max_batch]). */
void* b2_model_buffer(b2_model* m, const char* name);

/* Synchronous copy of `bytes` bytes at byte `offset` of a named buffer (see
 * b2_model_buffer) into host memory. */
int b2_model_read(b2_model* m, const char* name, void* host_dst, size_t offset, size_t bytes);

/* Layout of the KV cache: [layer][batch][K=0,V=1][kv_head][max_seq][head_dim]
 * half, kv heads of this rank only.  Writes the element strides. */
int b2_model_kv_layout(const b2_model* m, int64_t* stride_layer, int64_t* stride_batch,
                       int64_t* stride_kv, int64_t* stride_head, int64_t* stride_pos);

/* Algorithmic HBM bytes of one decode step at `batch` sequences whose context
 * (before the step) is `ctx` tokens, for this rank. */
double b2_model_step_bytes(const b2_model* m, int batch, int ctx);

/* Times one kernel of the decode step in isolation for roofline reporting:
 * kind 0 qkv, 1 attention (+combine), 2 o-proj, 3 gate/up, 4 down, 5 lm_head.
 * Launches it once per layer (different weights each launch, as in a step),
 * `reps` times over all layers, back to back on the model's stream with the
 * same launch attributes as the step, and writes the average milliseconds
 * per launch.  Overwrites activation buffers (not the KV cache contents of
 * earlier positions).  Synchronises. */
int b2_model_time_kernel(b2_model* m, int kind, int batch, int reps, float* avg_ms);

/* Algorithmic HBM bytes of one launch of `kind` (as above) at `batch`
 * sequences with `ctx` context tokens. */
double b2_model_kernel_bytes(const b2_model* m, int kind, int batch, int ctx);

/* Number of kernel launches one decode step issues (for reporting). */
int b2_model_step_launches(const b2_model* m, int batch);

/* Runs one decode step (not from its captured graph) with every kernel
 * recording, in %globaltimer nanoseconds, when its first CTA passed its
 * programmatic-launch wait and when its last CTA finished: host_ns receives
 * (start, end) pairs in launch order, *n_slots the number of launches.
 * Advances the sequences like b2_model_decode_step (tokens and positions
 * from the device state).  Allocates its buffer on first use; synchronises.
 * Under tensor parallelism every rank calls it together.  No reference
 * counterpart beyond its per-launch CudaTimer records
 * (src/model/forward_gpu.cu:542-551). */
int b2_model_trace_step(b2_model* m, int batch, unsigned long long* host_ns, int max_slots, int* n_slots);

/* ------------------------------------------------------------------------
 * Tokenizer (host only; no CUDA call).  Byte-level BPE read from a HF
 * tokenizer.json: the reference's Qwen2 vocabulary and, beyond it, Llama-3
 * and GPT-2 ones.  Replaces engine::BPETokenizer (src/tokenizer/bpe.h:17-58);
 * that class is kept over these calls in serving-engine_b200/compat
 * (src/tokenizer/bpe.h).  A tokenizer is immutable after loading: calls on
 * one object from several threads at once are safe.  Output buffers follow
 * one rule: *n (ids or bytes) always receives the full length, and when it is
 * above `cap` nothing is written and B2_ERR_WORKSPACE is returned. */
typedef struct b2_tokenizer b2_tokenizer;

/* b2_tokenizer_encode flags */
enum {
    B2_TOK_SPLIT_SPECIAL = 1, /* special added tokens in the text become their ids
                                 (the reference's allowed_special); without it they
                                 are encoded as plain text */
    B2_TOK_ADD_SPECIAL = 2    /* apply the file's TemplateProcessing post-processor
                                 (Llama-3: <|begin_of_text|> first) */
};

/* b2_tokenizer_info.pre_tokenizer */
enum { B2_PRE_QWEN2 = 1, B2_PRE_LLAMA3 = 2, B2_PRE_GPT2 = 3 };
/* b2_tokenizer_info.chat_format */
enum { B2_CHAT_NONE = 0, B2_CHAT_CHATML = 1, B2_CHAT_LLAMA3 = 2 };

typedef struct b2_tokenizer_info {
    int64_t vocab_size;    /* distinct token strings, vocab and added (BPETokenizer::vocab_size) */
    int64_t n_ids;         /* highest id + 1 */
    int64_t n_merges;
    int32_t pre_tokenizer; /* B2_PRE_* */
    int32_t nfc;           /* 1: text is NFC-normalised before splitting */
    int32_t ignore_merges; /* 1: a piece that is a vocab entry is one token */
    int32_t chat_format;   /* B2_CHAT_* */
    int32_t bos_id;        /* -1 if none */
    int32_t eos_id;        /* end of a chat turn (<|im_end|>, <|eot_id|>); -1 if none */
    int32_t n_stop;        /* ids that end generation, in stop_ids[0..n_stop) */
    int32_t stop_ids[4];
    int32_t n_added;
} b2_tokenizer_info;

/* BPETokenizer::load (src/tokenizer/bpe.cpp:87-158).  Reads and checks the
 * whole file; B2_ERR_UNSUPPORTED (with the reason in b2_last_error()) for a
 * normaliser, pre-tokenizer or model this tokenizer does not implement. */
int b2_tokenizer_load(const char* tokenizer_json_path, b2_tokenizer** out);
/* The same from the file's contents in memory. */
int b2_tokenizer_load_json(const char* json, size_t len, b2_tokenizer** out);
void b2_tokenizer_destroy(b2_tokenizer* t);

/* BPETokenizer::encode (src/tokenizer/bpe.cpp:386-447): UTF-8 text (bytes
 * that are not valid UTF-8 are kept as byte tokens) -> ids. */
int b2_tokenizer_encode(const b2_tokenizer* t, const char* text, size_t len, int flags, int32_t* ids, size_t cap,
                        size_t* n_ids);

/* BPETokenizer::decode (src/tokenizer/bpe.cpp:449-483): ids -> the bytes they
 * stand for (ids outside the vocabulary are skipped; special tokens too when
 * skip_special != 0).  The bytes of a partial sequence may end inside a
 * UTF-8 character. */
int b2_tokenizer_decode(const b2_tokenizer* t, const int32_t* ids, size_t n, int skip_special, char* out, size_t cap,
                        size_t* out_len);

/* BPETokenizer::apply_chat_template (src/tokenizer/bpe.cpp:485-506): the
 * ChatML prompt for Qwen vocabularies (the reference's format, with its
 * default system message when the first message is not a system one), the
 * Llama-3 header/eot format for Llama-3 vocabularies.  B2_ERR_UNSUPPORTED for
 * a vocabulary with neither set of control tokens. */
int b2_tokenizer_apply_chat_template(const b2_tokenizer* t, const char* const* roles, const char* const* contents,
                                     size_t n_messages, int add_generation_prompt, char* out, size_t cap,
                                     size_t* out_len);

/* Id of an added token (by its content) or of a vocab entry (as written in
 * tokenizer.json); B2_ERR_INVALID and *id = -1 if there is none.  Serves
 * BPETokenizer::im_start_id / im_end_id / endoftext_id (bpe.h:33-35). */
int b2_tokenizer_token_to_id(const b2_tokenizer* t, const char* token, size_t len, int32_t* id);

int b2_tokenizer_get_info(const b2_tokenizer* t, b2_tokenizer_info* info);

#ifdef __cplusplus
}
#endif

#endif /* B2ENGINE_H */
