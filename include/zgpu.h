/*
 * zgpu.h — C ABI of zero-b200, the B200 (sm_100a) decode hot path that drops
 * in under silicatetech/zero's `zero-llm-inference` forward/matmul API.
 *
 * Conventions
 *   - Plain C types only: pointers, sizes, integer status codes.  No CUDA or
 *     torch types cross the ABI (streams are passed as `void*`, a
 *     cudaStream_t; NULL means the context's own stream).
 *   - Every entry point returns a zgpu_status.  Codes map 1:1 onto the Rust
 *     error enums the reference returns (see each code's comment);
 *     zgpu_last_error() gives a human-readable message for the last failure
 *     on a context.  No C++ exception ever crosses the ABI.
 *   - The caller owns every host buffer.  Weights are registered once, keyed
 *     by the host address of the tensor payload, mirroring
 *     kernel/src/weight_layout.rs:40 (register) / :133 (group_of); the
 *     library keeps a device copy.  Contexts are not thread-safe (the
 *     reference's decode API is single-caller, kv_cache.rs:60).
 *   - There is no CPU fallback: every compute entry point runs CUDA kernels
 *     built for sm_100a and fails with ZGPU_ERR_NO_DEVICE when no device is
 *     usable.
 */
#ifndef ZGPU_H
#define ZGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZGPU_ABI_VERSION 1u

/* ggml / .smodel dtype ids (zero-gguf-parser lib.rs:95-126; .smodel v2 ids
 * tools/silicatepack.py:75-83). */
enum zgpu_dtype {
  ZGPU_F32 = 0,
  ZGPU_F16 = 1,
  ZGPU_Q4_0 = 2,
  ZGPU_Q8_0 = 8,
  /* GGUF K-quants, plain rows of 256-element super-blocks (the GGUF-compat
   * path: dequant.rs:63-138, 286-356): 144 / 210 bytes per super-block. */
  ZGPU_Q4_K = 12,
  ZGPU_Q6_K = 14,
  ZGPU_Q4_0X4 = 100,
  ZGPU_Q8_0X4 = 101
};

typedef enum zgpu_status {
  ZGPU_OK = 0,
  ZGPU_ERR_INVALID_ARG = 1,
  /* LinearDispatchError::UnsupportedQuant (ops.rs:461); the reference panics
   * at ops.rs:520 and inference_avx512.rs:1178. */
  ZGPU_ERR_UNSUPPORTED_QUANT = 2,
  /* a weight key that was never registered (no counterpart: the reference
   * reads host memory directly). */
  ZGPU_ERR_UNREGISTERED_WEIGHT = 3,
  /* KvCacheError (kv_cache.rs:68-83). */
  ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE = 10,
  ZGPU_ERR_KV_LAYER_OUT_OF_RANGE = 11,
  ZGPU_ERR_KV_INVALID_SLICE_LENGTH = 12,
  ZGPU_ERR_KV_TOKEN_COUNT_EXCEEDS_MAX = 13,
  /* AttentionError::NumericalInstability (attention.rs:26-31). */
  ZGPU_ERR_NUMERICAL_INSTABILITY = 20,
  /* EmbedDispatchError (forward_pass.rs:276-286). */
  ZGPU_ERR_EMBED_UNSUPPORTED_QUANT = 30,
  ZGPU_ERR_EMBED_DIM_MISALIGNMENT = 31,
  /* LmHeadError (lm_head.rs:31-38). */
  ZGPU_ERR_LM_NON_FINITE_LOGITS = 40,
  ZGPU_ERR_LM_ARGMAX_IN_PADDING = 41,
  /* LoadError (kernel/src/model_loader.rs:151-160) of a .smodel container:
   * MagicMismatch, UnsupportedFormat, InvalidContainer; and a file that
   * cannot be opened or mapped. */
  ZGPU_ERR_MODEL_MAGIC = 50,
  ZGPU_ERR_MODEL_UNSUPPORTED = 51,
  ZGPU_ERR_MODEL_INVALID = 52,
  ZGPU_ERR_MODEL_IO = 53,
  /* runtime */
  ZGPU_ERR_NO_DEVICE = 90,
  ZGPU_ERR_CUDA = 91,
  ZGPU_ERR_OUT_OF_MEMORY = 92,
  /* a device-side bounded wait gave up (no counterpart; the reference's SMP
   * barrier times out after 1 s, smp.rs:311). */
  ZGPU_ERR_DEVICE_TIMEOUT = 93
} zgpu_status;

typedef struct zgpu_ctx zgpu_ctx;
typedef struct zgpu_kv zgpu_kv;
typedef struct zgpu_model zgpu_model;

typedef struct zgpu_opts {
  uint32_t abi_version;  /* must be ZGPU_ABI_VERSION */
  int32_t device;        /* CUDA device ordinal */
  uint32_t flags;        /* ZGPU_FLAG_* */
} zgpu_opts;

/* Capture the decode step into a CUDA graph (default on). */
#define ZGPU_FLAG_NO_GRAPH 0x1u
/* Launch kernels with programmatic dependent launch (default on). */
#define ZGPU_FLAG_NO_PDL 0x2u
/* Run decode steps as one persistent cooperative kernel per call (default
 * on where the device and the model geometry allow it); with this flag the
 * step is a sequence of per-op kernels instead. */
#define ZGPU_FLAG_NO_PERSISTENT 0x4u

/* ---------------------------------------------------------------- context */
zgpu_status zgpu_init(const zgpu_opts *opts, zgpu_ctx **out);
void zgpu_destroy(zgpu_ctx *ctx);
const char *zgpu_last_error(const zgpu_ctx *ctx);
const char *zgpu_status_string(zgpu_status s);
/* Number of streaming multiprocessors on the context's device. */
zgpu_status zgpu_device_info(const zgpu_ctx *ctx, int32_t *sm_count, int32_t *cc_major,
                             int32_t *cc_minor);
zgpu_status zgpu_synchronize(zgpu_ctx *ctx);

/* ------------------------------------------------------- weight registry */
/* Upload one tensor and key it by `host_ptr` (weight_layout.rs:40 register,
 * model_loader.rs:532-570).  dtype is ZGPU_Q4_0 / ZGPU_Q8_0 (plain row
 * blocks), ZGPU_Q4_0X4 / ZGPU_Q8_0X4 (.smodel v2 4-row interleave),
 * ZGPU_Q4_K / ZGPU_Q6_K (plain rows of 144 / 210-byte super-blocks, cols a
 * multiple of 256) or ZGPU_F32.  rows/cols give the logical matrix
 * (cols = in_dim). */
zgpu_status zgpu_register_weights(zgpu_ctx *ctx, const void *host_ptr, size_t len,
                                  uint32_t dtype, uint64_t rows, uint64_t cols);
/* weight_layout.rs:133 group_of: 4 for an interleaved registration, 1
 * otherwise (also for unregistered addresses). */
uint32_t zgpu_group_of(const zgpu_ctx *ctx, const void *host_ptr);
/* weight_layout.rs:58 clear. Frees every device copy. */
zgpu_status zgpu_clear_weights(zgpu_ctx *ctx);

/* ------------------------------------------------------------ matmul API */
/* out[out_dim] = W[out_dim x in_dim] . x[in_dim] with host x/out buffers.
 * Mirrors linear_dispatch (ops.rs:486-523) and linear_dispatch_avx512
 * (inference_avx512.rs:1147-1185); `w_key` is the registered host address.
 * quant is the ggml type of the tensor (Q4_0, Q8_0, Q4_K or Q6_K: the four
 * linear_dispatch accepts; any other is ZGPU_ERR_UNSUPPORTED_QUANT where the
 * reference panics); the stored layout (plain or X4) comes from the
 * registry, as group_of decides at inference_avx512.rs:638.  Q4_K / Q6_K
 * follow linear_q4k / linear_q6k (ops.rs:179-292). */
zgpu_status zgpu_linear_dispatch(zgpu_ctx *ctx, const float *x, const void *w_key, float *out,
                                 uint64_t in_dim, uint64_t out_dim, uint32_t quant);
/* Same with device-resident x/out on `stream` (no host copies, async). */
zgpu_status zgpu_linear_dispatch_device(zgpu_ctx *ctx, const float *d_x, const void *w_key,
                                        float *d_out, uint64_t in_dim, uint64_t out_dim,
                                        uint32_t quant, void *stream);
/* Q8_0 activation quantiser: x[n] -> n/32 blocks of {fp16 d, i8 q[32]} with
 * the packer's rule (tools/silicatepack.py:893-907).  No counterpart on the
 * reference's decode path (it multiplies f32 activations). */
zgpu_status zgpu_quantize_q8_0(zgpu_ctx *ctx, const float *x, void *blocks_out, uint64_t n);
/* Q4_0 weight x Q8_0 activation GEMV (int8 dot products, per-block fp16
 * scales): out = sum_b d_w*d_x*sum_j (n-8)*q.  Host buffers. */
zgpu_status zgpu_linear_q8act(zgpu_ctx *ctx, const void *xq_blocks, const void *w_key, float *out,
                              uint64_t in_dim, uint64_t out_dim);
/* Same with device-resident Q8_0 blocks / output on `stream` (async). */
zgpu_status zgpu_linear_q8act_device(zgpu_ctx *ctx, const void *d_xq_blocks, const void *w_key,
                                     float *d_out, uint64_t in_dim, uint64_t out_dim, void *stream);

/* linear_dispatch (ops.rs:486) of n_vec (1..256) f32 vectors x[n_vec][in_dim]
 * against one registered Q4_0 or Q8_0 weight on the tensor cores
 * (tcgen05 int8 MMA over the three 8-bit digits of the GEMV's activation
 * integers): out[v] equals zgpu_linear_dispatch(x[v]) bit for bit for every
 * v, whatever n_vec is.  The reference multiplies one vector at a time; this
 * is the batched-decode form of the same product.  Host buffers. */
zgpu_status zgpu_linear_dispatch_batch(zgpu_ctx *ctx, const float *x, const void *w_key, float *out,
                                       uint64_t n_vec, uint64_t in_dim, uint64_t out_dim, uint32_t quant);

/* Batched form on the tensor cores (tcgen05 int8 MMA): T rows of f32
 * activations x[T][in_dim] are quantised per 32-block with the Q8_0 rule
 * above, then out[t][r] = sum_b (sum_j w_j*q_j * d_w) * d_x, accumulated in
 * block order, with w_j = n-8 for Q4_0 weights and the int8 value for Q8_0
 * weights (bit-identical to the single-row product).  No counterpart in the
 * reference, which decodes one token at a time: this is the prefill /
 * multi-token path.  out_dim must be a multiple of 128.  Host buffers. */
zgpu_status zgpu_linear_q8act_batch(zgpu_ctx *ctx, const float *x, const void *w_key, float *out,
                                    uint64_t T, uint64_t in_dim, uint64_t out_dim);
/* Same with device-resident f32 activations / output on `stream` (async). */
zgpu_status zgpu_linear_q8act_batch_device(zgpu_ctx *ctx, const float *d_x, const void *w_key,
                                           float *d_out, uint64_t T, uint64_t in_dim,
                                           uint64_t out_dim, void *stream);

/* ------------------------------------------------------------- small ops */
/* rmsnorm (ops.rs:29-52). */
zgpu_status zgpu_rmsnorm(zgpu_ctx *ctx, const float *x, const float *w, float *out, uint64_t n,
                         float eps);
/* RopeContext::new (ops.rs:79-93) + rope_sincos_lut_avx512/rope_apply_avx512
 * (trig.rs:148,192) on `n_heads` heads of `head_dim`, in place. */
zgpu_status zgpu_rope(zgpu_ctx *ctx, float *qk, uint32_t n_heads, uint32_t head_dim,
                      uint32_t pos, float freq_base);
/* silu_mul_avx512 (activation.rs:115-148). */
zgpu_status zgpu_silu_mul(zgpu_ctx *ctx, const float *gate, const float *up, float *out,
                          uint64_t n);

/* --------------------------------------------------------------- KV cache */
/* KvCache::new (kv_cache.rs:100-126): layer-major [K block | V block], each
 * block max_tokens x n_kv_heads x head_dim f32, in device memory. */
zgpu_status zgpu_kv_create(zgpu_ctx *ctx, uint32_t max_tokens, uint32_t n_layers,
                           uint32_t n_kv_heads, uint32_t head_dim, zgpu_kv **out);
void zgpu_kv_destroy(zgpu_kv *kv);
/* KvCache::store_kv (kv_cache.rs:139-183), host k/v of n_kv_heads*head_dim. */
zgpu_status zgpu_kv_store(zgpu_kv *kv, uint32_t layer, uint32_t token, const float *k,
                          const float *v, uint64_t len);
/* get_k_slice / get_v_slice (kv_cache.rs:186-222) copied to host:
 * token_count * n_kv_heads * head_dim floats each (either may be NULL). */
zgpu_status zgpu_kv_read(zgpu_kv *kv, uint32_t layer, uint32_t token_count, float *k_out,
                         float *v_out);

/* ------------------------------------------------------ decode attention */
/* Steps 2-5 of gqa_attention_single_token_dispatch
 * (crates/zero-llm-inference/src/attention.rs:344-425) for one layer, given
 * the raw projections qkv = [q (n_q_heads*hd) | k (n_kv*hd) | v (n_kv*hd)]:
 * per-head QK RMSNorm with q_norm / k_norm [hd] (ops.rs:29-52), RoPE at `pos`
 * with the RopeContext of freq_base (ops.rs:79-132), KvCache::store_kv of k
 * and v at `pos` (kv_cache.rs:139), then per q head softmax(q.k/sqrt(hd))
 * (attention.rs:48-84) over tokens 0..pos and sum_t p_t v_t into
 * out [n_q_heads*hd].  Requires head_dim 128 and n_q_heads = 1..4 x n_kv.
 * Errors: ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE
 * (pos >= max_tokens), ZGPU_ERR_NUMERICAL_INSTABILITY (AttentionError::
 * NumericalInstability).  Synchronous; host buffers. */
/* The prefill's causal attention over a cache layer: T queries q
 * [T][n_q_heads*128] (already QK-normed and rotated) at positions pos0 ..
 * pos0+T-1; query i attends to cached tokens 0..pos0+i with
 * softmax(q.k/sqrt(hd)) and writes out [T][n_q_heads*128] — the per-token
 * attention of gqa_attention_single_token_dispatch (attention.rs:278-433)
 * for a run of prompt tokens, in another f32 summation order.  The keys
 * must be in the cache (zgpu_kv_store or a prefill).  Errors as
 * zgpu_gqa_attention_decode.  Synchronous; host buffers. */
zgpu_status zgpu_causal_attention(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer, uint32_t pos0, uint32_t T,
                                  uint32_t n_q_heads, const float *q, float *out);
zgpu_status zgpu_gqa_attention_decode(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer, uint32_t pos,
                                      uint32_t n_q_heads, const float *qkv, const float *q_norm,
                                      const float *k_norm, float freq_base, float eps, float *out);
/* Device-buffer form: d_inv_freqs is the RopeContext table [hd/2]; launches
 * on `stream` (NULL = the context stream) without synchronising.  The split
 * partials live in context-owned device memory grown on first use.  Device-
 * side numerical errors are recorded in the context status block and
 * reported by the context's next synchronous entry point. */
zgpu_status zgpu_gqa_attention_decode_device(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer,
                                             uint32_t pos, uint32_t n_q_heads, const float *d_qkv,
                                             const float *d_q_norm, const float *d_k_norm,
                                             const float *d_inv_freqs, float eps, float *d_out,
                                             void *stream);
/* Has no counterpart in the reference: an added variant of
 * zgpu_gqa_attention_decode_device (same arguments, same results) for callers
 * that must not allocate device memory while they run.  Examples are hosts
 * that reserve all device memory up front and hand out fixed buffers,
 * per-token loops where an allocation could synchronise the device, and
 * plugins whose memory belongs to another allocator.  The call allocates
 * nothing.  Its split partials and counters live in a 1 MiB array built into
 * the library's device image, which every GPU that loads the library keeps
 * until the process exits.  Limits: n_q_heads x ceil(max_tokens / 256) x
 * (head_dim + 2) must be at most 261888 floats (16 q heads: caches up to
 * 32000 tokens), and n_kv at most 256.  Larger requests return
 * ZGPU_ERR_INVALID_ARG with a message and launch nothing.  The first call on
 * a device looks up the array's device address, so make that first call
 * before any stream capture.  The address is kept until the process exits:
 * resetting the device (cudaDeviceReset) or destroying its primary context
 * after that first call is not supported, since the array would move.  All calls on a device share the one array, and
 * each call clears the counters on its stream.  Calls that overlap on the GPU
 * race, whether from other streams or other contexts on the same device. */
zgpu_status zgpu_gqa_attention_decode_noalloc(zgpu_ctx *ctx, zgpu_kv *kv, uint32_t layer,
                                              uint32_t pos, uint32_t n_q_heads, const float *d_qkv,
                                              const float *d_q_norm, const float *d_k_norm,
                                              const float *d_inv_freqs, float eps, float *d_out,
                                              void *stream);

/* ------------------------------------------------------------ Qwen3 model */
/* One decoder layer's tensors, each a registered host key (LayerWeights,
 * forward_pass.rs:226-239).  Matmul tensors are Q4_0 (plain) or Q4_0X4;
 * norms are f32 host arrays (copied at model creation). */
typedef struct zgpu_qwen3_layer {
  const float *attn_norm;
  const void *attn_q, *attn_k, *attn_v, *attn_o;
  const float *q_norm, *k_norm;
  const float *ffn_norm;
  const void *ffn_gate, *ffn_up, *ffn_down;
} zgpu_qwen3_layer;

typedef struct zgpu_qwen3_desc {
  uint32_t n_layers, hidden, ffn, n_q_heads, n_kv_heads, head_dim;
  uint32_t vocab_padded, vocab_real;
  float rms_eps, rope_theta;
  uint32_t token_embd_quant;  /* ZGPU_Q8_0 or ZGPU_Q4_0, plain rows */
  const void *token_embd;     /* registered key */
  uint32_t output_quant;      /* ZGPU_Q8_0 or ZGPU_Q4_0 (stored X4 or plain) */
  const void *output;         /* registered key */
  const float *output_norm;
  const zgpu_qwen3_layer *layers;
} zgpu_qwen3_desc;

zgpu_status zgpu_qwen3_create(zgpu_ctx *ctx, const zgpu_qwen3_desc *desc, zgpu_model **out);
void zgpu_qwen3_destroy(zgpu_model *m);

/* Tensor parallelism (output rows sharded over 1-8 GPUs,
 * one process per GPU).  Rank `rank` of `world` keeps the q/k/v rows of its
 * kv heads (n_kv_heads / world of them; its attention and KV cache are
 * local: create the cache with n_kv_heads / world heads), gate/up SwiGLU
 * units, and row slices of O, down and the LM head, the slices the
 * reference's SMP partition splits by 4-row groups (smp_partition.rs:108-183)
 * spread over GPUs.  The decode step is one persistent kernel per GPU whose
 * stage epilogues store their rows straight into every rank's copy of the
 * activation vector over NVLink (peer stores of tagged words): the
 * all-gather is part of the kernel.  The LM head merges the ranks' argmax
 * (larger logit, smaller row on ties).  Every output row is reduced as on one
 * GPU, so tokens and logits equal the one-GPU decode bit for bit.
 * Requires n_kv_heads, hidden / 8, ffn / 8 and the LM-head units to divide by
 * world.  After creating every rank: zgpu_qwen3_tp_export on each, exchange
 * the handles (ZGPU_IPC_HANDLE_BYTES each, rank order), then
 * zgpu_qwen3_tp_connect on each, then a host barrier over the ranks (the
 * kernel's waits for a peer are bounded: no rank may start decoding while
 * another is still mapping handles).  A rank decodes through
 * zgpu_generate_greedy, or token by token through zgpu_forward_single_token
 * followed by zgpu_lm_head_argmax (all ranks make the same calls with the
 * same arguments, in the same order); logits_out then receives the rank's
 * vocab_padded / world rows per step, and every rank returns the same token.
 * Sampling (zgpu_lm_head_sample) and the per-op path are one-GPU only. */
#define ZGPU_IPC_HANDLE_BYTES 64
zgpu_status zgpu_qwen3_create_tp(zgpu_ctx *ctx, const zgpu_qwen3_desc *desc, uint32_t rank, uint32_t world,
                                 zgpu_model **out);
zgpu_status zgpu_qwen3_tp_export(zgpu_model *m, void *handle_out);
zgpu_status zgpu_qwen3_tp_connect(zgpu_model *m, const void *handles);
/* Has no counterpart in the reference: connects a tensor-parallel rank with
 * every other rank absent.  The other ranks' copies of the activation vectors
 * and argmax slots become local buffers that nothing reads, and the rows the
 * absent ranks own are never written, so the first stage that needs them
 * waits until its bounded device wait (1 s) expires; the call then returns
 * ZGPU_ERR_DEVICE_TIMEOUT and the context stays usable.  It exists to test,
 * on one GPU, how a rank whose peer never arrives fails. */
zgpu_status zgpu_qwen3_tp_connect_absent(zgpu_model *m);
/* forward_single_token (forward_pass.rs:515-631) /
 * forward_single_token_avx512 (inference_avx512.rs:1826-1987): token at
 * position `pos` through all layers, updating `kv`; the final hidden state
 * (pre-norm) is copied to hidden_out when non-NULL. */
zgpu_status zgpu_forward_single_token(zgpu_model *m, zgpu_kv *kv, uint32_t token, uint32_t pos,
                                      float *hidden_out);
/* lm_head_argmax_dynamic (lm_head.rs:98-166) / lm_head_argmax_avx512
 * (inference_avx512.rs:1200-1270) on the model's current hidden state:
 * final RMSNorm, logits over vocab_padded rows, first-max argmax, then the
 * non-finite / padding checks against vocab_real.  logits_out (nullable)
 * receives vocab_padded floats. */
zgpu_status zgpu_lm_head_argmax(zgpu_model *m, uint32_t vocab_real, uint32_t *token_out,
                                float *logits_out);
/* The reference's generation loop (inference.rs:1188-1320 prefill,
 * :1836-1999 decode): forward every prompt token, take the LM-head argmax
 * after the last one, then n_gen-1 greedy steps (forward + LM head).
 * tokens_out receives n_gen ids.  The decode step runs as one CUDA graph
 * replay with the token chained on the device.  logits_out (nullable)
 * receives n_gen * vocab_padded floats. */
zgpu_status zgpu_generate_greedy(zgpu_model *m, zgpu_kv *kv, const uint32_t *prompt,
                                 uint32_t n_prompt, uint32_t n_gen, uint32_t *tokens_out,
                                 float *logits_out);

/* Prompt prefill on the token-parallel path (no counterpart in the
 * reference, which runs forward_single_token per prompt token,
 * inference.rs:1188-1320): each layer's projections are batched Q4_0 x Q8_0
 * matmuls over all n tokens on the tensor cores (tcgen05 int8), attention is
 * causal over the prompt.  Writes cache positions [0, n) and returns the
 * LM-head argmax after the last token (logits_out, nullable: vocab_padded
 * floats).  Matmul inputs are quantised to Q8_0, so results agree with the
 * per-token path to that rounding.  Requires hidden, q+2kv and 2*ffn to be
 * multiples of 128.  zgpu_perf_snapshot's prefill_ms gives the device time. */
zgpu_status zgpu_prefill(zgpu_model *m, zgpu_kv *kv, const uint32_t *tokens, uint32_t n,
                         uint32_t *token_out, float *logits_out);
/* zgpu_prefill for n_seq prompts of n tokens each at once (BASELINE config 4
 * batch 8): sequence i's ids at tokens[i*n .. i*n+n), its cache kvs[i] (one
 * distinct cache per sequence), its next token in tokens_out[i] and (when
 * logits_out is non-NULL) its logits at logits_out[i*vocab_padded].  The
 * projections run over all n_seq*n rows; every result equals a one-sequence
 * zgpu_prefill of that prompt bit for bit. */
zgpu_status zgpu_prefill_batch(zgpu_model *m, zgpu_kv *const *kvs, uint32_t n_seq, const uint32_t *tokens,
                               uint32_t n, uint32_t *tokens_out, float *logits_out);
/* One greedy decode step for n_seq (1..256) independent sequences, each
 * with its own cache at its own position: per sequence the results of
 * zgpu_forward_single_token(kvs[i], tokens[i], positions[i]) followed by
 * zgpu_lm_head_argmax (forward_pass.rs:515-631, lm_head.rs:98-166), computed
 * as one batch.  The projections and the LM head run on the tensor cores over
 * Q8_0-quantised activation rows, as the prefill does (logits within the
 * prefill's tolerance of the per-token path, not bit-identical); the KV rows
 * are appended at positions[i].  tokens_out [n_seq]; logits_out
 * [n_seq][vocab_padded] or NULL.  An LM-head error of any sequence is
 * returned (its tokens_out entry still written).  Single-GPU models only;
 * head_dim 128, vocab_padded a multiple of 128. */
zgpu_status zgpu_decode_batch(zgpu_model *m, zgpu_kv *const *kvs, uint32_t n_seq, const uint32_t *tokens,
                              const uint32_t *positions, uint32_t *tokens_out, float *logits_out);

/* Per-kernel-class counters, mirroring Avx512PerfCounters
 * (inference_avx512.rs:274-330): calls and device milliseconds of the last
 * zgpu_generate_greedy decode phase. */
typedef struct zgpu_perf {
  uint64_t steps;
  uint64_t kernel_launches;   /* of this library's kernels, whole call */
  double decode_ms;           /* device time of the decode steps */
  double prefill_ms;
  uint64_t decode_launches;   /* kernel launches of the decode steps alone */
  double prefill_gemm_ms;     /* zgpu_prefill: device time of the projection GEMMs */
  double prefill_attn_ms;     /* zgpu_prefill: device time of the causal attention */
  double batch_gemm_ms;       /* zgpu_decode_batch: device time of the projection and LM-head GEMMs */
  double batch_attn_ms;       /* zgpu_decode_batch: device time of the attention launches */
} zgpu_perf;
zgpu_status zgpu_perf_snapshot(const zgpu_model *m, zgpu_perf *out);

/* ------------------------------------------- DeepSeek2: MoE routing */
/* MoeRoutingMode (crates/zero-llm-inference/src/moe.rs:55). */
#define ZGPU_ROUTE_SOFTMAX 0u
#define ZGPU_ROUTE_SIGMOID_NORMALIZE 1u
/* moe_route_f32 (moe.rs:132-317) on the GPU with host buffers: scores s_e =
 * sequential f32 dot(hidden, router row e) in the reference's order (+ bias
 * in Softmax mode; sigmoid in SigmoidNormalize mode), top-k by replacement of
 * the current minimum with a strict `>` (slot order, not sorted), weights =
 * softmax (or normalisation) over the selected k, the uniform 1/k fallback,
 * then expert_weight_scale.  Expert ids are bit-identical to the
 * reference's; weights agree to the rounding of expf.  router_key is a
 * registered ZGPU_F32 tensor [n_experts x dim]; router_bias (host, n_experts
 * floats) and scores_out (n_experts floats) may be NULL.  Where the
 * reference panics (top_k == 0 or top_k > n_experts) this returns
 * ZGPU_ERR_INVALID_ARG; top_k is at most 16 and dim at most 8192. */
zgpu_status zgpu_moe_route_f32(zgpu_ctx *ctx, const float *hidden, const void *router_key,
                               const float *router_bias, uint64_t dim, uint32_t n_experts,
                               uint32_t top_k, uint32_t mode, float expert_weight_scale,
                               float *scores_out, uint32_t *indices_out, float *weights_out);

/* ------------------------------------------------- DeepSeek2: MLA cache */
typedef struct zgpu_mla_kv zgpu_mla_kv;
/* MlaKvCache::new (kv_cache.rs:257-305): per layer max_tokens rows of
 * [kv_lora_rank | rope_dim] f32 (the normalised latent and the rotated
 * k_rope) in device memory. */
zgpu_status zgpu_mla_kv_create(zgpu_ctx *ctx, uint32_t max_tokens, uint32_t n_layers,
                               uint32_t kv_lora_rank, uint32_t rope_dim, zgpu_mla_kv **out);
void zgpu_mla_kv_destroy(zgpu_mla_kv *kv);
/* store_compressed (kv_cache.rs:318-360): c_kv [kv_lora_rank], k_rope
 * [rope_dim] (host). Errors: LayerOutOfRange, TokenIndexOutOfRange. */
zgpu_status zgpu_mla_kv_store(zgpu_mla_kv *kv, uint32_t layer, uint32_t token, const float *c_kv,
                              const float *k_rope);
/* get_c_kv / get_k_rope (kv_cache.rs:362-407) for tokens [0, token_count):
 * token_count rows of kv_lora_rank + rope_dim floats copied to host. */
zgpu_status zgpu_mla_kv_read(zgpu_mla_kv *kv, uint32_t layer, uint32_t token_count,
                             float *rows_out);
/* Device-to-device copy of rows [0, token_count) of every layer from src to
 * dst (same context and geometry), stream-ordered: a sequence forked from a
 * shared prompt without a second prefill.  Not in the reference (MlaKvCache
 * has no clone); the serving bench uses it to give 32 sequences one filled
 * context. */
zgpu_status zgpu_mla_kv_copy(zgpu_mla_kv *dst, const zgpu_mla_kv *src, uint32_t token_count);

/* ------------------------------------------------- DeepSeek2 model */
typedef struct zgpu_ds2_model zgpu_ds2_model;
/* One layer (Deepseek2LayerWeights, forward_pass.rs:640-700).  Matmul
 * tensors are registered keys (Q4_0 or Q8_0 = attn_quant, plain or X4);
 * norms are host f32 arrays copied at creation.  MLA: kv_b holds per head
 * nope rows then v rows; or k_b / v_b (both non-NULL) hold them split
 * (mla.rs:251-275).  Dense layers (moe == 0) use ffn_gate/up/down; MoE layers
 * use router_w (registered ZGPU_F32 [n_experts x hidden]), router_b (host,
 * nullable), the stacked experts gate_exps/up_exps [n_experts*expert_ffn x
 * hidden] and down_exps [n_experts*hidden x expert_ffn], and the stacked
 * shared experts (n_shared of width expert_ffn, same layout). */
typedef struct zgpu_ds2_layer {
  const float *attn_norm, *ffn_norm;
  const void *kv_a_mqa;          /* [kv_lora + rope] x hidden */
  const float *kv_a_norm;        /* [kv_lora] */
  const void *kv_b;              /* [n_heads*(nope+v)] x kv_lora, or NULL with k_b/v_b */
  const void *k_b, *v_b;
  const void *q_a;               /* q_lora x hidden */
  const float *q_a_norm;         /* [q_lora] */
  const void *q_b;               /* [n_heads*(nope+rope)] x q_lora */
  const void *attn_output;       /* hidden x [n_heads*v] */
  const float *k_norm;           /* [rope] or NULL */
  uint32_t moe;
  const void *ffn_gate, *ffn_up, *ffn_down;
  const void *router_w;
  const float *router_b;
  const void *gate_exps, *up_exps, *down_exps;
  const void *gate_shexp, *up_shexp, *down_shexp;
  /* AttnType (forward_pass.rs:51-57): ZGPU_ATTN_MLA, or ZGPU_ATTN_MHA for a
   * layer with standard attention (mla.rs:449-618): q_mha [n_heads*(nope+rope)
   * x hidden], k_mha [n_kv*(nope+rope) x hidden], v_mha [n_kv*v x hidden] and
   * attn_output; the MLA tensors and norms are then unused (may be NULL). */
  uint32_t attn_type;
  const void *q_mha, *k_mha, *v_mha;
} zgpu_ds2_layer;
#define ZGPU_ATTN_MLA 0u
#define ZGPU_ATTN_MHA 1u

typedef struct zgpu_ds2_desc {
  uint32_t n_layers, hidden, ffn, n_heads;
  uint32_t kv_lora_rank, q_lora_rank, nope_dim, rope_dim, v_dim;
  uint32_t n_experts, top_k, expert_ffn, n_shared;
  uint32_t vocab_padded, vocab_real;
  float rms_eps, rope_theta;
  uint32_t route_mode;           /* ZGPU_ROUTE_* */
  float expert_weight_scale;
  uint32_t attn_quant;           /* ZGPU_Q4_0 or ZGPU_Q8_0: every matmul of the layers */
  uint32_t token_embd_quant;     /* ZGPU_Q8_0 or ZGPU_Q4_0 */
  const void *token_embd;
  uint32_t output_quant;
  const void *output;
  const float *output_norm;
  const zgpu_ds2_layer *layers;
  uint32_t n_kv_heads;           /* kv heads of the MHA layers (0: n_heads) */
} zgpu_ds2_desc;

zgpu_status zgpu_ds2_create(zgpu_ctx *ctx, const zgpu_ds2_desc *desc, zgpu_ds2_model **out);

/* MhaKvCache (kv_cache.rs:433-560) in device memory, same layout: per MHA
 * layer a K block [max_tokens][n_kv*head_dim_qk] then a V block
 * [max_tokens][n_kv*head_dim_v].  store_kv / get_k_slice + get_v_slice as
 * zgpu_mha_kv_store / zgpu_mha_kv_read (host buffers). */
typedef struct zgpu_mha_kv zgpu_mha_kv;
zgpu_status zgpu_mha_kv_create(zgpu_ctx *ctx, uint32_t max_tokens, uint32_t n_mha_layers, uint32_t n_kv_heads,
                               uint32_t head_dim_qk, uint32_t head_dim_v, zgpu_mha_kv **out);
void zgpu_mha_kv_destroy(zgpu_mha_kv *kv);
zgpu_status zgpu_mha_kv_store(zgpu_mha_kv *kv, uint32_t layer, uint32_t token, const float *k, const float *v);
zgpu_status zgpu_mha_kv_read(zgpu_mha_kv *kv, uint32_t layer, uint32_t token_count, float *k_out, float *v_out);
/* The MHA cache the model's MHA layers use (forward_single_token_deepseek2's
 * mha_kv_cache argument, forward_pass.rs:730): the n-th MHA layer uses slot n.
 * Required before a forward when the model has MHA layers (without it the
 * forward returns ZGPU_ERR_NUMERICAL_INSTABILITY, as the reference's
 * forward_pass.rs:791-793); NULL unbinds. */
zgpu_status zgpu_ds2_set_mha_kv(zgpu_ds2_model *m, zgpu_mha_kv *kv);
void zgpu_ds2_destroy(zgpu_ds2_model *m);
/* Expert parallelism (experts sharded over 1-8 GPUs, one
 * process per GPU).  Rank `rank` of `world` runs routed experts
 * [rank*E/world, (rank+1)*E/world) of every MoE layer (moe_ffn, moe.rs:486-590);
 * the router, attention, dense layers, shared experts and LM head run on
 * every rank.  After the grouped expert GEMVs, a rank stores its selected
 * experts' outputs as tagged words into slot k of every rank's exchange
 * buffer over NVLink, and every rank's combine waits (bounded) for all top_k
 * slots and adds them in the reference's k order, so tokens, logits and
 * expert ids equal the one-GPU model bit for bit.  Requires n_experts to
 * divide by world.  Bring-up as zgpu_qwen3_create_tp: create every rank,
 * zgpu_ds2_ep_export on each, exchange the ZGPU_IPC_HANDLE_BYTES handles in
 * rank order, zgpu_ds2_ep_connect on each, then a host barrier over the
 * ranks (no rank's first exchange may start while a peer is still mapping
 * handles); then every rank makes the same calls (forward, LM head,
 * generate) with the same arguments.  A combine wait for another rank that
 * runs out (5 s) fails the call with ZGPU_ERR_DEVICE_TIMEOUT,
 * naming the wait in zgpu_last_error, and aborts the model's exchange:
 * every later call fails at once the same way; create the ranks again to
 * recover.  Status of this build: its two-GPU tests end with such timeouts
 * (an open defect), so bit identity with one GPU is not established. */
zgpu_status zgpu_ds2_create_ep(zgpu_ctx *ctx, const zgpu_ds2_desc *desc, uint32_t rank, uint32_t world,
                               zgpu_ds2_model **out);
zgpu_status zgpu_ds2_ep_export(zgpu_ds2_model *m, void *handle_out);
zgpu_status zgpu_ds2_ep_connect(zgpu_ds2_model *m, const void *handles);
/* forward_single_token_deepseek2 (forward_pass.rs:703-909) for MLA layers:
 * per layer rmsnorm -> MLA (mla.rs:122-414, with the kv_b projection
 * absorbed into the query and the output: same results to f32 rounding)
 * -> residual -> rmsnorm -> dense SwiGLU or moe_ffn -> residual. */
zgpu_status zgpu_ds2_forward_single_token(zgpu_ds2_model *m, zgpu_mla_kv *kv, uint32_t token,
                                          uint32_t pos, float *hidden_out);
/* lm_head_argmax_dynamic (lm_head.rs:98-166) on the model's hidden state. */
zgpu_status zgpu_ds2_lm_head_argmax(zgpu_ds2_model *m, uint32_t vocab_real, uint32_t *token_out,
                                    float *logits_out);
/* Expert ids / weights each MoE layer routed to in the last forward:
 * [n_layers][top_k] each (zeros for dense layers); either may be NULL. */
zgpu_status zgpu_ds2_expert_ids(zgpu_ds2_model *m, uint32_t *ids_out, float *weights_out);
/* Prompt prefill + n_gen greedy steps as zgpu_generate_greedy; the step is
 * one CUDA graph replay with the token chained on the device. */
zgpu_status zgpu_ds2_generate_greedy(zgpu_ds2_model *m, zgpu_mla_kv *kv, const uint32_t *prompt,
                                     uint32_t n_prompt, uint32_t n_gen, uint32_t *tokens_out,
                                     float *logits_out);
/* One decode step of n_seq (1..32) independent sequences, each with its own
 * MLA cache (all of one capacity, none twice) at its own position: for every
 * b, the result equals zgpu_ds2_forward_single_token(kvs[b], tokens[b],
 * positions[b]) followed by zgpu_ds2_lm_head_argmax(vocab_real) (tokens_out[b],
 * logits row b of n_seq x vocab_padded when logits_out is not NULL; the
 * cache rows appended) -- bit for bit while both split the attention into
 * 16-token pieces (a cache capacity below 2 * SMs * 16 / n_seq rows), to f32
 * rounding beyond that, where the batch takes longer splits.  It replaces the serving loop that
 * calls forward_single_token_deepseek2 (forward_pass.rs:703-909) and
 * lm_head_argmax_dynamic (lm_head.rs:98-166) once per sequence: each
 * weight tile is fetched once per step for the whole batch.  With expert
 * parallelism every rank makes the same call; each rank runs its own
 * experts for every token that selected them and the outputs cross NVLink as
 * in the one-token step.  MLA layers only (a model with MHA layers returns
 * ZGPU_ERR_INVALID_ARG). */
zgpu_status zgpu_ds2_decode_batch(zgpu_ds2_model *m, zgpu_mla_kv *const *kvs, uint32_t n_seq,
                                  const uint32_t *tokens, const uint32_t *positions, uint32_t *tokens_out,
                                  float *logits_out);
/* Expert ids / weights of the last zgpu_ds2_decode_batch: [n_layers][n_seq][top_k]
 * each (zeros for dense layers); either may be NULL. */
zgpu_status zgpu_ds2_batch_expert_ids(zgpu_ds2_model *m, uint32_t n_seq, uint32_t *ids_out, float *weights_out);
zgpu_status zgpu_ds2_perf_snapshot(const zgpu_ds2_model *m, zgpu_perf *out);

/* ------------------------------------------ synthetic .smodel generation */
/* Deterministic seeded tensors for the BASELINE configs (counter-based
 * SplitMix64, so any sub-range is reproducible).  Blocks are written in the
 * plain row-major layout; zgpu_pack_x4 re-lays them out as the packer's
 * writer does (tools/silicatepack.py:982-1022). */
/* Q4_0: nibbles uniform 0..15, d = fp16(|N(0, sigma)| / 8). */
void zgpu_synth_q4_0(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, float sigma,
                     void *out);
/* Q8_0: i8 uniform -127..127, d = fp16(scale). */
void zgpu_synth_q8_0(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, float scale,
                     void *out);
/* f32 N(mean, sigma) values (sigma 0 gives a constant). */
void zgpu_synth_f32(uint64_t seed, uint64_t stream, uint64_t n, float mean, float sigma,
                    float *out);
/* uniform token ids in [0, vocab). */
void zgpu_synth_tokens(uint64_t seed, uint64_t stream, uint64_t n, uint32_t vocab, uint32_t *out);
/* Plain -> X4 (quant ZGPU_Q4_0 or ZGPU_Q8_0); rows % 4 == 0, cols % 32 == 0. */
zgpu_status zgpu_pack_x4(const void *plain, void *x4, uint64_t rows, uint64_t cols,
                         uint32_t quant);

/* ------------------------------------------------------------ sampling */
/* lm_head_sample (kernel/src/sampler.rs:41-163) on the GPU: top-40 of
 * logits[0, min(len, vocab_real)) kept as the reference keeps them (the
 * running minimum replaced on a strict >, slot order preserved), scaled by
 * 1 / temperature, softmax with the reference's exp_approx, one draw
 * r = next_u32 / u32::MAX of the xorshift64 state *rng_state (rng.rs:23-46;
 * Rng::new(0) starts from 0x853c49e6748fea9b, the caller's job) against the
 * cumulative sum.  *rng_state advances by one draw.  Token and state equal
 * the reference's bit for bit.  The reference fixes vocab_real to 151643.
 * zgpu_sample_top_k takes host logits; zgpu_lm_head_sample samples the
 * model's logits of its last LM-head call (as inference.rs:2024 follows
 * lm_head with lm_head_sample). */
zgpu_status zgpu_sample_top_k(zgpu_ctx *ctx, const float *logits, uint32_t len, uint32_t vocab_real, float temperature,
                              uint64_t *rng_state, uint32_t *token_out);
zgpu_status zgpu_lm_head_sample(zgpu_model *m, uint32_t vocab_real, float temperature, uint64_t *rng_state,
                                uint32_t *token_out);

/* ------------------------------------------------ .smodel containers */
/* The SilicatePack native container (.smodel v1/v2) the reference's loader
 * boots from (kernel/src/model_loader.rs:256-661; writer
 * tools/silicatepack.py:1097-1410), mapped read-only with the loader's
 * validation: header, SIDX index (<= 10000 entries of 104 bytes), names,
 * tensor ranges, row-interleaved dtypes only on rank-2 tensors with rows a
 * multiple of 4.  Only native payloads are read (a GGUF-compat payload gives
 * ZGPU_ERR_MODEL_UNSUPPORTED). */
typedef struct zgpu_smodel zgpu_smodel;
typedef struct zgpu_smodel_info {
  uint32_t version, payload_kind, flags, tensor_count;
  uint64_t manifest_offset, manifest_len, payload_offset, payload_len, data_base;
  /* the SIDX model fields (ModelConfig, model_loader.rs:430-480); 0xFFFFFFFF: none */
  uint32_t architecture_id, block_count, context_length, embedding_length, feed_forward_length;
  uint32_t head_count, head_count_kv, key_length, value_length;
  float rope_freq_base, layer_norm_rms_epsilon;
  uint32_t vocab_size, eos_token_id, expert_count, expert_used_count, expert_shared_count;
  uint32_t expert_feed_forward_length, kv_lora_rank, q_lora_rank, qk_nope_head_dim, qk_rope_head_dim;
  uint32_t v_head_dim;
  float expert_weights_scale;
} zgpu_smodel_info;
typedef struct zgpu_smodel_tensor {
  const char *name;             /* owned by the handle */
  uint32_t dtype, rank;         /* SIDX dtype id (0 F32, 2 Q4_0, 8 Q8_0, 100 Q4_0X4, 101 Q8_0X4, ...) */
  uint64_t shape[8];            /* HF order: shape[0] = output rows of a matmul */
  uint64_t payload_offset, byte_len, elements;
  const void *data;             /* the mapped bytes (the tensor's registry key) */
} zgpu_smodel_tensor;
zgpu_status zgpu_smodel_open(const char *path, zgpu_smodel **out);
void zgpu_smodel_close(zgpu_smodel *m);
/* message of the last zgpu_smodel_* failure of this thread */
const char *zgpu_smodel_error(void);
zgpu_status zgpu_smodel_info_get(const zgpu_smodel *m, zgpu_smodel_info *out);
zgpu_status zgpu_smodel_manifest(const zgpu_smodel *m, const char **json, uint64_t *len);
zgpu_status zgpu_smodel_tensor_at(const zgpu_smodel *m, uint32_t i, zgpu_smodel_tensor *out);
zgpu_status zgpu_smodel_find(const zgpu_smodel *m, const char *name, zgpu_smodel_tensor *out);
/* zgpu_register_weights for every rank-2 F32 / Q4_0 / Q8_0 / Q4_0X4 / Q8_0X4
 * tensor, keyed by its mapped address (weight_layout::register keys by the
 * same address, model_loader.rs:560-566); keep the container open while
 * models built from it are created. */
zgpu_status zgpu_smodel_register(zgpu_ctx *ctx, const zgpu_smodel *m, uint32_t *registered);

/* ---------------------------------------------------------- detokenizer */
/* Token ids -> bytes for streaming output (kernel/src/detokenizer.rs): a
 * vocabulary of byte strings, offsets[i] .. offsets[i + 1] being token i's
 * bytes (vocab_size + 1 little-endian u32 entries, the layout of the
 * reference's vocab_offsets.bin / tools/extract_vocab.py).  create copies
 * both tables (install_runtime_vocab, detokenizer.rs:208-256; vocab_size 0
 * is ZGPU_ERR_INVALID_ARG).  An id past the vocabulary, or an entry whose
 * offsets run backwards or past the byte table, decodes to no bytes
 * (decode_token, :110-205).  Host code; no device work. */
typedef struct zgpu_detok zgpu_detok;
zgpu_status zgpu_detok_create(const void *bytes, uint64_t n_bytes, const uint32_t *offsets, uint32_t vocab_size,
                              zgpu_detok **out);
void zgpu_detok_destroy(zgpu_detok *d);
uint32_t zgpu_detok_vocab_size(const zgpu_detok *d);
/* Token id's bytes: *bytes_out points into the detokenizer's table (valid
 * until destroy), *len_out may be 0. */
zgpu_status zgpu_detok_token(const zgpu_detok *d, uint32_t id, const uint8_t **bytes_out, uint64_t *len_out);
/* The bytes of n ids, concatenated into out[cap]; *written = the bytes they
 * take.  If that exceeds cap, nothing is written and the call returns
 * ZGPU_ERR_INVALID_ARG with *written the size needed. */
zgpu_status zgpu_detok_decode(const zgpu_detok *d, const uint32_t *ids, uint64_t n, uint8_t *out, uint64_t cap,
                              uint64_t *written);

#ifdef __cplusplus
}
#endif
#endif /* ZGPU_H */
