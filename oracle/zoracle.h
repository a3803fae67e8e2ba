/*
 * zoracle.h — CPU parity oracle for the zero-llm-inference decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is a plain-C restatement of the
 * reference's CPU algorithms (silicatetech/zero).  Only tests/, the smoke()
 * check in __graft_entry__.py and bench.py's cpu_baseline / reference arm
 * may load it, and only as the checker or the timed CPU baseline — never
 * as part of the product path (zero_b200/ never links or imports it).
 *
 * Two orders are restated:
 *   - "scalar": the crate `crates/zero-llm-inference` (sequential f32,
 *     unfused multiply-add, libm expf/sinf/cosf/powf/sqrtf), which reads
 *     plain Q4_0/Q8_0 blocks;
 *   - "avx512": the kernel-side SIMD path `kernel/src/inference_avx512.rs`
 *     + `kernel/src/arch/x86_64/math/{linear,activation,trig}.rs`, whose
 *     16-lane accumulator order, FMA use and horizontal-reduction tree are
 *     restated lane by lane (portable C with fmaf), and — when the host has
 *     AVX-512F — also with real intrinsics for the timed baseline.  Both
 *     forms must agree bit for bit (tested).
 *
 * Pinning: the block encoders and X4 permutation are pinned against golden
 * fixtures generated from the reference's own tools/silicatepack.py
 * (tests/golden/gen_packer_golden.py); the linear/dequant/rmsnorm/rope
 * known-answer values come from the reference's unit tests
 * (ops.rs:531-1160, dequant.rs:553-1088).  The libm crate 0.2.16
 * (Cargo.lock:331) is not vendored: glibc's expf/powf share its upstream
 * algorithm; sinf/cosf agreement is at the <=1 ULP level (unpinned).
 */
#ifndef ZORACLE_H
#define ZORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (zero-gguf-parser lib.rs GgmlType) and the .smodel v2 ids. */
enum { ZO_F32 = 0, ZO_F16 = 1, ZO_Q4_0 = 2, ZO_Q8_0 = 8, ZO_Q4_K = 12, ZO_Q6_K = 14, ZO_Q4_0X4 = 100, ZO_Q8_0X4 = 101 };

/* Error codes (mirror of the Rust enums the path returns). */
enum {
  ZO_OK = 0,
  ZO_ERR_ARG = 1,
  ZO_ERR_UNSUPPORTED_QUANT = 2,
  ZO_ERR_KV_TOKEN_OUT_OF_RANGE = 10,
  ZO_ERR_KV_LAYER_OUT_OF_RANGE = 11,
  ZO_ERR_KV_TOKEN_COUNT = 13,
  ZO_ERR_NUMERICAL_INSTABILITY = 20,
  ZO_ERR_LM_NON_FINITE = 40,
  ZO_ERR_LM_PADDING = 41,
};

/* ---- fp16 / block codecs ------------------------------------------------ */
float    zo_fp16_to_f32(uint16_t bits);
uint16_t zo_f64_to_fp16(double v);
void     zo_dequant_q4_0_block(const uint8_t *blk, float *out32);
void     zo_dequant_q8_0_block(const uint8_t *blk, float *out32);
void     zo_quantize_q4_0_block(const float *v32, uint8_t *out18);
void     zo_quantize_q8_0_block(const float *v32, uint8_t *out34);
/* Q8_0 activation quantiser (n % 32 == 0): one zo_quantize_q8_0_block per block. */
void     zo_quantize_row_q8_0(const float *x, uint8_t *out, size_t n);
/* dequant.rs:63-138: Q4_K super-block (144 bytes -> 256 floats). */
void     zo_dequant_q4_k_block(const uint8_t *blk, float *out);
/* dequant.rs:286-356: Q6_K super-block (210 bytes -> 256 floats), the
 * canonical half-half layout ("pattern C"). */
void     zo_dequant_q6_k_block(const uint8_t *blk, float *out);
/* ops.rs:179-292: linear_q4k / linear_q6k, plain rows of super-blocks. */
void     zo_linear_q4_k(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim);
void     zo_linear_q6_k(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim);
/* rng.rs:23-46: xorshift64 (13, 7, 17); next_u32 = high half of next_u64. */
uint32_t zo_rng_next_u32(uint64_t *state);
/* sampler.rs:123-163: the sampler's own exp approximation. */
float    zo_exp_approx(float x);
/* sampler.rs:41-120 lm_head_sample: top-40 of logits[0 .. min(len,
 * vocab_real)) by replacement of the running minimum (strict >, slot order
 * kept), / temperature, softmax with zo_exp_approx, one draw r =
 * next_u32 / u32::MAX against the cumulative sum in slot order.  The
 * reference fixes vocab_real to 151643. */
uint32_t zo_lm_head_sample(const float *logits, uint32_t len, uint64_t *rng_state, float temperature,
                           uint32_t vocab_real);
/* Plain -> .smodel-v2 4-row interleave.  quant = ZO_Q4_0 or ZO_Q8_0. */
int      zo_interleave_x4(const uint8_t *plain, uint8_t *x4, size_t rows, size_t cols, int quant);

/* Q4_0 weights (plain) x Q8_0 activation blocks: no counterpart in the
 * reference decode path; restates ggml's vec_dot_q4_0_q8_0 reference loop
 * (the GGUF ecosystem's definition of this product, zero-gguf-parser carries
 * the formats): per block sumi = sum_j (n_j - 8) * q_j exactly, then
 * acc += (sumi * d_w) * d_x in block order. */
void     zo_linear_q8_0_q8act(const uint8_t *xq, const uint8_t *w, float *out, size_t in_dim,
                              size_t out_dim);
void     zo_linear_q4_0_q8act(const uint8_t *xq, const uint8_t *w, float *out, size_t in_dim,
                              size_t out_dim);

/* ---- scalar crate ops --------------------------------------------------- */
void  zo_rmsnorm(const float *x, const float *w, float *out, size_t n, float eps);
void  zo_rope_ctx(float freq_base, size_t half, float *inv_freqs);
void  zo_rope(float *qk, const float *inv_freqs, size_t half, size_t pos);
void  zo_linear_q4_0(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim);
void  zo_linear_q8_0(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim);
int   zo_linear_dispatch(const float *x, const uint8_t *w, float *out, size_t in_dim,
                         size_t out_dim, int quant);
int   zo_softmax(float *scores, size_t len);
/* One layer of decode attention: QK-norm, RoPE, store_kv, softmax(q.k) . V
 * (attention.rs:344-425 for order 0, inference_avx512.rs:1612-1800 for
 * order 1); work = (n_q + n_kv + 1)*hd + max_tokens floats. */
int   zo_gqa_attention_decode(const float *q, const float *k, const float *v, const float *q_norm,
                              const float *k_norm, const float *inv_freqs, float *k_block,
                              float *v_block, uint32_t pos, uint32_t max_tokens, uint32_t n_q,
                              uint32_t n_kv, uint32_t hd, float eps, int order, float *work,
                              float *out);

/* ---- AVX-512-order ops (lane-exact restatement) -------------------------- */
/* threads <= 0 -> all cores.  simd: 0 portable lane emulation, 1 intrinsics
 * when available (falls back to emulation otherwise). */
void  zo_linear_q4_0x4_avx512(const float *x, const uint8_t *w_x4, float *out, size_t in_dim,
                              size_t out_dim, int threads, int simd);
void  zo_linear_q8_0x4_avx512(const float *x, const uint8_t *w_x4, float *out, size_t in_dim,
                              size_t out_dim, int threads, int simd);
/* Same per-row math on the plain layout (linear.rs:710, :1271). */
void  zo_linear_q4_0_avx512(const float *x, const uint8_t *w, float *out, size_t in_dim,
                            size_t out_dim, int threads, int simd);
void  zo_linear_q8_0_avx512(const float *x, const uint8_t *w, float *out, size_t in_dim,
                            size_t out_dim, int threads, int simd);
float zo_dot_product_avx512(const float *a, const float *b, size_t len);
void  zo_weighted_add_avx512(float weight, const float *vec, float *out, size_t len);
size_t zo_argmax_avx512(const float *v, size_t n, float *max_out);
void  zo_exp_avx512(const float *x, float *y, size_t n);
void  zo_silu_mul_avx512(const float *g, const float *u, float *out, size_t n);
void  zo_rope_sincos_lut_avx512(size_t pos, const float *inv_freqs, float *cos_out,
                                float *sin_out, size_t len);
void  zo_rope_apply_avx512(float *qk, const float *cos_lut, const float *sin_lut, size_t half);
int   zo_have_avx512(void);

/* ---- Qwen3-shaped model ------------------------------------------------- */
typedef struct zo_qwen3_layer {
  const float   *attn_norm;   /* [hidden] */
  const uint8_t *attn_q;      /* plain Q4_0 [q_dim x hidden] */
  const uint8_t *attn_k;      /* plain Q4_0 [kv_dim x hidden] */
  const uint8_t *attn_v;      /* plain Q4_0 [kv_dim x hidden] */
  const uint8_t *attn_o;      /* plain Q4_0 [hidden x q_dim] */
  const float   *q_norm;      /* [head_dim] */
  const float   *k_norm;      /* [head_dim] */
  const float   *ffn_norm;    /* [hidden] */
  const uint8_t *ffn_gate;    /* plain Q4_0 [ffn x hidden] */
  const uint8_t *ffn_up;      /* plain Q4_0 [ffn x hidden] */
  const uint8_t *ffn_down;    /* plain Q4_0 [hidden x ffn] */
} zo_qwen3_layer;

typedef struct zo_qwen3 {
  uint32_t n_layers, hidden, ffn, n_q_heads, n_kv_heads, head_dim;
  uint32_t vocab_padded, vocab_real;
  float    rms_eps, rope_theta;
  int      token_embd_quant;   /* ZO_Q8_0 (plain rows) */
  const uint8_t *token_embd;   /* [vocab x hidden] */
  int      output_quant;       /* ZO_Q8_0 or ZO_Q4_0 */
  const uint8_t *output;       /* plain [vocab x hidden] (tied: == token_embd) */
  const float   *output_norm;  /* [hidden] */
  const zo_qwen3_layer *layers;
} zo_qwen3;

/* order: 0 = scalar crate path (forward_pass.rs:515), 1 = AVX-512 kernel path
 * (inference_avx512.rs:1826).  The run keeps its own f32 KV cache with the
 * kv_cache.rs:100 layout. */
/* Persistent dispatcher of the timed baseline: threads <= 0 -> one
 * participant per physical core the process may use.  Worker threads are
 * pinned one per core; the calling thread is participant 0. */
typedef struct zo_pool zo_pool;
zo_pool *zo_pool_create(int threads);
void     zo_pool_destroy(zo_pool *p);
int      zo_pool_size(const zo_pool *p);
/* linear_dispatch_avx512 on plain Q4_0 / Q8_0 rows over the pool (NULL: the
 * calling thread); simd 0 runs the lane emulation (same bits). */
int      zo_linear_plain_pool(zo_pool *p, const float *x, const uint8_t *w, float *out,
                              size_t in_dim, size_t out_dim, int quant, int simd);

typedef struct zo_run zo_run;
zo_run *zo_run_create(const zo_qwen3 *m, uint32_t max_tokens, int order, int threads, int simd);
void    zo_run_destroy(zo_run *r);
int     zo_run_forward(zo_run *r, uint32_t token, uint32_t pos, float *hidden_out);
/* lm_head_argmax_dynamic (lm_head.rs:98) / lm_head_argmax_avx512 (inference_avx512.rs:1200). */
int     zo_run_lm_head(zo_run *r, uint32_t *token_out, float *logits_out);
const float *zo_run_kv(const zo_run *r);
/* Q4_0 matmuls on Q8_0-quantised inputs (the prefill path's arithmetic). */
void    zo_run_set_q8act(zo_run *r, int on);
/* Prefill the prompt (one forward per token) then n_gen greedy steps. tokens_out
 * receives n_gen ids; margins_out (nullable) the top1-top2 logit gap per step;
 * logits_last (nullable) the logits of the final step. Returns the status of the
 * first failing call, or ZO_OK. */
int     zo_run_generate(zo_run *r, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen,
                        uint32_t *tokens_out, float *margins_out, float *logits_all);

/* ---- DeepSeek2: MoE routing / experts / MLA (zoracle_ds2.c) ---------------- */
/* MoeRoutingMode (moe.rs:55). */
enum { ZO_ROUTE_SOFTMAX = 0, ZO_ROUTE_SIGMOID_NORMALIZE = 1 };

/* moe.rs:132-317.  router_w f32 [n_experts x dim]; router_bias nullable. */
int zo_moe_route_f32(const float *hidden, size_t dim, const float *router_w,
                     const float *router_bias, size_t n_experts, size_t top_k, float *score_buf,
                     uint32_t *indices, float *weights, int mode, float expert_weight_scale);
/* moe.rs:345-397; work 3 * inter floats. */
int zo_expert_swiglu(const float *x, const uint8_t *gate_w, const uint8_t *up_w,
                     const uint8_t *down_w, size_t dim, size_t inter, int quant, float *work,
                     float *out);
/* moe.rs:486-590 with n_shared stacked shared experts of width inter (1 is
 * the reference's case); work n_experts + 3 * inter + dim floats. */
int zo_moe_ffn(const float *x, const float *router_w, const float *router_bias,
               const uint8_t *gate_exps, const uint8_t *up_exps, const uint8_t *down_exps,
               const uint8_t *gate_sh, const uint8_t *up_sh, const uint8_t *down_sh,
               size_t n_shared, size_t n_experts, size_t top_k, size_t dim, size_t inter,
               int quant, int mode, float expert_weight_scale, float *work, uint32_t *ids_out,
               float *weights_out, float *out);

typedef struct zo_mla_dims {
  uint32_t hidden, n_heads, kv_lora_rank, q_lora_rank, nope_dim, rope_dim, v_dim;
  int      quant;        /* attn_quant: ZO_Q4_0 or ZO_Q8_0 (plain rows) */
  float    eps, rope_base;
} zo_mla_dims;

/* MlaWeights (mla.rs:47-58); plain row-major blocks. */
typedef struct zo_mla_weights {
  const uint8_t *kv_a_mqa;   /* [kv_lora + rope] x hidden */
  const float   *kv_a_norm;  /* [kv_lora] */
  const uint8_t *kv_b;       /* [n_heads * (nope + v)] x kv_lora (per head: nope rows, then v rows) */
  const uint8_t *k_b, *v_b;  /* optional split form: [n_heads*nope] x kv_lora, [n_heads*v] x kv_lora */
  const uint8_t *q_a;        /* q_lora x hidden */
  const float   *q_a_norm;   /* [q_lora] */
  const uint8_t *q_b;        /* [n_heads * (nope + rope)] x q_lora */
  const uint8_t *output;     /* hidden x [n_heads * v] */
  const float   *k_norm;     /* [rope] or NULL */
} zo_mla_weights;

size_t zo_mla_work_floats(const zo_mla_dims *d, uint32_t max_tokens);
/* mla.rs:122-414; cache_layer = [max_tokens][kv_lora | rope] of this layer. */
int zo_mla_attention(const float *x, const zo_mla_weights *w, const zo_mla_dims *d,
                     float *cache_layer, uint32_t pos, uint32_t max_tokens, float *work,
                     float *out);

typedef struct zo_ds2_layer {
  const float   *attn_norm, *ffn_norm;   /* [hidden] */
  zo_mla_weights mla;
  int            moe;                    /* 0: dense SwiGLU FFN */
  const uint8_t *ffn_gate, *ffn_up, *ffn_down;            /* dense: [ffn x hidden], [hidden x ffn] */
  const float   *router_w, *router_b;                     /* f32 [n_experts x hidden], bias nullable */
  const uint8_t *gate_exps, *up_exps, *down_exps;         /* stacked [n_experts][inter x hidden] ... */
  const uint8_t *gate_shexp, *up_shexp, *down_shexp;      /* stacked [n_shared][...] */
  int            mha;                    /* AttnType::Mha: standard attention instead of mla */
  const uint8_t *q_mha, *k_mha, *v_mha;  /* [n_heads*(nope+rope)], [n_kv*(nope+rope)], [n_kv*v] x hidden;
                                            the output projection is mla.output */
} zo_ds2_layer;

typedef struct zo_ds2 {
  uint32_t n_layers, ffn, n_experts, top_k, expert_ffn, n_shared;
  uint32_t vocab_padded, vocab_real;
  zo_mla_dims mla;
  int      route_mode;
  float    expert_weight_scale;
  int      token_embd_quant;   /* plain rows */
  const uint8_t *token_embd;
  int      output_quant;
  const uint8_t *output;       /* plain [vocab x hidden] */
  const float   *output_norm;
  const zo_ds2_layer *layers;
  uint32_t n_kv_heads;         /* MHA layers' kv heads (0: n_heads) */
} zo_ds2;

/* mla.rs:449-618 (mha_attention_single_token): k_cache / v_cache are this
 * MHA layer's K and V blocks ([max_tokens][n_kv * (nope + rope)] and
 * [max_tokens][n_kv * v], kv_cache.rs:433-560 MhaKvCache); work:
 * zo_mha_work_floats floats. */
size_t zo_mha_work_floats(const zo_mla_dims *d, uint32_t n_kv, uint32_t max_tokens);
int zo_mha_attention(const float *x, const uint8_t *wq, const uint8_t *wk, const uint8_t *wv,
                     const uint8_t *wo, const zo_mla_dims *d, uint32_t n_kv, float *k_cache,
                     float *v_cache, uint32_t pos, uint32_t max_tokens, float *work, float *out);

typedef struct zo_ds2_run zo_ds2_run;
/* The scalar crate order. */
zo_ds2_run *zo_ds2_run_create(const zo_ds2 *m, uint32_t max_tokens);
/* order 0: the scalar crate order; 1: the crate's AVX-512 kernel order
 * (inference_avx512.rs:2141-2825) over a persistent pool of `threads`
 * participants (<= 0: one per physical core); simd 0 runs its lane
 * emulation (same bits). */
zo_ds2_run *zo_ds2_run_create_order(const zo_ds2 *m, uint32_t max_tokens, int order, int threads,
                                    int simd);
int     zo_ds2_run_threads(const zo_ds2_run *r);
/* cached latent rows [t0, t0 + n) of one layer := rows ([n][kv_lora | rope]) */
int     zo_ds2_run_set_cache_rows(zo_ds2_run *r, uint32_t layer, uint32_t t0, uint32_t n,
                                  const float *rows);
void    zo_ds2_run_destroy(zo_ds2_run *r);
/* forward_pass.rs:703-909 */
int     zo_ds2_run_forward(zo_ds2_run *r, uint32_t token, uint32_t pos, float *hidden_out);
int     zo_ds2_run_lm_head(zo_ds2_run *r, uint32_t *token_out, float *logits_out);
int     zo_ds2_run_generate(zo_ds2_run *r, const uint32_t *prompt, uint32_t n_prompt,
                            uint32_t n_gen, uint32_t *tokens_out, float *margins_out,
                            float *logits_all);
const float    *zo_ds2_run_cache(const zo_ds2_run *r);
/* The MHA layers' cache: per MHA layer (in layer order) the K block then the V block. */
const float    *zo_ds2_run_mha_cache(const zo_ds2_run *r);
/* [n_layers][top_k] expert ids / weights chosen by the last forward (0 for dense layers). */
const uint32_t *zo_ds2_run_expert_ids(const zo_ds2_run *r);
const float    *zo_ds2_run_expert_weights(const zo_ds2_run *r);

#ifdef __cplusplus
}
#endif
#endif
