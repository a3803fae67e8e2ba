// mla.h — multi-head latent attention decode kernels (mla.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace zgpu {

constexpr uint32_t kMlaSplitTokens = 16;   // cached tokens per attention CTA (the shortest split)
constexpr uint32_t kMlaMaxLatent = 512;    // kv_lora_rank
constexpr uint32_t kMlaMaxRope = 64;       // qk_rope_head_dim
constexpr uint32_t kMlaMaxNope = 256;      // qk_nope_head_dim
constexpr uint32_t kMlaPrepThreads = 512;

struct MlaParams {
  const float *kv_a;          // [kv_lora + rope]: W_kv_a_mqa . rmsnorm(hidden)
  const float *kv_a_norm;     // [kv_lora]
  const float *k_norm;        // [rope] or null
  const float *q;             // [n_heads][nope + rope]: W_q_b . rmsnorm(c_q)
  const uint8_t *kb;          // group streams holding each head's k_nope rows (kv_b or k_b)
  uint64_t kb_gstride;
  uint32_t kb_quant;
  uint32_t kb_head_rows;      // rows from one head's first k_nope row to the next head's
  const float *inv_freqs;     // [rope / 2]: powf(base, -2 i / rope)
  float *cache;               // this layer's [max_tokens][kv_lora + rope]
  uint32_t max_tokens;
  const uint32_t *pos_ptr;    // device position, or null for pos_value
  uint32_t pos_value;
  float *q_abs;               // [n_heads][kv_lora]: W_k_nope^T q_nope per head
  float *q_pe;                // [n_heads][rope]: rotated q_rope
  float *ctx;                 // [n_heads][kv_lora]: sum_t p_t c_kv_t
  float *part;                // [n_heads][max_splits][kv_lora + 2]
  uint32_t *status;
  uint32_t n_heads, kv_lora, rope, nope, max_splits;
  float eps, scale;
  uint32_t slab_bytes;        // shared bytes of one head's k_nope slab (set by the launcher)
  // A batch of n_seq sequences (grid dimension y; 0 or 1: the one sequence
  // above).  Sequence b reads kv_a + b * kv_a_stride and q + b * q_stride,
  // writes q_abs / q_pe / ctx / part at b times their one-sequence sizes,
  // and uses its own cache seq_cache[b] + layer_off (this layer of its
  // zgpu_mla_kv, all of one capacity max_tokens) and position seq_pos[b].
  uint32_t n_seq;
  uint32_t kv_a_stride, q_stride;
  float *const *seq_cache;
  uint64_t layer_off;
  const uint32_t *seq_pos;
  // Tokens per attention split (a multiple of kMlaSplitTokens; 0: the
  // shortest).  part holds max_splits >= mla_max_splits(max_tokens) slots
  // per head either way.
  uint32_t split_tokens;
};

// Splits (attention CTAs) a cache of max_tokens needs at the shortest split.
inline uint32_t mla_max_splits(uint32_t max_tokens) {
  return (max_tokens + kMlaSplitTokens - 1) / kMlaSplitTokens;
}
// Split length for n_seq sequences on caches of max_tokens rows: the
// shortest, doubled while the launch would still hold at least two CTAs per
// SM (long contexts in a batch: fewer partial sums to write and merge).
// Depends on n_seq, so a batch and a lone sequence may split (and round)
// differently; below 2 * sm_count * 16 / n_seq tokens they agree.
inline uint32_t mla_split_tokens(uint32_t n_seq, uint32_t max_tokens, uint32_t sm_count) {
  uint32_t s = kMlaSplitTokens;
  while (s < 4096 && static_cast<uint64_t>(n_seq) * ((max_tokens + 2 * s - 1) / (2 * s)) >= 2ull * sm_count) s *= 2;
  return s;
}
cudaError_t mla_setup();
// latent RMSNorm + k_rope norm/RoPE + cache append, and the per-head query
// absorption (q_abs, q_pe)
cudaError_t launch_mla_prep(const MlaParams &p, const LaunchCfg &lc);
// split-K attention over the latent cache, then the split merge into ctx
cudaError_t launch_mla_attention(const MlaParams &p, const LaunchCfg &lc);

// ------------------------------------------------------------------ MHA
// DeepSeek2 layers with standard attention (AttnType::Mha, mla.rs:449-618),
// kernels in mha.cu.
constexpr uint32_t kMhaSplitTokens = 64;   // cached tokens per attention CTA
constexpr uint32_t kMhaMaxHead = 320;      // nope + rope
constexpr uint32_t kMhaMaxV = 256;         // v head width
constexpr uint32_t kMhaThreads = 128;

struct MhaParams {
  float *qkv;                 // [n_heads*hq | n_kv*hq | n_kv*v] projections; mha_prep rotates q in place
  const float *inv_freqs;     // [rope / 2]: powf(base, -2 i / rope)
  float *k_cache, *v_cache;   // this layer's K block [max_tokens][n_kv*hq] and V block [max_tokens][n_kv*v]
  uint32_t max_tokens;
  const uint32_t *pos_ptr;    // device position, or null for pos_value
  uint32_t pos_value;
  float *part;                // [n_heads][max_splits][v + 2]
  float *out;                 // [n_heads * v]
  uint32_t *status;
  uint32_t n_heads, n_kv, nope, rope, v, max_splits;
  float scale;                // 1 / sqrt(nope + rope)
};

inline uint32_t mha_max_splits(uint32_t max_tokens) {
  return (max_tokens + kMhaSplitTokens - 1) / kMhaSplitTokens;
}
// RoPE of the rope part of every q head (in place) and of the new k, and the
// cache append of k and v at the position (store_kv, kv_cache.rs:487-531)
cudaError_t launch_mha_prep(const MhaParams &p, const LaunchCfg &lc);
// split attention over [0, pos] per q head, then the in-order split merge into out
cudaError_t launch_mha_attention(const MhaParams &p, const LaunchCfg &lc);
cudaError_t mha_setup();

}  // namespace zgpu
