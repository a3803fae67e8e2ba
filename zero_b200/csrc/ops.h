// ops.h — parameter blocks and launchers of the non-GEMV kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace zgpu {

// Device-resident decode state: the CUDA graph of one step reads and
// advances it, so a replay needs no host-side parameter updates.
struct StepState {
  uint32_t step;            // forward index since the last reset
  uint32_t n_prompt;        // steps < n_prompt take their token from the prompt
  uint32_t pos_base;        // position of step 0
  uint32_t pos;             // position of the current step (written by embed)
  uint32_t token;           // token of the current step (written by embed)
  uint32_t next_token;      // argmax of the last LM head
  uint32_t n_gen_cap;       // capacity of tokens_out
  uint32_t vocab_real;
  uint32_t first_err_step;  // 0xFFFFFFFF when no LM-head error happened
  float last_max;
};

struct EmbedParams {
  const uint8_t *emb;       // device table (layout.h group streams)
  uint64_t gstride;
  uint32_t quant;           // ZGPU_Q8_0 / ZGPU_Q4_0
  uint32_t hidden;
  uint32_t vocab;           // rows of the table
  const uint32_t *prompt;
  StepState *state;
  float *hidden_out;
  uint32_t *status;
};

struct FinalizeParams {
  unsigned long long *argmax;
  StepState *state;
  uint32_t *tokens_out;
  uint32_t *status;
};

struct AttnParams {
  const float *qkv;          // [n_q*hd | n_kv*hd | n_kv*hd] raw projections
  const float *q_norm, *k_norm;
  const float *inv_freqs;    // [hd/2] RopeContext (ops.rs:79)
  float *kv_layer;           // K block of this layer; V block follows at +kv_block
  uint64_t kv_block;         // max_tokens * n_kv * hd
  uint32_t max_tokens;
  const uint32_t *pos_ptr;   // device position of the token, or null to use pos_value
  uint32_t pos_value;
  float *out;                // [n_q*hd]
  float *part;               // [n_q][max_splits][hd + 2]
  uint32_t *counters;        // [n_kv]
  uint32_t *status;
  uint32_t n_q, n_kv, max_splits;
  float eps, scale;
  // tagged mode (persistent step kernel): projections and output are tagged
  // words (version << 32 | f32 bits) instead of qkv / out
  const unsigned long long *qkv_t;
  unsigned long long *out_t;
  uint32_t ver_in, ver_out;
  // tensor parallel: the output goes to the n_out copies out_dst[0..n_out)
  // (device table, each offset to this rank's heads); n_out == 0 writes out_t
  unsigned long long *const *out_dst;
  uint32_t n_out;
  volatile uint32_t *abort;         // this CTA's abort flag (shared memory)
  uint32_t *gabort;                 // the launch's abort flag
};

// Launch configuration with programmatic dependent launch when lc.pdl is set
// (attr must outlive the launch call).
inline cudaLaunchConfig_t make_launch_cfg(dim3 grid, dim3 block, size_t smem, const LaunchCfg &lc,
                                          cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lc.stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  return cfg;
}

// Batched Q4_0 x Q8_0 matmul on tcgen05 (mma_gemm.cu): y[t * ldy + m] for
// t < T, m < rows, from the layout.h weight streams and planar Q8_0
// activations (q int8 [T][bpr*32], d f32 [T][bpr]).
// Operand tiles of the batched Q4_0 x Q8_0 matmul (mma_gemm.cu): per
// 128-row (or 128-token) tile and 32-element block, 4096 bytes of int8 in the
// tensor core's canonical K-major layout (8-row x 16-byte core matrices, row r
// and K half h at (r % 8) * 16 + (r / 8) * 256 + h * 128), tiles laid out
// [tile][block], each block followed by its 128 rows' f32 scales.  Weights hold n - 8 of their
// Q4_0 nibbles; activations the Q8_0 digits, rows past T zero.
constexpr uint32_t kMmaTile = 128;
// A (tile, block) is kMmaBlockBytes: the 4 KB of int8 digits, then the 128
// rows' f32 scales, so that one copy brings a block and its scales.  The
// scales are addressed through the same allocation: callers pass
// reinterpret_cast<float *>(tiles) as the scale pointer.
constexpr uint32_t kMmaBlockBytes = 4096 + 4 * kMmaTile;
inline size_t mma_tile_bytes(uint64_t rows, uint32_t bpr) {
  return ((rows + kMmaTile - 1) / kMmaTile) * bpr * static_cast<uint64_t>(kMmaBlockBytes);
}
__host__ __device__ inline size_t mma_tile_off(uint32_t r, uint32_t b, uint32_t bpr, uint32_t h) {
  return (static_cast<size_t>(r / kMmaTile) * bpr + b) * kMmaBlockBytes + (r % 8) * 16u +
         ((r % kMmaTile) / 8) * 256u + h * 128u;
}
// f32 index of row r's scale of block b, from the tile allocation's start
__host__ __device__ inline size_t mma_scale_off(uint32_t r, uint32_t b, uint32_t bpr) {
  return ((static_cast<size_t>(r / kMmaTile) * bpr + b) * kMmaBlockBytes + 4096u) / 4u + r % kMmaTile;
}

struct MmaGemmParams {
  const int8_t *wt;         // weight tiles, rows / 128 of them
  const float *ws;          // weight block scales
  const int8_t *xt;         // activation tiles, ceil(T / 128)
  const float *xs;          // activation block scales
  float *y;                 // [T][ldy], columns [0, rows)
  uint32_t rows, bpr, T, ldy;
  uint32_t *status;
  uint32_t resadd;          // 0: y = result; 1: y = y + result (residual add)
  // K split (small T): ksplit > 1 runs each weight tile as ksplit block
  // ranges in parallel, each summed in block order into part [ksplit][T][rows]
  // (scratch), then added in split order; 0 or 1: no split
  uint32_t ksplit;
  float *part;
};
constexpr uint32_t kMmaMaxSplit = 16;
cudaError_t mma_setup();
cudaError_t launch_q4q8_mma(const MmaGemmParams &p, cudaStream_t s);
// The K split for a weight of rows x (32 bpr): a function of the weight's
// shape alone, so a row's result never depends on T.
uint32_t mma_ksplit(uint32_t rows, uint32_t bpr);
// Q4_0 group streams (layout.h) -> weight tiles + scales; rows % 128 == 0.
cudaError_t launch_build_w8_tiles(const uint8_t *w, uint64_t gstride, uint32_t rows, uint32_t bpr, uint32_t quant,
                                  int8_t *wt, float *ws, cudaStream_t s);
// x [T][K] f32 -> Q8_0 activation tiles + scales (the packer's rule); the
// padding rows of the last tile are zeroed.
cudaError_t launch_quantize_q8_0_tiles(const float *x, int8_t *xt, float *xs, uint32_t T, uint32_t K,
                                       uint32_t *status, cudaStream_t s);

// Token-parallel prefill kernels (prefill.cu).
cudaError_t prefill_setup();
// RMSNorm of each row, then Q8_0 into activation tiles (as launch_quantize_q8_0_tiles)
// Per row of n logits: the reference's greedy pick, tok[row], and its LM-head
// error (0, ZGPU_ERR_LM_NON_FINITE_LOGITS or ZGPU_ERR_LM_ARGMAX_IN_PADDING) in
// codes[row]; errors also set the status bits.
cudaError_t launch_rows_argmax(const float *logits, uint32_t rows, uint32_t n, uint32_t vocab_real, uint32_t *tok,
                               uint32_t *codes, uint32_t *status, cudaStream_t s);
cudaError_t launch_rows_rmsnorm_quant(const float *x, const float *g, float eps, uint32_t T, uint32_t n, int8_t *xt,
                                      float *xs, uint32_t *status, cudaStream_t s);
cudaError_t launch_rows_embed(const uint8_t *emb, uint64_t gstride, uint32_t quant, uint32_t hidden, uint32_t vocab,
                              const uint32_t *tokens, uint32_t T, float *out, uint32_t *status, cudaStream_t s);
cudaError_t launch_qk_rope_kv(const float *qkv, const float *q_norm, const float *k_norm, const float *inv_freqs,
                              float *kv_layer, uint64_t kv_block, uint32_t n_q, uint32_t n_kv, uint32_t pos0,
                              uint32_t T, float eps, float *q_out, cudaStream_t s);
cudaError_t launch_causal_attn(const float *q, const float *kv_layer, uint64_t kv_block, uint32_t n_q, uint32_t n_kv,
                               uint32_t pos0, uint32_t T, float scale, float *out, uint32_t *status,
                               cudaStream_t s);
cudaError_t launch_swiglu_rows(const float *y, float *act, uint32_t T, uint32_t ffn, cudaStream_t s);
// SwiGLU of the gate/up rows, Q8_0-quantised into activation tiles (as
// launch_quantize_q8_0_tiles of swiglu_rows' output, in one pass)
cudaError_t launch_swiglu_quant_tiles(const float *y, int8_t *xt, float *xs, uint32_t T, uint32_t ffn,
                                      uint32_t *status, cudaStream_t s);

// Device bytes per Q6_K super-block: the 210-byte block padded so that its
// fields start on 8-byte boundaries (registration pads, kquant.cu reads).
constexpr uint32_t kQ6kStride = 224;
// y = W x over K-quant rows (kquant.cu): quant ZGPU_Q4_K (plain rows) or
// ZGPU_Q6_K (kQ6kStride-byte blocks), in_dim % 256 == 0, at most 65536.
cudaError_t launch_gemv_kquant(const uint8_t *w, uint32_t quant, uint32_t rows, uint32_t in_dim, const float *x,
                               float *y, cudaStream_t s);

// lm_head_sample (sampler.rs:41-163) over logits[0, min(len, vocab_real)):
// one warp; *rng is the xorshift64 state, advanced by one draw; *out the token.
cudaError_t launch_sample_topk(const float *logits, uint32_t len, uint32_t vocab_real, float temperature,
                               unsigned long long *rng, uint32_t *out, cudaStream_t s);

cudaError_t launch_attention(const AttnParams &ap, const LaunchCfg &lc);
// One sequence of a batched decode step: its cache (K block of layer 0;
// layer l starts 2 l block floats further), block size, capacity and the
// position of its token.
struct AttnBatchSeq {
  float *kv;
  uint64_t block;
  uint32_t max_tokens, pos;
};
// The decode attention of one layer for n_seq sequences at once (grid z =
// sequence): sequence z reads qkv + z * qkv_stride, writes out + z *
// out_stride, and uses its own partials and arrival counters (part + z *
// n_q * max_splits * (hd + 2), counters + z * n_kv); ap.kv_layer / kv_block /
// max_tokens / pos come from seqs[z] (device).  ap.max_splits must cover
// every sequence's cache.
cudaError_t launch_attention_batch(const AttnParams &ap, const AttnBatchSeq *seqs, uint32_t layer, uint32_t n_seq,
                                   uint32_t qkv_stride, uint32_t out_stride, const LaunchCfg &lc);
// Number of attention splits (CTAs per kv-head) a cache of max_tokens needs.
uint32_t attention_max_splits(uint32_t max_tokens);
cudaError_t attention_setup();
cudaError_t ops_setup();
cudaError_t launch_embed(const EmbedParams &p, const LaunchCfg &lc);
cudaError_t launch_finalize(const FinalizeParams &p, const LaunchCfg &lc);
cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, uint32_t n, float eps,
                           cudaStream_t s);
cudaError_t launch_rope(float *qk, const float *inv_freqs, uint32_t n_heads, uint32_t head_dim,
                        uint32_t pos, cudaStream_t s);
cudaError_t launch_silu_mul(const float *g, const float *u, float *out, uint64_t n,
                            cudaStream_t s);
cudaError_t launch_quantize_q8_0(const float *x, uint8_t *out, uint64_t n, uint32_t *status,
                                 cudaStream_t s);

}  // namespace zgpu
