// moe.h — MoE router and combine kernels (moe.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"
#include "layout.h"

namespace zgpu {

constexpr uint32_t kMoeMaxTopK = 16;
constexpr uint32_t kMoeMaxDim = 8192;

struct RouteParams {
  const float *x;            // hidden [dim]: routed as is, or rmsnorm(x) * norm_w
  const float *norm_w;       // null: route x unchanged
  float eps;
  const float *w;            // router rows f32 [n_experts][dim]
  const float *bias;         // [n_experts] or null
  uint32_t dim, n_experts, top_k, mode;   // mode: 0 Softmax, 1 SigmoidNormalize
  float scale;               // expert_weight_scale
  float *scores;             // [n_experts]
  uint32_t *ids;             // [top_k]
  float *weights;            // [top_k]
  uint32_t *counter;         // arrival counter, zero between launches
  // dispatch tables of the grouped expert GEMVs (null: not written)
  unsigned long long *seg_gu, *seg_dn;       // [n_shared + top_k]
  unsigned long long gu_base, dn_base;       // routed experts' streams
  unsigned long long sh_gu_base, sh_dn_base; // shared experts' streams
  unsigned long long gu_bytes, dn_bytes;     // bytes per expert
  uint32_t n_shared;
  uint32_t experts_per_cta;  // set by the launcher
  uint32_t *status;
  // expert parallelism: this rank runs experts [ep_rank * ep_per_rank,
  // (ep_rank + 1) * ep_per_rank); a selected expert of another rank gets a
  // zero table entry (its GEMV segments do nothing).  ep_per_rank == 0: all.
  uint32_t ep_rank, ep_per_rank;
  // A batch of n_seq tokens (grid dimension y; 0 or 1: one token): token b
  // routes x + b * x_stride and writes its scores, ids, weights, arrival
  // counter and dispatch tables at b times their one-token sizes.
  uint32_t n_seq, x_stride;
};

// A combine wait that gives up records itself in words 4..7 of the status
// block (the first one only): the site, the version it waited for, the tag
// it last read, and which word (the rank for an arrival word, b * top_k + k
// for a slot).
// Site ZDEV_WAIT_EP_ABORTED: the exchange was already aborted (abort word
// set) and the combine did not wait.
enum : uint32_t { ZDEV_WAIT_EP_ARRIVAL = 2, ZDEV_WAIT_EP_SLOT = 3, ZDEV_WAIT_EP_ABORTED = 4 };

struct CombineParams {
  const float *exp_out;      // [n_shared + top_k][dim]
  const float *weights;      // [top_k]
  float *mlp_out;            // [dim] or null
  float *hidden;             // residual (+= mlp_out) or null
  uint32_t dim, n_shared, top_k;
  // expert parallelism: the routed slots' outputs come from this rank's
  // exchange buffer (tagged words [2][top_k][dim], filled by every rank's
  // moe_ep_publish) at version *ep_seq + 1; null: from exp_out.  The
  // combine also waits until every rank's arrival word (ep_arrive_words
  // after the slots, one per rank) carries that version.
  unsigned long long *xslots;
  const uint32_t *ep_seq;
  uint32_t world;
  uint32_t *status;
  // A batch of n_seq tokens (grid dimension y): token b combines exp_out +
  // b * (n_shared + top_k) * dim with weights + b * top_k into hidden /
  // mlp_out + b * dim, and reads its routed slots at (b * top_k + k) * dim
  // of the exchange buffer; each half of it holds slot_cap slots.
  uint32_t n_seq;
  uint32_t slot_cap;
};

// Expert parallelism: the outputs of this rank's selected experts, as tagged
// words into slot k of every rank's exchange buffer (buffer (v & 1), v =
// *ep_seq + 1), plus this rank's arrival word for invocation v in every
// rank's buffer.  A combine waits for all ranks' arrival words, so no rank
// finishes invocation v + 1 before every rank has finished invocation v and
// its reads of buffer (v & 1): publishing invocation v + 2 into that buffer
// is then safe however the experts are routed.
struct EpPublishParams {
  const float *exp_out;                    // [n_shared + top_k][dim] (per token of a batch)
  const uint32_t *ids;                     // [top_k] this layer's experts (per token)
  unsigned long long *const *dst;          // [world] every rank's exchange buffer
  const uint32_t *ep_seq;
  uint32_t dim, n_shared, top_k, world, ep_rank, ep_per_rank;
  uint32_t n_seq;                          // tokens of a batch (grid dimension z; 0 or 1: one)
  uint32_t slot_cap;                       // slots per half of the exchange buffer
};

// Words of one rank's exchange buffer: two buffers of slots x dim tagged
// words (slots = top_k per token of the largest batch), then one arrival
// word per rank.
constexpr uint32_t kEpMaxRanks = 8;
ZGPU_HD size_t ep_slot_words(uint32_t slots, uint32_t dim) { return 2 * static_cast<size_t>(slots) * dim; }
// After the arrival words, this rank's abort word: nonzero once one of its
// combine waits expired.  Every later combine then gives up at once (the
// ranks are out of step, so every wait would run to its limit); the
// exchange stays aborted for the model's lifetime.
ZGPU_HD size_t ep_abort_word(uint32_t slots, uint32_t dim) { return ep_slot_words(slots, dim) + kEpMaxRanks; }
ZGPU_HD size_t ep_exchange_words(uint32_t slots, uint32_t dim) { return ep_abort_word(slots, dim) + 1; }

// Grouping of a batch's (token, expert) pairs by expert for the tensor-core
// expert matvecs (digit_mma.h).  Segment s < n_local is this rank's routed
// expert ep_rank * ep_per_rank + s (all experts without expert
// parallelism), segment n_local + i the shared expert i.  Per segment:
// n_vec[s] tokens (at most 32, each token selects an expert once); for its
// j-th token b and that token's slot (shared experts first, then the k-th
// selection) the pair row p = b * (n_shared + top_k) + slot:
//   x_rows_gu[s * 32 + j] = b,           out_gu[s * 32 + j] = act + p * act_row
//   x_rows_dn[s * 32 + j] = p,           out_dn[s * 32 + j] = exp_out + p * dim
// and the tile tables tab_gu[s] / tab_dn[s] = the segment's weight tiles,
// 0 when no token selected it.  Which column a token takes inside its
// segment does not change any result.
struct MoeDispatchParams {
  const uint32_t *ids;               // [n_seq][top_k] this layer's selections
  uint32_t n_seq, top_k, n_shared, n_local, ep_rank, ep_per_rank;   // ep_per_rank 0: no expert parallelism
  float *act, *exp_out;
  uint32_t act_row, dim;
  const uint8_t *tiles_gu, *tiles_dn;          // routed experts' tiles, tiles_*_stride bytes apart
  const uint8_t *sh_tiles_gu, *sh_tiles_dn;    // shared experts' tiles
  uint64_t tiles_gu_stride, tiles_dn_stride;
  uint32_t *n_vec, *x_rows_gu, *x_rows_dn;
  float **out_gu, **out_dn;
  unsigned long long *tab_gu, *tab_dn;
  // every (segment, token slot) pair in use, segment << 8 | slot, and their count
  uint32_t *pairs, *n_pairs;
};
constexpr uint32_t kMoeMaxSegs = 256;

cudaError_t moe_setup();
cudaError_t launch_moe_route(const RouteParams &p, const LaunchCfg &lc);
cudaError_t launch_moe_dispatch(const MoeDispatchParams &p, const LaunchCfg &lc);
cudaError_t launch_moe_combine(const CombineParams &p, const LaunchCfg &lc);
cudaError_t launch_moe_ep_publish(const EpPublishParams &p, const LaunchCfg &lc);
// ++*ep_seq (one thread), after the layer's combine
cudaError_t launch_moe_ep_advance(uint32_t *ep_seq, const LaunchCfg &lc);

}  // namespace zgpu
