// step.h — the persistent decode-step kernel: descriptors shared by the host
// (model.cu builds them) and the kernel (step.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"
#include "ops.h"

namespace zgpu {

enum StageKind : uint32_t { STG_GEMV = 0, STG_ATTN = 1 };
// flag: the GEMV input is the embedding row of the step's token (layer 0)
constexpr uint32_t kStageEmbed = 1u;

// One stage of the step.  GEMV stages stream `w` (layout.h group streams);
// the producer warp of every CTA walks the same descriptors to prefetch.
struct StageDesc {
  uint32_t kind;
  uint32_t quant, pro, epi, flags;  // GemvPro / GemvEpi
  uint32_t rows;                    // valid output rows
  uint32_t units;                   // units of `gpu` groups
  uint32_t gpu;                     // groups per unit: 2 (Q4_0) or 1 (Q8_0)
  uint32_t bpr, ks;                 // blocks per row, K-chunks per unit
  uint32_t in_dim;
  uint32_t gbytes;                  // slot offset of the unit's second group
  uint32_t layer;                   // STG_ATTN
  uint32_t in_buf, out_buf;         // StepBuf of the input / output vector
  uint32_t out_row0;                // first row of this rank's slice in the output vector
  uint32_t bcast;                   // 1: store the output into every rank's copy (tensor parallel)
  uint32_t pad;
  const uint8_t *w;
  uint64_t gstride, wbytes;
  const float *norm_w;              // PRO_RMSNORM gain
  float *out;                       // plain f32 output (the LM head's logits)
  const unsigned long long *tin;    // tagged input vector (in_buf), or null
  unsigned long long *tout;         // tagged output vector (out_buf), or null
  const float *q_norm, *k_norm;     // STG_ATTN
};

// The inter-stage vectors of the step, held as tagged words
// (version << 32 | f32 bits): consumers wait for the version they expect
// instead of meeting at a grid barrier.
enum StepBuf : uint32_t { BUF_HIDDEN = 0, BUF_QKV = 1, BUF_ATTN = 2, BUF_ACT = 3, BUF_TOKEN = 4,
                          BUF_NONE = 5 };
constexpr int kStepBufs = 5;

constexpr uint32_t kStagesInGlobal = 0xFFFFFFFFu;

enum StepMode : uint32_t { STEP_GENERATE = 0, STEP_FORWARD = 1, STEP_LM = 2 };

// Tensor parallelism: ranks of one model, each running the step kernel on
// its own GPU over its slice of every stage's output rows.
constexpr uint32_t kMaxRanks = 8;
// Per-rank argmax slot of the LM head: {key, version} (8-byte words).
struct ArgSlot {
  unsigned long long key, ver;
};

struct StepParams {
  const StageDesc *stages;
  uint32_t n_layer_stages;          // stages[0, n_layer_stages): the forward pass
  uint32_t lm_stage;                // stages[lm_stage]: the LM-head GEMV
  uint32_t mode, step0, n_steps;
  uint32_t fwd_token, fwd_pos;      // STEP_FORWARD
  uint32_t n_q, n_kv, max_splits, max_tokens;
  float eps, scale;
  const uint8_t *emb;               // embedding table (layout.h), plain rows
  uint64_t emb_gstride;
  uint32_t emb_quant, emb_rows, hidden, pad;
  unsigned long long *tv[kStepBufs];  // tagged vectors (BUF_TOKEN: one word)
  uint32_t ver[kStepBufs];            // their versions before this launch
  const float *inv_freqs;
  float *kv_base;
  uint64_t kv_block;                // floats per K (or V) block of one layer
  float *attn_part;
  uint32_t *attn_counters;
  unsigned long long *argmax;
  StepState *state;
  const uint32_t *prompt;
  uint32_t *tokens_out;
  uint32_t *status;
  uint32_t *bar;                    // [0] LM-head arrival counter, [1] abort flag (zero at launch)
  uint32_t xbytes, part_bytes, hown_off, ring_off, smem_bytes;
  uint32_t hown_units, hown_rows;  // residual rows kept per CTA (units of 8 rows)
  uint32_t hid_row0;               // first hidden row of this rank's residual slice (0 on one GPU)
  uint32_t rank, world;            // tensor-parallel rank / ranks (0 / 1 on one GPU)
  uint32_t attn_out_off;           // words: this rank's first q head in the attention vector
  uint32_t pad2;
  // device tables (world > 1): peer_tv[d * kStepBufs + b] = rank d's tagged
  // vector b; peer_arg[d] = rank d's argmax slots [kMaxRanks]; attn_dst[d] =
  // rank d's attention vector at this rank's heads
  unsigned long long *const *peer_tv;
  ArgSlot *const *peer_arg;
  unsigned long long *const *attn_dst;
  uint32_t stages_off, n_stages;   // shared-memory copy of the stage list (kStagesInGlobal: none)
};

// Version advances of the tagged vectors for one step (what the kernel
// writes), so that the host can follow them across launches.
inline void step_advance_versions(uint32_t *ver, uint32_t n_layers, bool fwd, bool lm) {
  if (fwd) {
    ver[BUF_QKV] += n_layers;
    ver[BUF_ATTN] += n_layers;
    ver[BUF_ACT] += n_layers;
    ver[BUF_HIDDEN] += 2 * n_layers;
  }
  if (lm) ver[BUF_TOKEN] += 1;
}

// Shared-memory geometry for a stage list; false if it cannot fit.
bool step_geometry(const StageDesc *stages, uint32_t n, uint32_t grid, StepParams *p);
cudaError_t step_setup();
// Cooperative launch over `grid` CTAs (one per SM).
cudaError_t step_launch(const StepParams &p, uint32_t grid, cudaStream_t s);
// CTAs the step kernel can keep resident on the device (0 if it cannot run).
uint32_t step_max_grid(int sm_count);

}  // namespace zgpu
