// ds2.cu — the DeepSeek2-shaped (MLA + MoE) decode step: compressed-latent
// cache, device weight layout, per-step kernel sequence, CUDA-graph capture,
// the greedy loop and the MoE routing entry point.
//
// One decode step (forward_single_token_deepseek2, forward_pass.rs:703-909,
// then lm_head_argmax_dynamic, lm_head.rs:98) is, per layer:
//   [RMSNorm + fused kv_a_mqa | q_a GEMV]
//   [RMSNorm(c_q) + q_b GEMV]
//   [mla_prep: latent RMSNorm, k_rope norm + RoPE, cache append; per-head
//    query absorption W_kn^T q_nope and q_rope RoPE]
//   [mla_attn + mla_merge: split-K softmax over the latent cache]
//   [per-head V GEMV (segmented: head h reads its ctx_h and its v rows)]
//   [O GEMV + residual]
// then either the dense FFN
//   [RMSNorm + fused gate|up GEMV + SiLU*up] [down GEMV + residual]
// or the MoE FFN (moe_ffn, moe.rs:486-590)
//   [router: exact-order scores, top-k, weights, dispatch tables]
//   [grouped gate|up GEMV + SiLU*up over the shared and selected experts]
//   [grouped down GEMV] [weighted combine in the reference's order + residual]
// and the LM head [RMSNorm + GEMV + argmax] -> finalize.  Every kernel is
// launched with programmatic dependent launch and the whole step is captured
// once into a CUDA graph whose replays read token and position from device
// memory.  Expert ids never leave the device between the router and the
// expert GEMVs: the router writes the GEMVs' per-segment weight addresses.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "common.cuh"
#include "digit_mma.h"
#include "internal.h"
#include "layout.h"
#include "mla.h"
#include "moe.h"
#include "ops.h"

using namespace zgpu;

struct zgpu_mla_kv {
  zgpu_ctx *ctx = nullptr;
  float *d = nullptr;
  uint32_t max_tokens = 0, n_layers = 0, kv_lora = 0, rope = 0;
  uint64_t layer_floats = 0;   // max_tokens * (kv_lora + rope)
};

// MhaKvCache (kv_cache.rs:433-560): per MHA layer a K block
// [max_tokens][n_kv * head_dim_qk] then a V block [max_tokens][n_kv * head_dim_v].
struct zgpu_mha_kv {
  zgpu_ctx *ctx = nullptr;
  float *d = nullptr;
  uint32_t max_tokens = 0, n_layers = 0, n_kv = 0, hd_qk = 0, hd_v = 0;
  uint64_t k_block = 0, v_block = 0;   // floats
};

namespace {

constexpr uint32_t kMaxEpRanks = 8;
// Sequences of one zgpu_ds2_decode_batch call (the expert exchange buffers
// are sized for it when the model is created).
constexpr uint32_t kDs2MaxBatch = 32;

struct Ds2Layer {
  // attention
  uint8_t *cat_a = nullptr;          // owned: kv_a groups | q_a groups (| one zero group)
  uint32_t cat_a_groups = 0;
  const DeviceTensor *q_b = nullptr, *o = nullptr;
  const DeviceTensor *kb = nullptr;  // k_nope rows (kv_b or k_b)
  uint32_t kb_head_rows = 0;
  unsigned long long *d_vseg = nullptr;   // owned: per-head v-row stream addresses
  uint64_t v_seg_bytes = 0;
  uint64_t v_gstride = 0;
  // ffn
  uint32_t moe = 0;
  uint8_t *gateup = nullptr;         // owned: gate/up groups interleaved (dense or routed experts)
  uint8_t *sh_gateup = nullptr;      // owned: shared experts, interleaved
  const DeviceTensor *down = nullptr, *sh_down = nullptr, *router = nullptr;
  float *d_router_b = nullptr;       // owned (nullable)
  unsigned long long *d_seg_gu = nullptr, *d_seg_dn = nullptr;   // owned [n_shared + top_k]
  // standard attention (AttnType::Mha): fused q|k|v group streams, slot in the MHA cache
  uint32_t mha = 0, mha_idx = 0;
  uint8_t *cat_qkv = nullptr;        // owned
  uint32_t qkv_groups = 0;
  // tiles of the batch's tensor-core projections (digit_mma.h), built by
  // the first zgpu_ds2_decode_batch: kv_a|q_a, q_b, O, per-head V, dense
  // gate|up and down
  uint8_t *t_cat = nullptr, *t_qb = nullptr, *t_o = nullptr, *t_v = nullptr, *t_gu = nullptr, *t_dn = nullptr;
  // MoE layers: this rank's routed experts' and the shared experts' tiles
  uint8_t *t_egu = nullptr, *t_edn = nullptr, *t_sgu = nullptr, *t_sdn = nullptr;
  // norms (views into the model's norm block)
  const float *attn_norm = nullptr, *ffn_norm = nullptr, *kv_a_norm = nullptr, *q_a_norm = nullptr,
              *k_norm = nullptr;
};

}  // namespace

struct zgpu_ds2_model {
  zgpu_ctx *ctx = nullptr;
  zgpu_ds2_desc desc = {};
  std::vector<Ds2Layer> layers;
  uint64_t gs_h = 0, gs_e = 0, gs_f = 0;   // group strides for in_dim hidden / expert_ffn / ffn
  uint64_t gu_bytes = 0, dn_bytes = 0;     // per expert (interleaved gate/up, down)
  const DeviceTensor *emb = nullptr, *out = nullptr;
  float *d_norms = nullptr;                // every f32 vector of the model
  float *d_out_norm = nullptr;
  float *d_inv_freqs = nullptr;
  // activations
  float *d_hidden = nullptr, *d_ca = nullptr, *d_q = nullptr, *d_qabs = nullptr, *d_qpe = nullptr,
        *d_ctx = nullptr, *d_concat = nullptr, *d_act = nullptr, *d_expout = nullptr,
        *d_scores = nullptr, *d_logits = nullptr, *d_wts = nullptr;
  uint32_t *d_ids = nullptr, *d_route_counter = nullptr;
  unsigned long long *d_argmax = nullptr;
  StepState *d_state = nullptr;
  uint32_t *d_prompt = nullptr, *d_tokens = nullptr;
  uint32_t prompt_cap = 0, tokens_cap = 0;
  float *d_part = nullptr;
  uint32_t max_splits = 0;
  uint32_t *d_status = nullptr;
  cudaGraphExec_t step_graph = nullptr, fwd_graph = nullptr, lm_graph = nullptr;
  zgpu_mla_kv *graph_kv = nullptr;
  uint32_t step_kernels = 0, fwd_kernels = 0, lm_kernels = 0;
  zgpu_perf perf = {};
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  // expert parallelism (world > 1): rank `rank` runs routed experts
  // [rank * ep_per_rank, (rank + 1) * ep_per_rank); everything else is
  // replicated.  Selected experts' outputs cross over the exchange buffers.
  uint32_t rank = 0, world = 1, ep_per_rank = 0;
  unsigned long long *d_xslots = nullptr;   // this rank's exchange buffer: slots, arrival words, abort word
  uint32_t *d_ep_seq = nullptr;             // MoE invocations so far (the exchange version)
  unsigned long long **d_ep_dst = nullptr;  // [world] every rank's exchange buffer
  std::vector<void *> ipc_opened;
  bool ep_connected = false;
  // MHA layers: their count, kv heads, the bound cache and the attention scratch
  uint32_t n_mha = 0, n_kv = 0;
  zgpu_mha_kv *mha_kv = nullptr;
  float *d_mha_qkv = nullptr, *d_mha_part = nullptr;
  uint32_t mha_splits = 0;
  // zgpu_ds2_decode_batch: per-sequence activations of kDs2MaxBatch
  // sequences, allocated by the first batch call.  Sequence b's vectors sit
  // at b times the one-sequence sizes; the router writes layer l's ids,
  // weights and dispatch tables at l times the batch's sizes.
  struct Batch {
    float *hidden = nullptr, *ca = nullptr, *q = nullptr, *qabs = nullptr, *qpe = nullptr, *ctx = nullptr,
          *concat = nullptr, *act = nullptr, *expout = nullptr, *scores = nullptr, *logits = nullptr,
          *wts = nullptr, *part = nullptr;
    uint32_t *ids = nullptr, *counter = nullptr, *tok = nullptr, *pos = nullptr, *out = nullptr,
             *codes = nullptr;
    float **cache = nullptr;             // [kDs2MaxBatch] each sequence's zgpu_mla_kv rows
    uint8_t *t_out = nullptr;            // LM-head tiles
    // the expert grouping of the current MoE layer (moe.h MoeDispatchParams)
    uint32_t *dn_vec = nullptr, *x_rows_gu = nullptr, *x_rows_dn = nullptr, *pairs = nullptr;
    float **out_gu = nullptr, **out_dn = nullptr;
    unsigned long long *tab_gu = nullptr, *tab_dn = nullptr;
    uint8_t *img = nullptr;              // digit images of the tensor-core projections
    float *dpart = nullptr;              // their chunk partials
    uint32_t ca_stride = 0, act_stride = 0, splits = 0, max_tokens = 0;
    cudaGraphExec_t graph = nullptr;
    uint32_t graph_n = 0, graph_kernels = 0;
  } b;
};

namespace {

LaunchCfg launch_cfg(zgpu_ds2_model *m, uint32_t *counter) {
  LaunchCfg lc;
  lc.stream = m->ctx->stream;
  lc.pdl = !(m->ctx->flags & ZGPU_FLAG_NO_PDL);
  lc.sm_count = m->ctx->sm_count;
  lc.launch_counter = counter;
  return lc;
}

// Enqueue embed + all layers of one step.
cudaError_t ds2_enqueue_forward(zgpu_ds2_model *m, zgpu_mla_kv *kv, uint32_t *counter) {
  const zgpu_ds2_desc &d = m->desc;
  LaunchCfg lc = launch_cfg(m, counter);
  cudaError_t e;
  EmbedParams ep;
  ep.emb = m->emb->d;
  ep.gstride = m->emb->gstride;
  ep.quant = m->emb->quant;
  ep.hidden = d.hidden;
  ep.vocab = static_cast<uint32_t>(m->emb->rows);
  ep.prompt = m->d_prompt;
  ep.state = m->d_state;
  ep.hidden_out = m->d_hidden;
  ep.status = m->d_status;
  if ((e = launch_embed(ep, lc)) != cudaSuccess) return e;

  const uint32_t H = d.hidden, R = d.kv_lora_rank, RD = d.rope_dim, QL = d.q_lora_rank;
  const uint32_t NH = d.n_heads, hq = d.nope_dim + d.rope_dim;
  const uint32_t n_seg = d.n_shared + d.top_k;
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    const Ds2Layer &L = m->layers[l];
    GemvDesc g;
    GemvIo io;
    if (L.mha) {
      // standard attention (mla.rs:449-618): RMSNorm + fused q|k|v, RoPE and
      // cache append, attention into the head concat
      const uint32_t hqk = d.nope_dim + d.rope_dim;
      g.w = L.cat_qkv;
      g.gstride = m->gs_h;
      g.wbytes = static_cast<uint64_t>(L.qkv_groups) * m->gs_h;
      g.quant = d.attn_quant;
      g.rows = NH * hqk + m->n_kv * (hqk + d.v_dim);
      g.groups = L.qkv_groups;
      g.in_dim = H;
      io.x = m->d_hidden;
      io.norm_w = L.attn_norm;
      io.eps = d.rms_eps;
      io.out = m->d_mha_qkv;
      io.status = m->d_status;
      if ((e = launch_gemv(g, PRO_RMSNORM, EPI_STORE, io, lc)) != cudaSuccess) return e;
      MhaParams hp = {};
      hp.qkv = m->d_mha_qkv;
      hp.inv_freqs = m->d_inv_freqs;
      hp.k_cache = m->mha_kv->d + static_cast<size_t>(L.mha_idx) * (m->mha_kv->k_block + m->mha_kv->v_block);
      hp.v_cache = hp.k_cache + m->mha_kv->k_block;
      hp.max_tokens = m->mha_kv->max_tokens;
      hp.pos_ptr = &m->d_state->pos;
      hp.part = m->d_mha_part;
      hp.out = m->d_concat;
      hp.status = m->d_status;
      hp.n_heads = NH;
      hp.n_kv = m->n_kv;
      hp.nope = d.nope_dim;
      hp.rope = d.rope_dim;
      hp.v = d.v_dim;
      hp.max_splits = m->mha_splits;
      hp.scale = 1.0f / sqrtf(static_cast<float>(hqk));
      if ((e = launch_mha_prep(hp, lc)) != cudaSuccess) return e;
      if ((e = launch_mha_attention(hp, lc)) != cudaSuccess) return e;
    } else {
    // RMSNorm + fused kv_a_mqa | q_a
    g.w = L.cat_a;
    g.gstride = m->gs_h;
    g.wbytes = static_cast<uint64_t>(L.cat_a_groups) * m->gs_h;
    g.quant = d.attn_quant;
    g.rows = R + RD + QL;
    g.groups = L.cat_a_groups;
    g.in_dim = H;
    io.x = m->d_hidden;
    io.norm_w = L.attn_norm;
    io.eps = d.rms_eps;
    io.out = m->d_ca;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_RMSNORM, EPI_STORE, io, lc)) != cudaSuccess) return e;
    // RMSNorm(c_q, q_a_norm) + q_b
    g = GemvDesc();
    g.w = L.q_b->d;
    g.gstride = L.q_b->gstride;
    g.wbytes = L.q_b->bytes;
    g.quant = d.attn_quant;
    g.rows = NH * hq;
    g.groups = static_cast<uint32_t>(L.q_b->groups);
    g.in_dim = QL;
    io = GemvIo();
    io.x = m->d_ca + R + RD;
    io.norm_w = L.q_a_norm;
    io.eps = d.rms_eps;
    io.out = m->d_q;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_RMSNORM, EPI_STORE, io, lc)) != cudaSuccess) return e;
    // latent append + query absorption, attention, merge
    MlaParams mp = {};
    mp.kv_a = m->d_ca;
    mp.kv_a_norm = L.kv_a_norm;
    mp.k_norm = L.k_norm;
    mp.q = m->d_q;
    mp.kb = L.kb->d;
    mp.kb_gstride = L.kb->gstride;
    mp.kb_quant = L.kb->quant;
    mp.kb_head_rows = L.kb_head_rows;
    mp.inv_freqs = m->d_inv_freqs;
    mp.cache = kv->d + static_cast<size_t>(l) * kv->layer_floats;
    mp.max_tokens = kv->max_tokens;
    mp.pos_ptr = &m->d_state->pos;
    mp.q_abs = m->d_qabs;
    mp.q_pe = m->d_qpe;
    mp.ctx = m->d_ctx;
    mp.part = m->d_part;
    mp.status = m->d_status;
    mp.n_heads = NH;
    mp.kv_lora = R;
    mp.rope = RD;
    mp.nope = d.nope_dim;
    mp.max_splits = m->max_splits;
    mp.eps = d.rms_eps;
    mp.scale = 1.0f / sqrtf(static_cast<float>(hq));
    mp.split_tokens = mla_split_tokens(1, kv->max_tokens, m->ctx->sm_count);
    if ((e = launch_mla_prep(mp, lc)) != cudaSuccess) return e;
    if ((e = launch_mla_attention(mp, lc)) != cudaSuccess) return e;
    // per-head V projection of the merged latent context
    g = GemvDesc();
    g.gstride = L.v_gstride;
    g.wbytes = L.v_seg_bytes;
    g.quant = d.attn_quant;
    g.rows = d.v_dim;
    g.groups = d.v_dim / 4;
    g.in_dim = R;
    g.seg_w = L.d_vseg;
    g.seg_count = NH;
    g.seg_x_stride = R;
    g.seg_out_stride = d.v_dim;
    io = GemvIo();
    io.x = m->d_ctx;
    io.out = m->d_concat;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_PLAIN, EPI_STORE, io, lc)) != cudaSuccess) return e;
    }
    // O projection + residual
    g = GemvDesc();
    g.w = L.o->d;
    g.gstride = L.o->gstride;
    g.wbytes = L.o->bytes;
    g.quant = d.attn_quant;
    g.rows = H;
    g.groups = H / 4;
    g.in_dim = NH * d.v_dim;
    io = GemvIo();
    io.x = m->d_concat;
    io.out = m->d_hidden;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_PLAIN, EPI_RESADD, io, lc)) != cudaSuccess) return e;

    if (!L.moe) {
      g = GemvDesc();
      g.w = L.gateup;
      g.gstride = m->gs_h;
      g.wbytes = static_cast<uint64_t>(2 * d.ffn / 4) * m->gs_h;
      g.quant = ZGPU_Q4_0;
      g.rows = d.ffn;
      g.groups = 2 * d.ffn / 4;
      g.in_dim = H;
      io = GemvIo();
      io.x = m->d_hidden;
      io.norm_w = L.ffn_norm;
      io.eps = d.rms_eps;
      io.out = m->d_act;
      io.status = m->d_status;
      if ((e = launch_gemv(g, PRO_RMSNORM, EPI_SWIGLU, io, lc)) != cudaSuccess) return e;
      g = GemvDesc();
      g.w = L.down->d;
      g.gstride = L.down->gstride;
      g.wbytes = L.down->bytes;
      g.quant = ZGPU_Q4_0;
      g.rows = H;
      g.groups = H / 4;
      g.in_dim = d.ffn;
      io = GemvIo();
      io.x = m->d_act;
      io.out = m->d_hidden;
      io.status = m->d_status;
      if ((e = launch_gemv(g, PRO_PLAIN, EPI_RESADD, io, lc)) != cudaSuccess) return e;
      continue;
    }
    // router: ids / weights of this layer and the expert dispatch tables
    RouteParams rp = {};
    rp.x = m->d_hidden;
    rp.norm_w = L.ffn_norm;
    rp.eps = d.rms_eps;
    rp.w = reinterpret_cast<const float *>(L.router->d);
    rp.bias = L.d_router_b;
    rp.dim = H;
    rp.n_experts = d.n_experts;
    rp.top_k = d.top_k;
    rp.mode = d.route_mode;
    rp.scale = d.expert_weight_scale;
    rp.scores = m->d_scores;
    rp.ids = m->d_ids + static_cast<size_t>(l) * d.top_k;
    rp.weights = m->d_wts + static_cast<size_t>(l) * d.top_k;
    rp.counter = m->d_route_counter;
    rp.seg_gu = L.d_seg_gu;
    rp.seg_dn = L.d_seg_dn;
    rp.gu_base = reinterpret_cast<unsigned long long>(L.gateup);
    rp.dn_base = reinterpret_cast<unsigned long long>(L.down->d);
    rp.sh_gu_base = reinterpret_cast<unsigned long long>(L.sh_gateup);
    rp.sh_dn_base = L.sh_down ? reinterpret_cast<unsigned long long>(L.sh_down->d) : 0ull;
    rp.gu_bytes = m->gu_bytes;
    rp.dn_bytes = m->dn_bytes;
    rp.n_shared = d.n_shared;
    rp.status = m->d_status;
    rp.ep_rank = m->rank;
    rp.ep_per_rank = m->world > 1 ? m->ep_per_rank : 0;
    if ((e = launch_moe_route(rp, lc)) != cudaSuccess) return e;
    // grouped gate|up + SiLU*up: segment s = shared s, then the k-th selected expert
    g = GemvDesc();
    g.gstride = m->gs_h;
    g.wbytes = m->gu_bytes;
    g.quant = ZGPU_Q4_0;
    g.rows = d.expert_ffn;
    g.groups = 2 * d.expert_ffn / 4;
    g.in_dim = H;
    g.seg_w = L.d_seg_gu;
    g.seg_count = n_seg;
    g.seg_x_stride = 0;
    g.seg_out_stride = d.expert_ffn;
    g.seg_dynamic = true;
    io = GemvIo();
    io.x = m->d_hidden;
    io.norm_w = L.ffn_norm;
    io.eps = d.rms_eps;
    io.out = m->d_act;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_RMSNORM, EPI_SWIGLU, io, lc)) != cudaSuccess) return e;
    // grouped down projections
    g = GemvDesc();
    g.gstride = m->gs_e;
    g.wbytes = m->dn_bytes;
    g.quant = ZGPU_Q4_0;
    g.rows = H;
    g.groups = H / 4;
    g.in_dim = d.expert_ffn;
    g.seg_w = L.d_seg_dn;
    g.seg_count = n_seg;
    g.seg_x_stride = d.expert_ffn;
    g.seg_out_stride = H;
    g.seg_dynamic = true;
    io = GemvIo();
    io.x = m->d_act;
    io.out = m->d_expout;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_PLAIN, EPI_STORE, io, lc)) != cudaSuccess) return e;
    if (m->world > 1) {
      // this rank's selected experts' outputs into every rank's exchange buffer
      EpPublishParams pp = {};
      pp.exp_out = m->d_expout;
      pp.ids = m->d_ids + static_cast<size_t>(l) * d.top_k;
      pp.dst = m->d_ep_dst;
      pp.ep_seq = m->d_ep_seq;
      pp.dim = H;
      pp.n_shared = d.n_shared;
      pp.top_k = d.top_k;
      pp.world = m->world;
      pp.ep_rank = m->rank;
      pp.ep_per_rank = m->ep_per_rank;
      pp.slot_cap = d.top_k * kDs2MaxBatch;
      if ((e = launch_moe_ep_publish(pp, lc)) != cudaSuccess) return e;
    }
    CombineParams cp = {};
    cp.exp_out = m->d_expout;
    cp.weights = m->d_wts + static_cast<size_t>(l) * d.top_k;
    cp.hidden = m->d_hidden;
    cp.dim = H;
    cp.n_shared = d.n_shared;
    cp.top_k = d.top_k;
    cp.xslots = m->world > 1 ? m->d_xslots : nullptr;
    cp.ep_seq = m->d_ep_seq;
    cp.world = m->world;
    cp.slot_cap = d.top_k * kDs2MaxBatch;
    cp.status = m->d_status;
    if ((e = launch_moe_combine(cp, lc)) != cudaSuccess) return e;
    if (m->world > 1 && (e = launch_moe_ep_advance(m->d_ep_seq, lc)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t ds2_enqueue_lm_head(zgpu_ds2_model *m, uint32_t *counter) {
  const zgpu_ds2_desc &d = m->desc;
  LaunchCfg lc = launch_cfg(m, counter);
  GemvDesc g;
  g.w = m->out->d;
  g.wbytes = m->out->bytes;
  g.gstride = m->out->gstride;
  g.quant = m->out->quant;
  g.rows = d.vocab_padded;
  g.groups = static_cast<uint32_t>(m->out->groups);
  g.in_dim = d.hidden;
  GemvIo io;
  io.x = m->d_hidden;
  io.norm_w = m->d_out_norm;
  io.eps = d.rms_eps;
  io.out = m->d_logits;
  io.argmax = m->d_argmax;
  io.status = m->d_status;
  cudaError_t e = launch_gemv(g, PRO_RMSNORM, EPI_ARGMAX, io, lc);
  if (e != cudaSuccess) return e;
  FinalizeParams fp;
  fp.argmax = m->d_argmax;
  fp.state = m->d_state;
  fp.tokens_out = m->d_tokens;
  fp.status = m->d_status;
  return launch_finalize(fp, lc);
}

// One decode step of ns sequences (each at its own position of its own
// cache): the single-sequence kernel sequence with every launch widened over
// the batch, so each sequence's arithmetic, and so its results, are those of
// zgpu_ds2_forward_single_token + zgpu_ds2_lm_head_argmax bit for bit.  The
// projections are same-weight segmented GEMVs (segment b = sequence b), the
// MLA kernels and the router take the sequence as grid dimension y, and the
// grouped expert GEMVs run ns * (n_shared + top_k) segments from the
// router's per-token tables.  MLA layers only.
cudaError_t ds2_enqueue_batch(zgpu_ds2_model *m, uint32_t ns, uint32_t *counter) {
  const zgpu_ds2_desc &d = m->desc;
  auto &B = m->b;
  LaunchCfg lc = launch_cfg(m, counter);
  cudaError_t e = launch_rows_embed(m->emb->d, m->emb->gstride, m->emb->quant, d.hidden,
                                    static_cast<uint32_t>(m->emb->rows), B.tok, ns, B.hidden, m->d_status, lc.stream);
  if (counter) ++*counter;
  if (e != cudaSuccess) return e;
  const uint32_t H = d.hidden, R = d.kv_lora_rank, RD = d.rope_dim, QL = d.q_lora_rank;
  const uint32_t NH = d.n_heads, hq = d.nope_dim + d.rope_dim, VD = d.v_dim;
  // One projection of every sequence on the tensor cores (digit_mma.h):
  // the digit image of the inputs (RMSNorm first when norm_w), the MMA
  // partials, then the GEMV's epilogue.  n_img > 1: image / segment i uses
  // the inputs at x + i * x_img_stride and the i-th of n_img tile sets.
  // Each sequence's result is the single-sequence GEMV's bit for bit.
  auto dm = [&](const float *x, uint64_t x_stride, uint64_t x_img_stride, uint32_t n_img, const float *norm_w,
                const uint8_t *tiles, uint32_t rows, uint32_t in_dim, float *out, uint64_t out_seg_stride,
                uint64_t out_vec_stride, GemvEpi epi) -> cudaError_t {
    DigitImageParams ip = {};
    ip.x = x;
    ip.x_stride = x_stride;
    ip.x_img_stride = x_img_stride;
    ip.norm_w = norm_w;
    ip.eps = d.rms_eps;
    ip.in_dim = in_dim;
    ip.n_vec = ns;
    ip.n_img = n_img;
    ip.img = B.img;
    ip.status = m->d_status;
    cudaError_t e2 = launch_digit_image(ip, lc);
    if (e2 != cudaSuccess) return e2;
    DmGemmParams gp = {};
    gp.wt = tiles;
    gp.wt_seg_stride = dm_tile_bytes(rows, in_dim / 32);
    gp.rows = rows;
    gp.in_dim = in_dim;
    gp.img = B.img;
    gp.img_seg = n_img > 1 ? 1 : 0;
    gp.n_vec = ns;
    gp.n_seg = n_img;
    gp.part = B.dpart;
    gp.status = m->d_status;
    if ((e2 = launch_dm_gemm(gp, lc)) != cudaSuccess) return e2;
    DmCombineParams cp = {};
    cp.part = B.dpart;
    cp.rows = rows;
    cp.ks = (in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks;
    cp.n_vec = ns;
    cp.n_seg = n_img;
    cp.out = out;
    cp.out_seg_stride = out_seg_stride;
    cp.out_vec_stride = out_vec_stride;
    cp.epi = epi;
    return launch_dm_combine(cp, lc);
  };
  // The expert matvecs: n_segs segments of up to 32 vectors each (count
  // B.dn_vec[s]); vector j of segment s reads row x_rows[s * 32 + j] of x,
  // multiplies the tiles tab[s] and writes out_rows[s * 32 + j].
  auto dm_grouped = [&](const float *x, uint64_t x_stride, const float *norm_w, const uint32_t *x_rows,
                        const unsigned long long *tab, uint32_t n_segs, uint32_t rows, uint32_t in_dim,
                        float *const *out_rows, GemvEpi epi) -> cudaError_t {
    DigitImageParams ip = {};
    ip.x = x;
    ip.x_stride = x_stride;
    ip.x_rows = x_rows;
    ip.n_vec_of = B.dn_vec;
    ip.norm_w = norm_w;
    ip.eps = d.rms_eps;
    ip.in_dim = in_dim;
    ip.n_vec = kDmMaxVec;
    ip.n_img = n_segs;
    ip.img = B.img;
    ip.status = m->d_status;
    ip.pairs = B.pairs;
    ip.n_pairs = B.dn_vec + kMoeMaxSegs;
    ip.max_pairs = ns * (d.n_shared + d.top_k);
    cudaError_t e2 = launch_digit_image(ip, lc);
    if (e2 != cudaSuccess) return e2;
    DmGemmParams gp = {};
    gp.w_tab = tab;
    gp.w_tab_mod = n_segs;
    gp.rows = rows;
    gp.in_dim = in_dim;
    gp.img = B.img;
    gp.img_seg = 1;
    gp.n_vec = kDmMaxVec;
    gp.n_seg = n_segs;
    gp.n_vec_of = B.dn_vec;
    gp.part = B.dpart;
    gp.status = m->d_status;
    if ((e2 = launch_dm_gemm(gp, lc)) != cudaSuccess) return e2;
    DmCombineParams cp = {};
    cp.part = B.dpart;
    cp.rows = rows;
    cp.ks = (in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks;
    cp.n_vec = kDmMaxVec;
    cp.n_seg = n_segs;
    cp.n_vec_of = B.dn_vec;
    cp.out_rows = out_rows;
    cp.epi = epi;
    // only the (expert, token) pairs in use: at most n_seq x (n_shared + top_k)
    cp.pairs = B.pairs;
    cp.n_pairs = B.dn_vec + kMoeMaxSegs;
    cp.max_pairs = ns * (d.n_shared + d.top_k);
    return launch_dm_combine(cp, lc);
  };
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    const Ds2Layer &L = m->layers[l];
    // RMSNorm + fused kv_a_mqa | q_a; RMSNorm(c_q) + q_b
    if ((e = dm(B.hidden, H, 0, 1, L.attn_norm, L.t_cat, R + RD + QL, H, B.ca, 0,
                B.ca_stride, EPI_STORE)) != cudaSuccess)
      return e;
    if ((e = dm(B.ca + R + RD, B.ca_stride, 0, 1, L.q_a_norm, L.t_qb, NH * hq, QL, B.q, 0, NH * hq,
                EPI_STORE)) != cudaSuccess)
      return e;
    // latent append + query absorption, attention, merge: each sequence on
    // its own cache rows and position
    MlaParams mp = {};
    mp.kv_a = B.ca;
    mp.kv_a_norm = L.kv_a_norm;
    mp.k_norm = L.k_norm;
    mp.q = B.q;
    mp.kb = L.kb->d;
    mp.kb_gstride = L.kb->gstride;
    mp.kb_quant = L.kb->quant;
    mp.kb_head_rows = L.kb_head_rows;
    mp.inv_freqs = m->d_inv_freqs;
    mp.max_tokens = B.max_tokens;
    mp.q_abs = B.qabs;
    mp.q_pe = B.qpe;
    mp.ctx = B.ctx;
    mp.part = B.part;
    mp.status = m->d_status;
    mp.n_heads = NH;
    mp.kv_lora = R;
    mp.rope = RD;
    mp.nope = d.nope_dim;
    mp.max_splits = B.splits;
    mp.eps = d.rms_eps;
    mp.scale = 1.0f / sqrtf(static_cast<float>(hq));
    mp.n_seq = ns;
    mp.kv_a_stride = B.ca_stride;
    mp.q_stride = NH * hq;
    mp.seq_cache = B.cache;
    mp.layer_off = static_cast<uint64_t>(l) * B.max_tokens * (R + RD);
    mp.seq_pos = B.pos;
    mp.split_tokens = mla_split_tokens(ns, B.max_tokens, m->ctx->sm_count);
    if ((e = launch_mla_prep(mp, lc)) != cudaSuccess) return e;
    if ((e = launch_mla_attention(mp, lc)) != cudaSuccess) return e;
    // per-head V projection: image h holds every sequence's ctx row of
    // head h, segment h streams head h's v rows
    if ((e = dm(B.ctx, static_cast<uint64_t>(NH) * R, R, NH, nullptr, L.t_v, VD, R, B.concat, VD,
                static_cast<uint64_t>(NH) * VD, EPI_STORE)) != cudaSuccess)
      return e;
    // O projection + residual
    if ((e = dm(B.concat, static_cast<uint64_t>(NH) * VD, 0, 1, nullptr, L.t_o, H, NH * VD, B.hidden, 0, H,
                EPI_RESADD)) != cudaSuccess)
      return e;

    if (!L.moe) {
      if ((e = dm(B.hidden, H, 0, 1, L.ffn_norm, L.t_gu, 2 * d.ffn, H, B.act, 0, B.act_stride, EPI_SWIGLU)) != cudaSuccess)
        return e;
      if ((e = dm(B.act, B.act_stride, 0, 1, nullptr, L.t_dn, H, d.ffn, B.hidden, 0, H, EPI_RESADD)) != cudaSuccess)
        return e;
      continue;
    }
    RouteParams rp = {};
    rp.x = B.hidden;
    rp.norm_w = L.ffn_norm;
    rp.eps = d.rms_eps;
    rp.w = reinterpret_cast<const float *>(L.router->d);
    rp.bias = L.d_router_b;
    rp.dim = H;
    rp.n_experts = d.n_experts;
    rp.top_k = d.top_k;
    rp.mode = d.route_mode;
    rp.scale = d.expert_weight_scale;
    rp.scores = B.scores;
    rp.ids = B.ids + static_cast<size_t>(l) * kDs2MaxBatch * d.top_k;
    rp.weights = B.wts + static_cast<size_t>(l) * kDs2MaxBatch * d.top_k;
    rp.counter = B.counter;
    rp.seg_gu = nullptr;   // the expert grouping below replaces the per-token tables
    rp.seg_dn = nullptr;
    rp.gu_base = reinterpret_cast<unsigned long long>(L.gateup);
    rp.dn_base = reinterpret_cast<unsigned long long>(L.down->d);
    rp.sh_gu_base = reinterpret_cast<unsigned long long>(L.sh_gateup);
    rp.sh_dn_base = L.sh_down ? reinterpret_cast<unsigned long long>(L.sh_down->d) : 0ull;
    rp.gu_bytes = m->gu_bytes;
    rp.dn_bytes = m->dn_bytes;
    rp.n_shared = d.n_shared;
    rp.status = m->d_status;
    rp.ep_rank = m->rank;
    rp.ep_per_rank = m->world > 1 ? m->ep_per_rank : 0;
    rp.n_seq = ns;
    rp.x_stride = H;
    if ((e = launch_moe_route(rp, lc)) != cudaSuccess) return e;
    // the batch's (token, expert) pairs grouped by expert, then the grouped
    // gate|up + SiLU*up and down matvecs on the tensor cores: segment =
    // expert, vectors = the tokens that selected it
    const uint32_t n_local = m->world > 1 ? m->ep_per_rank : d.n_experts, n_segs = n_local + d.n_shared;
    MoeDispatchParams dp = {};
    dp.ids = rp.ids;
    dp.n_seq = ns;
    dp.top_k = d.top_k;
    dp.n_shared = d.n_shared;
    dp.n_local = n_local;
    dp.ep_rank = m->rank;
    dp.ep_per_rank = m->world > 1 ? m->ep_per_rank : 0;
    dp.act = B.act;
    dp.exp_out = B.expout;
    dp.act_row = d.expert_ffn;
    dp.dim = H;
    dp.tiles_gu = L.t_egu;
    dp.tiles_dn = L.t_edn;
    dp.sh_tiles_gu = L.t_sgu;
    dp.sh_tiles_dn = L.t_sdn;
    dp.tiles_gu_stride = dm_tile_bytes(2ull * d.expert_ffn, H / 32);
    dp.tiles_dn_stride = dm_tile_bytes(H, d.expert_ffn / 32);
    dp.n_vec = B.dn_vec;
    dp.x_rows_gu = B.x_rows_gu;
    dp.x_rows_dn = B.x_rows_dn;
    dp.out_gu = B.out_gu;
    dp.out_dn = B.out_dn;
    dp.tab_gu = B.tab_gu;
    dp.tab_dn = B.tab_dn;
    dp.pairs = B.pairs;
    dp.n_pairs = B.dn_vec + kMoeMaxSegs;
    if ((e = launch_moe_dispatch(dp, lc)) != cudaSuccess) return e;
    if ((e = dm_grouped(B.hidden, H, L.ffn_norm, B.x_rows_gu, B.tab_gu, n_segs, 2 * d.expert_ffn, H, B.out_gu,
                        EPI_SWIGLU)) != cudaSuccess)
      return e;
    if ((e = dm_grouped(B.act, d.expert_ffn, nullptr, B.x_rows_dn, B.tab_dn, n_segs, H, d.expert_ffn, B.out_dn,
                        EPI_STORE)) != cudaSuccess)
      return e;
    if (m->world > 1) {
      EpPublishParams pp = {};
      pp.exp_out = B.expout;
      pp.ids = rp.ids;
      pp.dst = m->d_ep_dst;
      pp.ep_seq = m->d_ep_seq;
      pp.dim = H;
      pp.n_shared = d.n_shared;
      pp.top_k = d.top_k;
      pp.world = m->world;
      pp.ep_rank = m->rank;
      pp.ep_per_rank = m->ep_per_rank;
      pp.n_seq = ns;
      pp.slot_cap = d.top_k * kDs2MaxBatch;
      if ((e = launch_moe_ep_publish(pp, lc)) != cudaSuccess) return e;
    }
    CombineParams cp = {};
    cp.exp_out = B.expout;
    cp.weights = rp.weights;
    cp.hidden = B.hidden;
    cp.dim = H;
    cp.n_shared = d.n_shared;
    cp.top_k = d.top_k;
    cp.xslots = m->world > 1 ? m->d_xslots : nullptr;
    cp.ep_seq = m->d_ep_seq;
    cp.world = m->world;
    cp.n_seq = ns;
    cp.slot_cap = d.top_k * kDs2MaxBatch;
    cp.status = m->d_status;
    if ((e = launch_moe_combine(cp, lc)) != cudaSuccess) return e;
    if (m->world > 1 && (e = launch_moe_ep_advance(m->d_ep_seq, lc)) != cudaSuccess) return e;
  }
  // LM head: RMSNorm + matvec per sequence, then the reference's greedy
  // pick per logits row
  if ((e = dm(B.hidden, H, 0, 1, m->d_out_norm, B.t_out, d.vocab_padded, H, B.logits, 0, d.vocab_padded, EPI_STORE)) != cudaSuccess)
    return e;
  if (counter) ++*counter;
  return launch_rows_argmax(B.logits, ns, d.vocab_padded, d.vocab_real, B.out, B.codes, m->d_status, lc.stream);
}

enum GraphPart { GRAPH_STEP = 0, GRAPH_FWD = 1, GRAPH_LM = 2 };

zgpu_status ds2_capture(zgpu_ds2_model *m, zgpu_mla_kv *kv, GraphPart part, cudaGraphExec_t *out,
                        uint32_t *kernels) {
  zgpu_ctx *ctx = m->ctx;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "begin capture");
  uint32_t n = 0;
  cudaError_t e1 = cudaSuccess;
  if (part != GRAPH_LM) e1 = ds2_enqueue_forward(m, kv, &n);
  if (e1 == cudaSuccess && part != GRAPH_FWD) e1 = ds2_enqueue_lm_head(m, &n);
  e = cudaStreamEndCapture(ctx->stream, &g);
  if (e1 != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return zgpu_cuda_fail(ctx, e1, "capture step");
  }
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "end capture");
  e = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "graph instantiate");
  *kernels = n;
  return ZGPU_OK;
}

void ds2_drop_graphs(zgpu_ds2_model *m) {
  for (cudaGraphExec_t *g : {&m->step_graph, &m->fwd_graph, &m->lm_graph}) {
    if (*g) cudaGraphExecDestroy(*g);
    *g = nullptr;
  }
  m->graph_kv = nullptr;
}

zgpu_status ds2_build_graphs(zgpu_ds2_model *m, zgpu_mla_kv *kv) {
  if (m->step_graph && m->graph_kv == kv) return ZGPU_OK;
  ds2_drop_graphs(m);
  zgpu_status s = ds2_capture(m, kv, GRAPH_STEP, &m->step_graph, &m->step_kernels);
  if (!s) s = ds2_capture(m, kv, GRAPH_FWD, &m->fwd_graph, &m->fwd_kernels);
  if (!s) s = ds2_capture(m, nullptr, GRAPH_LM, &m->lm_graph, &m->lm_kernels);
  if (s) {
    ds2_drop_graphs(m);
    return s;
  }
  m->graph_kv = kv;
  return ZGPU_OK;
}

zgpu_status ds2_set_state(zgpu_ds2_model *m, uint32_t n_prompt, uint32_t pos_base, uint32_t vocab_real,
                          uint32_t n_gen_cap) {
  StepState s = {};
  s.n_prompt = n_prompt;
  s.pos_base = pos_base;
  s.pos = pos_base;
  s.vocab_real = vocab_real;
  s.n_gen_cap = n_gen_cap;
  s.first_err_step = 0xFFFFFFFFu;
  cudaError_t e = cudaMemcpyAsync(m->d_state, &s, sizeof(s), cudaMemcpyHostToDevice, m->ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(m->ctx, e, "state upload");
  return ZGPU_OK;
}

template <class T>
cudaError_t grow(T **p, uint32_t *cap, uint32_t need) {
  if (need <= *cap) return cudaSuccess;
  cudaFree(*p);
  *p = nullptr;
  cudaError_t e = cudaMalloc(p, static_cast<size_t>(need) * sizeof(T));
  if (e == cudaSuccess) *cap = need;
  return e;
}

zgpu_status ds2_prepare_kv(zgpu_ds2_model *m, zgpu_mla_kv *kv) {
  zgpu_ctx *ctx = m->ctx;
  if (kv->n_layers != m->desc.n_layers)
    return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "mla cache layer count differs from the model");
  if (kv->kv_lora != m->desc.kv_lora_rank || kv->rope != m->desc.rope_dim)
    return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "mla cache geometry differs from the model");
  const uint32_t splits = mla_max_splits(kv->max_tokens);
  if (splits != m->max_splits || !m->d_part) {
    cudaFree(m->d_part);
    m->d_part = nullptr;
    const size_t n = static_cast<size_t>(m->desc.n_heads) * splits * (m->desc.kv_lora_rank + 2);
    cudaError_t e = cudaMalloc(&m->d_part, n * 4);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "mla attention scratch");
    m->max_splits = splits;
    ds2_drop_graphs(m);
  }
  // forward_pass.rs:790-793: an MHA layer without its cache is an error
  if (m->n_mha && !m->mha_kv)
    return zgpu_fail(ctx, ZGPU_ERR_NUMERICAL_INSTABILITY, "model has MHA layers: bind a cache with zgpu_ds2_set_mha_kv");
  return ZGPU_OK;
}

// Scratch of the batch's tensor-core projections (digit_mma.h): the largest
// digit image (32 vectors, per-head images for the V projection) and the
// largest set of chunk partials.
uint64_t ds2_dm_img_bytes(const zgpu_ds2_desc &d) {
  const uint32_t NB = kDs2MaxBatch;
  uint64_t b = std::max(dm_img_bytes(d.hidden, NB), static_cast<uint64_t>(d.n_heads) * dm_img_bytes(d.kv_lora_rank, NB));
  b = std::max(b, dm_img_bytes(d.q_lora_rank, NB));
  b = std::max(b, dm_img_bytes(d.n_heads * d.v_dim, NB));
  if (d.ffn % 32 == 0 && d.ffn) b = std::max(b, dm_img_bytes(d.ffn, NB));
  // expert groups: one image per expert segment
  const uint64_t segs = static_cast<uint64_t>(d.n_experts) + d.n_shared;
  if (d.expert_ffn % 32 == 0 && d.expert_ffn)
    b = std::max(b, segs * std::max(dm_img_bytes(d.hidden, NB), dm_img_bytes(d.expert_ffn, NB)));
  return b;
}
uint64_t ds2_dm_part_floats(const zgpu_ds2_desc &d, bool any_dense) {
  auto ks = [](uint32_t in_dim) { return static_cast<uint64_t>((in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks); };
  const uint64_t NB = kDs2MaxBatch, H = d.hidden, R = d.kv_lora_rank;
  const uint64_t cat_rows = (static_cast<uint64_t>(R + d.rope_dim + d.q_lora_rank) + 8) & ~7ull;
  uint64_t f = ks(d.hidden) * NB * std::max<uint64_t>(cat_rows, d.vocab_padded);
  if (any_dense) f = std::max(f, ks(d.hidden) * NB * 2 * d.ffn);
  f = std::max(f, ks(d.q_lora_rank) * NB * d.n_heads * (d.nope_dim + d.rope_dim));
  f = std::max(f, d.n_heads * ks(d.kv_lora_rank) * NB * d.v_dim);
  f = std::max(f, ks(d.n_heads * d.v_dim) * NB * H);
  if (any_dense) f = std::max(f, ks(d.ffn) * NB * H);
  const uint64_t segs = static_cast<uint64_t>(d.n_experts) + d.n_shared;
  if (d.expert_ffn % 32 == 0 && d.expert_ffn) {
    f = std::max(f, segs * ks(d.hidden) * NB * 2 * d.expert_ffn);
    f = std::max(f, segs * ks(d.expert_ffn) * NB * H);
  }
  return f;
}

// The weight tiles of every projection the batch step runs on the tensor
// cores (MLA layers: the batch refuses MHA layers).
bool ds2_build_tiles(zgpu_ds2_model *m) {
  const zgpu_ds2_desc &d = m->desc;
  cudaStream_t st = m->ctx->stream;
  auto tiles = [&](const uint8_t *w, uint64_t gstride, uint32_t quant, uint32_t rows, uint32_t in_dim,
                   uint8_t *dst) -> bool {
    return launch_build_dm_tiles(w, gstride, quant, rows, in_dim / 32, dst, st) == cudaSuccess;
  };
  auto alloc = [&](uint8_t **p, uint64_t rows, uint32_t in_dim, uint32_t copies) -> bool {
    return cudaMalloc(p, copies * dm_tile_bytes(rows, in_dim / 32)) == cudaSuccess;
  };
  const uint32_t H = d.hidden, R = d.kv_lora_rank, NH = d.n_heads, VD = d.v_dim, hq = d.nope_dim + d.rope_dim;
  for (Ds2Layer &L : m->layers) {
    if (L.mha) continue;
    const uint32_t cat_rows = R + d.rope_dim + d.q_lora_rank;
    if (!alloc(&L.t_cat, cat_rows, H, 1) || !tiles(L.cat_a, m->gs_h, d.attn_quant, cat_rows, H, L.t_cat)) return false;
    if (!alloc(&L.t_qb, NH * hq, d.q_lora_rank, 1) ||
        !tiles(L.q_b->d, L.q_b->gstride, d.attn_quant, NH * hq, d.q_lora_rank, L.t_qb))
      return false;
    if (!alloc(&L.t_o, H, NH * VD, 1) || !tiles(L.o->d, L.o->gstride, d.attn_quant, H, NH * VD, L.t_o)) return false;
    std::vector<unsigned long long> vseg(NH);
    if (cudaMemcpy(vseg.data(), L.d_vseg, NH * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return false;
    if (!alloc(&L.t_v, VD, R, NH)) return false;
    for (uint32_t h = 0; h < NH; ++h)
      if (!tiles(reinterpret_cast<const uint8_t *>(vseg[h]), L.v_gstride, d.attn_quant, VD, R,
                 L.t_v + h * dm_tile_bytes(VD, R / 32)))
        return false;
    if (!L.moe) {
      if (!alloc(&L.t_gu, 2ull * d.ffn, H, 1) || !tiles(L.gateup, m->gs_h, ZGPU_Q4_0, 2 * d.ffn, H, L.t_gu))
        return false;
      if (!alloc(&L.t_dn, H, d.ffn, 1) || !tiles(L.down->d, L.down->gstride, ZGPU_Q4_0, H, d.ffn, L.t_dn))
        return false;
      continue;
    }
    // this rank's routed experts, then the shared ones (each expert's
    // interleaved gate|up rows and its down rows as separate tile sets)
    const uint32_t EF = d.expert_ffn, n_local = m->world > 1 ? m->ep_per_rank : d.n_experts;
    const uint32_t e0 = m->world > 1 ? m->rank * m->ep_per_rank : 0;
    const uint64_t sgu = dm_tile_bytes(2ull * EF, H / 32), sdn = dm_tile_bytes(H, EF / 32);
    if (!alloc(&L.t_egu, 2ull * EF, H, n_local) || !alloc(&L.t_edn, H, EF, n_local)) return false;
    for (uint32_t i = 0; i < n_local; ++i) {
      if (!tiles(L.gateup + static_cast<uint64_t>(e0 + i) * m->gu_bytes, m->gs_h, ZGPU_Q4_0, 2 * EF, H,
                 L.t_egu + i * sgu) ||
          !tiles(L.down->d + static_cast<uint64_t>(e0 + i) * m->dn_bytes, m->gs_e, ZGPU_Q4_0, H, EF,
                 L.t_edn + i * sdn))
        return false;
    }
    if (d.n_shared) {
      if (!alloc(&L.t_sgu, 2ull * EF, H, d.n_shared) || !alloc(&L.t_sdn, H, EF, d.n_shared)) return false;
      for (uint32_t i = 0; i < d.n_shared; ++i) {
        if (!tiles(L.sh_gateup + static_cast<uint64_t>(i) * m->gu_bytes, m->gs_h, ZGPU_Q4_0, 2 * EF, H,
                   L.t_sgu + i * sgu) ||
            !tiles(L.sh_down->d + static_cast<uint64_t>(i) * m->dn_bytes, L.sh_down->gstride, ZGPU_Q4_0, H, EF,
                   L.t_sdn + i * sdn))
          return false;
      }
    }
  }
  auto &B = m->b;
  if (!alloc(&B.t_out, d.vocab_padded, H, 1) ||
      !tiles(m->out->d, m->out->gstride, m->out->quant, d.vocab_padded, H, B.t_out))
    return false;
  return cudaStreamSynchronize(st) == cudaSuccess;
}

void ds2_free_batch(zgpu_ds2_model *m) {
  auto &B = m->b;
  if (B.graph) cudaGraphExecDestroy(B.graph);
  for (float *p : {B.hidden, B.ca, B.q, B.qabs, B.qpe, B.ctx, B.concat, B.act, B.expout, B.scores, B.logits,
                   B.wts, B.part})
    cudaFree(p);
  for (uint32_t *p : {B.ids, B.counter, B.tok, B.pos, B.out, B.codes}) cudaFree(p);
  cudaFree(B.cache);
  cudaFree(B.img);
  cudaFree(B.dpart);
  cudaFree(B.t_out);
  cudaFree(B.dn_vec);
  cudaFree(B.pairs);
  cudaFree(B.x_rows_gu);
  cudaFree(B.x_rows_dn);
  cudaFree(B.out_gu);
  cudaFree(B.out_dn);
  cudaFree(B.tab_gu);
  cudaFree(B.tab_dn);
  for (Ds2Layer &L : m->layers)
    for (uint8_t **t : {&L.t_cat, &L.t_qb, &L.t_o, &L.t_v, &L.t_gu, &L.t_dn, &L.t_egu, &L.t_edn, &L.t_sgu, &L.t_sdn}) {
      cudaFree(*t);
      *t = nullptr;
    }
  B = zgpu_ds2_model::Batch();
}

// The batch buffers for caches of max_tokens rows (allocated once; the
// attention scratch again when the cache capacity changes).
zgpu_status ds2_prepare_batch(zgpu_ds2_model *m, uint32_t max_tokens) {
  zgpu_ctx *ctx = m->ctx;
  const zgpu_ds2_desc &d = m->desc;
  auto &B = m->b;
  const size_t NB = kDs2MaxBatch;
  const uint32_t H = d.hidden, R = d.kv_lora_rank, RD = d.rope_dim, NH = d.n_heads;
  const uint32_t n_seg = d.n_shared + d.top_k;
  if (!B.hidden) {
    bool any_moe = false, any_dense = false;
    for (const Ds2Layer &L : m->layers) (L.moe ? any_moe : any_dense) = true;
    B.ca_stride = R + RD + d.q_lora_rank + 8;
    B.act_stride = static_cast<uint32_t>(std::max<size_t>(any_dense ? d.ffn : 0, static_cast<size_t>(n_seg) * d.expert_ffn));
    const size_t topk = any_moe ? d.top_k : 1;
    const uint32_t hq = d.nope_dim + RD;
    if (cudaMalloc(&B.hidden, NB * H * 4) || cudaMalloc(&B.ca, NB * B.ca_stride * 4) ||
        cudaMalloc(&B.q, NB * NH * hq * 4) || cudaMalloc(&B.qabs, NB * NH * R * 4) ||
        cudaMalloc(&B.qpe, NB * NH * (RD ? RD : 1) * 4) || cudaMalloc(&B.ctx, NB * NH * R * 4) ||
        cudaMalloc(&B.concat, NB * NH * d.v_dim * 4) || cudaMalloc(&B.act, NB * (B.act_stride ? B.act_stride : 1) * 4) ||
        cudaMalloc(&B.expout, NB * (n_seg ? n_seg : 1) * H * 4) ||
        cudaMalloc(&B.scores, NB * (d.n_experts ? d.n_experts : 1) * 4) ||
        cudaMalloc(&B.logits, NB * d.vocab_padded * 4) || cudaMalloc(&B.wts, d.n_layers * NB * topk * 4) ||
        cudaMalloc(&B.ids, d.n_layers * NB * topk * 4) || cudaMalloc(&B.counter, NB * 4) ||
        cudaMalloc(&B.tok, NB * 4) || cudaMalloc(&B.pos, NB * 4) || cudaMalloc(&B.out, NB * 4) ||
        cudaMalloc(&B.codes, NB * 4) ||
        cudaMalloc(&B.cache, NB * sizeof(float *)) || cudaMalloc(&B.img, ds2_dm_img_bytes(d)) ||
        cudaMalloc(&B.dpart, ds2_dm_part_floats(d, any_dense) * 4) || cudaMalloc(&B.dn_vec, kMoeMaxSegs * 4 + 4) ||
        cudaMalloc(&B.pairs, kMoeMaxSegs * 32 * 4) ||
        cudaMalloc(&B.x_rows_gu, kMoeMaxSegs * 32 * 4) || cudaMalloc(&B.x_rows_dn, kMoeMaxSegs * 32 * 4) ||
        cudaMalloc(&B.out_gu, kMoeMaxSegs * 32 * sizeof(float *)) ||
        cudaMalloc(&B.out_dn, kMoeMaxSegs * 32 * sizeof(float *)) || cudaMalloc(&B.tab_gu, kMoeMaxSegs * 8) ||
        cudaMalloc(&B.tab_dn, kMoeMaxSegs * 8)) {
      ds2_free_batch(m);
      return zgpu_fail(ctx, ZGPU_ERR_OUT_OF_MEMORY, "batch activation buffers");
    }
    if (!ds2_build_tiles(m)) {
      ds2_free_batch(m);
      return zgpu_fail(ctx, ZGPU_ERR_OUT_OF_MEMORY, "batch weight tiles");
    }
    cudaMemset(B.counter, 0, NB * 4);
    cudaMemset(B.ids, 0, d.n_layers * NB * topk * 4);
    cudaMemset(B.wts, 0, d.n_layers * NB * topk * 4);
  }
  const uint32_t splits = mla_max_splits(max_tokens);
  if (splits != B.splits || max_tokens != B.max_tokens) {
    cudaFree(B.part);
    B.part = nullptr;
    B.splits = 0;
    if (B.graph) cudaGraphExecDestroy(B.graph);
    B.graph = nullptr;
    const size_t n = NB * NH * splits * (R + 2);
    cudaError_t e = cudaMalloc(&B.part, n * 4);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "batch attention scratch");
    B.splits = splits;
    B.max_tokens = max_tokens;
  }
  return ZGPU_OK;
}

// Interleave two tensors' group streams: group j of a at 2j, of b at 2j+1.
cudaError_t interleave_groups(uint8_t **dst, const DeviceTensor *a, const DeviceTensor *b) {
  cudaError_t e = cudaMalloc(dst, a->bytes + b->bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemcpy2D(*dst, 2 * a->gstride, a->d, a->gstride, a->gstride, a->groups, cudaMemcpyDeviceToDevice);
  if (e != cudaSuccess) return e;
  return cudaMemcpy2D(*dst + a->gstride, 2 * a->gstride, b->d, b->gstride, b->gstride, b->groups,
                      cudaMemcpyDeviceToDevice);
}

}  // namespace

extern "C" {

// ------------------------------------------------------------ MLA cache

zgpu_status zgpu_mla_kv_create(zgpu_ctx *ctx, uint32_t max_tokens, uint32_t n_layers,
                               uint32_t kv_lora_rank, uint32_t rope_dim, zgpu_mla_kv **out) {
  if (!ctx || !out || !max_tokens || !n_layers || !kv_lora_rank) return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  cudaSetDevice(ctx->device);
  zgpu_mla_kv *kv = new (std::nothrow) zgpu_mla_kv();
  if (!kv) return ZGPU_ERR_OUT_OF_MEMORY;
  kv->ctx = ctx;
  kv->max_tokens = max_tokens;
  kv->n_layers = n_layers;
  kv->kv_lora = kv_lora_rank;
  kv->rope = rope_dim;
  kv->layer_floats = static_cast<uint64_t>(max_tokens) * (kv_lora_rank + rope_dim);
  const size_t bytes = static_cast<size_t>(n_layers) * kv->layer_floats * sizeof(float);
  cudaError_t e = cudaMalloc(&kv->d, bytes);
  if (e == cudaSuccess) e = cudaMemset(kv->d, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(kv->d);
    delete kv;
    return zgpu_cuda_fail(ctx, e, "mla cache allocation");
  }
  *out = kv;
  return ZGPU_OK;
}

void zgpu_mla_kv_destroy(zgpu_mla_kv *kv) {
  if (!kv) return;
  cudaSetDevice(kv->ctx->device);
  cudaFree(kv->d);
  delete kv;
}

zgpu_status zgpu_mla_kv_store(zgpu_mla_kv *kv, uint32_t layer, uint32_t token, const float *c_kv,
                              const float *k_rope) {
  if (!kv || !c_kv || (!k_rope && kv->rope)) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = kv->ctx;
  if (layer >= kv->n_layers) return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "layer out of range");
  if (token >= kv->max_tokens) return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "token out of range");
  cudaSetDevice(ctx->device);
  float *row = kv->d + layer * kv->layer_floats + static_cast<uint64_t>(token) * (kv->kv_lora + kv->rope);
  cudaError_t e = cudaMemcpyAsync(row, c_kv, kv->kv_lora * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess && kv->rope)
    e = cudaMemcpyAsync(row + kv->kv_lora, k_rope, kv->rope * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "mla cache store");
  return ZGPU_OK;
}

zgpu_status zgpu_mla_kv_read(zgpu_mla_kv *kv, uint32_t layer, uint32_t token_count, float *rows_out) {
  if (!kv || !rows_out) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = kv->ctx;
  if (layer >= kv->n_layers) return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "layer out of range");
  if (token_count > kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_COUNT_EXCEEDS_MAX, "token count exceeds max_tokens");
  cudaSetDevice(ctx->device);
  const size_t n = static_cast<size_t>(token_count) * (kv->kv_lora + kv->rope);
  cudaError_t e = cudaMemcpyAsync(rows_out, kv->d + layer * kv->layer_floats, n * 4,
                                  cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "mla cache read");
  return ZGPU_OK;
}

zgpu_status zgpu_mla_kv_copy(zgpu_mla_kv *dst, const zgpu_mla_kv *src, uint32_t token_count) {
  if (!dst || !src || dst == src) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = dst->ctx;
  if (src->ctx != ctx || src->n_layers != dst->n_layers || src->kv_lora != dst->kv_lora || src->rope != dst->rope)
    return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "mla cache copy: geometry differs");
  if (token_count > src->max_tokens || token_count > dst->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_COUNT_EXCEEDS_MAX, "token count exceeds max_tokens");
  cudaSetDevice(ctx->device);
  const size_t row = static_cast<size_t>(token_count) * (src->kv_lora + src->rope) * 4;
  cudaError_t e = cudaSuccess;
  if (row)
    e = cudaMemcpy2DAsync(dst->d, dst->layer_floats * 4, src->d, src->layer_floats * 4, row, src->n_layers,
                          cudaMemcpyDeviceToDevice, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "mla cache copy");
  return ZGPU_OK;
}

// ------------------------------------------------------------ MoE routing

zgpu_status zgpu_moe_route_f32(zgpu_ctx *ctx, const float *hidden, const void *router_key,
                               const float *router_bias, uint64_t dim, uint32_t n_experts,
                               uint32_t top_k, uint32_t mode, float expert_weight_scale,
                               float *scores_out, uint32_t *indices_out, float *weights_out) {
  if (!ctx || !hidden || !indices_out || !weights_out) return ZGPU_ERR_INVALID_ARG;
  if (top_k == 0) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "moe_route_f32: top_k must be > 0");
  if (top_k > n_experts) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "moe_route_f32: top_k must be <= n_experts");
  if (top_k > kMoeMaxTopK || dim == 0 || dim % 4 || dim > kMoeMaxDim || mode > 1)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "moe_route_f32: unsupported geometry or mode");
  const DeviceTensor *t = zgpu_lookup(ctx, router_key);
  if (!t) return zgpu_fail(ctx, ZGPU_ERR_UNREGISTERED_WEIGHT, "router weights not registered");
  if (t->quant != ZGPU_F32 || t->rows != n_experts || t->cols != dim)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "router weights must be f32 [n_experts x dim]");
  cudaSetDevice(ctx->device);
  // scratch: x [dim] | bias [n_experts] | scores [n_experts] | weights [top_k] | ids [top_k]
  const size_t need = dim + 2 * static_cast<size_t>(n_experts) + 2 * top_k;
  if (need > ctx->d_x_cap) {
    cudaFree(ctx->d_x);
    ctx->d_x = nullptr;
    cudaError_t e = cudaMalloc(&ctx->d_x, need * sizeof(float));
    if (e != cudaSuccess) {
      ctx->d_x_cap = 0;
      return zgpu_cuda_fail(ctx, e, "router scratch");
    }
    ctx->d_x_cap = need;
  }
  float *d_x = ctx->d_x, *d_bias = d_x + dim, *d_scores = d_bias + n_experts, *d_w = d_scores + n_experts;
  uint32_t *d_ids = reinterpret_cast<uint32_t *>(d_w + top_k);
  cudaError_t e = cudaMemcpyAsync(d_x, hidden, dim * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess && router_bias)
    e = cudaMemcpyAsync(d_bias, router_bias, n_experts * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "router upload");
  RouteParams rp = {};
  rp.x = d_x;
  rp.w = reinterpret_cast<const float *>(t->d);
  rp.bias = router_bias ? d_bias : nullptr;
  rp.dim = static_cast<uint32_t>(dim);
  rp.n_experts = n_experts;
  rp.top_k = top_k;
  rp.mode = mode;
  rp.scale = expert_weight_scale;
  rp.scores = d_scores;
  rp.ids = d_ids;
  rp.weights = d_w;
  rp.counter = ctx->d_route_counter;
  rp.status = ctx->d_status;
  LaunchCfg lc;
  lc.stream = ctx->stream;
  lc.sm_count = ctx->sm_count;
  lc.launch_counter = &ctx->launches;
  e = launch_moe_route(rp, lc);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "router launch");
  e = cudaMemcpyAsync(indices_out, d_ids, top_k * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(weights_out, d_w, top_k * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess && scores_out)
    e = cudaMemcpyAsync(scores_out, d_scores, n_experts * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "router results");
  uint32_t st = 0;
  zgpu_status s = zgpu_read_device_status(ctx, ctx->d_status, &st);
  if (s) return s;
  return zgpu_map_device_status(ctx, st);
}

// ------------------------------------------------------------ MHA cache

zgpu_status zgpu_mha_kv_create(zgpu_ctx *ctx, uint32_t max_tokens, uint32_t n_mha_layers, uint32_t n_kv_heads,
                               uint32_t head_dim_qk, uint32_t head_dim_v, zgpu_mha_kv **out) {
  if (!ctx || !out || !max_tokens || !n_mha_layers || !n_kv_heads || !head_dim_qk || !head_dim_v)
    return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  cudaSetDevice(ctx->device);
  zgpu_mha_kv *kv = new (std::nothrow) zgpu_mha_kv();
  if (!kv) return ZGPU_ERR_OUT_OF_MEMORY;
  kv->ctx = ctx;
  kv->max_tokens = max_tokens;
  kv->n_layers = n_mha_layers;
  kv->n_kv = n_kv_heads;
  kv->hd_qk = head_dim_qk;
  kv->hd_v = head_dim_v;
  kv->k_block = static_cast<uint64_t>(max_tokens) * n_kv_heads * head_dim_qk;
  kv->v_block = static_cast<uint64_t>(max_tokens) * n_kv_heads * head_dim_v;
  const size_t bytes = static_cast<size_t>(n_mha_layers) * (kv->k_block + kv->v_block) * 4;
  if (cudaMalloc(&kv->d, bytes) != cudaSuccess) {
    delete kv;
    return zgpu_fail(ctx, ZGPU_ERR_OUT_OF_MEMORY, "mha cache allocation");
  }
  cudaMemset(kv->d, 0, bytes);
  *out = kv;
  return ZGPU_OK;
}

void zgpu_mha_kv_destroy(zgpu_mha_kv *kv) {
  if (!kv) return;
  cudaSetDevice(kv->ctx->device);
  cudaFree(kv->d);
  delete kv;
}

zgpu_status zgpu_mha_kv_store(zgpu_mha_kv *kv, uint32_t layer, uint32_t token, const float *k, const float *v) {
  if (!kv || !k || !v) return ZGPU_ERR_INVALID_ARG;
  if (layer >= kv->n_layers) return zgpu_fail(kv->ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "mha cache layer");
  if (token >= kv->max_tokens) return zgpu_fail(kv->ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "mha cache token");
  cudaSetDevice(kv->ctx->device);
  const size_t ks = static_cast<size_t>(kv->n_kv) * kv->hd_qk, vs = static_cast<size_t>(kv->n_kv) * kv->hd_v;
  float *base = kv->d + static_cast<size_t>(layer) * (kv->k_block + kv->v_block);
  cudaError_t e = cudaMemcpy(base + token * ks, k, ks * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(base + kv->k_block + token * vs, v, vs * 4, cudaMemcpyHostToDevice);
  return e == cudaSuccess ? ZGPU_OK : zgpu_cuda_fail(kv->ctx, e, "mha cache store");
}

zgpu_status zgpu_mha_kv_read(zgpu_mha_kv *kv, uint32_t layer, uint32_t token_count, float *k_out, float *v_out) {
  if (!kv || !k_out || !v_out) return ZGPU_ERR_INVALID_ARG;
  if (layer >= kv->n_layers) return zgpu_fail(kv->ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "mha cache layer");
  if (token_count > kv->max_tokens)
    return zgpu_fail(kv->ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "mha cache token count");
  cudaSetDevice(kv->ctx->device);
  cudaStreamSynchronize(kv->ctx->stream);
  const size_t ks = static_cast<size_t>(kv->n_kv) * kv->hd_qk, vs = static_cast<size_t>(kv->n_kv) * kv->hd_v;
  const float *base = kv->d + static_cast<size_t>(layer) * (kv->k_block + kv->v_block);
  cudaError_t e = cudaMemcpy(k_out, base, token_count * ks * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(v_out, base + kv->k_block, token_count * vs * 4, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? ZGPU_OK : zgpu_cuda_fail(kv->ctx, e, "mha cache read");
}

zgpu_status zgpu_ds2_set_mha_kv(zgpu_ds2_model *m, zgpu_mha_kv *kv) {
  if (!m) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  if (kv) {
    const zgpu_ds2_desc &d = m->desc;
    if (kv->n_layers != m->n_mha)
      return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "mha cache layer count differs from the model's MHA layers");
    if (kv->n_kv != m->n_kv || kv->hd_qk != d.nope_dim + d.rope_dim || kv->hd_v != d.v_dim)
      return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "mha cache geometry differs from the model");
    const uint32_t splits = mha_max_splits(kv->max_tokens);
    if (splits > m->mha_splits) {
      cudaFree(m->d_mha_part);
      m->d_mha_part = nullptr;
      m->mha_splits = 0;
      cudaError_t e = cudaMalloc(&m->d_mha_part, static_cast<size_t>(d.n_heads) * splits * (d.v_dim + 2) * 4);
      if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "mha attention scratch");
      m->mha_splits = splits;
    }
  }
  m->mha_kv = kv;
  ds2_drop_graphs(m);   // the step graphs hold the cache's addresses
  return ZGPU_OK;
}

// ------------------------------------------------------------ model

void zgpu_ds2_destroy(zgpu_ds2_model *m) {
  if (!m) return;
  cudaSetDevice(m->ctx->device);
  ds2_drop_graphs(m);
  ds2_free_batch(m);
  for (Ds2Layer &L : m->layers) {
    cudaFree(L.cat_a);
    cudaFree(L.d_vseg);
    cudaFree(L.gateup);
    cudaFree(L.sh_gateup);
    cudaFree(L.d_router_b);
    cudaFree(L.d_seg_gu);
    cudaFree(L.d_seg_dn);
    cudaFree(L.cat_qkv);
  }
  cudaFree(m->d_mha_qkv);
  cudaFree(m->d_mha_part);
  for (float *p : {m->d_norms, m->d_inv_freqs, m->d_hidden, m->d_ca, m->d_q, m->d_qabs, m->d_qpe,
                   m->d_ctx, m->d_concat, m->d_act, m->d_expout, m->d_scores, m->d_logits, m->d_wts,
                   m->d_part})
    cudaFree(p);
  cudaFree(m->d_ids);
  cudaFree(m->d_route_counter);
  cudaFree(m->d_argmax);
  cudaFree(m->d_state);
  cudaFree(m->d_prompt);
  cudaFree(m->d_tokens);
  cudaFree(m->d_status);
  for (auto &ev : m->ev)
    if (ev) cudaEventDestroy(ev);
  for (void *p : m->ipc_opened) cudaIpcCloseMemHandle(p);
  cudaFree(m->d_xslots);
  cudaFree(m->d_ep_seq);
  cudaFree(m->d_ep_dst);
  delete m;
}

}  // extern "C"

namespace {

zgpu_status ds2_create(zgpu_ctx *ctx, const zgpu_ds2_desc *d, uint32_t rank, uint32_t world, zgpu_ds2_model **out) {
  if (!ctx || !d || !out || !d->layers || !d->output_norm) return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  if (world == 0 || world > kMaxEpRanks || rank >= world)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "expert parallel: 1..8 ranks");
  if (world > 1 && (d->n_experts == 0 || d->n_experts % world))
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "expert parallel: n_experts must divide by the ranks");
  cudaSetDevice(ctx->device);
  const uint32_t H = d->hidden, R = d->kv_lora_rank, RD = d->rope_dim, QL = d->q_lora_rank;
  const uint32_t NH = d->n_heads, NO = d->nope_dim, VD = d->v_dim, hq = NO + RD, L_ = d->n_layers;
  const uint32_t NKV = d->n_kv_heads ? d->n_kv_heads : NH;
  auto bad = [&](const char *msg) { return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, msg); };
  if (!L_ || !NH) return bad("ds2: n_layers and n_heads must be > 0");
  if (d->attn_quant != ZGPU_Q4_0)
    return zgpu_fail(ctx, ZGPU_ERR_UNSUPPORTED_QUANT, "ds2: the layers' matmuls must be Q4_0");
  if (H % 32 || H % 8) return bad("ds2: hidden must be a multiple of 32");
  if (R == 0 || R % 32 || R > kMlaMaxLatent) return bad("ds2: kv_lora_rank must be a multiple of 32, at most 512");
  if (RD % 2 || RD > kMlaMaxRope || (R + RD) % 4) return bad("ds2: rope_dim must be even, at most 64");
  if (NO == 0 || NO % 4 || NO > kMlaMaxNope) return bad("ds2: nope_dim must be a multiple of 4, at most 256");
  if (VD == 0 || VD % 8 || (NH * VD) % 32) return bad("ds2: v_dim must be a multiple of 8");
  if (QL == 0 || QL % 32) return bad("ds2: q_lora_rank must be a multiple of 32");
  if ((NH * hq) % 8 || (R + RD + QL) % 4) return bad("ds2: projection rows must fill 4-row groups");
  if (d->vocab_real > d->vocab_padded) return bad("ds2: vocab_real > vocab_padded");
  bool any_mha = false;
  for (uint32_t l = 0; l < L_; ++l) any_mha |= d->layers[l].attn_type == ZGPU_ATTN_MHA;
  if (any_mha && (NH % NKV || hq > kMhaMaxHead || VD > kMhaMaxV || (NKV * hq) % 4 || (NKV * VD) % 4))
    return bad("ds2: MHA layers need n_heads % n_kv_heads == 0, nope + rope <= 320, v_dim <= 256");
  if (d->route_mode > 1) return bad("ds2: unknown routing mode");
  bool any_moe = false, any_dense = false;
  for (uint32_t l = 0; l < L_; ++l) (d->layers[l].moe ? any_moe : any_dense) = true;
  if (any_dense && (d->ffn == 0 || d->ffn % 32)) return bad("ds2: ffn must be a multiple of 32");
  if (any_moe) {
    if (d->top_k == 0 || d->top_k > d->n_experts || d->top_k > kMoeMaxTopK)
      return bad("ds2: need 0 < top_k <= n_experts, top_k <= 16");
    if (d->expert_ffn == 0 || d->expert_ffn % 32) return bad("ds2: expert_ffn must be a multiple of 32");
    if (H > kMoeMaxDim) return bad("ds2: router input above 8192");
  }
  zgpu_ds2_model *m = new (std::nothrow) zgpu_ds2_model();
  if (!m) return ZGPU_ERR_OUT_OF_MEMORY;
  m->ctx = ctx;
  m->desc = *d;
  m->desc.layers = nullptr;
  m->desc.output_norm = nullptr;
  m->layers.resize(L_);
  auto fail = [&](zgpu_status s, const std::string &msg) {
    zgpu_ds2_destroy(m);
    return zgpu_fail(ctx, s, msg);
  };
  auto need = [&](const void *key, uint32_t quant, uint64_t rows, uint64_t cols,
                  const char *what) -> const DeviceTensor * {
    const DeviceTensor *t = zgpu_lookup(ctx, key);
    if (!t || t->quant != quant || t->rows != rows || t->cols != cols) {
      ctx->last_error = std::string("ds2_create: bad or unregistered tensor ") + what;
      return nullptr;
    }
    return t;
  };
  m->emb = need(d->token_embd, d->token_embd_quant, d->vocab_padded, H, "token_embd");
  if (!m->emb) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
  m->out = need(d->output, d->output_quant, d->vocab_padded, H, "output");
  if (!m->out) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);

  // f32 vectors: per layer attn | ffn | kv_a_norm | q_a_norm | k_norm, then the output norm
  const size_t per_layer = 2 * static_cast<size_t>(H) + R + QL + RD;
  std::vector<float> norms(per_layer * L_ + H, 1.0f);
  const uint32_t n_seg = d->n_shared + d->top_k;
  cudaError_t e = cudaSuccess;
  for (uint32_t l = 0; l < L_; ++l) {
    const zgpu_ds2_layer &ly = d->layers[l];
    Ds2Layer &L = m->layers[l];
    if (ly.attn_type > ZGPU_ATTN_MHA) return fail(ZGPU_ERR_INVALID_ARG, "ds2_create: unknown attention type");
    L.mha = ly.attn_type == ZGPU_ATTN_MHA;
    if (!ly.attn_norm || !ly.ffn_norm || (!L.mha && (!ly.kv_a_norm || !ly.q_a_norm)))
      return fail(ZGPU_ERR_INVALID_ARG, "ds2_create: missing norm weights");
    float *nb = norms.data() + per_layer * l;
    std::memcpy(nb, ly.attn_norm, H * 4);
    std::memcpy(nb + H, ly.ffn_norm, H * 4);
    L.o = need(ly.attn_output, ZGPU_Q4_0, H, static_cast<uint64_t>(NH) * VD, "attn_output");
    if (!L.o) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
    if (L.mha) {
      // standard attention (AttnType::Mha): q | k | v fused into one group stream
      const DeviceTensor *wq = need(ly.q_mha, ZGPU_Q4_0, static_cast<uint64_t>(NH) * hq, H, "q_mha");
      const DeviceTensor *wk = need(ly.k_mha, ZGPU_Q4_0, static_cast<uint64_t>(NKV) * hq, H, "k_mha");
      const DeviceTensor *wv = need(ly.v_mha, ZGPU_Q4_0, static_cast<uint64_t>(NKV) * VD, H, "v_mha");
      if (!wq || !wk || !wv) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
      m->gs_h = wq->gstride;
      const uint32_t gq = static_cast<uint32_t>(wq->groups + wk->groups + wv->groups);
      L.qkv_groups = (gq + 1) & ~1u;
      const size_t cb = static_cast<size_t>(L.qkv_groups) * m->gs_h;
      if ((e = cudaMalloc(&L.cat_qkv, cb)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "q|k|v allocation");
      cudaMemset(L.cat_qkv, 0, cb);
      cudaMemcpy(L.cat_qkv, wq->d, wq->bytes, cudaMemcpyDeviceToDevice);
      cudaMemcpy(L.cat_qkv + wq->bytes, wk->d, wk->bytes, cudaMemcpyDeviceToDevice);
      cudaMemcpy(L.cat_qkv + wq->bytes + wk->bytes, wv->d, wv->bytes, cudaMemcpyDeviceToDevice);
      L.mha_idx = m->n_mha++;
    } else {
    std::memcpy(nb + 2 * H, ly.kv_a_norm, R * 4);
    std::memcpy(nb + 2 * H + R, ly.q_a_norm, QL * 4);
    if (ly.k_norm) std::memcpy(nb + 2 * H + R + QL, ly.k_norm, RD * 4);
    const DeviceTensor *kva = need(ly.kv_a_mqa, ZGPU_Q4_0, R + RD, H, "kv_a_mqa");
    const DeviceTensor *qa = need(ly.q_a, ZGPU_Q4_0, QL, H, "q_a");
    L.q_b = need(ly.q_b, ZGPU_Q4_0, static_cast<uint64_t>(NH) * hq, QL, "q_b");
    if (!kva || !qa || !L.q_b) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
    const DeviceTensor *vb = nullptr;
    if (ly.k_b && ly.v_b) {
      L.kb = need(ly.k_b, ZGPU_Q4_0, static_cast<uint64_t>(NH) * NO, R, "k_b");
      vb = need(ly.v_b, ZGPU_Q4_0, static_cast<uint64_t>(NH) * VD, R, "v_b");
      L.kb_head_rows = NO;
    } else {
      L.kb = need(ly.kv_b, ZGPU_Q4_0, static_cast<uint64_t>(NH) * (NO + VD), R, "kv_b");
      vb = L.kb;
      L.kb_head_rows = NO + VD;
    }
    if (!L.kb || !vb) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
    m->gs_h = kva->gstride;
    // fused kv_a | q_a, padded to an even group count with a zero group
    const uint32_t ga = static_cast<uint32_t>(kva->groups + qa->groups);
    L.cat_a_groups = (ga + 1) & ~1u;
    const size_t cat_bytes = static_cast<size_t>(L.cat_a_groups) * m->gs_h;
    if ((e = cudaMalloc(&L.cat_a, cat_bytes)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "kv_a|q_a allocation");
    cudaMemset(L.cat_a, 0, cat_bytes);
    cudaMemcpy(L.cat_a, kva->d, kva->bytes, cudaMemcpyDeviceToDevice);
    cudaMemcpy(L.cat_a + kva->bytes, qa->d, qa->bytes, cudaMemcpyDeviceToDevice);
    // per-head V row streams
    std::vector<unsigned long long> vseg(NH);
    for (uint32_t h = 0; h < NH; ++h) {
      const uint64_t row = (ly.k_b && ly.v_b) ? static_cast<uint64_t>(h) * VD
                                              : static_cast<uint64_t>(h) * (NO + VD) + NO;
      vseg[h] = reinterpret_cast<unsigned long long>(vb->d + (row / 4) * vb->gstride);
    }
    L.v_gstride = vb->gstride;
    L.v_seg_bytes = static_cast<uint64_t>(VD / 4) * vb->gstride;
    if ((e = cudaMalloc(&L.d_vseg, NH * 8)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "v table");
    cudaMemcpy(L.d_vseg, vseg.data(), NH * 8, cudaMemcpyHostToDevice);
    }
    L.moe = ly.moe;
    if (!ly.moe) {
      const DeviceTensor *gt = need(ly.ffn_gate, ZGPU_Q4_0, d->ffn, H, "ffn_gate");
      const DeviceTensor *up = need(ly.ffn_up, ZGPU_Q4_0, d->ffn, H, "ffn_up");
      L.down = need(ly.ffn_down, ZGPU_Q4_0, H, d->ffn, "ffn_down");
      if (!gt || !up || !L.down) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
      if ((e = interleave_groups(&L.gateup, gt, up)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "gate/up");
      continue;
    }
    const uint64_t EF = d->expert_ffn;
    const DeviceTensor *gt = need(ly.gate_exps, ZGPU_Q4_0, d->n_experts * EF, H, "gate_exps");
    const DeviceTensor *up = need(ly.up_exps, ZGPU_Q4_0, d->n_experts * EF, H, "up_exps");
    L.down = need(ly.down_exps, ZGPU_Q4_0, static_cast<uint64_t>(d->n_experts) * H, EF, "down_exps");
    L.router = need(ly.router_w, ZGPU_F32, d->n_experts, H, "router_w");
    if (!gt || !up || !L.down || !L.router) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
    if ((e = interleave_groups(&L.gateup, gt, up)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "expert gate/up");
    m->gs_e = L.down->gstride;
    m->gu_bytes = 2 * (EF / 4) * gt->gstride;
    m->dn_bytes = (H / 4) * L.down->gstride;
    if (d->n_shared) {
      const DeviceTensor *sg = need(ly.gate_shexp, ZGPU_Q4_0, d->n_shared * EF, H, "gate_shexp");
      const DeviceTensor *su = need(ly.up_shexp, ZGPU_Q4_0, d->n_shared * EF, H, "up_shexp");
      L.sh_down = need(ly.down_shexp, ZGPU_Q4_0, static_cast<uint64_t>(d->n_shared) * H, EF, "down_shexp");
      if (!sg || !su || !L.sh_down) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
      if ((e = interleave_groups(&L.sh_gateup, sg, su)) != cudaSuccess)
        return fail(ZGPU_ERR_OUT_OF_MEMORY, "shared gate/up");
    }
    if (ly.router_b) {
      if ((e = cudaMalloc(&L.d_router_b, d->n_experts * 4)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "router bias");
      cudaMemcpy(L.d_router_b, ly.router_b, d->n_experts * 4, cudaMemcpyHostToDevice);
    }
    if (cudaMalloc(&L.d_seg_gu, n_seg * 8) != cudaSuccess || cudaMalloc(&L.d_seg_dn, n_seg * 8) != cudaSuccess)
      return fail(ZGPU_ERR_OUT_OF_MEMORY, "expert tables");
    cudaMemset(L.d_seg_gu, 0, n_seg * 8);
    cudaMemset(L.d_seg_dn, 0, n_seg * 8);
  }
  std::memcpy(norms.data() + per_layer * L_, d->output_norm, H * 4);
  if ((e = cudaMalloc(&m->d_norms, norms.size() * 4)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "norms");
  cudaMemcpy(m->d_norms, norms.data(), norms.size() * 4, cudaMemcpyHostToDevice);
  for (uint32_t l = 0; l < L_; ++l) {
    Ds2Layer &L = m->layers[l];
    float *nb = m->d_norms + per_layer * l;
    L.attn_norm = nb;
    L.ffn_norm = nb + H;
    L.kv_a_norm = nb + 2 * H;
    L.q_a_norm = nb + 2 * H + R;
    L.k_norm = d->layers[l].k_norm ? nb + 2 * H + R + QL : nullptr;
  }
  m->d_out_norm = m->d_norms + per_layer * L_;
  // mla.rs:165-171: freq_i = powf(base, -2 i / rope_dim)
  std::vector<float> inv(RD / 2 ? RD / 2 : 1, 0.f);
  for (uint32_t i = 0; i < RD / 2; ++i)
    inv[i] = powf(d->rope_theta, -2.0f * static_cast<float>(i) / static_cast<float>(RD));
  if ((e = cudaMalloc(&m->d_inv_freqs, inv.size() * 4)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "rope");
  cudaMemcpy(m->d_inv_freqs, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice);

  const size_t act = std::max<size_t>(any_dense ? d->ffn : 0, static_cast<size_t>(n_seg) * d->expert_ffn);
  const size_t topk = any_moe ? d->top_k : 1;
  if (cudaMalloc(&m->d_hidden, H * 4) || cudaMalloc(&m->d_ca, (R + RD + QL + 8) * 4) ||
      cudaMalloc(&m->d_q, static_cast<size_t>(NH) * hq * 4) || cudaMalloc(&m->d_qabs, static_cast<size_t>(NH) * R * 4) ||
      cudaMalloc(&m->d_qpe, static_cast<size_t>(NH) * (RD ? RD : 1) * 4) ||
      cudaMalloc(&m->d_ctx, static_cast<size_t>(NH) * R * 4) ||
      cudaMalloc(&m->d_concat, static_cast<size_t>(NH) * VD * 4) || cudaMalloc(&m->d_act, (act ? act : 1) * 4) ||
      cudaMalloc(&m->d_expout, static_cast<size_t>(n_seg ? n_seg : 1) * H * 4) ||
      cudaMalloc(&m->d_scores, (d->n_experts ? d->n_experts : 1) * 4) ||
      cudaMalloc(&m->d_logits, static_cast<size_t>(d->vocab_padded) * 4) ||
      cudaMalloc(&m->d_wts, L_ * topk * 4) || cudaMalloc(&m->d_ids, L_ * topk * 4) ||
      cudaMalloc(&m->d_route_counter, 4) || cudaMalloc(&m->d_argmax, 8) ||
      cudaMalloc(&m->d_state, sizeof(StepState)) || cudaMalloc(&m->d_status, kStatusWords * 4))
    return fail(ZGPU_ERR_OUT_OF_MEMORY, "activation buffers");
  const unsigned long long init = kArgmaxInitKey;
  cudaMemcpy(m->d_argmax, &init, 8, cudaMemcpyHostToDevice);
  cudaMemset(m->d_status, 0, kStatusWords * 4);
  cudaMemset(m->d_route_counter, 0, 4);
  cudaMemset(m->d_hidden, 0, H * 4);
  cudaMemset(m->d_ids, 0, L_ * topk * 4);
  cudaMemset(m->d_wts, 0, L_ * topk * 4);
  m->n_kv = NKV;
  // + 8: the GEMV writes the rows of the zero padding group as well
  if (m->n_mha && cudaMalloc(&m->d_mha_qkv, (static_cast<size_t>(NH) * hq + static_cast<size_t>(NKV) * (hq + VD) + 8) * 4))
    return fail(ZGPU_ERR_OUT_OF_MEMORY, "MHA projections");
  for (auto &ev : m->ev) cudaEventCreate(&ev);
  m->rank = rank;
  m->world = world;
  m->ep_per_rank = world > 1 ? d->n_experts / world : 0;
  if (world > 1) {
    const size_t xw = ep_exchange_words(d->top_k * kDs2MaxBatch, H);
    if (cudaMalloc(&m->d_xslots, xw * 8) || cudaMalloc(&m->d_ep_seq, 4))
      return fail(ZGPU_ERR_OUT_OF_MEMORY, "expert-parallel exchange buffers");
    cudaMemset(m->d_xslots, 0, xw * 8);
    cudaMemset(m->d_ep_seq, 0, 4);
  }
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(ZGPU_ERR_CUDA, std::string("ds2 upload: ") + cudaGetErrorString(e));
  *out = m;
  return ZGPU_OK;
}

}  // namespace

extern "C" {

zgpu_status zgpu_ds2_create(zgpu_ctx *ctx, const zgpu_ds2_desc *d, zgpu_ds2_model **out) {
  return ds2_create(ctx, d, 0, 1, out);
}

zgpu_status zgpu_ds2_create_ep(zgpu_ctx *ctx, const zgpu_ds2_desc *d, uint32_t rank, uint32_t world,
                               zgpu_ds2_model **out) {
  return ds2_create(ctx, d, rank, world, out);
}

zgpu_status zgpu_ds2_ep_export(zgpu_ds2_model *m, void *handle_out) {
  if (!m || !handle_out || m->world < 2 || !m->d_xslots) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(m->ctx->device);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, m->d_xslots);
  if (e != cudaSuccess) return zgpu_cuda_fail(m->ctx, e, "expert parallel: export the exchange buffer");
  std::memcpy(handle_out, &h, sizeof(h));
  return ZGPU_OK;
}

zgpu_status zgpu_ds2_ep_connect(zgpu_ds2_model *m, const void *handles) {
  if (!m || !handles || m->world < 2 || !m->d_xslots) return ZGPU_ERR_INVALID_ARG;
  if (m->ep_connected) return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "expert parallel: already connected");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  std::vector<unsigned long long *> dst(m->world, nullptr);
  for (uint32_t r = 0; r < m->world; ++r) {
    if (r == m->rank) {
      dst[r] = m->d_xslots;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t *>(handles) + static_cast<size_t>(r) * sizeof(h), sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "expert parallel: open a peer's exchange buffer");
    m->ipc_opened.push_back(p);
    dst[r] = static_cast<unsigned long long *>(p);
  }
  cudaError_t e = cudaMalloc(&m->d_ep_dst, m->world * sizeof(void *));
  if (e == cudaSuccess) e = cudaMemcpy(m->d_ep_dst, dst.data(), m->world * sizeof(void *), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "expert parallel: peer table");
  m->ep_connected = true;
  return ZGPU_OK;
}

zgpu_status zgpu_ds2_forward_single_token(zgpu_ds2_model *m, zgpu_mla_kv *kv, uint32_t token,
                                          uint32_t pos, float *hidden_out) {
  if (!m || !kv) return ZGPU_ERR_INVALID_ARG;
  if (m->world > 1 && !m->ep_connected)
    return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "expert parallel: zgpu_ds2_ep_connect first");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  zgpu_status s = ds2_prepare_kv(m, kv);
  if (s) return s;
  if (pos >= kv->max_tokens) return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "position beyond the cache");
  if (token >= m->desc.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "token id beyond the vocab");
  cudaError_t e = grow(&m->d_prompt, &m->prompt_cap, 1);
  if (e == cudaSuccess) e = grow(&m->d_tokens, &m->tokens_cap, 1);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  if ((s = ds2_set_state(m, 1, pos, m->desc.vocab_real, 1))) return s;
  const bool use_graph = !(ctx->flags & ZGPU_FLAG_NO_GRAPH);
  if (use_graph && (s = ds2_build_graphs(m, kv))) return s;
  e = cudaMemcpyAsync(m->d_prompt, &token, 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) {
    if (use_graph) {
      e = cudaGraphLaunch(m->fwd_graph, ctx->stream);
      ctx->launches += m->fwd_kernels;
    } else {
      e = ds2_enqueue_forward(m, kv, &ctx->launches);
    }
  }
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "forward");
  if (hidden_out) {
    e = cudaMemcpyAsync(hidden_out, m->d_hidden, m->desc.hidden * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "hidden d2h");
  }
  uint32_t st = 0;
  if ((s = zgpu_read_device_status(ctx, m->d_status, &st))) return s;
  return zgpu_map_device_status(ctx, st);
}

zgpu_status zgpu_ds2_lm_head_argmax(zgpu_ds2_model *m, uint32_t vocab_real, uint32_t *token_out,
                                    float *logits_out) {
  if (!m || !token_out) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  if (vocab_real > m->desc.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "vocab_real > padded");
  cudaError_t e = grow(&m->d_prompt, &m->prompt_cap, 1);
  if (e == cudaSuccess) e = grow(&m->d_tokens, &m->tokens_cap, 1);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  zgpu_status s = ds2_set_state(m, 1, 0, vocab_real, 1);
  if (s) return s;
  const bool use_graph = !(ctx->flags & ZGPU_FLAG_NO_GRAPH) && m->lm_graph;
  if (use_graph) {
    e = cudaGraphLaunch(m->lm_graph, ctx->stream);
    ctx->launches += m->lm_kernels;
  } else {
    e = ds2_enqueue_lm_head(m, &ctx->launches);
  }
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "lm head");
  if (logits_out) {
    e = cudaMemcpyAsync(logits_out, m->d_logits, static_cast<size_t>(m->desc.vocab_padded) * 4,
                        cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "logits d2h");
  }
  e = cudaMemcpyAsync(token_out, m->d_tokens, 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "token d2h");
  uint32_t st = 0;
  if ((s = zgpu_read_device_status(ctx, m->d_status, &st))) return s;
  return zgpu_map_device_status(ctx, st);
}

zgpu_status zgpu_ds2_expert_ids(zgpu_ds2_model *m, uint32_t *ids_out, float *weights_out) {
  if (!m) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  bool any_moe = false;
  for (const Ds2Layer &L : m->layers) any_moe |= L.moe != 0;
  const size_t n = static_cast<size_t>(m->desc.n_layers) * (any_moe ? m->desc.top_k : 1);
  cudaError_t e = cudaSuccess;
  if (ids_out) e = cudaMemcpyAsync(ids_out, m->d_ids, n * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess && weights_out)
    e = cudaMemcpyAsync(weights_out, m->d_wts, n * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "expert ids");
  return ZGPU_OK;
}

zgpu_status zgpu_ds2_generate_greedy(zgpu_ds2_model *m, zgpu_mla_kv *kv, const uint32_t *prompt,
                                     uint32_t n_prompt, uint32_t n_gen, uint32_t *tokens_out,
                                     float *logits_out) {
  if (!m || !kv || !prompt || !tokens_out || n_prompt == 0 || n_gen == 0) return ZGPU_ERR_INVALID_ARG;
  if (m->world > 1 && !m->ep_connected)
    return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "expert parallel: zgpu_ds2_ep_connect first");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  zgpu_status s = ds2_prepare_kv(m, kv);
  if (s) return s;
  const uint32_t steps = n_prompt + n_gen - 1;
  if (steps > kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "prompt + generation exceeds the cache");
  for (uint32_t i = 0; i < n_prompt; ++i)
    if (prompt[i] >= m->desc.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "prompt id beyond the vocab");
  cudaError_t e = grow(&m->d_prompt, &m->prompt_cap, n_prompt);
  if (e == cudaSuccess) e = grow(&m->d_tokens, &m->tokens_cap, n_gen);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  if ((s = ds2_set_state(m, n_prompt, 0, m->desc.vocab_real, n_gen))) return s;
  e = cudaMemcpyAsync(m->d_prompt, prompt, n_prompt * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "prompt upload");
  const bool use_graph = !(ctx->flags & ZGPU_FLAG_NO_GRAPH);
  if (use_graph && (s = ds2_build_graphs(m, kv))) return s;
  const size_t V = m->desc.vocab_padded;
  uint32_t launches = 0, prefill_launches = 0;
  auto run_step = [&](uint32_t step) -> cudaError_t {
    cudaError_t err;
    if (use_graph) {
      err = cudaGraphLaunch(m->step_graph, ctx->stream);
      launches += m->step_kernels;
    } else {
      err = ds2_enqueue_forward(m, kv, &launches);
      if (err == cudaSuccess) err = ds2_enqueue_lm_head(m, &launches);
    }
    if (err == cudaSuccess && logits_out && step + 1 >= n_prompt)
      err = cudaMemcpyAsync(logits_out + static_cast<size_t>(step + 1 - n_prompt) * V, m->d_logits, V * 4,
                            cudaMemcpyDeviceToHost, ctx->stream);
    return err;
  };
  cudaEventRecord(m->ev[0], ctx->stream);
  for (uint32_t st = 0; st < n_prompt && e == cudaSuccess; ++st) e = run_step(st);
  prefill_launches = launches;
  cudaEventRecord(m->ev[1], ctx->stream);
  for (uint32_t st = n_prompt; st < steps && e == cudaSuccess; ++st) e = run_step(st);
  cudaEventRecord(m->ev[2], ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "generate");
  e = cudaMemcpyAsync(tokens_out, m->d_tokens, n_gen * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "tokens d2h");
  uint32_t st = 0;
  if ((s = zgpu_read_device_status(ctx, m->d_status, &st))) return s;
  float pre = 0.f, dec = 0.f;
  cudaEventElapsedTime(&pre, m->ev[0], m->ev[1]);
  cudaEventElapsedTime(&dec, m->ev[1], m->ev[2]);
  m->perf.steps = n_gen - 1;
  m->perf.kernel_launches = launches;
  m->perf.decode_launches = launches - prefill_launches;
  m->perf.prefill_ms = pre;
  m->perf.decode_ms = dec;
  ctx->launches += launches;
  return zgpu_map_device_status(ctx, st);
}

zgpu_status zgpu_ds2_decode_batch(zgpu_ds2_model *m, zgpu_mla_kv *const *kvs, uint32_t n_seq,
                                  const uint32_t *tokens, const uint32_t *positions, uint32_t *tokens_out,
                                  float *logits_out) {
  if (!m || !kvs || !tokens || !positions || !tokens_out || n_seq == 0) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  if (n_seq > kDs2MaxBatch) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "ds2 batch: at most 32 sequences");
  if (m->world > 1 && !m->ep_connected)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "expert parallel: zgpu_ds2_ep_connect first");
  if (m->n_mha) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "ds2 batch: MLA layers only");
  cudaSetDevice(ctx->device);
  const zgpu_ds2_desc &d = m->desc;
  const uint32_t max_tokens = kvs[0] ? kvs[0]->max_tokens : 0;
  float *caches[kDs2MaxBatch];
  for (uint32_t b = 0; b < n_seq; ++b) {
    zgpu_mla_kv *kv = kvs[b];
    if (!kv) return ZGPU_ERR_INVALID_ARG;
    if (kv->n_layers != d.n_layers)
      return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "mla cache layer count differs from the model");
    if (kv->kv_lora != d.kv_lora_rank || kv->rope != d.rope_dim)
      return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "mla cache geometry differs from the model");
    if (kv->max_tokens != max_tokens)
      return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "ds2 batch: every cache needs the same capacity");
    for (uint32_t c = 0; c < b; ++c)
      if (kvs[c] == kv) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "ds2 batch: a cache appears twice");
    if (positions[b] >= max_tokens)
      return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "position beyond the cache");
    if (tokens[b] >= d.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "token id beyond the vocab");
    caches[b] = kv->d;
  }
  zgpu_status s = ds2_prepare_batch(m, max_tokens);
  if (s) return s;
  auto &B = m->b;
  cudaStream_t st = ctx->stream;
  cudaError_t e = cudaMemcpyAsync(B.tok, tokens, n_seq * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(B.pos, positions, n_seq * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(B.cache, caches, n_seq * sizeof(float *), cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "batch upload");
  const bool use_graph = !(ctx->flags & ZGPU_FLAG_NO_GRAPH);
  uint32_t launches = 0;
  if (use_graph && (!B.graph || B.graph_n != n_seq)) {
    if (B.graph) cudaGraphExecDestroy(B.graph);
    B.graph = nullptr;
    cudaGraph_t g = nullptr;
    e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "begin capture");
    uint32_t n = 0;
    cudaError_t e1 = ds2_enqueue_batch(m, n_seq, &n);
    e = cudaStreamEndCapture(st, &g);
    if (e1 != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return zgpu_cuda_fail(ctx, e1, "capture batch step");
    }
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "end capture");
    e = cudaGraphInstantiate(&B.graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "graph instantiate");
    B.graph_n = n_seq;
    B.graph_kernels = n;
  }
  cudaEventRecord(m->ev[0], st);
  if (use_graph) {
    e = cudaGraphLaunch(B.graph, st);
    launches = B.graph_kernels;
  } else {
    e = ds2_enqueue_batch(m, n_seq, &launches);
  }
  cudaEventRecord(m->ev[1], st);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "batch step");
  ctx->launches += launches;
  if (logits_out) {
    e = cudaMemcpyAsync(logits_out, B.logits, static_cast<size_t>(n_seq) * d.vocab_padded * 4,
                        cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "logits d2h");
  }
  e = cudaMemcpyAsync(tokens_out, B.out, n_seq * 4, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "tokens d2h");
  uint32_t stw = 0;
  if ((s = zgpu_read_device_status(ctx, m->d_status, &stw))) return s;
  // the step's device time and launches (zgpu_ds2_perf_snapshot)
  float ms = 0.f;
  cudaEventElapsedTime(&ms, m->ev[0], m->ev[1]);
  m->perf = zgpu_perf();
  m->perf.steps = 1;
  m->perf.kernel_launches = launches;
  m->perf.decode_launches = launches;
  m->perf.decode_ms = ms;
  return zgpu_map_device_status(ctx, stw);
}

zgpu_status zgpu_ds2_batch_expert_ids(zgpu_ds2_model *m, uint32_t n_seq, uint32_t *ids_out, float *weights_out) {
  if (!m || n_seq == 0 || n_seq > kDs2MaxBatch) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  if (!m->b.ids) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "ds2 batch: no batch step has run");
  cudaSetDevice(ctx->device);
  bool any_moe = false;
  for (const Ds2Layer &L : m->layers) any_moe |= L.moe != 0;
  const uint32_t k = any_moe ? m->desc.top_k : 1;
  // device rows are [layer][kDs2MaxBatch][k]: copy the first n_seq of each layer
  cudaError_t e = cudaSuccess;
  if (ids_out)
    e = cudaMemcpy2DAsync(ids_out, n_seq * k * 4, m->b.ids, kDs2MaxBatch * k * 4, n_seq * k * 4,
                          m->desc.n_layers, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess && weights_out)
    e = cudaMemcpy2DAsync(weights_out, n_seq * k * 4, m->b.wts, kDs2MaxBatch * k * 4, n_seq * k * 4,
                          m->desc.n_layers, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "batch expert ids");
  return ZGPU_OK;
}

zgpu_status zgpu_ds2_perf_snapshot(const zgpu_ds2_model *m, zgpu_perf *out) {
  if (!m || !out) return ZGPU_ERR_INVALID_ARG;
  *out = m->perf;
  return ZGPU_OK;
}

}  // extern "C"
