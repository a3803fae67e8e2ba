// model.cu — the Qwen3-shaped decode step: KV cache, device weight layout,
// per-step kernel sequence, CUDA-graph capture and the greedy loop.
//
// One decode step (forward_single_token_avx512, inference_avx512.rs:1826, then
// lm_head_argmax_avx512, :1200) is 5 kernels per layer plus 3:
//   embed (token select + row dequant)
//   per layer: [RMSNorm + fused Q|K|V GEMV] -> [QK-norm + RoPE + KV append +
//              split-K attention] -> [O GEMV + residual] -> [RMSNorm + fused
//              gate|up GEMV + SiLU*up] -> [down GEMV + residual]
//   [final RMSNorm + LM-head GEMV + argmax] -> finalize (checks, token chain)
// Every kernel is launched with programmatic dependent launch, so each one's
// weight prefetch (TMA into shared memory) starts while its predecessor
// drains; the whole step is captured once into a CUDA graph whose replays
// read the token and position from device memory.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "digit_mma.h"
#include "internal.h"
#include "layout.h"
#include "moe.h"
#include "ops.h"
#include "step.h"

using namespace zgpu;

namespace {
constexpr uint32_t kMaxDecodeBatch = 256;
}

struct zgpu_model {
  zgpu_ctx *ctx = nullptr;
  zgpu_qwen3_desc desc = {};
  uint32_t q_dim = 0, kv_dim = 0;
  // weights (group streams in the layout.h format on the device)
  std::vector<uint8_t *> qkv;       // owned: q|k|v groups concatenated
  std::vector<uint8_t *> gateup;    // owned: gate/up groups interleaved
  std::vector<const DeviceTensor *> o, down;
  uint64_t gs_h = 0;                // group stride for in_dim = hidden
  uint64_t gs_f = 0;                // group stride for in_dim = ffn (down)
  uint64_t gs_q = 0;                // group stride for in_dim = q_dim (O)
  const DeviceTensor *emb = nullptr, *out = nullptr;
  float *d_norms = nullptr;         // attn[L][H] | ffn[L][H] | qn[L][hd] | kn[L][hd] | out[H]
  float *d_inv_freqs = nullptr;
  // activations / state
  float *d_hidden = nullptr, *d_qkvo = nullptr, *d_attn = nullptr, *d_act = nullptr,
        *d_logits = nullptr;
  unsigned long long *d_argmax = nullptr;
  StepState *d_state = nullptr;
  uint32_t *d_prompt = nullptr, *d_tokens = nullptr;
  uint32_t prompt_cap = 0, tokens_cap = 0;
  float *d_part = nullptr;
  uint32_t *d_counters = nullptr;
  uint32_t max_splits = 0, part_tokens = 0;
  uint32_t *d_status = nullptr;
  // graphs (replays read token / position from d_state)
  cudaGraphExec_t step_graph = nullptr;   // embed + layers + LM head + finalize
  cudaGraphExec_t fwd_graph = nullptr;    // embed + layers
  cudaGraphExec_t lm_graph = nullptr;     // LM head + finalize
  zgpu_kv *graph_kv = nullptr;
  uint32_t step_kernels = 0, fwd_kernels = 0, lm_kernels = 0;
  zgpu_perf perf = {};
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  // persistent step kernel (step.cu): stage list and launch geometry
  std::vector<StageDesc> stages;
  StageDesc *d_stages = nullptr;
  uint32_t n_layer_stages = 0, lm_stage = 0;
  uint32_t *d_bar = nullptr;        // grid-barrier counter + abort flag
  uint32_t step_grid = 0;           // 0: the persistent path is not used
  StepParams step_geom = {};
  unsigned long long *d_tv = nullptr;   // tagged vectors: hidden | qkv | attn | act | token
  unsigned long long *tv[kStepBufs] = {};
  uint32_t ver[kStepBufs] = {};
  bool last_fwd_persistent = false; // the path the last forward used (the LM head follows it)
  // token-parallel prefill scratch (grown on demand)
  uint8_t *d_pf = nullptr;
  size_t pf_cap = 0;
  std::vector<cudaEvent_t> pf_ev;   // one pair per timed prefill launch (GEMM / attention)
  // the prefill's weight operand tiles (ops.h), built on the first prefill:
  // per layer QKV, O, gate/up, down
  std::vector<int8_t *> pf_w8;
  std::vector<float *> pf_ws8;
  // batched decode (zgpu_decode_batch): a block holding the sequence table,
  // attention partials and arrival counters, logits, tokens, per-row codes,
  // the digit images and the matvec partials
  // the tensor-core matvec's weight tiles (digit_mma.h), built on the first
  // batched decode: per layer QKV, O, gate/up, down, then the LM head
  std::vector<uint8_t *> dm_tiles;
  uint8_t *d_bd = nullptr;
  size_t bd_cap = 0;
  // tensor parallelism (world > 1): this rank's slice of every stage
  uint32_t rank = 0, world = 1;
  uint32_t q_loc = 0, kv_loc = 0;   // this rank's q / k rows (all of them on one GPU)
  uint32_t lm_rows = 0;             // LM-head (vocabulary) rows on this rank
  std::vector<DeviceTensor *> owned;   // row slices made for this rank (O, down, LM head)
  size_t tv_words = 0, arg_off = 0;    // tagged arena size; its argmax slots (words)
  size_t tv_off[kStepBufs] = {};
  bool tp_connected = false;
  std::vector<void *> ipc_opened;      // peers' arenas mapped into this process
  std::vector<void *> absent_arenas;   // stand-ins for absent peers (zgpu_qwen3_tp_connect_absent)
  unsigned long long **d_peer_tv = nullptr;
  ArgSlot **d_peer_arg = nullptr;
  unsigned long long **d_attn_dst = nullptr;
};

// Status block of a step: copy back (synchronising the stream), clear it
// when set, report a failed device bounds check.
zgpu_status zgpu_read_device_status(zgpu_ctx *ctx, uint32_t *d_status, uint32_t *st_out) {
  uint32_t sw[kStatusWords] = {0};
  cudaError_t e = cudaMemcpyAsync(sw, d_status, sizeof(sw), cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "step status");
  *st_out = sw[0];
  for (int i = 0; i < 4; ++i) ctx->last_wait[i] = (sw[0] & ZDEV_ERR_TIMEOUT) ? sw[4 + i] : 0u;
  if (sw[0]) cudaMemsetAsync(d_status, 0, sizeof(sw), ctx->stream);
  if (sw[1])
    return zgpu_fail(ctx, ZGPU_ERR_CUDA, "device bounds check " + std::to_string(sw[1]) + " failed (" +
                                             std::to_string(sw[2]) + ", " + std::to_string(sw[3]) + ")");
  return ZGPU_OK;
}

zgpu_status zgpu_map_device_status(zgpu_ctx *ctx, uint32_t st) {
  if (!st) return ZGPU_OK;
  if (st & ZDEV_ERR_TIMEOUT) {
    std::string what = "device wait timed out";
    const uint32_t *w = ctx->last_wait;
    if (w[0] == ZDEV_WAIT_EP_ABORTED)
      what += " (the expert-parallel exchange was aborted by an earlier expired wait; create the model again)";
    else if (w[0] == ZDEV_WAIT_EP_ARRIVAL || w[0] == ZDEV_WAIT_EP_SLOT)
      what += std::string(w[0] == ZDEV_WAIT_EP_ARRIVAL ? " (expert-parallel arrival word of rank "
                                                        : " (expert-parallel slot ") +
              std::to_string(w[3]) + ": waited for version " + std::to_string(w[1]) + ", read " +
              std::to_string(w[2]) + ")";
    return zgpu_fail(ctx, ZGPU_ERR_DEVICE_TIMEOUT, what);
  }
  if (st & ZDEV_ERR_BOUNDS)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "token or position outside the cache");
  if (st & ZDEV_ERR_NUMERICAL)
    return zgpu_fail(ctx, ZGPU_ERR_NUMERICAL_INSTABILITY, "softmax: non-finite max or bad sum");
  if (st & ZDEV_ERR_LM_NONFINITE)
    return zgpu_fail(ctx, ZGPU_ERR_LM_NON_FINITE_LOGITS, "lm head: non-finite max logit");
  if (st & ZDEV_ERR_LM_PADDING)
    return zgpu_fail(ctx, ZGPU_ERR_LM_ARGMAX_IN_PADDING, "lm head: argmax in padding region");
  return zgpu_fail(ctx, ZGPU_ERR_CUDA, "device status " + std::to_string(st));
}

namespace {

float *norm_attn(zgpu_model *m, uint32_t l) { return m->d_norms + static_cast<size_t>(l) * m->desc.hidden; }
float *norm_ffn(zgpu_model *m, uint32_t l) {
  return m->d_norms + static_cast<size_t>(m->desc.n_layers + l) * m->desc.hidden;
}
float *norm_q(zgpu_model *m, uint32_t l) {
  return m->d_norms + static_cast<size_t>(2 * m->desc.n_layers) * m->desc.hidden +
         static_cast<size_t>(l) * m->desc.head_dim;
}
float *norm_k(zgpu_model *m, uint32_t l) {
  return norm_q(m, 0) + static_cast<size_t>(m->desc.n_layers + l) * m->desc.head_dim;
}
float *norm_out(zgpu_model *m) {
  return norm_q(m, 0) + static_cast<size_t>(2 * m->desc.n_layers) * m->desc.head_dim;
}

LaunchCfg launch_cfg(zgpu_model *m, uint32_t *counter) {
  LaunchCfg lc;
  lc.stream = m->ctx->stream;
  lc.pdl = !(m->ctx->flags & ZGPU_FLAG_NO_PDL);
  lc.sm_count = m->ctx->sm_count;
  lc.launch_counter = counter;
  return lc;
}

// Enqueue the forward part of one step (embed + all layers).
cudaError_t enqueue_forward(zgpu_model *m, zgpu_kv *kv, uint32_t *counter) {
  const zgpu_qwen3_desc &d = m->desc;
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

  const uint32_t qkv_rows = m->q_dim + 2 * m->kv_dim;
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    GemvDesc g;
    GemvIo io;
    // RMSNorm + fused Q|K|V projection
    g.w = m->qkv[l];
    g.wbytes = static_cast<uint64_t>(qkv_rows / 4) * m->gs_h;
    g.gstride = m->gs_h;
    g.quant = ZGPU_Q4_0;
    g.rows = qkv_rows;
    g.groups = qkv_rows / 4;
    g.in_dim = d.hidden;
    io = GemvIo();
    io.x = m->d_hidden;
    io.norm_w = norm_attn(m, l);
    io.eps = d.rms_eps;
    io.out = m->d_qkvo;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_RMSNORM, EPI_STORE, io, lc)) != cudaSuccess) return e;

    AttnParams ap = {};
    ap.qkv = m->d_qkvo;
    ap.q_norm = norm_q(m, l);
    ap.k_norm = norm_k(m, l);
    ap.inv_freqs = m->d_inv_freqs;
    ap.kv_layer = kv->d + static_cast<size_t>(l) * 2 * kv->block;
    ap.kv_block = kv->block;
    ap.max_tokens = kv->max_tokens;
    ap.pos_ptr = &m->d_state->pos;
    ap.out = m->d_attn;
    ap.part = m->d_part;
    ap.counters = m->d_counters;
    ap.status = m->d_status;
    ap.n_q = d.n_q_heads;
    ap.n_kv = d.n_kv_heads;
    ap.max_splits = m->max_splits;
    ap.eps = d.rms_eps;
    ap.scale = 1.0f / sqrtf(static_cast<float>(d.head_dim));
    if ((e = launch_attention(ap, lc)) != cudaSuccess) return e;

    // O projection + residual
    g.w = m->o[l]->d;
    g.wbytes = m->o[l]->bytes;
    g.gstride = m->gs_q;
    g.rows = d.hidden;
    g.groups = d.hidden / 4;
    g.in_dim = m->q_dim;
    io = GemvIo();
    io.x = m->d_attn;
    io.out = m->d_hidden;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_PLAIN, EPI_RESADD, io, lc)) != cudaSuccess) return e;

    // RMSNorm + fused gate|up + SiLU(gate)*up
    g.w = m->gateup[l];
    g.wbytes = static_cast<uint64_t>(2 * d.ffn / 4) * m->gs_h;
    g.gstride = m->gs_h;
    g.rows = d.ffn;
    g.groups = 2 * d.ffn / 4;
    g.in_dim = d.hidden;
    io = GemvIo();
    io.x = m->d_hidden;
    io.norm_w = norm_ffn(m, l);
    io.eps = d.rms_eps;
    io.out = m->d_act;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_RMSNORM, EPI_SWIGLU, io, lc)) != cudaSuccess) return e;

    // down projection + residual
    g.w = m->down[l]->d;
    g.wbytes = m->down[l]->bytes;
    g.gstride = m->gs_f;
    g.rows = d.hidden;
    g.groups = d.hidden / 4;
    g.in_dim = d.ffn;
    io = GemvIo();
    io.x = m->d_act;
    io.out = m->d_hidden;
    io.status = m->d_status;
    if ((e = launch_gemv(g, PRO_PLAIN, EPI_RESADD, io, lc)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t enqueue_lm_head(zgpu_model *m, uint32_t *counter) {
  const zgpu_qwen3_desc &d = m->desc;
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
  io.norm_w = norm_out(m);
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

enum GraphPart { GRAPH_STEP = 0, GRAPH_FWD = 1, GRAPH_LM = 2 };

zgpu_status capture(zgpu_model *m, zgpu_kv *kv, GraphPart part, cudaGraphExec_t *out,
                    uint32_t *kernels) {
  zgpu_ctx *ctx = m->ctx;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "begin capture");
  uint32_t n = 0;
  cudaError_t e1 = cudaSuccess;
  if (part != GRAPH_LM) e1 = enqueue_forward(m, kv, &n);
  if (e1 == cudaSuccess && part != GRAPH_FWD) e1 = enqueue_lm_head(m, &n);
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

void drop_graphs(zgpu_model *m) {
  for (cudaGraphExec_t *g : {&m->step_graph, &m->fwd_graph, &m->lm_graph}) {
    if (*g) cudaGraphExecDestroy(*g);
    *g = nullptr;
  }
  m->graph_kv = nullptr;
}

// Capture the three step graphs for this cache (once per cache).
zgpu_status build_graphs(zgpu_model *m, zgpu_kv *kv) {
  if (m->step_graph && m->graph_kv == kv) return ZGPU_OK;
  drop_graphs(m);
  zgpu_status s = capture(m, kv, GRAPH_STEP, &m->step_graph, &m->step_kernels);
  if (!s) s = capture(m, kv, GRAPH_FWD, &m->fwd_graph, &m->fwd_kernels);
  if (!s) s = capture(m, nullptr, GRAPH_LM, &m->lm_graph, &m->lm_kernels);
  if (s) {
    drop_graphs(m);
    return s;
  }
  m->graph_kv = kv;
  return ZGPU_OK;
}

zgpu_status read_status(zgpu_model *m, uint32_t *st_out) {
  return zgpu_read_device_status(m->ctx, m->d_status, st_out);
}

zgpu_status map_status(zgpu_ctx *ctx, uint32_t st) { return zgpu_map_device_status(ctx, st); }

zgpu_status set_state(zgpu_model *m, uint32_t n_prompt, uint32_t pos_base, uint32_t vocab_real,
                      uint32_t n_gen_cap) {
  StepState s = {};
  s.step = 0;
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

// Stage list of one decode step for the persistent kernel (step.cu).  The
// model keeps the multi-kernel path when the device or the geometry does not
// suit the persistent kernel, or when the context asks for it.
zgpu_status build_step(zgpu_model *m) {
  zgpu_ctx *ctx = m->ctx;
  m->step_grid = 0;
  if (ctx->flags & ZGPU_FLAG_NO_PERSISTENT) return ZGPU_OK;
  const uint32_t grid = step_max_grid(ctx->sm_count);
  if (!grid) return ZGPU_OK;
  const zgpu_qwen3_desc &d = m->desc;
  const uint32_t H = d.hidden, F = d.ffn, L = d.n_layers;
  const uint32_t N = m->world, r = m->rank;
  const uint32_t qkv_rows = m->q_loc + 2 * m->kv_loc;   // this rank's heads only: attention is local
  const uint32_t H_loc = H / N, F_loc = F / N;
  auto gemv = [&](uint32_t quant, uint32_t pro, uint32_t epi, uint32_t rows, uint32_t units,
                  uint32_t in_dim, const uint8_t *w, uint64_t gstride, uint64_t wbytes, uint32_t in_buf,
                  const float *norm_w, uint32_t out_buf) {
    StageDesc s = {};
    s.kind = STG_GEMV;
    s.quant = quant;
    s.pro = pro;
    s.epi = epi;
    s.rows = rows;
    s.units = units;
    s.gpu = quant == ZGPU_Q4_0 ? 2 : 1;
    s.bpr = in_dim / 32;
    s.ks = (s.bpr + kChunkBlocks - 1) / kChunkBlocks;
    s.in_dim = in_dim;
    s.gbytes = static_cast<uint32_t>(chunk_bytes(quant, s.bpr < kChunkBlocks ? s.bpr : kChunkBlocks));
    s.w = w;
    s.gstride = gstride;
    s.wbytes = wbytes;
    s.in_buf = in_buf;
    s.out_buf = out_buf;
    s.norm_w = norm_w;
    return s;
  };
  // gate/up units (a gate group and its up group each) as the model stores
  // them: padded to an even count on one GPU, F / 4 / N on a rank
  const uint64_t gu_groups = N == 1 ? (((F + 3) / 4 + 1) & ~uint64_t(1)) : F_loc / 4;
  // tensor parallel: the O, gate/up, down and LM-head stages own a row slice
  // and store it into every rank's copy of the vector
  auto slice = [&](StageDesc s, uint32_t row0) {
    s.out_row0 = row0;
    s.bcast = N > 1 ? 1u : 0u;
    return s;
  };
  std::vector<StageDesc> st;
  for (uint32_t l = 0; l < L; ++l) {
    StageDesc q = gemv(ZGPU_Q4_0, PRO_RMSNORM, EPI_STORE, qkv_rows, qkv_rows / 8, H, m->qkv[l], m->gs_h,
                       static_cast<uint64_t>(qkv_rows / 4) * m->gs_h, BUF_HIDDEN, norm_attn(m, l), BUF_QKV);
    if (l == 0) q.flags = kStageEmbed;
    st.push_back(q);
    StageDesc a = {};
    a.kind = STG_ATTN;
    a.layer = l;
    a.q_norm = norm_q(m, l);
    a.k_norm = norm_k(m, l);
    st.push_back(a);
    const DeviceTensor *o = m->o[l], *dn = m->down[l];
    st.push_back(slice(gemv(ZGPU_Q4_0, PRO_PLAIN, EPI_RESADD, H_loc, static_cast<uint32_t>(o->groups / 2),
                            m->q_dim, o->d, o->gstride, o->bytes, BUF_ATTN, nullptr, BUF_HIDDEN),
                       r * H_loc));
    st.push_back(slice(gemv(ZGPU_Q4_0, PRO_RMSNORM, EPI_SWIGLU, F_loc, static_cast<uint32_t>(gu_groups), H,
                            m->gateup[l], m->gs_h, 2 * gu_groups * m->gs_h, BUF_HIDDEN, norm_ffn(m, l), BUF_ACT),
                       r * F_loc));
    st.push_back(slice(gemv(ZGPU_Q4_0, PRO_PLAIN, EPI_RESADD, H_loc, static_cast<uint32_t>(dn->groups / 2), F,
                            dn->d, dn->gstride, dn->bytes, BUF_ACT, nullptr, BUF_HIDDEN),
                       r * H_loc));
  }
  const DeviceTensor *ot = m->out;
  const uint32_t gpu = ot->quant == ZGPU_Q4_0 ? 2 : 1;
  const uint32_t lm = static_cast<uint32_t>(st.size());
  st.push_back(slice(gemv(ot->quant, PRO_RMSNORM, EPI_ARGMAX, m->lm_rows, static_cast<uint32_t>(ot->groups / gpu),
                          H, ot->d, ot->gstride, ot->bytes, BUF_HIDDEN, norm_out(m), BUF_NONE),
                     r * m->lm_rows));
  st.back().bcast = 0;   // the argmax keys meet in the LM head's own exchange
  st.back().out = m->d_logits;
  StepParams g = {};
  if (!step_geometry(st.data(), static_cast<uint32_t>(st.size()), grid, &g)) return ZGPU_OK;
  g.hid_row0 = r * H_loc;
  g.rank = r;
  g.world = N;
  cudaError_t e = cudaMalloc(&m->d_stages, st.size() * sizeof(StageDesc));
  if (e == cudaSuccess)
    e = cudaMemcpy(m->d_stages, st.data(), st.size() * sizeof(StageDesc), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&m->d_bar, 2 * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(m->d_bar, 0, 2 * sizeof(uint32_t));
  // tagged vectors (version 0 everywhere: nothing written yet), then the
  // argmax slots of the tensor-parallel LM head; every rank lays its arena
  // out the same way
  const size_t tv_len[kStepBufs] = {H, qkv_rows, m->q_dim, F, 2};
  size_t tv_total = 0;
  for (int b = 0; b < kStepBufs; ++b) {
    m->tv_off[b] = tv_total;
    tv_total += tv_len[b];
  }
  m->arg_off = tv_total;
  tv_total += 2 * kMaxRanks;
  m->tv_words = tv_total;
  if (e == cudaSuccess) e = cudaMalloc(&m->d_tv, tv_total * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(m->d_tv, 0, tv_total * sizeof(unsigned long long));
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "step kernel set-up");
  for (int b = 0; b < kStepBufs; ++b) {
    m->tv[b] = m->d_tv + m->tv_off[b];
    m->ver[b] = 0;
  }
  for (StageDesc &sd : st) {
    if (sd.kind != STG_GEMV) continue;
    sd.tin = (sd.flags & kStageEmbed) ? nullptr : m->tv[sd.in_buf];
    sd.tout = sd.out_buf < kStepBufs ? m->tv[sd.out_buf] : nullptr;
  }
  if (e == cudaSuccess)
    e = cudaMemcpy(m->d_stages, st.data(), st.size() * sizeof(StageDesc), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "step kernel set-up");
  m->stages = st;
  m->n_layer_stages = 5 * L;
  m->lm_stage = lm;
  m->step_geom = g;
  m->step_grid = grid;
  return ZGPU_OK;
}

bool step_usable(const zgpu_model *m, const zgpu_kv *kv) {
  if (!m->step_grid) return false;
  return !kv || static_cast<uint64_t>(m->desc.n_kv_heads / m->world) * m->max_splits <= m->step_grid;
}

// One persistent launch: `n_steps` steps from global step `step0`.
cudaError_t run_step(zgpu_model *m, zgpu_kv *kv, StepMode mode, uint32_t step0, uint32_t n_steps,
                     uint32_t token, uint32_t pos, uint32_t n_prompt) {
  const zgpu_qwen3_desc &d = m->desc;
  StepParams p = m->step_geom;
  p.stages = m->d_stages;
  p.n_layer_stages = m->n_layer_stages;
  p.lm_stage = m->lm_stage;
  p.mode = mode;
  p.step0 = step0;
  p.n_steps = n_steps;
  p.fwd_token = token;
  p.fwd_pos = pos;
  p.n_q = d.n_q_heads / m->world;
  p.n_kv = d.n_kv_heads / m->world;
  p.peer_tv = m->d_peer_tv;
  p.peer_arg = m->d_peer_arg;
  p.attn_dst = m->d_attn_dst;
  p.max_splits = m->max_splits;
  p.max_tokens = kv ? kv->max_tokens : 0;
  p.eps = d.rms_eps;
  p.scale = 1.0f / sqrtf(static_cast<float>(d.head_dim));
  p.emb = m->emb->d;
  p.emb_gstride = m->emb->gstride;
  p.emb_quant = m->emb->quant;
  p.emb_rows = static_cast<uint32_t>(m->emb->rows);
  p.hidden = d.hidden;
  for (int b = 0; b < kStepBufs; ++b) {
    p.tv[b] = m->tv[b];
    p.ver[b] = m->ver[b];
  }
  p.inv_freqs = m->d_inv_freqs;
  p.kv_base = kv ? kv->d : nullptr;
  p.kv_block = kv ? kv->block : 0;
  p.attn_part = m->d_part;
  p.attn_counters = m->d_counters;
  p.argmax = m->d_argmax;
  p.state = m->d_state;
  p.prompt = m->d_prompt;
  p.tokens_out = m->d_tokens;
  p.status = m->d_status;
  p.bar = m->d_bar;
  cudaError_t e = cudaMemsetAsync(m->d_bar, 0, 2 * sizeof(uint32_t), m->ctx->stream);
  if (e != cudaSuccess) return e;
  e = step_launch(p, m->step_grid, m->ctx->stream);
  if (e != cudaSuccess) return e;
  // the versions the launch leaves behind (the kernel walks the same steps)
  for (uint32_t i = 0; i < n_steps; ++i) {
    const uint32_t gstep = step0 + i;
    const bool fwd = mode != STEP_LM;
    const bool lm = mode == STEP_LM || (mode == STEP_GENERATE && gstep + 1 >= n_prompt);
    step_advance_versions(m->ver, d.n_layers, fwd, lm);
  }
  if (mode != STEP_LM) m->last_fwd_persistent = true;
  return cudaSuccess;
}

// After a device-side timeout the tagged vectors may hold any version: start
// them over.
void reset_step_tags(zgpu_model *m) {
  if (!m->d_tv) return;
  cudaMemsetAsync(m->d_tv, 0, m->tv_words * sizeof(unsigned long long), m->ctx->stream);
  cudaMemsetAsync(m->d_counters, 0, m->desc.n_kv_heads * sizeof(uint32_t), m->ctx->stream);
  for (int b = 0; b < kStepBufs; ++b) m->ver[b] = 0;
}

}  // namespace

extern "C" {

zgpu_status zgpu_kv_create(zgpu_ctx *ctx, uint32_t max_tokens, uint32_t n_layers,
                           uint32_t n_kv_heads, uint32_t head_dim, zgpu_kv **out) {
  if (!ctx || !out || !max_tokens || !n_layers || !n_kv_heads || !head_dim)
    return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  zgpu_kv *kv = new (std::nothrow) zgpu_kv();
  if (!kv) return ZGPU_ERR_OUT_OF_MEMORY;
  kv->ctx = ctx;
  kv->max_tokens = max_tokens;
  kv->n_layers = n_layers;
  kv->n_kv = n_kv_heads;
  kv->head_dim = head_dim;
  kv->block = static_cast<uint64_t>(max_tokens) * n_kv_heads * head_dim;
  const size_t bytes = 2ull * n_layers * kv->block * sizeof(float);
  cudaError_t e = cudaMalloc(&kv->d, bytes);
  if (e == cudaSuccess) e = cudaMemset(kv->d, 0, bytes);
  if (e != cudaSuccess) {
    delete kv;
    return zgpu_cuda_fail(ctx, e, "kv cache allocation");
  }
  *out = kv;
  return ZGPU_OK;
}

void zgpu_kv_destroy(zgpu_kv *kv) {
  if (!kv) return;
  cudaSetDevice(kv->ctx->device);
  cudaFree(kv->d);
  delete kv;
}

zgpu_status zgpu_kv_store(zgpu_kv *kv, uint32_t layer, uint32_t token, const float *k,
                          const float *v, uint64_t len) {
  if (!kv || !k || !v) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = kv->ctx;
  if (layer >= kv->n_layers) return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "layer out of range");
  if (token >= kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "token index out of range");
  const uint64_t stride = static_cast<uint64_t>(kv->n_kv) * kv->head_dim;
  if (len != stride) return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "invalid slice length");
  cudaSetDevice(ctx->device);
  float *kd = kv->d + static_cast<size_t>(layer) * 2 * kv->block + token * stride;
  cudaError_t e = cudaMemcpy(kd, k, stride * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(kd + kv->block, v, stride * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "kv store");
  return ZGPU_OK;
}

zgpu_status zgpu_kv_read(zgpu_kv *kv, uint32_t layer, uint32_t token_count, float *k_out,
                         float *v_out) {
  if (!kv) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = kv->ctx;
  if (layer >= kv->n_layers) return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "layer out of range");
  if (token_count > kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_COUNT_EXCEEDS_MAX, "token count exceeds max");
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  const uint64_t n = static_cast<uint64_t>(token_count) * kv->n_kv * kv->head_dim;
  const float *kd = kv->d + static_cast<size_t>(layer) * 2 * kv->block;
  cudaError_t e = cudaSuccess;
  if (k_out) e = cudaMemcpy(k_out, kd, n * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && v_out) e = cudaMemcpy(v_out, kd + kv->block, n * 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "kv read");
  return ZGPU_OK;
}

void zgpu_qwen3_destroy(zgpu_model *m) {
  if (m) cudaFree(m->d_pf);
  if (!m) return;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  drop_graphs(m);
  for (auto p : m->qkv) cudaFree(p);
  for (auto p : m->gateup) cudaFree(p);
  cudaFree(m->d_norms);
  cudaFree(m->d_inv_freqs);
  cudaFree(m->d_hidden);
  cudaFree(m->d_qkvo);
  cudaFree(m->d_attn);
  cudaFree(m->d_act);
  cudaFree(m->d_logits);
  cudaFree(m->d_argmax);
  cudaFree(m->d_state);
  cudaFree(m->d_prompt);
  cudaFree(m->d_tokens);
  cudaFree(m->d_part);
  cudaFree(m->d_counters);
  cudaFree(m->d_status);
  cudaFree(m->d_stages);
  cudaFree(m->d_bar);
  cudaFree(m->d_tv);
  for (auto &e : m->ev)
    if (e) cudaEventDestroy(e);
  for (auto &e : m->pf_ev) cudaEventDestroy(e);
  for (int8_t *p : m->pf_w8) cudaFree(p);
  for (uint8_t *p : m->dm_tiles) cudaFree(p);
  cudaFree(m->d_bd);
  for (DeviceTensor *t : m->owned) {
    cudaFree(t->d);
    delete t;
  }
  for (void *p : m->ipc_opened) cudaIpcCloseMemHandle(p);
  for (void *p : m->absent_arenas) cudaFree(p);
  cudaFree(m->d_peer_tv);
  cudaFree(m->d_peer_arg);
  cudaFree(m->d_attn_dst);
  delete m;
}

}  // extern "C"

namespace {

// A model, or (world > 1) rank `rank` of a tensor-parallel model: the rank
// keeps q/k/v rows of its kv heads, gate/up units, and O / down / LM-head
// row slices; the embedding and the norms are whole on every rank.
zgpu_status create_model(zgpu_ctx *ctx, const zgpu_qwen3_desc *d, uint32_t rank, uint32_t world, zgpu_model **out) {
  if (!ctx || !d || !out || !d->layers) return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  cudaSetDevice(ctx->device);
  if (d->head_dim != 128)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "decode attention kernel requires head_dim 128");
  if (!d->n_kv_heads || d->n_q_heads % d->n_kv_heads || d->n_q_heads / d->n_kv_heads > 4)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "unsupported GQA geometry");
  if (d->hidden % 32 || d->ffn % 32 || d->hidden % 4 || d->ffn % 4)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "hidden/ffn must be multiples of 32");
  if (d->vocab_real > d->vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "vocab_real > vocab_padded");
  if (world == 0 || world > kMaxRanks || rank >= world)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: 1..8 ranks");
  const uint32_t lm_unit = d->output_quant == ZGPU_Q4_0 ? 8u : 4u;
  if (world > 1 && (d->n_kv_heads % world || d->hidden % (8 * world) || d->ffn % (8 * world) ||
                    d->vocab_padded % (lm_unit * world)))
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG,
                     "tensor parallel: kv heads, hidden / 8, ffn / 8 and the LM-head units must divide by the ranks");
  zgpu_model *m = new (std::nothrow) zgpu_model();
  if (!m) return ZGPU_ERR_OUT_OF_MEMORY;
  m->ctx = ctx;
  m->desc = *d;
  m->desc.layers = nullptr;
  m->desc.output_norm = nullptr;
  m->q_dim = d->n_q_heads * d->head_dim;
  m->kv_dim = d->n_kv_heads * d->head_dim;
  m->rank = rank;
  m->world = world;
  m->q_loc = m->q_dim / world;
  m->kv_loc = m->kv_dim / world;
  m->lm_rows = d->vocab_padded / world;
  const uint32_t H = d->hidden, F = d->ffn, L = d->n_layers, hd = d->head_dim;
  auto fail = [&](zgpu_status s, const std::string &msg) {
    zgpu_qwen3_destroy(m);
    return zgpu_fail(ctx, s, msg);
  };
  // rows [row0, row0 + rows) of a registered tensor as a tensor of this rank
  // (group streams: whole groups of 4 rows)
  auto row_slice = [&](const DeviceTensor *t, uint64_t row0, uint64_t rows) -> const DeviceTensor * {
    if (world == 1) return t;
    DeviceTensor *sl = new (std::nothrow) DeviceTensor(*t);
    if (!sl) return nullptr;
    sl->rows = rows;
    sl->groups = rows / 4;
    sl->bytes = sl->groups * t->gstride;
    sl->d = nullptr;
    if (cudaMalloc(&sl->d, sl->bytes) != cudaSuccess) {
      delete sl;
      return nullptr;
    }
    m->owned.push_back(sl);
    cudaMemcpy(sl->d, t->d + (row0 / 4) * t->gstride, sl->bytes, cudaMemcpyDeviceToDevice);
    return sl;
  };
  auto need = [&](const void *key, uint32_t quant, uint64_t rows, uint64_t cols,
                  const char *what) -> const DeviceTensor * {
    const DeviceTensor *t = zgpu_lookup(ctx, key);
    if (!t || t->quant != quant || t->rows != rows || t->cols != cols) {
      ctx->last_error = std::string("qwen3_create: bad or unregistered tensor ") + what;
      return nullptr;
    }
    return t;
  };
  m->emb = need(d->token_embd, d->token_embd_quant, d->vocab_padded, H, "token_embd");
  if (!m->emb) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
  m->out = need(d->output, d->output_quant, d->vocab_padded, H, "output");
  if (!m->out) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
  m->out = row_slice(m->out, static_cast<uint64_t>(rank) * m->lm_rows, m->lm_rows);
  if (!m->out) return fail(ZGPU_ERR_OUT_OF_MEMORY, "LM-head slice");

  cudaError_t e = cudaSuccess;
  for (uint32_t l = 0; l < L; ++l) {
    const zgpu_qwen3_layer &ly = d->layers[l];
    const DeviceTensor *q = need(ly.attn_q, ZGPU_Q4_0, m->q_dim, H, "attn_q");
    const DeviceTensor *k = need(ly.attn_k, ZGPU_Q4_0, m->kv_dim, H, "attn_k");
    const DeviceTensor *v = need(ly.attn_v, ZGPU_Q4_0, m->kv_dim, H, "attn_v");
    const DeviceTensor *o = need(ly.attn_o, ZGPU_Q4_0, H, m->q_dim, "attn_o");
    const DeviceTensor *gt = need(ly.ffn_gate, ZGPU_Q4_0, F, H, "ffn_gate");
    const DeviceTensor *up = need(ly.ffn_up, ZGPU_Q4_0, F, H, "ffn_up");
    const DeviceTensor *dn = need(ly.ffn_down, ZGPU_Q4_0, H, F, "ffn_down");
    if (!q || !k || !v || !o || !gt || !up || !dn) return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, ctx->last_error);
    // the fused Q|K|V stream concatenates whole units of two groups
    if (q->groups * 4 != q->rows || k->groups * 4 != k->rows || v->groups * 4 != v->rows)
      return fail(ZGPU_ERR_INVALID_ARG, "q/k/v rows must be multiples of 8");
    m->gs_h = q->gstride;
    m->gs_q = o->gstride;
    m->gs_f = dn->gstride;
    // fused Q|K|V of this rank's heads: q rows of its q heads, then the k and
    // v rows of its kv heads (everything on one GPU)
    const uint64_t qb = static_cast<uint64_t>(m->q_loc / 4) * q->gstride;
    const uint64_t kb = static_cast<uint64_t>(m->kv_loc / 4) * k->gstride;
    uint8_t *cat = nullptr;
    e = cudaMalloc(&cat, qb + 2 * kb);
    if (e != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "qkv allocation");
    m->qkv.push_back(cat);
    cudaMemcpy(cat, q->d + rank * qb, qb, cudaMemcpyDeviceToDevice);
    cudaMemcpy(cat + qb, k->d + rank * kb, kb, cudaMemcpyDeviceToDevice);
    cudaMemcpy(cat + qb + kb, v->d + rank * kb, kb, cudaMemcpyDeviceToDevice);
    // gate/up units of this rank, interleaved (gate group u, up group u)
    const uint64_t gu_n = world == 1 ? gt->groups : F / 4 / world, gu_0 = world == 1 ? 0 : rank * gu_n;
    uint8_t *gu = nullptr;
    e = cudaMalloc(&gu, world == 1 ? gt->bytes + up->bytes : 2 * gu_n * gt->gstride);
    if (e != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "gate/up allocation");
    m->gateup.push_back(gu);
    cudaMemcpy2D(gu, 2 * gt->gstride, gt->d + gu_0 * gt->gstride, gt->gstride, gt->gstride, gu_n,
                 cudaMemcpyDeviceToDevice);
    cudaMemcpy2D(gu + gt->gstride, 2 * gt->gstride, up->d + gu_0 * up->gstride, up->gstride, up->gstride, gu_n,
                 cudaMemcpyDeviceToDevice);
    const DeviceTensor *os = row_slice(o, static_cast<uint64_t>(rank) * (H / world), H / world);
    const DeviceTensor *ds = row_slice(dn, static_cast<uint64_t>(rank) * (H / world), H / world);
    if (!os || !ds) return fail(ZGPU_ERR_OUT_OF_MEMORY, "O / down slices");
    m->o.push_back(os);
    m->down.push_back(ds);
  }
  // norms
  const size_t nn = static_cast<size_t>(2) * L * H + static_cast<size_t>(2) * L * hd + H;
  std::vector<float> norms(nn);
  for (uint32_t l = 0; l < L; ++l) {
    std::memcpy(&norms[static_cast<size_t>(l) * H], d->layers[l].attn_norm, H * 4);
    std::memcpy(&norms[static_cast<size_t>(L + l) * H], d->layers[l].ffn_norm, H * 4);
    std::memcpy(&norms[static_cast<size_t>(2) * L * H + static_cast<size_t>(l) * hd], d->layers[l].q_norm, hd * 4);
    std::memcpy(&norms[static_cast<size_t>(2) * L * H + static_cast<size_t>(L + l) * hd], d->layers[l].k_norm,
                hd * 4);
  }
  std::memcpy(&norms[static_cast<size_t>(2) * L * H + static_cast<size_t>(2) * L * hd], d->output_norm, H * 4);
  if ((e = cudaMalloc(&m->d_norms, nn * 4)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "norms");
  cudaMemcpy(m->d_norms, norms.data(), nn * 4, cudaMemcpyHostToDevice);
  // RopeContext::new (ops.rs:79-93)
  std::vector<float> inv(hd / 2);
  for (uint32_t i = 0; i < hd / 2; ++i)
    inv[i] = powf(d->rope_theta, -2.0f * static_cast<float>(i) / static_cast<float>(hd));
  if ((e = cudaMalloc(&m->d_inv_freqs, inv.size() * 4)) != cudaSuccess) return fail(ZGPU_ERR_OUT_OF_MEMORY, "rope");
  cudaMemcpy(m->d_inv_freqs, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice);

  const uint32_t qkv_rows = m->q_dim + 2 * m->kv_dim;
  if (cudaMalloc(&m->d_hidden, H * 4) || cudaMalloc(&m->d_qkvo, qkv_rows * 4) ||
      cudaMalloc(&m->d_attn, m->q_dim * 4) || cudaMalloc(&m->d_act, F * 4) ||
      cudaMalloc(&m->d_logits, static_cast<size_t>(d->vocab_padded) * 4) ||
      cudaMalloc(&m->d_argmax, 8) || cudaMalloc(&m->d_state, sizeof(StepState)) ||
      cudaMalloc(&m->d_status, kStatusWords * 4) || cudaMalloc(&m->d_counters, d->n_kv_heads * 4))
    return fail(ZGPU_ERR_OUT_OF_MEMORY, "activation buffers");
  const unsigned long long init = kArgmaxInitKey;
  cudaMemcpy(m->d_argmax, &init, 8, cudaMemcpyHostToDevice);
  cudaMemset(m->d_status, 0, kStatusWords * 4);
  cudaMemset(m->d_counters, 0, d->n_kv_heads * 4);
  cudaMemset(m->d_hidden, 0, H * 4);
  for (auto &ev : m->ev) cudaEventCreate(&ev);
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(ZGPU_ERR_CUDA, "model upload");
  zgpu_status bs = build_step(m);
  if (bs) {
    zgpu_qwen3_destroy(m);
    return bs;
  }
  if (world > 1 && !m->step_grid)
    return fail(ZGPU_ERR_INVALID_ARG, "tensor parallel: the persistent step kernel does not fit this model");
  *out = m;
  return ZGPU_OK;
}

}  // namespace

extern "C" {

zgpu_status zgpu_qwen3_create(zgpu_ctx *ctx, const zgpu_qwen3_desc *d, zgpu_model **out) {
  return create_model(ctx, d, 0, 1, out);
}

zgpu_status zgpu_qwen3_create_tp(zgpu_ctx *ctx, const zgpu_qwen3_desc *d, uint32_t rank, uint32_t world,
                                 zgpu_model **out) {
  return create_model(ctx, d, rank, world, out);
}

zgpu_status zgpu_qwen3_tp_export(zgpu_model *m, void *handle_out) {
  if (!m || !handle_out || m->world < 2 || !m->d_tv) return ZGPU_ERR_INVALID_ARG;
  cudaSetDevice(m->ctx->device);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, m->d_tv);
  if (e != cudaSuccess) return zgpu_cuda_fail(m->ctx, e, "tensor parallel: export the tagged vectors");
  std::memcpy(handle_out, &h, sizeof(h));
  return ZGPU_OK;
}

}  // extern "C"

namespace {

// The device tables of every rank's arena (base[d]: rank d's tagged vectors
// as this rank addresses them).
zgpu_status tp_tables(zgpu_model *m, const std::vector<unsigned long long *> &base) {
  zgpu_ctx *ctx = m->ctx;
  const uint32_t N = m->world;
  std::vector<unsigned long long *> tv(static_cast<size_t>(N) * kStepBufs), dst(N);
  std::vector<ArgSlot *> arg(N);
  for (uint32_t d = 0; d < N; ++d) {
    for (int b = 0; b < kStepBufs; ++b) tv[static_cast<size_t>(d) * kStepBufs + b] = base[d] + m->tv_off[b];
    arg[d] = reinterpret_cast<ArgSlot *>(base[d] + m->arg_off);
    dst[d] = base[d] + m->tv_off[BUF_ATTN] + static_cast<size_t>(m->rank) * m->q_loc;
  }
  cudaError_t e = cudaMalloc(&m->d_peer_tv, tv.size() * sizeof(void *));
  if (e == cudaSuccess) e = cudaMalloc(&m->d_peer_arg, arg.size() * sizeof(void *));
  if (e == cudaSuccess) e = cudaMalloc(&m->d_attn_dst, dst.size() * sizeof(void *));
  if (e == cudaSuccess) e = cudaMemcpy(m->d_peer_tv, tv.data(), tv.size() * sizeof(void *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(m->d_peer_arg, arg.data(), arg.size() * sizeof(void *), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(m->d_attn_dst, dst.data(), dst.size() * sizeof(void *), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "tensor parallel: peer tables");
  m->tp_connected = true;
  return ZGPU_OK;
}

}  // namespace

extern "C" {

zgpu_status zgpu_qwen3_tp_connect(zgpu_model *m, const void *handles) {
  if (!m || !handles || m->world < 2 || !m->d_tv) return ZGPU_ERR_INVALID_ARG;
  if (m->tp_connected) return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: already connected");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  const uint32_t N = m->world;
  std::vector<unsigned long long *> base(N, nullptr);
  for (uint32_t d = 0; d < N; ++d) {
    if (d == m->rank) {
      base[d] = m->d_tv;
      continue;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t *>(handles) + static_cast<size_t>(d) * sizeof(h), sizeof(h));
    void *p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "tensor parallel: open a peer's tagged vectors");
    m->ipc_opened.push_back(p);
    base[d] = static_cast<unsigned long long *>(p);
  }
  return tp_tables(m, base);
}

zgpu_status zgpu_qwen3_tp_connect_absent(zgpu_model *m) {
  if (!m || m->world < 2 || !m->d_tv) return ZGPU_ERR_INVALID_ARG;
  if (m->tp_connected) return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: already connected");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  const uint32_t N = m->world;
  std::vector<unsigned long long *> base(N, nullptr);
  for (uint32_t d = 0; d < N; ++d) {
    if (d == m->rank) {
      base[d] = m->d_tv;
      continue;
    }
    // a local arena that no kernel reads stands in for the absent rank
    void *p = nullptr;
    cudaError_t e = cudaMalloc(&p, m->tv_words * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(p, 0, m->tv_words * sizeof(unsigned long long));
    if (e != cudaSuccess) {
      cudaFree(p);
      return zgpu_cuda_fail(ctx, e, "tensor parallel: stand-in arena");
    }
    m->absent_arenas.push_back(p);
    base[d] = static_cast<unsigned long long *>(p);
  }
  return tp_tables(m, base);
}

}  // extern "C"

namespace {

// Size the attention split scratch for a cache (one partial per split).
zgpu_status prepare_kv(zgpu_model *m, zgpu_kv *kv) {
  zgpu_ctx *ctx = m->ctx;
  if (kv->n_layers != m->desc.n_layers)
    return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "kv cache layer count differs from the model");
  // a tensor-parallel rank caches its own kv heads only
  if (kv->n_kv != m->desc.n_kv_heads / m->world || kv->head_dim != m->desc.head_dim)
    return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "kv cache geometry differs from the model");
  const uint32_t splits = attention_max_splits(kv->max_tokens);
  if (splits != m->max_splits || !m->d_part) {
    cudaFree(m->d_part);
    m->d_part = nullptr;
    const size_t n = static_cast<size_t>(m->desc.n_q_heads) * splits * (m->desc.head_dim + 2);
    cudaError_t e = cudaMalloc(&m->d_part, n * 4);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "attention scratch");
    m->max_splits = splits;
    drop_graphs(m);
  }
  return ZGPU_OK;
}

}  // namespace

extern "C" {

zgpu_status zgpu_forward_single_token(zgpu_model *m, zgpu_kv *kv, uint32_t token, uint32_t pos,
                                      float *hidden_out) {
  if (!m || !kv) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  if (m->world > 1 && !m->tp_connected)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: zgpu_qwen3_tp_connect first");
  zgpu_status s = prepare_kv(m, kv);
  if (s) return s;
  if (pos >= kv->max_tokens) return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "position beyond the cache");
  if (token >= m->desc.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "token id beyond the vocab");
  cudaError_t e = grow(&m->d_prompt, &m->prompt_cap, 1);
  if (e == cudaSuccess) e = grow(&m->d_tokens, &m->tokens_cap, 1);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  if ((s = set_state(m, 1, pos, m->desc.vocab_real, 1))) return s;
  const bool persistent = step_usable(m, kv);
  // a tensor-parallel rank runs the step kernel only (its stage outputs
  // cross NVLink inside it); every rank makes the same call
  if (m->world > 1 && !persistent)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: the cache needs more attention CTAs than the step kernel has");
  const bool use_graph = !persistent && !(ctx->flags & ZGPU_FLAG_NO_GRAPH);
  if (use_graph && (s = build_graphs(m, kv))) return s;
  e = cudaMemcpyAsync(m->d_prompt, &token, 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) {
    if (persistent) {
      e = run_step(m, kv, STEP_FORWARD, 0, 1, token, pos, 1);
      ++ctx->launches;
    } else if (use_graph) {
      e = cudaGraphLaunch(m->fwd_graph, ctx->stream);
      ctx->launches += m->fwd_kernels;
      m->last_fwd_persistent = false;
    } else {
      e = enqueue_forward(m, kv, &ctx->launches);
      m->last_fwd_persistent = false;
    }
  }
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "forward");
  std::vector<unsigned long long> tagged;
  if (hidden_out) {
    if (persistent) {
      tagged.resize(m->desc.hidden);
      e = cudaMemcpyAsync(tagged.data(), m->tv[BUF_HIDDEN], m->desc.hidden * sizeof(unsigned long long),
                          cudaMemcpyDeviceToHost, ctx->stream);
    } else {
      e = cudaMemcpyAsync(hidden_out, m->d_hidden, m->desc.hidden * 4, cudaMemcpyDeviceToHost, ctx->stream);
    }
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "hidden d2h");
  }
  uint32_t st = 0;
  if ((s = read_status(m, &st))) return s;   // synchronises the stream
  if (persistent && (st & ZDEV_ERR_TIMEOUT)) reset_step_tags(m);
  if (hidden_out && persistent)
    for (uint32_t i = 0; i < m->desc.hidden; ++i) {
      const uint32_t bits = static_cast<uint32_t>(tagged[i]);
      std::memcpy(&hidden_out[i], &bits, 4);
    }
  return map_status(ctx, st);
}

zgpu_status zgpu_lm_head_argmax(zgpu_model *m, uint32_t vocab_real, uint32_t *token_out,
                                float *logits_out) {
  if (!m || !token_out) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  if (m->world > 1 && !m->tp_connected)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: zgpu_qwen3_tp_connect first");
  if (vocab_real > m->desc.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "vocab_real > padded");
  cudaError_t e = grow(&m->d_prompt, &m->prompt_cap, 1);
  if (e == cudaSuccess) e = grow(&m->d_tokens, &m->tokens_cap, 1);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  zgpu_status s = set_state(m, 1, 0, vocab_real, 1);
  if (s) return s;
  const bool persistent = step_usable(m, nullptr) && m->last_fwd_persistent;
  if (m->world > 1 && !persistent)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: the LM head follows a zgpu_forward_single_token");
  const bool use_graph = !persistent && !(ctx->flags & ZGPU_FLAG_NO_GRAPH) && m->lm_graph;
  if (persistent) {
    e = run_step(m, nullptr, STEP_LM, 0, 1, 0, 0, 1);
    ++ctx->launches;
  } else if (use_graph) {
    e = cudaGraphLaunch(m->lm_graph, ctx->stream);
    ctx->launches += m->lm_kernels;
  } else {
    e = enqueue_lm_head(m, &ctx->launches);
  }
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "lm head");
  if (logits_out) {   // a tensor-parallel rank holds the logits of its own vocabulary rows
    e = cudaMemcpyAsync(logits_out, m->d_logits, static_cast<size_t>(m->lm_rows) * 4,
                        cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "logits d2h");
  }
  e = cudaMemcpyAsync(token_out, m->d_tokens, 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "token d2h");
  uint32_t st = 0;
  if ((s = read_status(m, &st))) return s;
  if (persistent && (st & ZDEV_ERR_TIMEOUT)) reset_step_tags(m);
  return map_status(ctx, st);
}

zgpu_status zgpu_generate_greedy(zgpu_model *m, zgpu_kv *kv, const uint32_t *prompt,
                                 uint32_t n_prompt, uint32_t n_gen, uint32_t *tokens_out,
                                 float *logits_out) {
  if (!m || !kv || !prompt || !tokens_out || n_prompt == 0 || n_gen == 0) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  if (m->world > 1 && !m->tp_connected)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: zgpu_qwen3_tp_connect first");
  zgpu_status s = prepare_kv(m, kv);
  if (s) return s;
  const uint32_t steps = n_prompt + n_gen - 1;
  if (steps > kv->max_tokens)
    return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "prompt + generation exceeds the cache");
  for (uint32_t i = 0; i < n_prompt; ++i)
    if (prompt[i] >= m->desc.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "prompt id beyond the vocab");
  cudaError_t e = grow(&m->d_prompt, &m->prompt_cap, n_prompt);
  if (e == cudaSuccess) e = grow(&m->d_tokens, &m->tokens_cap, n_gen);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  if ((s = set_state(m, n_prompt, 0, m->desc.vocab_real, n_gen))) return s;
  e = cudaMemcpyAsync(m->d_prompt, prompt, n_prompt * 4, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "prompt upload");
  const bool persistent = step_usable(m, kv);
  if (m->world > 1 && !persistent)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor parallel: the cache needs more attention CTAs than the step kernel has");
  const bool use_graph = !persistent && !(ctx->flags & ZGPU_FLAG_NO_GRAPH);
  if (use_graph && (s = build_graphs(m, kv))) return s;
  const size_t V = m->desc.vocab_padded;
  uint32_t launches = 0, prefill_launches = 0;
  if (persistent) {
    // one launch for the prompt (the LM head runs after its last token) and
    // one for the decode steps; with logits requested, one launch per step so
    // that each step's logits can be copied out
    // (a tensor-parallel rank has the logits of its own vocabulary rows)
    const size_t VL = m->lm_rows;
    auto copy_logits = [&](uint32_t step) -> cudaError_t {
      if (!logits_out || step + 1 < n_prompt) return cudaSuccess;
      return cudaMemcpyAsync(logits_out + static_cast<size_t>(step + 1 - n_prompt) * VL, m->d_logits, VL * 4,
                             cudaMemcpyDeviceToHost, ctx->stream);
    };
    auto phase = [&](uint32_t first, uint32_t last) -> cudaError_t {
      cudaError_t err = cudaSuccess;
      if (first >= last) return err;
      if (!logits_out) {
        err = run_step(m, kv, STEP_GENERATE, first, last - first, 0, 0, n_prompt);
        ++launches;
        return err;
      }
      for (uint32_t st = first; st < last && err == cudaSuccess; ++st) {
        err = run_step(m, kv, STEP_GENERATE, st, 1, 0, 0, n_prompt);
        ++launches;
        if (err == cudaSuccess) err = copy_logits(st);
      }
      return err;
    };
    cudaEventRecord(m->ev[0], ctx->stream);
    e = phase(0, n_prompt);
    prefill_launches = launches;
    cudaEventRecord(m->ev[1], ctx->stream);
    if (e == cudaSuccess) e = phase(n_prompt, steps);
    cudaEventRecord(m->ev[2], ctx->stream);
  }
  auto run_step_graph = [&](uint32_t step) -> cudaError_t {
    cudaError_t err;
    if (use_graph) {
      err = cudaGraphLaunch(m->step_graph, ctx->stream);
      launches += m->step_kernels;
    } else {
      err = enqueue_forward(m, kv, &launches);
      if (err == cudaSuccess) err = enqueue_lm_head(m, &launches);
    }
    if (err == cudaSuccess && logits_out && step + 1 >= n_prompt) {
      err = cudaMemcpyAsync(logits_out + static_cast<size_t>(step + 1 - n_prompt) * V, m->d_logits,
                            V * 4, cudaMemcpyDeviceToHost, ctx->stream);
    }
    return err;
  };
  if (!persistent) {
    cudaEventRecord(m->ev[0], ctx->stream);
    for (uint32_t st = 0; st < n_prompt && e == cudaSuccess; ++st) e = run_step_graph(st);
    prefill_launches = launches;
    cudaEventRecord(m->ev[1], ctx->stream);
    for (uint32_t st = n_prompt; st < steps && e == cudaSuccess; ++st) e = run_step_graph(st);
    cudaEventRecord(m->ev[2], ctx->stream);
  }
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "generate");
  e = cudaMemcpyAsync(tokens_out, m->d_tokens, n_gen * 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "tokens d2h");
  uint32_t st = 0;
  if ((s = read_status(m, &st))) return s;
  if (persistent && (st & ZDEV_ERR_TIMEOUT)) reset_step_tags(m);
  float pre = 0.f, dec = 0.f;
  cudaEventElapsedTime(&pre, m->ev[0], m->ev[1]);
  cudaEventElapsedTime(&dec, m->ev[1], m->ev[2]);
  m->perf.steps = n_gen - 1;
  m->perf.kernel_launches = launches;
  m->perf.decode_launches = launches - prefill_launches;
  m->perf.prefill_ms = pre;
  m->perf.decode_ms = dec;
  m->perf.prefill_gemm_ms = 0;
  m->perf.prefill_attn_ms = 0;
  ctx->launches += launches;
  return map_status(ctx, st);
}

zgpu_status zgpu_lm_head_sample(zgpu_model *m, uint32_t vocab_real, float temperature, uint64_t *rng_state,
                                uint32_t *token_out) {
  if (!m || !rng_state || !token_out || vocab_real == 0) return ZGPU_ERR_INVALID_ARG;
  if (m->world > 1)
    return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "tensor-parallel ranks decode through zgpu_generate_greedy");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  cudaError_t e = grow(&m->d_tokens, &m->tokens_cap, 1);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "state buffers");
  unsigned long long *d_rng = nullptr;
  if ((e = cudaMallocAsync(reinterpret_cast<void **>(&d_rng), 8, ctx->stream)) != cudaSuccess)
    return zgpu_cuda_fail(ctx, e, "rng state");
  e = cudaMemcpyAsync(d_rng, rng_state, 8, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess)
    e = launch_sample_topk(m->d_logits, m->desc.vocab_padded, vocab_real, temperature, d_rng, m->d_tokens, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(token_out, m->d_tokens, 4, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(rng_state, d_rng, 8, cudaMemcpyDeviceToHost, ctx->stream);
  cudaFreeAsync(d_rng, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "lm_head_sample");
  ++ctx->launches;
  return ZGPU_OK;
}

zgpu_status zgpu_perf_snapshot(const zgpu_model *m, zgpu_perf *out) {
  if (!m || !out) return ZGPU_ERR_INVALID_ARG;
  *out = m->perf;
  return ZGPU_OK;
}

}  // extern "C"

extern "C" {

// Prompt prefill on the token-parallel path: every projection of a layer is
// one batched Q4_0 x Q8_0 matmul over all prompt tokens on the tensor cores
// (mma_gemm.cu), attention is causal over the prompt (prefill.cu).  The
// reference runs forward_single_token once per prompt token
// (inference.rs:1188-1320) with f32 activations; this path quantises the
// matmul inputs to Q8_0, so its KV cache and logits agree to that rounding,
// not bit for bit.  Fills cache positions [0, n) and returns the LM-head
// argmax after the last prompt token (lm_head.rs:98-166).
}  // extern "C"

namespace {

// Token-parallel prefill of n_seq prompts of n tokens each (sequence i's
// tokens at tokens[i*n ..], its cache kvs[i]).  Embedding, RMSNorm + Q8_0,
// the projections and SwiGLU run over all n_seq * n rows at once; QK-norm /
// RoPE / KV append and the causal attention run per sequence into its own
// cache; the LM head runs on each sequence's last token.  Every row is
// computed exactly as a one-sequence prefill computes it.
// The tensor-core operand tiles (ops.h) of every projection, built once per
// model on the first multi-token call: per layer QKV, O, gate/up, down.
zgpu_status ensure_pf_tiles(zgpu_model *m) {
  if (!m->pf_w8.empty()) return ZGPU_OK;
  const zgpu_qwen3_desc &d = m->desc;
  const uint32_t H = d.hidden, F = d.ffn, QD = m->q_dim, QKV = QD + 2 * m->kv_dim;
  struct Mat {
    const uint8_t *w;
    uint64_t gstride;
    uint32_t rows, in_dim;
  };
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    const Mat mats[4] = {{m->qkv[l], m->gs_h, QKV, H},
                         {m->o[l]->d, m->o[l]->gstride, H, QD},
                         {m->gateup[l], m->gs_h, 2 * F, H},
                         {m->down[l]->d, m->down[l]->gstride, H, F}};
    for (const Mat &mt : mats) {
      int8_t *wt = nullptr;
      float *ws = nullptr;
      cudaError_t e = cudaMalloc(&wt, mma_tile_bytes(mt.rows, mt.in_dim / 32));
      ws = reinterpret_cast<float *>(wt);   // the scales sit beside each 4 KB tile
      m->pf_w8.push_back(wt);
      m->pf_ws8.push_back(ws);
      if (e == cudaSuccess)
        e = launch_build_w8_tiles(mt.w, mt.gstride, mt.rows, mt.in_dim / 32, ZGPU_Q4_0, wt, ws, m->ctx->stream);
      if (e != cudaSuccess) {
        for (int8_t *p : m->pf_w8) cudaFree(p);
        m->pf_w8.clear();
        m->pf_ws8.clear();
        return zgpu_cuda_fail(m->ctx, e, "prefill weight tiles");
      }
    }
  }
  return ZGPU_OK;
}

zgpu_status prefill_run(zgpu_model *m, zgpu_kv *const *kvs, uint32_t n_seq, const uint32_t *tokens, uint32_t n,
                        uint32_t *tokens_out, float *logits_out) {
  if (!m || !kvs || !tokens || !tokens_out || n == 0 || n_seq == 0) return ZGPU_ERR_INVALID_ARG;
  if (m->world > 1)
    return zgpu_fail(m->ctx, ZGPU_ERR_INVALID_ARG, "tensor-parallel ranks decode through zgpu_generate_greedy");
  zgpu_ctx *ctx = m->ctx;
  cudaSetDevice(ctx->device);
  const zgpu_qwen3_desc &d = m->desc;
  zgpu_status st;
  for (uint32_t i = 0; i < n_seq; ++i) {
    if (!kvs[i]) return ZGPU_ERR_INVALID_ARG;
    if ((st = prepare_kv(m, kvs[i]))) return st;
    if (n > kvs[i]->max_tokens)
      return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "prompt longer than the cache");
    for (uint32_t j = 0; j < i; ++j)
      if (kvs[j] == kvs[i]) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "prefill: one cache per sequence");
  }
  const uint64_t NT = static_cast<uint64_t>(n_seq) * n;   // rows through the projections
  if (NT > 0xFFFFFFFFull / 16) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "prefill: too many tokens");
  for (uint64_t i = 0; i < NT; ++i)
    if (tokens[i] >= d.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "prompt id beyond the vocab");
  const uint32_t H = d.hidden, F = d.ffn, QD = m->q_dim, KVD = m->kv_dim, QKV = QD + 2 * KVD;
  if (H % 128 || QKV % 128 || (2 * F) % 128 || QD % 32 || F % 32)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "prefill: projection rows must be multiples of 128");
  if ((st = ensure_pf_tiles(m))) return st;
  // scratch: tokens | hidden [NT][H] | qkv [NT][QKV] | qrot [NT][QD] | attn [NT][QD] | gu [NT][2F]
  //          | activation tiles and scales for the widest input
  const size_t N = NT, maxk = std::max(std::max(H, QD), F);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t o_tok = 0, o_hid = al(N * 4), o_qkv = o_hid + al(N * H * 4), o_qr = o_qkv + al(N * QKV * 4),
               o_at = o_qr + al(N * QD * 4), o_gu = o_at + al(N * QD * 4), o_q8 = o_gu + al(N * 2 * F * 4),
               o_d8 = o_q8, total = o_q8 + al(mma_tile_bytes(N, maxk / 32));   // scales inside the tiles
  if (total > m->pf_cap) {
    cudaFree(m->d_pf);
    m->d_pf = nullptr;
    m->pf_cap = 0;
    cudaError_t e = cudaMalloc(&m->d_pf, total);
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "prefill scratch");
    m->pf_cap = total;
  }
  uint8_t *B = m->d_pf;
  uint32_t *d_tok = reinterpret_cast<uint32_t *>(B + o_tok);
  float *hid = reinterpret_cast<float *>(B + o_hid), *qkv = reinterpret_cast<float *>(B + o_qkv),
        *qr = reinterpret_cast<float *>(B + o_qr), *at = reinterpret_cast<float *>(B + o_at),
        *gu = reinterpret_cast<float *>(B + o_gu);
  int8_t *q8 = reinterpret_cast<int8_t *>(B + o_q8);
  float *d8 = reinterpret_cast<float *>(B + o_d8);
  cudaStream_t s = ctx->stream;
  uint32_t launches = 0;
  // an event pair around every GEMM and attention phase: per-class device time
  const size_t n_ev = static_cast<size_t>(d.n_layers) * 10;
  while (m->pf_ev.size() < n_ev) {
    cudaEvent_t ev;
    cudaError_t ee = cudaEventCreate(&ev);
    if (ee != cudaSuccess) return zgpu_cuda_fail(ctx, ee, "prefill events");
    m->pf_ev.push_back(ev);
  }
  size_t ev_i = 0;
  auto mark = [&]() { cudaEventRecord(m->pf_ev[ev_i++], s); };
  auto gemm = [&](uint32_t l, uint32_t which, uint32_t rows, uint32_t in_dim, float *y, bool resadd) {
    MmaGemmParams p = {};
    p.wt = m->pf_w8[4 * l + which];
    p.ws = m->pf_ws8[4 * l + which];
    p.rows = rows;
    p.bpr = in_dim / 32;
    p.T = static_cast<uint32_t>(NT);
    p.ldy = rows;
    p.xt = q8;
    p.xs = d8;
    p.y = y;
    p.status = m->d_status;
    p.resadd = resadd ? 1u : 0u;
    ++launches;
    mark();
    cudaError_t ge = launch_q4q8_mma(p, s);
    mark();
    return ge;
  };
  cudaError_t e = cudaMemcpyAsync(d_tok, tokens, N * 4, cudaMemcpyHostToDevice, s);
  cudaEventRecord(m->ev[0], s);
  if (e == cudaSuccess)
    e = launch_rows_embed(m->emb->d, m->emb->gstride, m->emb->quant, H, static_cast<uint32_t>(m->emb->rows), d_tok,
                          static_cast<uint32_t>(NT), hid, m->d_status, s), ++launches;
  const float scale = 1.0f / sqrtf(static_cast<float>(d.head_dim));
  const uint32_t T = static_cast<uint32_t>(NT);
  for (uint32_t l = 0; l < d.n_layers && e == cudaSuccess; ++l) {
    if ((e = launch_rows_rmsnorm_quant(hid, norm_attn(m, l), d.rms_eps, T, H, q8, d8, m->d_status, s))) break;
    if ((e = gemm(l, 0, QKV, H, qkv, false))) break;
    for (uint32_t i = 0; i < n_seq && e == cudaSuccess; ++i, ++launches) {
      float *kvl = kvs[i]->d + static_cast<size_t>(l) * 2 * kvs[i]->block;
      const size_t r0 = static_cast<size_t>(i) * n;
      e = launch_qk_rope_kv(qkv + r0 * QKV, norm_q(m, l), norm_k(m, l), m->d_inv_freqs, kvl, kvs[i]->block,
                            d.n_q_heads, d.n_kv_heads, 0, n, d.rms_eps, qr + r0 * QD, s);
    }
    if (e) break;
    mark();
    for (uint32_t i = 0; i < n_seq && e == cudaSuccess; ++i, ++launches) {
      float *kvl = kvs[i]->d + static_cast<size_t>(l) * 2 * kvs[i]->block;
      const size_t r0 = static_cast<size_t>(i) * n;
      e = launch_causal_attn(qr + r0 * QD, kvl, kvs[i]->block, d.n_q_heads, d.n_kv_heads, 0, n, scale, at + r0 * QD,
                             m->d_status, s);
    }
    mark();
    if (e) break;
    if ((e = launch_quantize_q8_0_tiles(at, q8, d8, T, QD, m->d_status, s))) break;
    if ((e = gemm(l, 1, H, QD, hid, true))) break;
    if ((e = launch_rows_rmsnorm_quant(hid, norm_ffn(m, l), d.rms_eps, T, H, q8, d8, m->d_status, s))) break;
    if ((e = gemm(l, 2, 2 * F, H, gu, false))) break;
    if ((e = launch_swiglu_quant_tiles(gu, q8, d8, T, F, m->d_status, s))) break;
    if ((e = gemm(l, 3, H, F, hid, true))) break;
    launches += 4;
  }
  cudaEventRecord(m->ev[1], s);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "prefill");
  // LM head on each sequence's last prompt token
  cudaError_t e2 = grow(&m->d_prompt, &m->prompt_cap, 1);
  if (e2 == cudaSuccess) e2 = grow(&m->d_tokens, &m->tokens_cap, 1);
  if (e2 != cudaSuccess) return zgpu_cuda_fail(ctx, e2, "state buffers");
  const size_t V = d.vocab_padded;
  for (uint32_t i = 0; i < n_seq; ++i) {
    if ((st = set_state(m, 1, n - 1, d.vocab_real, 1))) return st;
    e = cudaMemcpyAsync(m->d_hidden, hid + (static_cast<size_t>(i) * n + n - 1) * H, H * 4, cudaMemcpyDeviceToDevice,
                        s);
    if (e == cudaSuccess) e = enqueue_lm_head(m, &launches);
    m->last_fwd_persistent = false;
    if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "prefill lm head");
    if (logits_out)
      if ((e = cudaMemcpyAsync(logits_out + i * V, m->d_logits, V * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
        return zgpu_cuda_fail(ctx, e, "logits d2h");
    if ((e = cudaMemcpyAsync(tokens_out + i, m->d_tokens, 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
      return zgpu_cuda_fail(ctx, e, "token d2h");
  }
  uint32_t sw = 0;
  if ((st = read_status(m, &sw))) return st;
  float ms = 0.f;
  cudaEventElapsedTime(&ms, m->ev[0], m->ev[1]);
  m->perf.prefill_ms = ms;
  // five event pairs per layer, in launch order: QKV GEMM, attention, O, gate/up and down GEMMs
  double gemm_ms = 0, attn_ms = 0;
  for (size_t i = 0; i + 1 < ev_i; i += 2) {
    float t = 0.f;
    cudaEventElapsedTime(&t, m->pf_ev[i], m->pf_ev[i + 1]);
    if ((i / 2) % 5 == 1)
      attn_ms += t;
    else
      gemm_ms += t;
  }
  m->perf.prefill_gemm_ms = gemm_ms;
  m->perf.prefill_attn_ms = attn_ms;
  m->perf.kernel_launches = launches;
  m->perf.steps = 0;
  m->perf.decode_ms = 0;
  m->perf.decode_launches = 0;
  ctx->launches += launches;
  return map_status(ctx, sw);
}

// One greedy decode step for n_seq independent sequences, each at its own
// position: forward_single_token (forward_pass.rs:515-631) + the LM head pick
// (lm_head.rs:98-166) per sequence, computed as one batch.  The projections
// and the LM head run on the tensor cores over Q8_0-quantised activation rows
// (the prefill arithmetic, with the LM head's Q8_0 weights as int8 tiles);
// the attention is the decode kernel with a sequence grid dimension.
// The tensor-core matvec's weight tiles of every projection and the LM
// head, built once per model by the first batched decode.
zgpu_status ensure_dm_tiles(zgpu_model *m) {
  if (!m->dm_tiles.empty()) return ZGPU_OK;
  const zgpu_qwen3_desc &d = m->desc;
  const uint32_t H = d.hidden, F = d.ffn, QD = m->q_dim, QKV = QD + 2 * m->kv_dim;
  struct Mat {
    const uint8_t *w;
    uint64_t gstride;
    uint32_t quant, rows, in_dim;
  };
  std::vector<Mat> mats;
  for (uint32_t l = 0; l < d.n_layers; ++l) {
    mats.push_back({m->qkv[l], m->gs_h, ZGPU_Q4_0, QKV, H});
    mats.push_back({m->o[l]->d, m->o[l]->gstride, ZGPU_Q4_0, H, QD});
    mats.push_back({m->gateup[l], m->gs_h, ZGPU_Q4_0, 2 * F, H});
    mats.push_back({m->down[l]->d, m->down[l]->gstride, ZGPU_Q4_0, H, F});
  }
  mats.push_back({m->out->d, m->out->gstride, m->out->quant, d.vocab_padded, H});
  for (const Mat &mt : mats) {
    uint8_t *t = nullptr;
    cudaError_t e = cudaMalloc(&t, dm_tile_bytes(mt.rows, mt.in_dim / 32));
    if (e == cudaSuccess) {
      m->dm_tiles.push_back(t);
      e = launch_build_dm_tiles(mt.w, mt.gstride, mt.quant, mt.rows, mt.in_dim / 32, t, m->ctx->stream);
    }
    if (e != cudaSuccess) {
      for (uint8_t *p : m->dm_tiles) cudaFree(p);
      m->dm_tiles.clear();
      return zgpu_cuda_fail(m->ctx, e, "batched decode weight tiles");
    }
  }
  return ZGPU_OK;
}

zgpu_status decode_batch_run(zgpu_model *m, zgpu_kv *const *kvs, uint32_t n_seq, const uint32_t *tokens,
                             const uint32_t *positions, uint32_t *tokens_out, float *logits_out) {
  if (!m || !kvs || !tokens || !positions || !tokens_out || n_seq == 0) return ZGPU_ERR_INVALID_ARG;
  zgpu_ctx *ctx = m->ctx;
  if (m->world > 1)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "tensor-parallel ranks decode through zgpu_generate_greedy");
  if (n_seq > kMaxDecodeBatch) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "decode batch: at most 256 sequences");
  cudaSetDevice(ctx->device);
  const zgpu_qwen3_desc &d = m->desc;
  const uint32_t H = d.hidden, F = d.ffn, QD = m->q_dim, KVD = m->kv_dim, QKV = QD + 2 * KVD;
  const uint32_t V = d.vocab_padded, hd = d.head_dim;
  if (H % 32 || QD % 32 || F % 32 || F % 4)
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "decode batch: hidden, q and ffn widths must be multiples of 32");
  if (hd != 128)   // the decode attention kernel's head size
    return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "decode batch: head_dim must be 128");
  uint32_t splits = 0;
  std::vector<AttnBatchSeq> seqs(n_seq);
  for (uint32_t i = 0; i < n_seq; ++i) {
    const zgpu_kv *kv = kvs[i];
    if (!kv) return ZGPU_ERR_INVALID_ARG;
    if (kv->n_layers != d.n_layers)
      return zgpu_fail(ctx, ZGPU_ERR_KV_LAYER_OUT_OF_RANGE, "kv cache layer count differs from the model");
    if (kv->n_kv != d.n_kv_heads || kv->head_dim != hd)
      return zgpu_fail(ctx, ZGPU_ERR_KV_INVALID_SLICE_LENGTH, "kv cache geometry differs from the model");
    if (positions[i] >= kv->max_tokens)
      return zgpu_fail(ctx, ZGPU_ERR_KV_TOKEN_OUT_OF_RANGE, "decode batch: position beyond the cache");
    if (tokens[i] >= d.vocab_padded) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "token id beyond the vocab");
    for (uint32_t j = 0; j < i; ++j)
      if (kvs[j] == kv) return zgpu_fail(ctx, ZGPU_ERR_INVALID_ARG, "decode batch: one cache per sequence");
    seqs[i] = {kv->d, kv->block, kv->max_tokens, positions[i]};
    splits = std::max(splits, attention_max_splits(kv->max_tokens));
  }
  zgpu_status st;
  if ((st = ensure_dm_tiles(m))) return st;
  cudaStream_t s = ctx->stream;
  cudaError_t e = cudaSuccess;
  // scratch (n_seq rows each): tokens | residual | q|k|v | attention output |
  // SwiGLU output
  const size_t N = n_seq, maxk = std::max(std::max(H, QD), F);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t o_tok = 0, o_hid = al(N * 4), o_qkv = o_hid + al(N * H * 4), o_at = o_qkv + al(N * QKV * 4),
               o_gu = o_at + al(N * QD * 4), total = o_gu + al(N * F * 4);
  if (total > m->pf_cap) {
    cudaFree(m->d_pf);
    m->d_pf = nullptr;
    m->pf_cap = 0;
    if ((e = cudaMalloc(&m->d_pf, total)) != cudaSuccess) return zgpu_cuda_fail(ctx, e, "decode batch scratch");
    m->pf_cap = total;
  }
  // the matvec partials: the largest chunks x rows of the step's products
  auto ks_of = [](uint32_t in_dim) { return static_cast<size_t>((in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks); };
  size_t part_f = 0;
  {
    const uint32_t shapes[5][2] = {{QKV, H}, {H, QD}, {2 * F, H}, {H, F}, {V, H}};
    for (const auto &sh : shapes) part_f = std::max(part_f, ks_of(sh[1]) * sh[0]);
  }
  // batch block: seq table | partials | counters | logits | tokens | codes | digit image | matvec partials
  const size_t b_seq = 0, b_part = al(N * sizeof(AttnBatchSeq)),
               b_cnt = b_part + al(N * d.n_q_heads * splits * (hd + 2) * 4),
               b_log = b_cnt + al(N * d.n_kv_heads * 4), b_tok = b_log + al(N * V * 4), b_code = b_tok + al(N * 4),
               b_img = b_code + al(N * 4), b_dpart = b_img + al(dm_img_bytes(maxk, n_seq)),
               b_total = b_dpart + al(part_f * N * 4);
  if (b_total > m->bd_cap) {
    cudaFree(m->d_bd);
    m->d_bd = nullptr;
    m->bd_cap = 0;
    if ((e = cudaMalloc(&m->d_bd, b_total)) != cudaSuccess) return zgpu_cuda_fail(ctx, e, "decode batch buffers");
    m->bd_cap = b_total;
  }
  // the arrival counters start at zero (their offset moves with n_seq and the
  // split count; within the step the attention resets them after use)
  if ((e = cudaMemsetAsync(m->d_bd + b_cnt, 0, N * d.n_kv_heads * 4, s)) != cudaSuccess)
    return zgpu_cuda_fail(ctx, e, "memset");
  uint8_t *B = m->d_pf, *BB = m->d_bd;
  uint32_t *d_tok = reinterpret_cast<uint32_t *>(B + o_tok);
  float *hid = reinterpret_cast<float *>(B + o_hid), *qkv = reinterpret_cast<float *>(B + o_qkv),
        *at = reinterpret_cast<float *>(B + o_at), *act = reinterpret_cast<float *>(B + o_gu);
  AttnBatchSeq *d_seqs = reinterpret_cast<AttnBatchSeq *>(BB + b_seq);
  float *logits = reinterpret_cast<float *>(BB + b_log);
  uint32_t *d_out_tok = reinterpret_cast<uint32_t *>(BB + b_tok),
           *d_codes = reinterpret_cast<uint32_t *>(BB + b_code);
  uint8_t *img = BB + b_img;
  float *dpart = reinterpret_cast<float *>(BB + b_dpart);
  const uint32_t T = n_seq;
  uint32_t launches = 0;
  // an event pair around every projection and attention launch: per-class device time
  const size_t n_ev = static_cast<size_t>(d.n_layers) * 10 + 2;
  while (m->pf_ev.size() < n_ev) {
    cudaEvent_t ev;
    if ((e = cudaEventCreate(&ev)) != cudaSuccess) return zgpu_cuda_fail(ctx, e, "decode batch events");
    m->pf_ev.push_back(ev);
  }
  size_t ev_i = 0;
  std::vector<uint8_t> ev_attn;   // per event pair: 1 for an attention launch
  auto mark = [&]() { cudaEventRecord(m->pf_ev[ev_i++], s); };
  LaunchCfg lc;
  lc.stream = s;
  lc.pdl = !(ctx->flags & ZGPU_FLAG_NO_PDL);
  lc.sm_count = ctx->sm_count;
  lc.launch_counter = &launches;
  // One projection of every sequence on the tensor cores (digit_mma.h):
  // digit image (RMSNorm first when norm_w), MMA partials, the GEMV's
  // epilogue.  Each sequence's row equals the one-token GEMV's bit for bit.
  auto proj = [&](const float *x, uint32_t in_dim, const float *norm_w, const uint8_t *tiles, uint32_t rows, float *y,
                  uint32_t ldy, GemvEpi epi) -> cudaError_t {
    mark();
    ev_attn.push_back(0);
    DigitImageParams ip = {};
    ip.x = x;
    ip.x_stride = in_dim;
    ip.norm_w = norm_w;
    ip.eps = d.rms_eps;
    ip.in_dim = in_dim;
    ip.n_vec = T;
    ip.n_img = 1;
    ip.img = img;
    ip.status = m->d_status;
    cudaError_t pe = launch_digit_image(ip, lc);
    if (pe != cudaSuccess) return pe;
    DmGemmParams gp = {};
    gp.wt = tiles;
    gp.rows = rows;
    gp.in_dim = in_dim;
    gp.img = img;
    gp.n_vec = T;
    gp.n_seg = 1;
    gp.part = dpart;
    gp.status = m->d_status;
    if ((pe = launch_dm_gemm(gp, lc)) != cudaSuccess) return pe;
    DmCombineParams cp = {};
    cp.part = dpart;
    cp.rows = rows;
    cp.ks = static_cast<uint32_t>(ks_of(in_dim));
    cp.n_vec = T;
    cp.n_seg = 1;
    cp.out = y;
    cp.out_vec_stride = ldy;
    cp.epi = epi;
    pe = launch_dm_combine(cp, lc);
    mark();
    return pe;
  };
  e = cudaMemcpyAsync(d_tok, tokens, N * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_seqs, seqs.data(), N * sizeof(AttnBatchSeq), cudaMemcpyHostToDevice, s);
  cudaEventRecord(m->ev[0], s);
  if (e == cudaSuccess) {
    e = launch_rows_embed(m->emb->d, m->emb->gstride, m->emb->quant, H, static_cast<uint32_t>(m->emb->rows), d_tok,
                          T, hid, m->d_status, s);
    ++launches;
  }
  LaunchCfg alc = lc;
  alc.pdl = false;
  AttnParams ap = {};
  ap.qkv = qkv;
  ap.inv_freqs = m->d_inv_freqs;
  ap.out = at;
  ap.part = reinterpret_cast<float *>(BB + b_part);
  ap.counters = reinterpret_cast<uint32_t *>(BB + b_cnt);
  ap.status = m->d_status;
  ap.n_q = d.n_q_heads;
  ap.n_kv = d.n_kv_heads;
  ap.max_splits = splits;
  ap.eps = d.rms_eps;
  ap.scale = 1.0f / sqrtf(static_cast<float>(hd));
  for (uint32_t l = 0; l < d.n_layers && e == cudaSuccess; ++l) {
    uint8_t *const *tl = m->dm_tiles.data() + 4 * l;
    if ((e = proj(hid, H, norm_attn(m, l), tl[0], QKV, qkv, QKV, EPI_STORE))) break;
    ap.q_norm = norm_q(m, l);
    ap.k_norm = norm_k(m, l);
    mark();
    ev_attn.push_back(1);
    e = launch_attention_batch(ap, d_seqs, l, T, QKV, QD, alc);
    mark();
    if (e) break;
    if ((e = proj(at, QD, nullptr, tl[1], H, hid, H, EPI_RESADD))) break;
    if ((e = proj(hid, H, norm_ffn(m, l), tl[2], 2 * F, act, F, EPI_SWIGLU))) break;
    if ((e = proj(act, F, nullptr, tl[3], H, hid, H, EPI_RESADD))) break;
  }
  if (e == cudaSuccess) e = proj(hid, H, norm_out(m), m->dm_tiles.back(), V, logits, V, EPI_STORE);
  if (e == cudaSuccess) {
    e = launch_rows_argmax(logits, T, V, d.vocab_real, d_out_tok, d_codes, m->d_status, s);
    ++launches;
  }
  cudaEventRecord(m->ev[1], s);
  if (e != cudaSuccess) return zgpu_cuda_fail(ctx, e, "decode batch");
  std::vector<uint32_t> codes(N);
  if ((e = cudaMemcpyAsync(tokens_out, d_out_tok, N * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(codes.data(), d_codes, N * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return zgpu_cuda_fail(ctx, e, "tokens d2h");
  if (logits_out && (e = cudaMemcpyAsync(logits_out, logits, N * V * 4, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return zgpu_cuda_fail(ctx, e, "logits d2h");
  uint32_t sw = 0;
  if ((st = read_status(m, &sw))) return st;   // synchronises the stream
  float ms = 0.f;
  cudaEventElapsedTime(&ms, m->ev[0], m->ev[1]);
  m->perf.decode_ms = ms;
  double gemm_ms = 0, attn_ms = 0;
  for (size_t i = 0; i + 1 < ev_i; i += 2) {
    float t = 0.f;
    cudaEventElapsedTime(&t, m->pf_ev[i], m->pf_ev[i + 1]);
    (ev_attn[i / 2] ? attn_ms : gemm_ms) += t;
  }
  m->perf.batch_gemm_ms = gemm_ms;
  m->perf.batch_attn_ms = attn_ms;
  m->perf.steps = 1;
  m->perf.kernel_launches = launches;
  m->perf.decode_launches = launches;
  ctx->launches += launches;
  m->last_fwd_persistent = false;
  // the LM-head error of each sequence, as its own call would report it
  for (uint32_t i = 0; i < n_seq; ++i)
    if (codes[i])
      return zgpu_fail(ctx, static_cast<zgpu_status>(codes[i]),
                       "sequence " + std::to_string(i) +
                           (codes[i] == ZGPU_ERR_LM_NON_FINITE_LOGITS ? ": non-finite max logit"
                                                                       : ": argmax in padding region"));
  return map_status(ctx, sw);
}

}  // namespace

extern "C" {

zgpu_status zgpu_prefill(zgpu_model *m, zgpu_kv *kv, const uint32_t *tokens, uint32_t n, uint32_t *token_out,
                         float *logits_out) {
  if (!kv) return ZGPU_ERR_INVALID_ARG;
  return prefill_run(m, &kv, 1, tokens, n, token_out, logits_out);
}

zgpu_status zgpu_prefill_batch(zgpu_model *m, zgpu_kv *const *kvs, uint32_t n_seq, const uint32_t *tokens, uint32_t n,
                               uint32_t *tokens_out, float *logits_out) {
  return prefill_run(m, kvs, n_seq, tokens, n, tokens_out, logits_out);
}

zgpu_status zgpu_decode_batch(zgpu_model *m, zgpu_kv *const *kvs, uint32_t n_seq, const uint32_t *tokens,
                              const uint32_t *positions, uint32_t *tokens_out, float *logits_out) {
  return decode_batch_run(m, kvs, n_seq, tokens, positions, tokens_out, logits_out);
}

}  // extern "C"
