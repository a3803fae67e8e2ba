// step.cu — persistent decode-step kernel.
//
// One cooperative launch runs whole decode steps of the Qwen3 forward pass
// (forward_single_token_avx512, kernel/src/inference_avx512.rs:1826-1987)
// and the LM-head argmax (lm_head.rs:98-166): for every layer the stages
//   QKV GEMV (RMSNorm prologue; layer 0 embeds the token) -> attention ->
//   O GEMV + residual -> gate/up GEMV + SwiGLU (RMSNorm prologue) ->
//   down GEMV + residual,
// then the LM-head GEMV with its argmax and the token hand-off.  One CTA per
// SM; each CTA has 16 consumer warps and one producer warp.
//
//   * The producer warp never waits for another CTA: lane w walks the same
//     stage list as consumer warp w and streams that warp's weight items
//     (1-D TMA bulk copies, L2 evict-first) into the warp's own ring slots,
//     across stage and step boundaries, limited only by free slots.  Weights
//     do not depend on activations, so HBM keeps streaming while the
//     consumers wait at a stage boundary.
//   * There is no grid barrier.  The inter-stage vectors (residual stream,
//     fused QKV, attention output, SwiGLU output, the next token) are tagged
//     words (version << 32 | f32 bits, one 64-bit store each); a stage's
//     consumers wait, element by element, for the version they expect, so
//     waiting for the inputs and fetching them is one L2 round trip.  Every
//     stage's input is written by all CTAs' previous stage, so no CTA can
//     overwrite a vector another CTA has yet to read.  Reads go through L2
//     (ld.global.cg): L1 is not coherent within a kernel.
//   * Each CTA owns the same residual rows in every residual-adding stage and
//     keeps them in shared memory.  The LM head's CTAs count their arrivals;
//     CTA 0 then decodes the argmax and publishes the next token.
//   * A GEMV stage splits its units (8 rows for Q4_0, 4 for Q8_0) evenly
//     over the CTAs; within a CTA the warps take (unit, K-chunk) items and
//     the chunk partials are added in chunk order, so results do not depend
//     on timing.  The arithmetic is the standalone GEMV's (gemv_body.cuh).
//   * The attention stage runs on n_kv * splits CTAs with all their consumer
//     warps (attn_body.cuh); the other CTAs pass to the next stage.
// Any bounded wait that gives up sets ZDEV_ERR_TIMEOUT and the launch's abort
// flag; from then on every wait of every CTA fails at once, producers stop
// issuing and drain their copies in flight, and the launch runs out.
#include "attn_body.cuh"
#include "common.cuh"
#include "gemv_body.cuh"
#include "layout.h"
#include "step.h"

namespace zgpu {

namespace {

constexpr int kNW = 15;                        // consumer warps (16 warps per CTA: 128 registers)
constexpr int kNC = 32 * kNW;                  // consumer threads
constexpr int kStepThreads = kNC + 32;         // + one producer warp
constexpr uint32_t kSlots = 2;                 // ring slots per consumer warp
constexpr uint32_t kSlotBytes = 4608;          // 2 Q4_0 or 1 Q8_0 group-chunk of 32 blocks
constexpr uint32_t kBarConsumers = 1;          // named barrier ids (0 = __syncthreads)
constexpr uint32_t kBarAttn = 2;
constexpr size_t kStepSmemMax = 227 * 1024;
constexpr size_t kStepDynSmemMax = kStepSmemMax - 3072;   // the rest is the kernel's static shared memory

#ifdef ZGPU_STEP_TRACE
// Stage timeline of CTA 0 (profiling builds only): entry k holds
// (%globaltimer << 8) | event, event = stage kind + 8 * phase, where phase 0
// is the stage start (after its grid barrier) and 1 the stage end.
constexpr uint32_t kTraceCap = 1 << 17;
__device__ unsigned long long g_step_trace[kTraceCap];
__device__ uint32_t g_step_trace_n;
__shared__ uint32_t s_trace_n;   // entries this launch (thread 0 of CTA 0 only)
__device__ __forceinline__ void trace(uint32_t event) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const uint32_t n = s_trace_n;
    if (n < kTraceCap) g_step_trace[n] = (globaltimer_ns() << 8) | event;
    s_trace_n = n + 1;
  }
}
// Per-CTA stage timeline: (stage sequence, CTA) -> image ready, items done,
// epilogue done, stage done; plus each CTA's SM id.
constexpr uint32_t kCtaTraceCap = 1 << 21;
__device__ unsigned long long g_cta_trace[kCtaTraceCap];
__device__ uint32_t g_cta_smid[1024];
__shared__ uint32_t s_cta_seq;
__device__ __forceinline__ void trace_cta(uint32_t which) {
  if (threadIdx.x == 0) {
    const uint64_t i = (static_cast<uint64_t>(s_cta_seq) * gridDim.x + blockIdx.x) * 4 + which;
    if (i < kCtaTraceCap) g_cta_trace[i] = globaltimer_ns();
    if (which == 3) ++s_cta_seq;
  }
}
__device__ __forceinline__ void trace_begin() {
  if (blockIdx.x == 0 && threadIdx.x == 0) s_trace_n = g_step_trace_n;
  if (threadIdx.x == 0) {
    s_cta_seq = 0;
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    if (blockIdx.x < 1024) g_cta_smid[blockIdx.x] = smid;
  }
}
__device__ __forceinline__ void trace_end() {
  if (blockIdx.x == 0 && threadIdx.x == 0) g_step_trace_n = s_trace_n < kTraceCap ? s_trace_n : kTraceCap;
}
#else
__device__ __forceinline__ void trace(uint32_t) {}
__device__ __forceinline__ void trace_begin() {}
__device__ __forceinline__ void trace_end() {}
__device__ __forceinline__ void trace_cta(uint32_t) {}
#endif

__device__ __forceinline__ void red_release_add(uint32_t *p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// mbarrier phase wait that also gives up when the CTA is aborting.
__device__ bool wait_phase(uint32_t bar, uint32_t parity, uint32_t *status, volatile uint32_t *abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, ZDEV_ERR_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
}

// The attention CTAs run the attention on all their consumer warps.
using StepAttnSmem = AttnSmemT<kNW>;
struct AttnBar {
  __device__ __forceinline__ void operator()() const { named_bar_sync(kBarAttn, kNC); }
};
struct AttnMark {   // attention timeline events 121..123 (profiling builds)
  __device__ __forceinline__ void operator()(uint32_t e) const { trace(120 + e); }
};

// Whether step `gstep` of this launch runs the forward pass / the LM head.
__device__ __forceinline__ bool runs_fwd(const StepParams &P) { return P.mode != STEP_LM; }
__device__ __forceinline__ bool runs_lm(const StepParams &P, uint32_t gstep, uint32_t n_prompt) {
  return P.mode == STEP_LM || (P.mode == STEP_GENERATE && gstep + 1 >= n_prompt);
}

__device__ __forceinline__ void unit_range(uint32_t units, uint32_t *u0, uint32_t *u1) {
  const uint64_t G = gridDim.x, c = blockIdx.x;
  *u0 = static_cast<uint32_t>(static_cast<uint64_t>(units) * c / G);
  *u1 = static_cast<uint32_t>(static_cast<uint64_t>(units) * (c + 1) / G);
}

// ------------------------------------------------------------- producer
// Item k of a stage (this CTA's (unit, chunk) list) goes to warp
// (k + rot) % kNW, rot advancing by each stage's item count, so that every
// warp's ring slots carry an even share of the weight stream.
__device__ void produce_stage(const StepParams &P, const StageDesc &sd, uint8_t *ring, uint64_t *full,
                              uint64_t *empty, uint32_t lane, uint64_t pol, uint32_t *j, uint32_t *rot,
                              bool *stop, volatile uint32_t *abort) {
  if (*stop || sd.kind != STG_GEMV) return;
  uint32_t u0, u1;
  unit_range(sd.units, &u0, &u1);
  const uint32_t nitems = (u1 - u0) * sd.ks;
  const uint32_t first = (lane + kNW - *rot) % kNW;
  *rot = (*rot + nitems) % kNW;
  for (uint32_t k = first; k < nitems; k += kNW) {
    const uint32_t slot = lane * kSlots + (*j % kSlots);
    if (*j >= kSlots && !wait_phase(smem_addr(&empty[slot]), ((*j / kSlots) - 1) & 1, P.status, abort)) {
      *stop = true;
      return;
    }
    const uint32_t unit = u0 + k / sd.ks, chunk = k % sd.ks;
    const uint32_t bytes = static_cast<uint32_t>(chunk_bytes(sd.quant, chunk_blocks(sd.bpr, chunk)));
    const uint64_t off = chunk_offset(sd.quant, chunk);
    const uint64_t g0 = static_cast<uint64_t>(unit) * sd.gpu;
    if (!ZDEV_CHECK((g0 + sd.gpu - 1) * sd.gstride + off + bytes <= sd.wbytes &&
                        sd.gbytes * (sd.gpu - 1) + bytes <= kSlotBytes,
                    P.status, 30, unit, chunk)) {
      *stop = true;
      return;
    }
    const uint32_t fb = smem_addr(&full[slot]);
    const uint32_t dst = smem_addr(ring + static_cast<size_t>(slot) * kSlotBytes);
    mbar_arrive_expect_tx(fb, sd.gpu * bytes);
    for (uint32_t g = 0; g < sd.gpu; ++g)
      tma_bulk_g2s(dst + g * sd.gbytes, sd.w + (g0 + g) * sd.gstride + off, bytes, fb, pol);
    ++*j;
  }
}

__device__ void producer(const StepParams &P, const StageDesc *stages, uint8_t *ring, uint64_t *full,
                         uint64_t *empty, uint32_t lane, volatile uint32_t *abort) {
  if (lane >= kNW) return;
  const uint64_t pol = l2_evict_first_policy();
  const uint32_t n_prompt = P.state->n_prompt;
  uint32_t j = 0, rot = 0;
  bool stop = false;
  for (uint32_t i = 0; i < P.n_steps && !stop; ++i) {
    const uint32_t gstep = P.step0 + i;
    if (runs_fwd(P))
      for (uint32_t s = 0; s < P.n_layer_stages && !stop; ++s)
        produce_stage(P, stages[s], ring, full, empty, lane, pol, &j, &rot, &stop, abort);
    if (runs_lm(P, gstep, n_prompt))
      produce_stage(P, stages[P.lm_stage], ring, full, empty, lane, pol, &j, &rot, &stop, abort);
  }
  // Never leave a copy in flight when the CTA may exit.
  for (uint32_t s = 0; s < kSlots && s < j; ++s) {
    const uint32_t last = s + ((j - 1 - s) / kSlots) * kSlots;
    mbar_wait(smem_addr(&full[lane * kSlots + s]), (last / kSlots) & 1, P.status);
  }
}

// ------------------------------------------------------------- consumers
// Embedding row of `token` (embed_lookup_dispatch, forward_pass.rs:311-370):
// elements 4f..4f+3, dequantised from the table's plane layout.
__device__ __forceinline__ float4 embed_f4(const StepParams &P, uint32_t token, uint32_t f) {
  const uint32_t bpr = P.hidden / 32;
  const uint32_t e = 4 * f, b = e >> 5, jb = e & 31, l = token & 3;
  const uint8_t *grp = P.emb + static_cast<uint64_t>(token >> 2) * P.emb_gstride;
  const uint8_t *sc = grp + scale_entry(P.emb_quant, bpr, b) + 2 * l;
  const float d = h2f(static_cast<uint16_t>(__ldg(sc) | (__ldg(sc + 1) << 8)));
  float v[4];
  if (P.emb_quant == ZGPU_Q8_0) {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(
        grp + plane_entry(P.emb_quant, bpr, b, 2 * l + (jb >> 4)) + (jb & 15)));
#pragma unroll
    for (int k = 0; k < 4; ++k)
      v[k] = __fmul_rn(static_cast<float>(static_cast<int8_t>((w >> (8 * k)) & 0xFF)), d);
  } else {
    const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(grp + plane_entry(P.emb_quant, bpr, b, l) +
                                                                (jb & 15)));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t byte = (w >> (8 * k)) & 0xFF;
      const int n = (jb < 16) ? static_cast<int>(byte & 0x0F) : static_cast<int>(byte >> 4);
      v[k] = __fmul_rn(static_cast<float>(n - 8), d);
    }
  }
  return make_float4(v[0], v[1], v[2], v[3]);
}

struct Ctx {
  const StageDesc *stages;   // shared-memory copy of the stage list
  uint32_t *xsm;
  float *part;
  float *hown;       // this CTA's residual rows
  uint32_t hrow0;    // first residual row this CTA owns (in this rank's row slice)
  uint32_t hrow0g;   // the same row in the whole hidden vector
  uint8_t *ring;
  uint64_t *full, *empty;
  float *red;
  unsigned long long *best_w;
  uint32_t *s_token;
  volatile uint32_t *abort;
  uint32_t j;        // items this warp has consumed (matches its producer lane)
  uint32_t rot;      // item-to-warp rotation (matches the producer)
  uint32_t v_hidden, v_qkv, v_attn, v_act, v_token;   // versions of the tagged vectors
};

// Version of tagged vector b (kept in registers: no indexed arrays).
__device__ __forceinline__ uint32_t ver_of(const Ctx &c, uint32_t b) {
  switch (b) {
    case BUF_HIDDEN: return c.v_hidden;
    case BUF_QKV: return c.v_qkv;
    case BUF_ATTN: return c.v_attn;
    case BUF_ACT: return c.v_act;
    default: return c.v_token;
  }
}
__device__ __forceinline__ void ver_bump(Ctx &c, uint32_t b) {
  switch (b) {
    case BUF_HIDDEN: ++c.v_hidden; break;
    case BUF_QKV: ++c.v_qkv; break;
    case BUF_ATTN: ++c.v_attn; break;
    case BUF_ACT: ++c.v_act; break;
    default: ++c.v_token; break;
  }
}

// XR: float4s of the input per consumer thread (2 covers a 2048-wide input,
// 4 the 6144-wide one).
template <int QT, int PRO, int EPI, bool EMB, int XR>
__device__ __forceinline__ void gemv_stage(const StepParams &P, const StageDesc &sd, Ctx &c, uint32_t token) {
  constexpr int GPU = (QT == ZGPU_Q4_0) ? 2 : 1;
  constexpr int R = 4 * GPU;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t nf4 = sd.in_dim / 4;
  uint32_t u0, u1;
  unit_range(sd.units, &u0, &u1);

  // ---- input: each thread takes its float4s of x, XR at a time (one round
  // covers XR * kNC float4s), waiting for the expected version, for both the
  // sum of squares and the digits.  Within a round all of the thread's words
  // are polled together, so the wait ends one L2 round trip after the last
  // of them is published.
  const unsigned long long *xin = sd.tin;
  const uint32_t vin = EMB ? 0u : ver_of(c, sd.in_buf);
  float ss = 0.f;   // RMSNorm: this thread's sum of squares, its float4s in index order
  for (uint32_t base = 0; base < nf4; base += XR * kNC) {
    float4 xr[XR];
    if (!EMB) {
      ulonglong2 raw[XR][2];
      uint32_t todo = 0;
#pragma unroll
      for (int i = 0; i < XR; ++i) {
        const uint32_t f = base + warp * 32 + lane + i * kNC;
        if (f < nf4) {
          const ulonglong2 *q = reinterpret_cast<const ulonglong2 *>(xin + 4 * f);
          raw[i][0] = __ldcg(q);
          raw[i][1] = __ldcg(q + 1);
          todo |= 1u << i;
        } else {
          raw[i][0] = raw[i][1] = make_ulonglong2(0ull, 0ull);
        }
      }
      auto ready = [&](const ulonglong2 (&r)[2]) {
        return static_cast<uint32_t>(r[0].x >> 32) == vin && static_cast<uint32_t>(r[0].y >> 32) == vin &&
               static_cast<uint32_t>(r[1].x >> 32) == vin && static_cast<uint32_t>(r[1].y >> 32) == vin;
      };
#pragma unroll
      for (int i = 0; i < XR; ++i)
        if ((todo >> i & 1u) && ready(raw[i])) todo &= ~(1u << i);
      if (todo) {
        const uint64_t t0 = globaltimer_ns();
        while (todo) {
#pragma unroll
          for (int i = 0; i < XR; ++i) {
            if (todo >> i & 1u) {
              const ulonglong2 *q =
                  reinterpret_cast<const ulonglong2 *>(xin + 4 * (base + warp * 32 + lane + i * kNC));
              raw[i][0] = __ldcg(q);
              raw[i][1] = __ldcg(q + 1);
            }
          }
#pragma unroll
          for (int i = 0; i < XR; ++i)
            if ((todo >> i & 1u) && ready(raw[i])) todo &= ~(1u << i);
          if (!todo) break;
          if (*c.abort || ld_relaxed_u32(&P.bar[1])) {
            *c.abort = 1;
            break;
          }
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(P.status, ZDEV_ERR_TIMEOUT);
            atomicExch(&P.bar[1], 1u);
            *c.abort = 1;
            break;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < XR; ++i)
        xr[i] = make_float4(__uint_as_float(static_cast<uint32_t>(raw[i][0].x)),
                            __uint_as_float(static_cast<uint32_t>(raw[i][0].y)),
                            __uint_as_float(static_cast<uint32_t>(raw[i][1].x)),
                            __uint_as_float(static_cast<uint32_t>(raw[i][1].y)));
    }
#pragma unroll
    for (int i = 0; i < XR; ++i) {
      const uint32_t f = base + warp * 32 + lane + i * kNC;
      if (EMB) xr[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (f < nf4) {
        if (EMB) {
          xr[i] = embed_f4(P, token, f);
          // the embedding is the residual base of the rows this CTA owns
          const float ev[4] = {xr[i].x, xr[i].y, xr[i].z, xr[i].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t e = 4 * f + k;
            if (e >= c.hrow0g && e - c.hrow0g < P.hown_rows) c.hown[e - c.hrow0g] = ev[k];
          }
        }
      }
    }
    trace(16 + 2 + EPI);
    // RMSNorm (ops.rs:29-52) as y = inv * (W . (x * g)): the digits are taken
    // of x * g right away and the scalar inv = 1/sqrt(mean(x^2) + eps) scales
    // the row sums in the epilogue, so the sum of squares (fixed order: per
    // thread over its float4s, xor-tree in the warp, warps in order) needs no
    // barrier of its own: its per-warp parts cross the image barrier below.
    if (PRO == PRO_RMSNORM) {
#pragma unroll
      for (int i = 0; i < XR; ++i) {
        const float4 t = xr[i];
        ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(t.x, t.x), __fmul_rn(t.y, t.y)),
                                     __fadd_rn(__fmul_rn(t.z, t.z), __fmul_rn(t.w, t.w))));
      }
    }
#pragma unroll
    for (int i = 0; i < XR; ++i) {
      const uint32_t f0 = base + warp * 32 + i * kNC;
      if (f0 >= nf4) break;   // warp-uniform
      const uint32_t f = f0 + lane;
      const bool valid = f < nf4;
      float4 t = xr[i];
      if (PRO == PRO_RMSNORM && valid) {
        const float4 g = reinterpret_cast<const float4 *>(sd.norm_w)[f];
        t.x = __fmul_rn(t.x, g.x);
        t.y = __fmul_rn(t.y, g.y);
        t.z = __fmul_rn(t.z, g.z);
        t.w = __fmul_rn(t.w, g.w);
      }
      digitise_f4<QT>(t, f, valid, c.xsm, sd.bpr, P.xbytes, P.status);
    }
  }
  if (PRO == PRO_RMSNORM) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) c.red[warp] = ss;
  }
  named_bar_sync(kBarConsumers, kNC);
  trace(32 + 2 + EPI);
  trace_cta(0);
  float inv = 1.0f;
  if (PRO == PRO_RMSNORM) {
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) tot = __fadd_rn(tot, c.red[w]);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(sd.in_dim)), P.eps)));
  }

  // ---- items: warp (k + rot) % kNW takes item k of this CTA's list
  const uint32_t nloc = u1 - u0, nitems = nloc * sd.ks;
  const uint32_t first = (warp + kNW - c.rot) % kNW;
  c.rot = (c.rot + nitems) % kNW;
  bool failed = false;
  for (uint32_t k = first; k < nitems; k += kNW) {
    const uint32_t slot = warp * kSlots + (c.j % kSlots);
    trace(64);
    if (!failed && !wait_phase(smem_addr(&c.full[slot]), (c.j / kSlots) & 1, P.status, c.abort)) failed = true;
    trace(80);
    const uint32_t chunk = k % sd.ks;
    const uint32_t b = chunk * kChunkBlocks + lane;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    if (!failed && b < sd.bpr)
      item_rows<QT, GPU>(c.ring + static_cast<size_t>(slot) * kSlotBytes, sd.gbytes,
                         chunk_blocks(sd.bpr, chunk), lane, b, c.xsm, acc);
    __syncwarp();
    trace(96);
    if (lane == 0) mbar_arrive(smem_addr(&c.empty[slot]));
    ++c.j;
    const float v = reduce_scatter<R>(acc, lane);
    if ((lane & (32 / R - 1)) == 0) c.part[k * R + lane / (32 / R)] = v;
  }
  named_bar_sync(kBarConsumers, kNC);
  trace(48);
  trace_cta(1);

  // ---- epilogue: K-chunks in order, then per row
  unsigned long long *xout = sd.tout;
  const uint32_t vout = (EPI == EPI_ARGMAX) ? 0u : ver_of(c, sd.out_buf) + 1;
  // output word of local row `row`: this rank's vector, or (tensor parallel)
  // every rank's copy at the slice's place in the whole vector
  auto put = [&](uint32_t row, unsigned long long w) {
    if (sd.bcast) {
      for (uint32_t d = 0; d < P.world; ++d) P.peer_tv[d * kStepBufs + sd.out_buf][sd.out_row0 + row] = w;
    } else {
      xout[row] = w;
    }
  };
  unsigned long long best = kArgmaxInitKey;
  if (EPI == EPI_SWIGLU) {
    // unit = {gate rows 4u..4u+3, up rows 4u..4u+3}
    for (uint32_t t = tid; t < nloc * 4; t += kNC) {
      const uint32_t ul = t >> 2, r = t & 3;
      float yg = 0.f, yu = 0.f;
      for (uint32_t ch = 0; ch < sd.ks; ++ch) {
        yg += c.part[(ul * sd.ks + ch) * R + r];
        yu += c.part[(ul * sd.ks + ch) * R + 4 + r];
      }
      yg = __fmul_rn(yg, inv);
      yu = __fmul_rn(yu, inv);
      const uint32_t row = (u0 + ul) * 4 + r;
      if (row < sd.rows) put(row, tag_word(ref_silu_mul(yg, yu), vout));
    }
  } else {
    for (uint32_t t = tid; t < nloc * R; t += kNC) {
      const uint32_t ul = t / R, r = t % R;
      float y = 0.f;
      for (uint32_t ch = 0; ch < sd.ks; ++ch) y += c.part[(ul * sd.ks + ch) * R + r];
      if (PRO == PRO_RMSNORM) y = __fmul_rn(y, inv);
      const uint32_t row = (u0 + ul) * R + r;
      if (row < sd.rows) {
        if (EPI == EPI_STORE) {
          put(row, tag_word(y, vout));
        } else if (EPI == EPI_RESADD) {
          const uint32_t hr = row - c.hrow0;   // < hown_rows: this CTA owns the row
          const float h = c.hown[hr] + y;
          c.hown[hr] = h;
          put(row, tag_word(h, vout));
        } else {
          sd.out[row] = y;
          const unsigned long long key = argmax_key(y, sd.out_row0 + row);
          best = key > best ? key : best;
        }
      }
    }
  }
  if (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0) c.best_w[warp] = best;
    named_bar_sync(kBarConsumers, kNC);
    if (tid == 0) {
      unsigned long long b = kArgmaxInitKey;
      for (int w = 0; w < kNW; ++w) b = c.best_w[w] > b ? c.best_w[w] : b;
      if (b != kArgmaxInitKey) atomicMax(P.argmax, b);
    }
  } else {
    ver_bump(c, sd.out_buf);
  }
  trace_cta(2);
  named_bar_sync(kBarConsumers, kNC);
  trace_cta(3);
}

__device__ __forceinline__ void run_gemv(const StepParams &P, const StageDesc &sd, Ctx &c, uint32_t token) {
  const bool emb = (sd.flags & kStageEmbed) != 0;
  const bool wide = sd.in_dim > 2u * 4u * kNC;
  if (sd.quant == ZGPU_Q4_0) {
    if (sd.pro == PRO_RMSNORM) {
      if (sd.epi == EPI_STORE) {
        if (emb) gemv_stage<ZGPU_Q4_0, PRO_RMSNORM, EPI_STORE, true, 2>(P, sd, c, token);
        else gemv_stage<ZGPU_Q4_0, PRO_RMSNORM, EPI_STORE, false, 2>(P, sd, c, token);
      } else if (sd.epi == EPI_SWIGLU) {
        gemv_stage<ZGPU_Q4_0, PRO_RMSNORM, EPI_SWIGLU, false, 2>(P, sd, c, token);
      } else if (sd.epi == EPI_ARGMAX) {
        gemv_stage<ZGPU_Q4_0, PRO_RMSNORM, EPI_ARGMAX, false, 2>(P, sd, c, token);
      }
    } else if (sd.epi == EPI_RESADD) {
      if (wide) gemv_stage<ZGPU_Q4_0, PRO_PLAIN, EPI_RESADD, false, 4>(P, sd, c, token);
      else gemv_stage<ZGPU_Q4_0, PRO_PLAIN, EPI_RESADD, false, 2>(P, sd, c, token);
    }
  } else if (sd.pro == PRO_RMSNORM && sd.epi == EPI_ARGMAX) {
    gemv_stage<ZGPU_Q8_0, PRO_RMSNORM, EPI_ARGMAX, false, 2>(P, sd, c, token);
  }
}

// End of an LM-head step (CTA 0, one thread, after every CTA's argmax has
// arrived): decode the argmax key, apply the non-finite and padding checks of
// lm_head.rs:157-163, record the token, publish it for the next step, reset
// the key and advance the step.
__device__ void finalize(const StepParams &P, uint32_t gstep, uint32_t n_prompt, uint32_t tok_ver,
                         unsigned long long key) {
  StepState *st = P.state;
  const uint32_t idx = argmax_key_index(key);
  const float val = argmax_key_value(key);
  uint32_t err = 0;
  if (!(val > -INFINITY && val < INFINITY)) err |= ZDEV_ERR_LM_NONFINITE;
  else if (idx >= st->vocab_real) err |= ZDEV_ERR_LM_PADDING;
  if (err) {
    atomicOr(P.status, err);
    if (st->first_err_step == 0xFFFFFFFFu) st->first_err_step = gstep;
  }
  if (gstep + 1 >= n_prompt) {
    const uint32_t gi = gstep + 1 - n_prompt;
    if (gi < st->n_gen_cap) P.tokens_out[gi] = idx;
  }
  st->next_token = idx;
  st->last_max = val;
  st->step = gstep + 1;
  *P.argmax = kArgmaxInitKey;
  P.tv[BUF_TOKEN][0] = (static_cast<unsigned long long>(tok_ver) << 32) | idx;
}

__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Tensor parallel LM head (CTA 0, one thread): publish this rank's argmax key
// into slot [rank] of every rank (the key, then the version with release
// semantics), wait (bounded) until every slot of this rank carries `ver`, and
// merge: the larger key wins, i.e. the larger logit and, on ties, the
// smaller vocabulary row, as the one-GPU argmax over the whole vocabulary.
__device__ bool exchange_argmax(const StepParams &P, unsigned long long key, uint32_t ver,
                                unsigned long long *merged) {
  for (uint32_t d = 0; d < P.world; ++d) st_relaxed_sys(&P.peer_arg[d][P.rank].key, key);
  for (uint32_t d = 0; d < P.world; ++d) st_release_sys(&P.peer_arg[d][P.rank].ver, ver);
  ArgSlot *mine = P.peer_arg[P.rank];
  unsigned long long best = kArgmaxInitKey;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t r = 0; r < P.world; ++r) {
    while (ld_acquire_sys(&mine[r].ver) != ver) {
      if (ld_relaxed_u32(&P.bar[1])) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(P.status, ZDEV_ERR_TIMEOUT);
        atomicExch(&P.bar[1], 1u);
        return false;
      }
    }
    const unsigned long long k = ld_relaxed_sys(&mine[r].key);
    best = k > best ? k : best;
  }
  *merged = best;
  return true;
}

// The step's token: a prompt id, the previous step's argmax (waiting for its
// version), or the caller's.  Thread 0 fetches it and shares it through
// shared memory.
__device__ __forceinline__ uint32_t step_token(const StepParams &P, Ctx &c, uint32_t gstep, uint32_t n_prompt) {
  const uint32_t tid = threadIdx.x;
  if (tid == 0) {
    uint32_t token = 0;
    if (P.mode == STEP_FORWARD) {
      token = P.fwd_token;
    } else if (gstep < n_prompt) {
      token = P.prompt[gstep];
    } else {
      const unsigned long long *w = P.tv[BUF_TOKEN];
      const uint32_t want = c.v_token;
      unsigned long long v = __ldcg(w);
      const uint64_t t0 = globaltimer_ns();
      while (static_cast<uint32_t>(v >> 32) != want) {
        __nanosleep(64);
        v = __ldcg(w);
        if (*c.abort || ld_relaxed_u32(&P.bar[1])) {
          *c.abort = 1;
          break;
        }
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          atomicOr(P.status, ZDEV_ERR_TIMEOUT);
          atomicExch(&P.bar[1], 1u);
          *c.abort = 1;
          break;
        }
      }
      token = static_cast<uint32_t>(v);
    }
    if (token >= P.emb_rows) {
      if (blockIdx.x == 0) atomicOr(P.status, ZDEV_ERR_BOUNDS);
      token = 0;
    }
    *c.s_token = token;
  }
  named_bar_sync(kBarConsumers, kNC);
  return *c.s_token;
}

// Consumers never leave the stage loop early: a named barrier would then
// wait for them forever.  After an abort every wait fails at once, so the
// remaining stages run through quickly (their results are discarded: the
// host sees ZDEV_ERR_TIMEOUT).
__device__ __forceinline__ void consumer(const StepParams &P, Ctx &c) {
  const uint32_t tid = threadIdx.x;
  const uint32_t n_prompt = P.state->n_prompt;
  const uint32_t pos_base = P.state->pos_base;
  uint32_t lm_done = 0;
  for (uint32_t i = 0; i < P.n_steps; ++i) {
    const uint32_t gstep = P.step0 + i;
    const uint32_t pos = (P.mode == STEP_FORWARD) ? P.fwd_pos : pos_base + gstep;
    if (runs_fwd(P)) {
      const uint32_t token = step_token(P, c, gstep, n_prompt);
      if (blockIdx.x == 0 && tid == 0) {
        P.state->token = token;
        P.state->pos = pos;
      }
      for (uint32_t s = 0; s < P.n_layer_stages; ++s) {
        const StageDesc &sd = c.stages[s];
        trace(sd.kind == STG_GEMV ? 2 + sd.epi : 1);
        if (sd.kind == STG_GEMV) {
          run_gemv(P, sd, c, token);
        } else {
          if (blockIdx.x < P.n_kv * P.max_splits) {
            AttnParams ap = {};
            ap.q_norm = sd.q_norm;
            ap.k_norm = sd.k_norm;
            ap.inv_freqs = P.inv_freqs;
            ap.kv_layer = P.kv_base + static_cast<size_t>(sd.layer) * 2 * P.kv_block;
            ap.kv_block = P.kv_block;
            ap.max_tokens = P.max_tokens;
            ap.pos_ptr = nullptr;
            ap.pos_value = pos;
            ap.part = P.attn_part;
            ap.counters = P.attn_counters;
            ap.status = P.status;
            ap.n_q = P.n_q;
            ap.n_kv = P.n_kv;
            ap.max_splits = P.max_splits;
            ap.eps = P.eps;
            ap.scale = P.scale;
            ap.qkv_t = P.tv[BUF_QKV];
            ap.out_t = P.tv[BUF_ATTN];
            ap.n_out = P.world > 1 ? P.world : 0;
            ap.out_dst = P.attn_dst;
            ap.ver_in = c.v_qkv;
            ap.ver_out = c.v_attn + 1;
            ap.abort = c.abort;
            ap.gabort = &P.bar[1];
            trace(120);
            attn_decode_block<AttnBar, true, 4, kNW, AttnMark>(ap, blockIdx.x % P.n_kv, blockIdx.x / P.n_kv,
                                                               pos, tid, *reinterpret_cast<StepAttnSmem *>(c.xsm),
                                                               AttnBar(), AttnMark());
          }
          ++c.v_attn;
          // the x image area doubles as the attention's shared memory
          named_bar_sync(kBarConsumers, kNC);
        }
      }
    }
    if (runs_lm(P, gstep, n_prompt)) {
      trace(7);
      run_gemv(P, c.stages[P.lm_stage], c, 0);
      // count this CTA's arrival (its argmax is in), then CTA 0 hands the
      // token on once every CTA has arrived
      named_bar_sync(kBarConsumers, kNC);
      if (tid == 0) red_release_add(&P.bar[0], 1u);
      ++lm_done;
      if (blockIdx.x == 0 && tid == 0) {
        const uint32_t target = lm_done * gridDim.x;
        const uint64_t t0 = globaltimer_ns();
        bool ok = true;
        while (ld_acquire(&P.bar[0]) < target) {
          if (ld_relaxed_u32(&P.bar[1])) {
            ok = false;
            break;
          }
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(P.status, ZDEV_ERR_TIMEOUT);
            atomicExch(&P.bar[1], 1u);
            ok = false;
            break;
          }
        }
        unsigned long long key = __ldcg(P.argmax);
        if (ok && P.world > 1) ok = exchange_argmax(P, key, c.v_token + 1, &key);
        if (ok) finalize(P, gstep, n_prompt, c.v_token + 1, key);
        else *c.abort = 1;
      }
      ++c.v_token;
      trace(0);
    }
  }
}

__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const StepParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kNW];
  __shared__ unsigned long long best_w[kNW];
  __shared__ uint32_t s_abort, s_token;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t *ring = smem + P.ring_off;
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + static_cast<size_t>(kNW) * kSlots * kSlotBytes);
  uint64_t *empty = full + kNW * kSlots;
  // the stage list, read at every stage boundary, lives in shared memory
  // unless it did not fit there
  const StageDesc *stages = P.stages;
  if (P.stages_off != kStagesInGlobal) {
    StageDesc *sm = reinterpret_cast<StageDesc *>(smem + P.stages_off);
    const uint32_t words = P.n_stages * static_cast<uint32_t>(sizeof(StageDesc) / 4);
    const uint32_t *src = reinterpret_cast<const uint32_t *>(P.stages);
    uint32_t *dst = reinterpret_cast<uint32_t *>(sm);
    for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    stages = sm;
  }
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kNW * kSlots; ++i) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), 1);
    }
    fence_barrier_init();
    s_abort = 0;
  }
  __syncthreads();
  volatile uint32_t *abort = &s_abort;
  if (warp == kNW) {
    producer(P, stages, ring, full, empty, lane, abort);
    return;
  }
  Ctx c;
  c.stages = stages;
  c.xsm = reinterpret_cast<uint32_t *>(smem);
  c.part = reinterpret_cast<float *>(smem + P.xbytes);
  c.hown = reinterpret_cast<float *>(smem + P.hown_off);
  c.ring = ring;
  c.full = full;
  c.empty = empty;
  c.red = red;
  c.best_w = best_w;
  c.s_token = &s_token;
  c.abort = abort;
  c.j = 0;
  c.rot = 0;
  c.v_hidden = P.ver[BUF_HIDDEN];
  c.v_qkv = P.ver[BUF_QKV];
  c.v_attn = P.ver[BUF_ATTN];
  c.v_act = P.ver[BUF_ACT];
  c.v_token = P.ver[BUF_TOKEN];
  {
    // residual rows: the rows of this CTA's units in the residual-adding
    // stages (the same units in all of them)
    uint32_t u0, u1;
    unit_range(P.hown_units, &u0, &u1);
    c.hrow0 = u0 * 8;
    c.hrow0g = P.hid_row0 + u0 * 8;
  }
  trace_begin();
  consumer(P, c);
  trace_end();
  if (threadIdx.x == 0 && ld_relaxed_u32(&P.bar[1])) *abort = 1;
}

}  // namespace

bool step_geometry(const StageDesc *stages, uint32_t n, uint32_t grid, StepParams *p) {
  size_t xbytes = sizeof(StepAttnSmem);
  size_t part = 0;
  uint32_t hunits = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const StageDesc &s = stages[i];
    if (s.kind != STG_GEMV) continue;
    if (s.in_dim % 32 != 0 || s.bpr * 32 != s.in_dim) return false;
    const size_t img = static_cast<size_t>(s.bpr) * 128;
    if (img > xbytes) xbytes = img;
    const size_t upc = (static_cast<size_t>(s.units) + grid - 1) / grid;
    const size_t pb = upc * s.ks * 4 * s.gpu * sizeof(float);
    if (pb > part) part = pb;
    const uint64_t cb = chunk_bytes(s.quant, s.bpr < kChunkBlocks ? s.bpr : kChunkBlocks);
    if (s.gbytes * (s.gpu - 1) + cb > kSlotBytes) return false;
    if (s.gstride % 16 != 0 || s.gbytes % 16 != 0) return false;
    if (s.epi == EPI_RESADD) {
      // residual rows stay in shared memory: every residual-adding stage
      // must split the same 8-row units over the CTAs
      if (s.quant != ZGPU_Q4_0 || (hunits && hunits != s.units)) return false;
      hunits = s.units;
    }
  }
  if (!hunits) return false;
  const size_t hown = ((static_cast<size_t>(hunits) + grid - 1) / grid * 8 * sizeof(float) + 127) & ~size_t(127);
  xbytes = (xbytes + 127) & ~size_t(127);
  part = (part + 127) & ~size_t(127);
  const size_t hown_off = xbytes + part;
  const size_t stages_off = hown_off + hown;
  size_t stages_bytes = (static_cast<size_t>(n) * sizeof(StageDesc) + 127) & ~size_t(127);
  const size_t ring_bytes = static_cast<size_t>(kNW) * kSlots * kSlotBytes + 2 * kNW * kSlots * 8;
  // the stage list is copied to shared memory where it fits, else read from
  // global memory (one broadcast read per stage)
  if (stages_off + stages_bytes + ring_bytes > kStepDynSmemMax) stages_bytes = 0;
  const size_t ring_off = stages_off + stages_bytes;
  const size_t smem = ring_off + ring_bytes;
  if (smem > kStepDynSmemMax) return false;
  p->xbytes = static_cast<uint32_t>(xbytes);
  p->part_bytes = static_cast<uint32_t>(part);
  p->hown_off = static_cast<uint32_t>(hown_off);
  p->stages_off = stages_bytes ? static_cast<uint32_t>(stages_off) : kStagesInGlobal;
  p->n_stages = n;
  p->hown_units = hunits;
  p->hown_rows = static_cast<uint32_t>((static_cast<size_t>(hunits) + grid - 1) / grid * 8);
  p->ring_off = static_cast<uint32_t>(ring_off);
  p->smem_bytes = static_cast<uint32_t>(smem);
  return true;
}

cudaError_t step_setup() {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, step_kernel);
  if (e != cudaSuccess) return e;
  if (fa.sharedSizeBytes + kStepDynSmemMax > kStepSmemMax) return cudaErrorInvalidValue;
  e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kStepDynSmemMax));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(step_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared);
}

uint32_t step_max_grid(int sm_count) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel, kStepThreads,
                                                    kStepDynSmemMax) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return per_sm >= 1 ? static_cast<uint32_t>(sm_count) : 0u;
}

cudaError_t step_launch(const StepParams &p, uint32_t grid, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, p);
}

}  // namespace zgpu

#ifdef ZGPU_STEP_TRACE
// Profiling builds only: copy out and reset the stage timeline.
extern "C" int zgpu_debug_cta_trace(unsigned long long *out, int cap, uint32_t *smid, int n_smid) {
  if (cudaMemcpyFromSymbol(out, zgpu::g_cta_trace, static_cast<size_t>(cap) * 8) != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(smid, zgpu::g_cta_smid, static_cast<size_t>(n_smid) * 4) != cudaSuccess) return -1;
  return 0;
}

extern "C" int zgpu_debug_step_trace(unsigned long long *out, int cap) {
  uint32_t n = 0;
  if (cudaMemcpyFromSymbol(&n, zgpu::g_step_trace_n, sizeof(n)) != cudaSuccess) return -1;
  if (n > static_cast<uint32_t>(cap)) n = static_cast<uint32_t>(cap);
  if (n && cudaMemcpyFromSymbol(out, zgpu::g_step_trace, n * sizeof(unsigned long long)) != cudaSuccess)
    return -1;
  const uint32_t zero = 0;
  cudaMemcpyToSymbol(zgpu::g_step_trace_n, &zero, sizeof(zero));
  return static_cast<int>(n);
}
#endif
