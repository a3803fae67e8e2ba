// mla.cu — multi-head latent attention (MLA) decode over the compressed
// latent cache.
//
// Replaces mla_attention_single_token (crates/zero-llm-inference/src/mla.rs:
// 122-414) between the projections.  The reference re-expands every cached
// latent through kv_b twice per step (O(t * kv_b) work).  Here the
// projection is absorbed instead:
//   score_h,t = q_nope_h . (W_kn_h c_t) + q_rope_h . k_rope_t
//             = (W_kn_h^T q_nope_h) . c_t + q_rope_h . k_rope_t,
//   out_h     = sum_t p_h,t (W_v_h c_t) = W_v_h (sum_t p_h,t c_t),
// so attention reads only the cache's [kv_lora | rope] rows, all heads share
// every row (one CTA walks a token range for all heads), and the V
// projection is one GEMV per head after the merge (the segmented GEMV of
// gemv.cu).  The sums are reordered relative to the reference: results agree
// to f32 rounding, not bit for bit.
//
//   mla_prep   CTA h < n_heads: stage head h's k_nope rows of kv_b (one
//              contiguous slab of group streams) in shared memory, rotate
//              q_rope (mla.rs:229-252 RoPE), q_abs_h = W_kn_h^T q_nope_h;
//              last CTA: rmsnorm(c_kv, kv_a_norm), optional k_rope RMS norm,
//              RoPE at pos, append [c_kv | k_rope] at pos (store_compressed,
//              kv_cache.rs:318).
//   mla_attn   CTA (s, sequence, head group): tokens [S s, S s + S) of
//              [0, pos] (S = split_tokens, a multiple of 16) for up to 16
//              heads, 4 heads per warp, lane per 32nd latent column: online
//              softmax (scale 1 / sqrt(nope + rope)) over 8-token groups,
//              partial (m, l, sum p c) per head.
//   mla_merge  CTA per (head, 128 columns): merge the splits in order into
//              ctx_h; a non-finite max or a sum <= 0 raises the
//              NumericalInstability status (attention.rs:48-84).
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "gemv_body.cuh"
#include "internal.h"
#include "layout.h"
#include "mla.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr size_t kMlaSlabMax = 200 * 1024;
constexpr uint32_t kMlaAttnWarps = 4;                       // 4 heads per warp
constexpr uint32_t kMlaHeadsPerCta = 4 * kMlaAttnWarps;     // grid dimension z covers the rest
constexpr uint32_t kMlaSubTokens = 16;                      // rows per staged buffer
constexpr uint32_t kMlaMergeThreads = 128;

__device__ __forceinline__ uint32_t mla_pos(const MlaParams &p) {
  return p.seq_pos ? __ldcg(p.seq_pos + blockIdx.y) : (p.pos_ptr ? *p.pos_ptr : p.pos_value);
}

// This CTA's sequence (grid dimension y) of a batch: the per-sequence
// vectors and cache of MlaParams rebased on it.
__device__ __forceinline__ MlaParams mla_seq(const MlaParams &p0) {
  MlaParams p = p0;
  const uint32_t b = blockIdx.y;
  if (b) {
    const uint32_t R = p.kv_lora, RD = p.rope;
    p.kv_a += static_cast<size_t>(b) * p.kv_a_stride;
    p.q += static_cast<size_t>(b) * p.q_stride;
    p.q_abs += static_cast<size_t>(b) * p.n_heads * R;
    p.q_pe += static_cast<size_t>(b) * p.n_heads * RD;
    p.ctx += static_cast<size_t>(b) * p.n_heads * R;
    p.part += static_cast<size_t>(b) * p.n_heads * p.max_splits * (R + 2);
  }
  if (p.seq_cache) p.cache = p.seq_cache[b] + p.layer_off;
  return p;
}

// Fixed-order block sum over kMlaPrepThreads threads (thread partials, xor
// tree per warp, warps in order).  Every thread gets the total.
__device__ __forceinline__ float prep_block_sum(float v, float *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (uint32_t w = 0; w < kMlaPrepThreads / 32; ++w) s = __fadd_rn(s, red[w]);
  return s;
}

__device__ __forceinline__ void rope_pair(float x0, float x1, float theta, float *o0, float *o1) {
  float s, c;
  sincosf(theta, &s, &c);
  *o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  *o1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void __launch_bounds__(kMlaPrepThreads) mla_prep_kernel(const MlaParams p0) {
  const MlaParams p = mla_seq(p0);
  extern __shared__ __align__(16) uint8_t slab[];
  __shared__ float qn[kMlaMaxNope];
  __shared__ float red[kMlaPrepThreads / 32];
  __shared__ float kr[kMlaMaxRope];
  pdl_launch_dependents();
  const uint32_t tid = threadIdx.x;
  const uint32_t R = p.kv_lora, RD = p.rope, half = RD / 2;
  if (blockIdx.x < p.n_heads) {
    const uint32_t h = blockIdx.x;
    // the weights do not depend on the previous kernel: stage the head's
    // k_nope rows (one contiguous run of group streams) with one bulk copy
    __shared__ __align__(8) uint64_t sbar;
    const uint32_t sb = smem_addr(&sbar);
    if (tid == 0) {
      mbar_init(sb, 1);
      fence_barrier_init();
      mbar_arrive_expect_tx(sb, p.slab_bytes);
      bulk_copy_g2s(smem_addr(slab), p.kb + static_cast<uint64_t>(h * p.kb_head_rows / 4) * p.kb_gstride,
                    p.slab_bytes, sb);
    }
    pdl_wait();
    const uint32_t pos = mla_pos(p);
    const float *qh = p.q + static_cast<size_t>(h) * (p.nope + RD);
    for (uint32_t i = tid; i < p.nope; i += kMlaPrepThreads) qn[i] = __ldcg(qh + i);
    if (tid < half) {
      const float theta = __fmul_rn(static_cast<float>(pos), p.inv_freqs[tid]);
      float o0, o1;
      rope_pair(__ldcg(qh + p.nope + tid), __ldcg(qh + p.nope + tid + half), theta, &o0, &o1);
      p.q_pe[static_cast<size_t>(h) * RD + tid] = o0;
      p.q_pe[static_cast<size_t>(h) * RD + tid + half] = o1;
    }
    __syncthreads();
    if (!mbar_wait(sb, 0, p.status)) return;   // timed out: the status word says so
    const uint32_t bpr = R / 32;
    for (uint32_t c = tid; c < R; c += kMlaPrepThreads) {
      const uint32_t b = c >> 5, e = c & 31;
      const uint64_t sc_off = scale_entry(p.kb_quant, bpr, b);
      float acc = 0.f;
      if (p.kb_quant == ZGPU_Q4_0) {
#pragma unroll 4
        for (uint32_t i = 0; i < p.nope; ++i) {
          const uint8_t *g = slab + static_cast<size_t>(i >> 2) * p.kb_gstride;
          const uint32_t r = i & 3;
          const float d = h2f(*reinterpret_cast<const uint16_t *>(g + sc_off + 2 * r));
          const uint8_t byte = g[plane_entry(ZGPU_Q4_0, bpr, b, r) + (e & 15)];
          const int n = (e < 16) ? (byte & 0x0F) : (byte >> 4);
          acc = fmaf(qn[i], __fmul_rn(d, static_cast<float>(n - 8)), acc);
        }
      } else {
#pragma unroll 4
        for (uint32_t i = 0; i < p.nope; ++i) {
          const uint8_t *g = slab + static_cast<size_t>(i >> 2) * p.kb_gstride;
          const uint32_t r = i & 3;
          const float d = h2f(*reinterpret_cast<const uint16_t *>(g + sc_off + 2 * r));
          const int8_t q = static_cast<int8_t>(g[plane_entry(ZGPU_Q8_0, bpr, b, 2 * r + (e >> 4)) + (e & 15)]);
          acc = fmaf(qn[i], __fmul_rn(d, static_cast<float>(q)), acc);
        }
      }
      p.q_abs[static_cast<size_t>(h) * R + c] = acc;
    }
    return;
  }
  // ---- the latent CTA: normalise, rotate and append this token's row ----
  pdl_wait();
  const uint32_t pos = mla_pos(p);
  if (pos >= p.max_tokens) {
    if (tid == 0) atomicOr(p.status, ZDEV_ERR_BOUNDS);
    return;
  }
  float *row = p.cache + static_cast<size_t>(pos) * (R + RD);
  float ss = 0.f;
  for (uint32_t i = tid; i < R; i += kMlaPrepThreads) {
    const float v = __ldcg(p.kv_a + i);
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  const float tot = prep_block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(R)), p.eps)));
  for (uint32_t i = tid; i < R; i += kMlaPrepThreads)
    row[i] = __fmul_rn(__fmul_rn(__ldcg(p.kv_a + i), inv), p.kv_a_norm[i]);
  float v = tid < RD ? __ldcg(p.kv_a + R + tid) : 0.f;
  if (p.k_norm) {   // mla.rs:180-196
    const float t2 = prep_block_sum(__fmul_rn(v, v), red);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(t2, static_cast<float>(RD)), p.eps));
    const float inv2 = __fdiv_rn(1.0f, rms);
    if (tid < RD) v = __fmul_rn(__fmul_rn(v, inv2), p.k_norm[tid]);
  }
  if (tid < RD) kr[tid] = v;
  __syncthreads();
  if (tid < half) {
    const float theta = __fmul_rn(static_cast<float>(pos), p.inv_freqs[tid]);
    float o0, o1;
    rope_pair(kr[tid], kr[tid + half], theta, &o0, &o1);
    row[R + tid] = o0;
    row[R + tid + half] = o1;
  }
}

// Split-K attention over the latent cache.  CTA (split, sequence, head
// group): tokens [split * split_tokens, ...) of [0, pos] for up to 16 heads;
// warp w takes 4 heads, lane j holds latent columns j + 32 i of their
// queries and context sums.  The split's rows stream through two 16-token
// shared-memory buffers (bulk copies, double-buffered); scores are formed 8
// tokens at a time: each lane accumulates partial dots of 4 heads x 8 tokens
// and one reduce-scatter leaves lane l with head l / 8, token l % 8 (31
// shuffles per 32 scores).  Online softmax per 8-token group, then the
// context update from the same shared rows.  Output per head: the split's
// (sum p c, m, l).
// Any supported geometry; kv_lora 512 / rope 64 (DeepSeek2's) runs
// mla_attn512_kernel below.
__global__ void __launch_bounds__(32 * kMlaAttnWarps, 2) mla_attn_kernel(const MlaParams p0) {
  const MlaParams p = mla_seq(p0);
  extern __shared__ __align__(128) float chunk[];   // [2][kMlaSubTokens][kv_lora + rope]
  __shared__ __align__(8) uint64_t bar[2];
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = mla_pos(p);
  if (pos >= p.max_tokens) return;   // reported by mla_prep
  const uint32_t R = p.kv_lora, RD = p.rope, nr = R / 32, row = R + RD;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t split = blockIdx.x, st = p.split_tokens;
  const uint32_t t0 = split * st;
  if (t0 > pos) return;   // beyond the context: the merge reads only the splits up to pos
  const uint32_t t1 = min(t0 + st, pos + 1);
  const uint32_t nsub = (t1 - t0 + kMlaSubTokens - 1) / kMlaSubTokens;
  const uint32_t bars[2] = {smem_addr(&bar[0]), smem_addr(&bar[1])};
  // thread 0: sub-tile i (contiguous rows; row * 4 is a multiple of 16) into buffer i & 1
  auto issue = [&](uint32_t i) {
    const uint32_t ts = t0 + i * kMlaSubTokens, nt = min(kMlaSubTokens, t1 - ts);
    mbar_arrive_expect_tx(bars[i & 1], nt * row * 4);
    bulk_copy_g2s(smem_addr(chunk + (i & 1) * kMlaSubTokens * row), p.cache + static_cast<size_t>(ts) * row,
                  nt * row * 4, bars[i & 1]);
  };
  if (threadIdx.x == 0) {
    mbar_init(bars[0], 1);
    mbar_init(bars[1], 1);
    fence_barrier_init();
    issue(0);
    if (nsub > 1) issue(1);
  }
  // this warp's heads; a head beyond n_heads has zero queries and is not written
  const uint32_t hb = blockIdx.z * kMlaHeadsPerCta + warp * 4;
  float qa[4][16], qp[4][2], acc[4][16];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const bool hv = hb + h < p.n_heads;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      acc[h][j] = 0.f;
      qa[h][j] = (hv && j < static_cast<int>(nr)) ? __ldcg(p.q_abs + static_cast<size_t>(hb + h) * R + lane + 32 * j)
                                                   : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
      qp[h][j] = (hv && lane + 32 * j < RD) ? __ldcg(p.q_pe + static_cast<size_t>(hb + h) * RD + lane + 32 * j) : 0.f;
  }
  // one cached row's latent values (cv) and rope values (cr) for this lane
  auto load_row = [&](const float *ct, float (&cv)[16], float (&cr)[2]) {
#pragma unroll
    for (int j = 0; j < 16; ++j) cv[j] = (j < static_cast<int>(nr)) ? ct[lane + 32 * j] : 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) cr[j] = (lane + 32 * j < RD) ? ct[R + lane + 32 * j] : 0.f;
  };
  // lane l's score slot: head l / 8, token l % 8 of each group
  float m_mine = -INFINITY, l_mine = 0.f;
  __syncthreads();   // barriers initialised before anyone waits on them
  bool ok = true;
  for (uint32_t i = 0; i < nsub; ++i) {
    ok = __syncthreads_and(ok && mbar_wait(bars[i & 1], (i >> 1) & 1, p.status));
    if (!ok) {
      // a copy that did not land: wait (bounded) for the other buffer's
      // copy in flight, then report through a NaN sum
      if (threadIdx.x == 0) {
        mbar_wait(bars[i & 1], (i >> 1) & 1, p.status);
        if (i + 1 < nsub) mbar_wait(bars[(i + 1) & 1], ((i + 1) >> 1) & 1, p.status);
      }
      break;
    }
    const float *ch = chunk + (i & 1) * kMlaSubTokens * row;
    const uint32_t nt = min(kMlaSubTokens, t1 - (t0 + i * kMlaSubTokens));
    for (uint32_t g = 0; g < nt; g += 8) {
      const uint32_t ng = min(8u, nt - g);
      float v[32];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (static_cast<uint32_t>(k) < ng) {
          float cv[16], cr[2];
          load_row(ch + (g + k) * row, cv, cr);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float d = fmaf(qp[h][0], cr[0], 0.f);
            d = fmaf(qp[h][1], cr[1], d);
#pragma unroll
            for (int j = 0; j < 16; ++j) d = fmaf(qa[h][j], cv[j], d);
            v[h * 8 + k] = d;
          }
        } else {
#pragma unroll
          for (int h = 0; h < 4; ++h) v[h * 8 + k] = 0.f;
        }
      }
      const float dot = reduce_scatter<32>(v, lane);
      const float s = ((lane & 7) < ng) ? __fmul_rn(dot, p.scale) : -INFINITY;
      // this head's group max, new running max, rescale and weights
      float gm = s;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, off));
      const float mn = fmaxf(m_mine, gm);
      const float corr = (m_mine == mn) ? 1.0f : expf(m_mine - mn);
      const float pe = (s == -INFINITY) ? 0.0f : expf(s - mn);
      float ps = pe;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, off));
      l_mine = fmaf(l_mine, corr, ps);
      m_mine = mn;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float c = __shfl_sync(0xffffffffu, corr, h * 8);
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[h][j] = __fmul_rn(acc[h][j], c);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (static_cast<uint32_t>(k) < ng) {
          float pk[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) pk[h] = __shfl_sync(0xffffffffu, pe, h * 8 + k);
          float cv[16], cr[2];
          load_row(ch + (g + k) * row, cv, cr);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (j < static_cast<int>(nr)) {
#pragma unroll
              for (int h = 0; h < 4; ++h) acc[h][j] = fmaf(pk[h], cv[j], acc[h][j]);
            }
          }
        }
      }
    }
    __syncthreads();   // every warp is done with buffer i & 1
    if (threadIdx.x == 0 && i + 2 < nsub) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + 2);
    }
  }
  if (!ok) l_mine = __uint_as_float(0x7fc00000u);   // a failed copy surfaces as NumericalInstability
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    if (hb + h >= p.n_heads) break;
    float *pp = p.part + (static_cast<size_t>(hb + h) * p.max_splits + split) * (R + 2);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (j < static_cast<int>(nr)) pp[lane + 32 * j] = acc[h][j];
    if (lane == static_cast<uint32_t>(h) * 8) {
      pp[R] = m_mine;
      pp[R + 1] = l_mine;
    }
  }
}

// The DeepSeek2 geometry (kv_lora 512, rope 64) on packed f32x2 arithmetic:
// the structure of mla_attn_kernel, with lane l holding latent columns
// 128 i + 4 l .. + 3 as two column pairs each, so that a score's dot product
// runs as two interleaved chains (even and odd columns, added at the end) of
// fma.rn.f32x2 and the context update as one fma.rn.f32x2 per column pair;
// each lane rounds as the scalar instruction.
__global__ void __launch_bounds__(32 * kMlaAttnWarps, 2) mla_attn512_kernel(const MlaParams p0) {
  const MlaParams p = mla_seq(p0);
  extern __shared__ __align__(128) float chunk[];   // [2][kMlaSubTokens][576]
  __shared__ __align__(8) uint64_t bar[2];
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = mla_pos(p);
  if (pos >= p.max_tokens) return;   // reported by mla_prep
  constexpr uint32_t R = 512, RD = 64, row = R + RD;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t split = blockIdx.x, st = p.split_tokens;
  const uint32_t t0 = split * st;
  if (t0 > pos) return;   // beyond the context: the merge reads only the splits up to pos
  const uint32_t t1 = min(t0 + st, pos + 1);
  const uint32_t nsub = (t1 - t0 + kMlaSubTokens - 1) / kMlaSubTokens;
  const uint32_t bars[2] = {smem_addr(&bar[0]), smem_addr(&bar[1])};
  auto issue = [&](uint32_t i) {
    const uint32_t ts = t0 + i * kMlaSubTokens, nt = min(kMlaSubTokens, t1 - ts);
    mbar_arrive_expect_tx(bars[i & 1], nt * row * 4);
    bulk_copy_g2s(smem_addr(chunk + (i & 1) * kMlaSubTokens * row), p.cache + static_cast<size_t>(ts) * row,
                  nt * row * 4, bars[i & 1]);
  };
  if (threadIdx.x == 0) {
    mbar_init(bars[0], 1);
    mbar_init(bars[1], 1);
    fence_barrier_init();
    issue(0);
    if (nsub > 1) issue(1);
  }
  const uint32_t hb = blockIdx.z * kMlaHeadsPerCta + warp * 4;
  // column pair i of this lane: columns 128 (i / 2) + 4 lane + 2 (i % 2) + {0, 1}
  float2 qa[4][8], acc[4][8], qp[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const bool hv = hb + h < p.n_heads;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const float4 q4 = hv ? __ldcg(reinterpret_cast<const float4 *>(p.q_abs + static_cast<size_t>(hb + h) * R) +
                                    32 * jj + lane)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
      qa[h][2 * jj] = make_float2(q4.x, q4.y);
      qa[h][2 * jj + 1] = make_float2(q4.z, q4.w);
      acc[h][2 * jj] = acc[h][2 * jj + 1] = make_float2(0.f, 0.f);
    }
    qp[h] = hv ? __ldcg(reinterpret_cast<const float2 *>(p.q_pe + static_cast<size_t>(hb + h) * RD) + lane)
               : make_float2(0.f, 0.f);
  }
  auto load_row = [&](const float *ct, float2 (&cv)[8], float2 &cr) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const float4 c4 = reinterpret_cast<const float4 *>(ct)[32 * jj + lane];
      cv[2 * jj] = make_float2(c4.x, c4.y);
      cv[2 * jj + 1] = make_float2(c4.z, c4.w);
    }
    cr = reinterpret_cast<const float2 *>(ct + R)[lane];
  };
  float m_mine = -INFINITY, l_mine = 0.f;
  __syncthreads();   // barriers initialised before anyone waits on them
  bool ok = true;
  for (uint32_t i = 0; i < nsub; ++i) {
    ok = __syncthreads_and(ok && mbar_wait(bars[i & 1], (i >> 1) & 1, p.status));
    if (!ok) {
      if (threadIdx.x == 0) {
        mbar_wait(bars[i & 1], (i >> 1) & 1, p.status);
        if (i + 1 < nsub) mbar_wait(bars[(i + 1) & 1], ((i + 1) >> 1) & 1, p.status);
      }
      break;
    }
    const float *ch = chunk + (i & 1) * kMlaSubTokens * row;
    const uint32_t nt = min(kMlaSubTokens, t1 - (t0 + i * kMlaSubTokens));
    for (uint32_t g = 0; g < nt; g += 8) {
      const uint32_t ng = min(8u, nt - g);
      float v[32];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (static_cast<uint32_t>(k) < ng) {
          float2 cv[8], cr;
          load_row(ch + (g + k) * row, cv, cr);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float2 d = mul2_rn(qp[h], cr);
#pragma unroll
            for (int c = 0; c < 8; ++c) d = fma2_rn(qa[h][c], cv[c], d);
            v[h * 8 + k] = __fadd_rn(d.x, d.y);
          }
        } else {
#pragma unroll
          for (int h = 0; h < 4; ++h) v[h * 8 + k] = 0.f;
        }
      }
      const float dot = reduce_scatter<32>(v, lane);
      const float s = ((lane & 7) < ng) ? __fmul_rn(dot, p.scale) : -INFINITY;
      float gm = s;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, off));
      const float mn = fmaxf(m_mine, gm);
      const float corr = (m_mine == mn) ? 1.0f : expf(m_mine - mn);
      const float pe = (s == -INFINITY) ? 0.0f : expf(s - mn);
      float ps = pe;
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, off));
      l_mine = fmaf(l_mine, corr, ps);
      m_mine = mn;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float c = __shfl_sync(0xffffffffu, corr, h * 8);
        const float2 c2 = make_float2(c, c);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[h][j] = mul2_rn(acc[h][j], c2);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (static_cast<uint32_t>(k) < ng) {
          float2 cv[8], cr;
          load_row(ch + (g + k) * row, cv, cr);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float pk = __shfl_sync(0xffffffffu, pe, h * 8 + k);
            const float2 pk2 = make_float2(pk, pk);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[h][j] = fma2_rn(pk2, cv[j], acc[h][j]);
          }
        }
      }
    }
    __syncthreads();   // every warp is done with buffer i & 1
    if (threadIdx.x == 0 && i + 2 < nsub) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + 2);
    }
  }
  if (!ok) l_mine = __uint_as_float(0x7fc00000u);   // a failed copy surfaces as NumericalInstability
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    if (hb + h >= p.n_heads) break;
    float *pp = p.part + (static_cast<size_t>(hb + h) * p.max_splits + split) * (R + 2);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t c0 = 128u * (j / 2) + 4u * lane + 2u * (j % 2);
      pp[c0] = acc[h][j].x;
      pp[c0 + 1] = acc[h][j].y;
    }
    if (lane == static_cast<uint32_t>(h) * 8) {
      pp[R] = m_mine;
      pp[R + 1] = l_mine;
    }
  }
}

__global__ void __launch_bounds__(kMlaMergeThreads) mla_merge_kernel(const MlaParams p0) {
  const MlaParams p = mla_seq(p0);
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = mla_pos(p);
  if (pos >= p.max_tokens) return;
  const uint32_t R = p.kv_lora;
  const uint32_t nq = (R + kMlaMergeThreads - 1) / kMlaMergeThreads;
  const uint32_t h = blockIdx.x / nq;
  const uint32_t c = (blockIdx.x % nq) * kMlaMergeThreads + threadIdx.x;
  const uint32_t nsplit = pos / p.split_tokens + 1;
  const float *pb = p.part + static_cast<size_t>(h) * p.max_splits * (R + 2);
  float M = -INFINITY;
  for (uint32_t s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(pb + static_cast<size_t>(s) * (R + 2) + R));
  float L = 0.f, A = 0.f;
  for (uint32_t s = 0; s < nsplit; ++s) {
    const float *ps = pb + static_cast<size_t>(s) * (R + 2);
    const float ms = __ldcg(ps + R);
    const float f = (ms == -INFINITY) ? 0.0f : expf(ms - M);
    L = fmaf(f, __ldcg(ps + R + 1), L);
    if (c < R) A = fmaf(f, __ldcg(ps + c), A);
  }
  const bool bad = !(fabsf(M) <= FLT_MAX) || !(L > 0.0f) || !(L <= FLT_MAX);
  if (bad && c == 0) atomicOr(p.status, ZDEV_ERR_NUMERICAL);
  if (c < R) p.ctx[static_cast<size_t>(h) * R + c] = bad ? 0.0f : __fdiv_rn(A, L);
}

}  // namespace

cudaError_t mla_setup() {
  cudaError_t e = cudaFuncSetAttribute(mla_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kMlaSlabMax));
  if (e != cudaSuccess) return e;
  const int smem = static_cast<int>(2 * kMlaSubTokens * (kMlaMaxLatent + kMlaMaxRope) * sizeof(float));
  e = cudaFuncSetAttribute(mla_attn512_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(mla_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

cudaError_t launch_mla_prep(const MlaParams &mp, const LaunchCfg &lc) {
  if (mp.kv_lora == 0 || mp.kv_lora % 32 || mp.kv_lora > kMlaMaxLatent || mp.rope % 2 ||
      mp.rope > kMlaMaxRope || mp.nope == 0 || mp.nope % 4 || mp.nope > kMlaMaxNope ||
      mp.kb_head_rows % 4 || mp.n_heads == 0 || (mp.kv_lora + mp.rope) % 4 ||
      (mp.kb_quant != ZGPU_Q4_0 && mp.kb_quant != ZGPU_Q8_0))
    return cudaErrorInvalidValue;
  MlaParams p = mp;
  const uint64_t slab = static_cast<uint64_t>(p.nope / 4) * p.kb_gstride;
  if (slab > kMlaSlabMax || p.kb_gstride % 16) return cudaErrorInvalidValue;
  p.slab_bytes = static_cast<uint32_t>(slab);
  cudaLaunchAttribute attr[1];
  const uint32_t ns = p.n_seq > 1 ? p.n_seq : 1;
  if (ns > 1 && (!p.seq_cache || !p.seq_pos)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(p.n_heads + 1, ns), dim3(kMlaPrepThreads), slab, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, mla_prep_kernel, p);
}

cudaError_t launch_mla_attention(const MlaParams &mp, const LaunchCfg &lc) {
  MlaParams p = mp;
  if (p.split_tokens == 0) p.split_tokens = kMlaSplitTokens;
  if (p.kv_lora == 0 || p.kv_lora % 32 || p.kv_lora > kMlaMaxLatent || p.rope > kMlaMaxRope ||
      (p.kv_lora + p.rope) % 4 || p.split_tokens % kMlaSplitTokens ||
      p.max_splits < mla_max_splits(p.max_tokens) || p.n_heads == 0)
    return cudaErrorInvalidValue;
  const uint32_t hg = (p.n_heads + kMlaHeadsPerCta - 1) / kMlaHeadsPerCta;
  const uint32_t warps = hg > 1 ? kMlaAttnWarps : (p.n_heads + 3) / 4;
  cudaLaunchAttribute attr[1];
  const size_t chunk = 2 * static_cast<size_t>(kMlaSubTokens) * (p.kv_lora + p.rope) * sizeof(float);
  const uint32_t ns = p.n_seq > 1 ? p.n_seq : 1;
  if (ns > 1 && (!p.seq_cache || !p.seq_pos)) return cudaErrorInvalidValue;
  const uint32_t splits = (p.max_tokens + p.split_tokens - 1) / p.split_tokens;
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(splits, ns, hg), dim3(32 * warps), chunk, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  cudaError_t e = (p.kv_lora == 512 && p.rope == 64) ? cudaLaunchKernelEx(&cfg, mla_attn512_kernel, p)
                                                      : cudaLaunchKernelEx(&cfg, mla_attn_kernel, p);
  if (e != cudaSuccess) return e;
  const uint32_t nq = (p.kv_lora + kMlaMergeThreads - 1) / kMlaMergeThreads;
  cudaLaunchAttribute attr2[1];
  cudaLaunchConfig_t cfg2 = make_launch_cfg(dim3(p.n_heads * nq, ns), dim3(kMlaMergeThreads), 0, lc, attr2);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg2, mla_merge_kernel, p);
}

}  // namespace zgpu
