// attn_body.cuh — single-token GQA decode attention for one (kv head, split),
// shared by the standalone kernel (attention.cu) and the persistent step
// kernel (step.cu).
//
// Replaces, for one layer, steps 2-5 of gqa_attention_single_token_avx512
// (kernel/src/inference_avx512.rs:1612-1800) and of the scalar
// gqa_attention_single_token_dispatch (crates/zero-llm-inference/src/
// attention.rs:344-425):
//   per-head QK RMSNorm (ops.rs:29) -> RoPE with the per-token sin/cos LUT
//   (trig.rs:148, :192) -> KvCache::store_kv (kv_cache.rs:139) -> scores
//   q.k / sqrt(head_dim) -> softmax (attention.rs:48) -> sum_t p_t v_t.
//
// 256 threads (8 warps) run one (kv head h, split s); split s covers a
// contiguous range of at most kAttnSplitTokens tokens, so a short context
// runs as one split with no cross-CTA combine; longer contexts use
// flash-decoding partials (running max m, sum l, unnormalised o) merged in
// split order by the last split of the kv head to arrive (arrival counter,
// reset in place so that later launches and graph replays stay valid).
//   * warp j < G normalises and rotates q head h*G+j, warp G the new k, all
//     with shuffles (lane l holds dims 4l..4l+3; the RoPE partner of dim i is
//     dim i+64, held by lane l^16); the (cos, sin) pairs come from the
//     reference's own sincos polynomial;
//   * the split whose range holds the current position appends k and v;
//   * each warp takes runs of kAttnUnroll tokens (8, or 4 where registers
//     are scarcer), loads their K and V rows together and keeps a running max, sum
//     and unnormalised output per q head (online softmax); the warps' states
//     are merged in warp order through shared memory.
// Softmax errors follow the reference: a non-finite max or a non-positive /
// non-finite sum flags ZDEV_ERR_NUMERICAL.  Every read of data another CTA
// may have written during the same kernel (projections, cache rows,
// partials) goes through L2 (ld.global.cg).
#pragma once

#include <cfloat>

#include "common.cuh"
#include "ops.h"

namespace zgpu {

constexpr int kAttnHd = 128;          // head_dim handled by this code
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kAttnMaxGqa = 4;
constexpr int kAttnSplitTokens = 256;
constexpr int kAttnUnrollMax = 8;        // tokens per warp per round (K and V rows in flight)

template <int NW>
struct AttnSmemT {
  float cs[kAttnHd / 2], sn[kAttnHd / 2];
  __align__(16) float qs[kAttnMaxGqa][kAttnHd];
  __align__(16) float kn[kAttnHd];
  __align__(16) float vn[kAttnHd];
  __align__(16) float opart[NW][kAttnMaxGqa][kAttnHd];
  float wm[NW][kAttnMaxGqa], wl[NW][kAttnMaxGqa];   // per-warp running max / sum
  float wf[NW][kAttnMaxGqa];                         // merge weights exp(m_w - max)
  float wL[kAttnMaxGqa];                             // merged sums
  uint32_t s_last;
};
using AttnSmem = AttnSmemT<kAttnWarps>;

// QK-norm (rmsnorm over one head, ops.rs:29) then RoPE (trig.rs:192) for the
// four dims 4l..4l+3 a lane holds; every lane of the warp participates.
__device__ __forceinline__ float4 attn_norm_rope_lane(float4 x, float4 w, float eps, const float *cs,
                                                      const float *sn, uint32_t lane) {
  float ss = __fadd_rn(__fadd_rn(__fmul_rn(x.x, x.x), __fmul_rn(x.y, x.y)),
                       __fadd_rn(__fmul_rn(x.z, x.z), __fmul_rn(x.w, x.w)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(kAttnHd)), eps)));
  float4 n;
  n.x = __fmul_rn(__fmul_rn(x.x, inv), w.x);
  n.y = __fmul_rn(__fmul_rn(x.y, inv), w.y);
  n.z = __fmul_rn(__fmul_rn(x.z, inv), w.z);
  n.w = __fmul_rn(__fmul_rn(x.w, inv), w.w);
  float4 p;   // partner dims (i + 64 or i - 64) from lane ^ 16
  p.x = __shfl_xor_sync(0xffffffffu, n.x, 16);
  p.y = __shfl_xor_sync(0xffffffffu, n.y, 16);
  p.z = __shfl_xor_sync(0xffffffffu, n.z, 16);
  p.w = __shfl_xor_sync(0xffffffffu, n.w, 16);
  const uint32_t i0 = (4 * lane) & (kAttnHd / 2 - 1);
  const bool upper = lane >= 16;   // dims 64..127: y' = x*s + y*c with x = partner
  float4 r;
  if (!upper) {
    r.x = __fmaf_rn(n.x, cs[i0 + 0], -__fmul_rn(p.x, sn[i0 + 0]));
    r.y = __fmaf_rn(n.y, cs[i0 + 1], -__fmul_rn(p.y, sn[i0 + 1]));
    r.z = __fmaf_rn(n.z, cs[i0 + 2], -__fmul_rn(p.z, sn[i0 + 2]));
    r.w = __fmaf_rn(n.w, cs[i0 + 3], -__fmul_rn(p.w, sn[i0 + 3]));
  } else {
    r.x = __fmaf_rn(p.x, sn[i0 + 0], __fmul_rn(n.x, cs[i0 + 0]));
    r.y = __fmaf_rn(p.y, sn[i0 + 1], __fmul_rn(n.y, cs[i0 + 1]));
    r.z = __fmaf_rn(p.z, sn[i0 + 2], __fmul_rn(n.z, cs[i0 + 2]));
    r.w = __fmaf_rn(p.w, sn[i0 + 3], __fmul_rn(n.w, cs[i0 + 3]));
  }
  return r;
}

// One (kv head, split) of the attention.  tid in [0, 256); bar() is a
// barrier over exactly those 256 threads.  Every branch that skips work is
// uniform over the 256 threads.
// Projection words of the q/k/v heads: plain floats, or (TAGGED) tagged
// words polled until they carry ver_in.
template <bool TAGGED>
__device__ __forceinline__ float4 attn_load_proj(const AttnParams &p, uint32_t off) {
  if (!TAGGED) return __ldcg(reinterpret_cast<const float4 *>(p.qkv + off));
  float4 v;
  tag_wait4(p.qkv_t + off, p.ver_in, &v, p.status, p.abort, p.gabort);
  return v;
}

template <bool TAGGED>
__device__ __forceinline__ void attn_store_out(const AttnParams &p, uint32_t i, float v) {
  if (TAGGED) {
    const unsigned long long w = tag_word(v, p.ver_out);
    if (p.n_out == 0) {
      p.out_t[i] = w;
    } else {
      for (uint32_t d = 0; d < p.n_out; ++d) p.out_dst[d][i] = w;
    }
  } else {
    p.out[i] = v;
  }
}

// Mark: optional timeline hook (event id) for profiling builds of the caller.
struct AttnNoMark {
  __device__ __forceinline__ void operator()(uint32_t) const {}
};

// FAST (the batched decode kernel): the run's scores of all q heads reduced
// together (one butterfly for four values per token) and exp by __expf; the
// result differs from the default path in the last bits of the sums.
template <class Bar, bool TAGGED = false, int kAttnUnroll = kAttnUnrollMax, int NW = kAttnWarps,
          class Mark = AttnNoMark, bool FAST = false>
__device__ __forceinline__ void attn_decode_block(const AttnParams &p, uint32_t kvh, uint32_t split,
                                                  uint32_t pos, uint32_t tid, AttnSmemT<NW> &sm, Bar bar,
                                                  Mark mark = Mark()) {
  constexpr uint32_t kThreads = 32 * NW;
  const uint32_t warp = tid >> 5, lane = tid & 31;
  const uint32_t G = p.n_q / p.n_kv;
  if (pos >= p.max_tokens) {
    if (tid == 0 && split == 0 && kvh == 0) atomicOr(p.status, ZDEV_ERR_BOUNDS);
    return;
  }
  const uint32_t total = pos + 1;
  const uint32_t nact = (total + kAttnSplitTokens - 1) / kAttnSplitTokens;
  const uint32_t t0 = split * kAttnSplitTokens;
  if (split >= nact) return;
  const uint32_t t1 = min(t0 + kAttnSplitTokens, total);
  const uint32_t qd = p.n_q * kAttnHd, kvd = p.n_kv * kAttnHd;
  float *kc = p.kv_layer, *vc = p.kv_layer + p.kv_block;

  // The cached rows of tokens before `pos` do not depend on this step: the
  // warp's first run of K and V rows is loaded before the projections are
  // waited for, so that round trip overlaps the wait.  The current token's
  // row is patched in from shared memory once it exists.
  float4 kk[kAttnUnroll], vv[kAttnUnroll];
  auto load_run = [&](uint32_t tb) {
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const uint32_t t = tb + u;
      kk[u] = vv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < t1 && t != pos &&
          ZDEV_CHECK(static_cast<uint64_t>(t + 1) * kvd <= p.kv_block && t - t0 < kAttnSplitTokens, p.status,
                     10, t, kvh)) {
        const size_t row = static_cast<size_t>(t) * kvd + kvh * kAttnHd;
        kk[u] = __ldcg(reinterpret_cast<const float4 *>(kc + row) + lane);
        vv[u] = __ldcg(reinterpret_cast<const float4 *>(vc + row) + lane);
      }
    }
  };
  uint32_t tb = t0 + warp * kAttnUnroll;
  load_run(tb);

  // RoPE LUT for this position (rope_sincos_lut_avx512, trig.rs:148).
  if (tid < kAttnHd / 2) {
    float s, c;
    ref_sincos(__fmul_rn(static_cast<float>(pos), p.inv_freqs[tid]), &s, &c);
    sm.cs[tid] = c;
    sm.sn[tid] = s;
  }
  bar();
  if (warp < G) {
    const float4 x = attn_load_proj<TAGGED>(p, (kvh * G + warp) * kAttnHd + 4 * lane);
    const float4 w = *reinterpret_cast<const float4 *>(p.q_norm + 4 * lane);
    *reinterpret_cast<float4 *>(&sm.qs[warp][4 * lane]) = attn_norm_rope_lane(x, w, p.eps, sm.cs, sm.sn, lane);
  } else if (warp == G) {
    const float4 x = attn_load_proj<TAGGED>(p, qd + kvh * kAttnHd + 4 * lane);
    const float4 w = *reinterpret_cast<const float4 *>(p.k_norm + 4 * lane);
    *reinterpret_cast<float4 *>(&sm.kn[4 * lane]) = attn_norm_rope_lane(x, w, p.eps, sm.cs, sm.sn, lane);
  } else if (warp == G + 1) {
    *reinterpret_cast<float4 *>(&sm.vn[4 * lane]) = attn_load_proj<TAGGED>(p, qd + kvd + kvh * kAttnHd + 4 * lane);
  }
  bar();
  mark(1);

  if (t1 == total && tid < kAttnHd) {
    // KvCache::store_kv at `pos` (kv_cache.rs:175-181).
    kc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + tid] = sm.kn[tid];
    vc[static_cast<size_t>(pos) * kvd + kvh * kAttnHd + tid] = sm.vn[tid];
  }

  // Online softmax over this warp's runs of kAttnUnroll tokens; lane holds
  // dims 4l..4l+3 of q, k, v and of the running output.
  float4 q[kAttnMaxGqa], o[kAttnMaxGqa];
  float m[kAttnMaxGqa], l[kAttnMaxGqa];
#pragma unroll
  for (int j = 0; j < kAttnMaxGqa; ++j) {
    q[j] = (j < static_cast<int>(G)) ? *reinterpret_cast<const float4 *>(&sm.qs[j][4 * lane])
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
    o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    m[j] = -INFINITY;
    l[j] = 0.f;
  }
  for (; tb < t1; tb += NW * kAttnUnroll) {
    if (tb + kAttnUnroll > pos && tb <= pos) {   // the run holds the current token
#pragma unroll
      for (int u = 0; u < kAttnUnroll; ++u) {
        if (tb + u == pos) {
          kk[u] = *reinterpret_cast<const float4 *>(&sm.kn[4 * lane]);
          vv[u] = *reinterpret_cast<const float4 *>(&sm.vn[4 * lane]);
        }
      }
    }
    if constexpr (FAST) {
      static_assert(kAttnMaxGqa == 4, "the butterfly reduces four heads");
      // per token: lane l holds the partial dots of the four heads over its
      // 4 dims; after exchanging pairs (xor 16), singles (xor 8) and three
      // more rounds, lanes 8(2a + b).. hold the full dot of head 2a + b,
      // which is then broadcast
      float sc4[kAttnMaxGqa][kAttnUnroll];
      const bool hi = lane & 16, bt = lane & 8;
#pragma unroll
      for (int u = 0; u < kAttnUnroll; ++u) {
        float d[kAttnMaxGqa];
#pragma unroll
        for (int j = 0; j < kAttnMaxGqa; ++j)
          d[j] = __fmaf_rn(q[j].w, kk[u].w, __fmaf_rn(q[j].z, kk[u].z, __fmaf_rn(q[j].y, kk[u].y, __fmul_rn(q[j].x, kk[u].x))));
        const float r0 = __shfl_xor_sync(0xffffffffu, hi ? d[0] : d[2], 16);
        const float r1 = __shfl_xor_sync(0xffffffffu, hi ? d[1] : d[3], 16);
        const float a0 = (hi ? d[2] : d[0]) + r0, a1 = (hi ? d[3] : d[1]) + r1;
        float c = (bt ? a1 : a0) + __shfl_xor_sync(0xffffffffu, bt ? a0 : a1, 8);
        c += __shfl_xor_sync(0xffffffffu, c, 4);
        c += __shfl_xor_sync(0xffffffffu, c, 2);
        c += __shfl_xor_sync(0xffffffffu, c, 1);
#pragma unroll
        for (int j = 0; j < kAttnMaxGqa; ++j) {
          const float dj = __shfl_sync(0xffffffffu, c, (j >> 1) * 16 + (j & 1) * 8);
          sc4[j][u] = (tb + u < t1) ? __fmul_rn(dj, p.scale) : -INFINITY;
        }
      }
#pragma unroll
      for (int j = 0; j < kAttnMaxGqa; ++j) {
        if (j >= static_cast<int>(G)) break;
        float mx = m[j];
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) mx = fmaxf(mx, sc4[j][u]);
        const float corr = __expf(m[j] - mx);
        float lj = l[j] * corr;
        float4 oj = make_float4(o[j].x * corr, o[j].y * corr, o[j].z * corr, o[j].w * corr);
#pragma unroll
        for (int u = 0; u < kAttnUnroll; ++u) {
          const float e = (tb + u < t1) ? __expf(sc4[j][u] - mx) : 0.f;
          lj += e;
          oj.x = __fmaf_rn(e, vv[u].x, oj.x);
          oj.y = __fmaf_rn(e, vv[u].y, oj.y);
          oj.z = __fmaf_rn(e, vv[u].z, oj.z);
          oj.w = __fmaf_rn(e, vv[u].w, oj.w);
        }
        m[j] = mx;
        l[j] = lj;
        o[j] = oj;
      }
    } else
#pragma unroll
    for (int j = 0; j < kAttnMaxGqa; ++j) {
      if (j >= static_cast<int>(G)) break;
      float sc[kAttnUnroll];
      float mx = m[j];
#pragma unroll
      for (int u = 0; u < kAttnUnroll; ++u) {
        float d = __fmaf_rn(q[j].w, kk[u].w,
                            __fmaf_rn(q[j].z, kk[u].z, __fmaf_rn(q[j].y, kk[u].y, __fmul_rn(q[j].x, kk[u].x))));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
        sc[u] = (tb + u < t1) ? __fmul_rn(d, p.scale) : -INFINITY;
        mx = fmaxf(mx, sc[u]);
      }
      const float corr = expf(m[j] - mx);
      float lj = l[j] * corr;
      float4 oj = make_float4(o[j].x * corr, o[j].y * corr, o[j].z * corr, o[j].w * corr);
#pragma unroll
      for (int u = 0; u < kAttnUnroll; ++u) {
        const float e = (tb + u < t1) ? expf(sc[u] - mx) : 0.f;
        lj += e;
        oj.x = __fmaf_rn(e, vv[u].x, oj.x);
        oj.y = __fmaf_rn(e, vv[u].y, oj.y);
        oj.z = __fmaf_rn(e, vv[u].z, oj.z);
        oj.w = __fmaf_rn(e, vv[u].w, oj.w);
      }
      m[j] = mx;
      l[j] = lj;
      o[j] = oj;
    }
    if (tb + NW * kAttnUnroll < t1) load_run(tb + NW * kAttnUnroll);
  }
  mark(2);
#pragma unroll
  for (int j = 0; j < kAttnMaxGqa; ++j) {
    if (j >= static_cast<int>(G)) break;
    *reinterpret_cast<float4 *>(&sm.opart[warp][j][4 * lane]) = o[j];
    if (lane == 0) {
      sm.wm[warp][j] = m[j];
      sm.wl[warp][j] = l[j];
    }
  }
  bar();

  // Merge the warps' states in warp order; thread (j, d) finalises head j,
  // dim d.  Warps without tokens carry m = -inf, l = 0, o = 0.  The merge
  // weights exp(m_w - max) and the merged sum depend only on the head: one
  // thread per (warp, head) computes each weight, one per head the sum.
  const bool single = (nact == 1);
  if (tid < NW * G) {
    const uint32_t w = tid / G, j = tid % G;
    float mm = -INFINITY;
#pragma unroll
    for (int v = 0; v < NW; ++v) mm = fmaxf(mm, sm.wm[v][j]);
    sm.wf[w][j] = (sm.wm[w][j] == -INFINITY) ? 0.f : expf(sm.wm[w][j] - mm);
    if (w == 0) sm.wL[j] = mm;   // the max, read back below
  }
  bar();
  if (tid < G) {
    float ll = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) ll = __fmaf_rn(sm.wf[w][tid], sm.wl[w][tid], ll);
    sm.wm[0][tid] = sm.wL[tid];   // keep the max for the split partials
    sm.wL[tid] = ll;
  }
  bar();
  for (uint32_t idx = tid; idx < G * kAttnHd; idx += kThreads) {
    const uint32_t j = idx / kAttnHd, d = idx % kAttnHd;
    const float mm = sm.wm[0][j], ll = sm.wL[j];
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) acc = __fmaf_rn(sm.wf[w][j], sm.opart[w][j][d], acc);
    const uint32_t qh = kvh * G + j;
    if (single) {
      if (d == 0 && (!(mm > -INFINITY && mm < INFINITY) || !(ll > 0.f) || !(ll < INFINITY)))
        atomicOr(p.status, ZDEV_ERR_NUMERICAL);
      attn_store_out<TAGGED>(p, qh * kAttnHd + d, __fdiv_rn(acc, ll));
    } else {
      if (!ZDEV_CHECK(qh < p.n_q && split < p.max_splits, p.status, 11, qh, split)) continue;
      float *pp = p.part + (static_cast<size_t>(qh) * p.max_splits + split) * (kAttnHd + 2);
      pp[d] = acc;
      if (d == 0) {
        pp[kAttnHd] = mm;
        pp[kAttnHd + 1] = ll;
      }
    }
  }
  mark(3);
  if (single) return;

  // Publish the partials, then let the last split of this kv head merge them.
  __threadfence();
  bar();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&p.counters[kvh], 1u);
    sm.s_last = (prev == nact - 1) ? 1u : 0u;
  }
  bar();
  if (!sm.s_last) return;
  __threadfence();
  for (uint32_t idx = tid; idx < G * kAttnHd; idx += kThreads) {
    const uint32_t j = idx / kAttnHd, d = idx % kAttnHd;
    const uint32_t qh = kvh * G + j;
    const float *base = p.part + static_cast<size_t>(qh) * p.max_splits * (kAttnHd + 2);
    float M = -INFINITY;
    for (uint32_t s = 0; s < nact; ++s) M = fmaxf(M, __ldcg(base + s * (kAttnHd + 2) + kAttnHd));
    float L = 0.f, O = 0.f;
    for (uint32_t s = 0; s < nact; ++s) {
      const float f = expf(__ldcg(base + s * (kAttnHd + 2) + kAttnHd) - M);
      L = __fmaf_rn(f, __ldcg(base + s * (kAttnHd + 2) + kAttnHd + 1), L);
      O = __fmaf_rn(f, __ldcg(base + s * (kAttnHd + 2) + d), O);
    }
    if (d == 0 && (!(M > -INFINITY && M < INFINITY) || !(L > 0.f) || !(L < INFINITY)))
      atomicOr(p.status, ZDEV_ERR_NUMERICAL);
    attn_store_out<TAGGED>(p, qh * kAttnHd + d, __fdiv_rn(O, L));
  }
  if (tid == 0) p.counters[kvh] = 0u;
}

}  // namespace zgpu
