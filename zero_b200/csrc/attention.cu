// attention.cu — single-token GQA decode attention over the f32 KV cache.
//
// Replaces, for one layer, steps 2-5 of gqa_attention_single_token_avx512
// (kernel/src/inference_avx512.rs:1612-1800) and of the scalar
// gqa_attention_single_token_dispatch (crates/zero-llm-inference/src/
// attention.rs:344-425):
//   per-head QK RMSNorm (ops.rs:29) -> RoPE with the per-token sin/cos LUT
//   (trig.rs:148, :192) -> KvCache::store_kv (kv_cache.rs:139) -> scores
//   q.k / sqrt(head_dim) -> softmax (attention.rs:48) -> sum_t p_t v_t.
//
// Grid: (n_kv_heads, max_splits), 256 threads.  Split s of kv-head h covers a
// contiguous range of at most kSplitTokens tokens, so a short context (every
// step of BASELINE config 0) runs as one CTA per kv-head with no cross-CTA
// combine; longer contexts use flash-decoding partials (running max m, sum l,
// unnormalised o) merged in split order by the last CTA of the kv-head to
// arrive (arrival counter, reset in place so CUDA-graph replays stay valid).
//   * warp j < G normalises and rotates q-head h*G+j, warp G the new k, all
//     with shuffles (lane l holds dims 4l..4l+3; the RoPE partner of dim i is
//     dim i+64, held by lane l^16); the (cos, sin) pairs come from the
//     reference's own sincos polynomial;
//   * the CTA whose range holds the current position appends k and v;
//   * warps stride over tokens for the scores and for sum_t p_t v_t, then
//     reduce across warps through shared memory in fixed order.
// Softmax errors follow the reference: a non-finite max or a non-positive /
// non-finite sum flags ZDEV_ERR_NUMERICAL.
#include <cfloat>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr int HD = 128;          // head_dim handled by this kernel
constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kMaxGqa = 4;
constexpr int kSplitTokens = 256;

// QK-norm (rmsnorm over one head, ops.rs:29) then RoPE (trig.rs:192) for the
// four dims 4l..4l+3 a lane holds; every lane of the warp participates.
__device__ __forceinline__ float4 norm_rope_lane(float4 x, float4 w, float eps, const float *cs,
                                                 const float *sn, uint32_t lane) {
  float ss = __fadd_rn(__fadd_rn(__fmul_rn(x.x, x.x), __fmul_rn(x.y, x.y)),
                       __fadd_rn(__fmul_rn(x.z, x.z), __fmul_rn(x.w, x.w)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(HD)), eps)));
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
  const uint32_t i0 = (4 * lane) & (HD / 2 - 1);
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

__global__ void __launch_bounds__(kThreads) attn_decode_kernel(const AttnParams p) {
  __shared__ float cs[HD / 2], sn[HD / 2];
  __shared__ __align__(16) float qs[kMaxGqa][HD];
  __shared__ __align__(16) float kn[HD], vn[HD];
  __shared__ float sc[kMaxGqa][kSplitTokens];
  __shared__ __align__(16) float opart[kWarps][kMaxGqa][HD];
  __shared__ float stat[kMaxGqa][2];
  __shared__ uint32_t s_last;

  pdl_launch_dependents();
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t kvh = blockIdx.x, split = blockIdx.y;
  const uint32_t G = p.n_q / p.n_kv;
  pdl_wait();
  const uint32_t pos = p.pos_ptr ? *p.pos_ptr : p.pos_value;
  if (pos >= p.max_tokens) {
    if (tid == 0 && split == 0 && kvh == 0) atomicOr(p.status, ZDEV_ERR_BOUNDS);
    return;
  }
  const uint32_t total = pos + 1;
  const uint32_t nact = (total + kSplitTokens - 1) / kSplitTokens;
  const uint32_t t0 = split * kSplitTokens;
  if (split >= nact) return;
  const uint32_t t1 = min(t0 + kSplitTokens, total);
  const uint32_t ntok = t1 - t0;
  const uint32_t qd = p.n_q * HD, kvd = p.n_kv * HD;

  // RoPE LUT for this position (rope_sincos_lut_avx512, trig.rs:148).
  if (tid < HD / 2) {
    float s, c;
    ref_sincos(__fmul_rn(static_cast<float>(pos), p.inv_freqs[tid]), &s, &c);
    cs[tid] = c;
    sn[tid] = s;
  }
  __syncthreads();
  if (warp < G) {
    const float4 x = *reinterpret_cast<const float4 *>(p.qkv + (kvh * G + warp) * HD + 4 * lane);
    const float4 w = *reinterpret_cast<const float4 *>(p.q_norm + 4 * lane);
    *reinterpret_cast<float4 *>(&qs[warp][4 * lane]) = norm_rope_lane(x, w, p.eps, cs, sn, lane);
  } else if (warp == G) {
    const float4 x = *reinterpret_cast<const float4 *>(p.qkv + qd + kvh * HD + 4 * lane);
    const float4 w = *reinterpret_cast<const float4 *>(p.k_norm + 4 * lane);
    *reinterpret_cast<float4 *>(&kn[4 * lane]) = norm_rope_lane(x, w, p.eps, cs, sn, lane);
  } else if (warp == G + 1) {
    *reinterpret_cast<float4 *>(&vn[4 * lane]) =
        *reinterpret_cast<const float4 *>(p.qkv + qd + kvd + kvh * HD + 4 * lane);
  }
  __syncthreads();

  float *kc = p.kv_layer, *vc = p.kv_layer + p.kv_block;
  if (t1 == total && tid < HD) {
    // KvCache::store_kv at `pos` (kv_cache.rs:175-181).
    kc[static_cast<size_t>(pos) * kvd + kvh * HD + tid] = kn[tid];
    vc[static_cast<size_t>(pos) * kvd + kvh * HD + tid] = vn[tid];
  }

  // Scores: warp w takes tokens t0+w, t0+w+8, ...; lane holds 4 dims.
  float4 q[kMaxGqa];
#pragma unroll
  for (int j = 0; j < kMaxGqa; ++j)
    q[j] = (j < static_cast<int>(G)) ? *reinterpret_cast<const float4 *>(&qs[j][4 * lane])
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t t = t0 + warp; t < t1; t += kWarps) {
    if (!ZDEV_CHECK(static_cast<uint64_t>(t + 1) * kvd <= p.kv_block && t - t0 < kSplitTokens,
                    p.status, 10, t, kvh))
      break;
    const float4 kk = (t == pos) ? *reinterpret_cast<const float4 *>(&kn[4 * lane])
                                 : *reinterpret_cast<const float4 *>(
                                       kc + static_cast<size_t>(t) * kvd + kvh * HD + 4 * lane);
#pragma unroll
    for (int j = 0; j < kMaxGqa; ++j) {
      if (j >= static_cast<int>(G)) break;
      float d = __fmaf_rn(q[j].w, kk.w,
                          __fmaf_rn(q[j].z, kk.z, __fmaf_rn(q[j].y, kk.y, __fmul_rn(q[j].x, kk.x))));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      if (lane == 0) sc[j][t - t0] = __fmul_rn(d, p.scale);
    }
  }
  __syncthreads();

  // Split-local softmax statistics: warp j owns q-head j.
  if (warp < G) {
    float m = -INFINITY;
    for (uint32_t t = lane; t < ntok; t += 32) m = fmaxf(m, sc[warp][t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float l = 0.f;
    for (uint32_t t = lane; t < ntok; t += 32) {
      const float e = expf(sc[warp][t] - m);
      sc[warp][t] = e;
      l += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (lane == 0) {
      stat[warp][0] = m;
      stat[warp][1] = l;
    }
  }
  __syncthreads();

  // sum_t e_t v_t: warp w takes tokens t0+w, t0+w+8, ...; lane holds 4 dims.
  float4 o[kMaxGqa];
#pragma unroll
  for (int j = 0; j < kMaxGqa; ++j) o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t t = t0 + warp; t < t1; t += kWarps) {
    const float4 vv = (t == pos) ? *reinterpret_cast<const float4 *>(&vn[4 * lane])
                                 : *reinterpret_cast<const float4 *>(
                                       vc + static_cast<size_t>(t) * kvd + kvh * HD + 4 * lane);
#pragma unroll
    for (int j = 0; j < kMaxGqa; ++j) {
      if (j >= static_cast<int>(G)) break;
      const float e = sc[j][t - t0];
      o[j].x = __fmaf_rn(e, vv.x, o[j].x);
      o[j].y = __fmaf_rn(e, vv.y, o[j].y);
      o[j].z = __fmaf_rn(e, vv.z, o[j].z);
      o[j].w = __fmaf_rn(e, vv.w, o[j].w);
    }
  }
#pragma unroll
  for (int j = 0; j < kMaxGqa; ++j)
    if (j < static_cast<int>(G)) *reinterpret_cast<float4 *>(&opart[warp][j][4 * lane]) = o[j];
  __syncthreads();

  // Cross-warp sum in warp order; thread (j, d) finalises head j, dim d.
  const bool single = (nact == 1);
  for (uint32_t idx = tid; idx < G * HD; idx += kThreads) {
    const uint32_t j = idx / HD, d = idx % HD;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) acc += opart[w][j][d];
    const float m = stat[j][0], l = stat[j][1];
    const uint32_t qh = kvh * G + j;
    if (single) {
      if (d == 0 && (!(m > -INFINITY && m < INFINITY) || !(l > 0.f) || !(l < INFINITY)))
        atomicOr(p.status, ZDEV_ERR_NUMERICAL);
      p.out[qh * HD + d] = __fdiv_rn(acc, l);
    } else {
      if (!ZDEV_CHECK(qh < p.n_q && split < p.max_splits, p.status, 11, qh, split)) continue;
      float *pp = p.part + (static_cast<size_t>(qh) * p.max_splits + split) * (HD + 2);
      pp[d] = acc;
      if (d == 0) {
        pp[HD] = m;
        pp[HD + 1] = l;
      }
    }
  }
  if (single) return;

  // Publish the partials, then let the last CTA of this kv-head merge them.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&p.counters[kvh], 1u);
    s_last = (prev == nact - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (uint32_t idx = tid; idx < G * HD; idx += kThreads) {
    const uint32_t j = idx / HD, d = idx % HD;
    const uint32_t qh = kvh * G + j;
    const float *base = p.part + static_cast<size_t>(qh) * p.max_splits * (HD + 2);
    float M = -INFINITY;
    for (uint32_t s = 0; s < nact; ++s) M = fmaxf(M, __ldcg(base + s * (HD + 2) + HD));
    float L = 0.f, O = 0.f;
    for (uint32_t s = 0; s < nact; ++s) {
      const float f = expf(__ldcg(base + s * (HD + 2) + HD) - M);
      L = __fmaf_rn(f, __ldcg(base + s * (HD + 2) + HD + 1), L);
      O = __fmaf_rn(f, __ldcg(base + s * (HD + 2) + d), O);
    }
    if (d == 0 && (!(M > -INFINITY && M < INFINITY) || !(L > 0.f) || !(L < INFINITY)))
      atomicOr(p.status, ZDEV_ERR_NUMERICAL);
    p.out[qh * HD + d] = __fdiv_rn(O, L);
  }
  if (tid == 0) p.counters[kvh] = 0u;
}

}  // namespace

uint32_t attention_max_splits(uint32_t max_tokens) {
  return (max_tokens + kSplitTokens - 1) / kSplitTokens;
}

cudaError_t attention_setup() {
  return cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared);
}

cudaError_t launch_attention(const AttnParams &ap, const LaunchCfg &lc) {
  if (ap.n_q % ap.n_kv != 0 || ap.n_q / ap.n_kv > kMaxGqa || ap.n_q / ap.n_kv + 2 > kWarps)
    return cudaErrorInvalidValue;
  if (ap.max_splits < attention_max_splits(ap.max_tokens)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ap.n_kv, ap.max_splits);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = lc.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, attn_decode_kernel, ap);
}

}  // namespace zgpu
