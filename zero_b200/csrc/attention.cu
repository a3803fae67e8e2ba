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
// Grid: (n_kv_heads, max_splits).  Split s of kv-head h covers a contiguous
// token range; its CTA recomputes the normalised, rotated q of the GQA group
// (gqa q-heads share the kv-head's K/V reads) and the new k, scores its
// tokens, and writes a flash-decoding partial (running max m, sum l, and the
// unnormalised o) to scratch.  The last CTA of the kv-head to finish
// (arrival counter, reset in place so CUDA-graph replays stay valid) merges
// the partials in split order.  The CTA whose range holds the current
// position appends k and v to the cache.  Softmax errors follow the
// reference: a non-finite max or a non-positive / non-finite sum flags
// ZDEV_ERR_NUMERICAL.
#include <cfloat>

#include "common.cuh"
#include "internal.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr int HD = 128;          // head_dim handled by this kernel
constexpr int kMaxGqa = 8;
constexpr int kMaxSplitTokens = 64;

// Fixed-order block sum over 128 threads (4 warps).
__device__ __forceinline__ float block_sum128(float v, float *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  return ((red[0] + red[1]) + red[2]) + red[3];
}

// rmsnorm over one 128-wide head held one value per thread, then RoPE
// rotation of the pair (i, i+64) with the LUT; result written to dst.
__device__ __forceinline__ void norm_rope(float x, const float *w, float eps, const float *cs,
                                          const float *sn, float *tmp, float *dst, float *red) {
  const float ss = block_sum128(__fmul_rn(x, x), red);
  const float mean = __fdiv_rn(ss, static_cast<float>(HD));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  const int i = threadIdx.x;
  tmp[i] = __fmul_rn(__fmul_rn(x, inv), w[i]);
  __syncthreads();
  if (i < HD / 2) {
    const float a = tmp[i], bb = tmp[i + HD / 2];
    dst[i] = __fmaf_rn(a, cs[i], -__fmul_rn(bb, sn[i]));
    dst[i + HD / 2] = __fmaf_rn(a, sn[i], __fmul_rn(bb, cs[i]));
  }
  __syncthreads();
}

__global__ void __launch_bounds__(HD) attn_decode_kernel(const AttnParams p) {
  __shared__ float cs[HD / 2], sn[HD / 2];
  __shared__ float qs[kMaxGqa][HD];
  __shared__ float ks_[HD], vs_[HD], tmp[HD];
  __shared__ float sc[kMaxGqa][kMaxSplitTokens];
  __shared__ float red[4];
  __shared__ uint32_t s_last;

  pdl_launch_dependents();
  pdl_wait();

  const uint32_t tid = threadIdx.x;
  const uint32_t kvh = blockIdx.x, split = blockIdx.y;
  const uint32_t G = p.n_q / p.n_kv;
  const uint32_t pos = *p.pos_ptr;
  if (pos >= p.max_tokens) {
    if (tid == 0 && split == 0 && kvh == 0) atomicOr(p.status, ZDEV_ERR_BOUNDS);
    return;
  }
  const uint32_t total = pos + 1;
  uint32_t ts = (total + p.max_splits - 1) / p.max_splits;
  const uint32_t nact = (total + ts - 1) / ts;
  const uint32_t t0 = split * ts;
  if (t0 >= total) return;
  const uint32_t t1 = min(t0 + ts, total);
  const uint32_t qd = p.n_q * HD, kvd = p.n_kv * HD;

  // RoPE LUT for this position (rope_sincos_lut_avx512, trig.rs:148).
  if (tid < HD / 2) {
    float s, c;
    ref_sincos(__fmul_rn(static_cast<float>(pos), p.inv_freqs[tid]), &s, &c);
    cs[tid] = c;
    sn[tid] = s;
  }
  __syncthreads();

  for (uint32_t j = 0; j < G; ++j) {
    const uint32_t qh = kvh * G + j;
    norm_rope(p.qkv[qh * HD + tid], p.q_norm, p.eps, cs, sn, tmp, qs[j], red);
  }
  norm_rope(p.qkv[qd + kvh * HD + tid], p.k_norm, p.eps, cs, sn, tmp, ks_, red);
  vs_[tid] = p.qkv[qd + kvd + kvh * HD + tid];
  __syncthreads();

  float *kc = p.kv_layer, *vc = p.kv_layer + p.kv_block;
  if (t1 == total) {
    // KvCache::store_kv at `pos` (kv_cache.rs:175-181).
    kc[static_cast<size_t>(pos) * kvd + kvh * HD + tid] = ks_[tid];
    vc[static_cast<size_t>(pos) * kvd + kvh * HD + tid] = vs_[tid];
  }

  // Scores: warp w takes tokens t0+w, t0+w+4, ...; lane holds 4 dims.
  const uint32_t warp = tid >> 5, lane = tid & 31;
  for (uint32_t t = t0 + warp; t < t1; t += 4) {
    float4 kk;
    if (t == pos) {
      kk = *reinterpret_cast<const float4 *>(&ks_[4 * lane]);
    } else {
      kk = *reinterpret_cast<const float4 *>(kc + static_cast<size_t>(t) * kvd + kvh * HD +
                                             4 * lane);
    }
    for (uint32_t j = 0; j < G; ++j) {
      const float4 q = *reinterpret_cast<const float4 *>(&qs[j][4 * lane]);
      float d = __fmaf_rn(q.w, kk.w, __fmaf_rn(q.z, kk.z, __fmaf_rn(q.y, kk.y, __fmul_rn(q.x, kk.x))));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      if (lane == 0) sc[j][t - t0] = __fmul_rn(d, p.scale);
    }
  }
  __syncthreads();

  for (uint32_t j = 0; j < G; ++j) {
    const uint32_t qh = kvh * G + j;
    // split-local softmax statistics
    float m = -INFINITY;
    for (uint32_t t = 0; t < t1 - t0; ++t) m = fmaxf(m, sc[j][t]);
    // every thread computed the same m (same order over shared values)
    float l = 0.f, o = 0.f;
    for (uint32_t t = t0; t < t1; ++t) {
      const float e = expf(sc[j][t - t0] - m);
      l += e;
      const float vv = (t == pos) ? vs_[tid]
                                  : vc[static_cast<size_t>(t) * kvd + kvh * HD + tid];
      o = __fmaf_rn(e, vv, o);
    }
    if (nact == 1) {
      if (!(m > -INFINITY && m < INFINITY) || !(l > 0.f) || !(l < INFINITY)) {
        if (tid == 0) atomicOr(p.status, ZDEV_ERR_NUMERICAL);
      }
      p.out[qh * HD + tid] = __fdiv_rn(o, l);
    } else {
      float *pp = p.part + (static_cast<size_t>(qh) * p.max_splits + split) * (HD + 2);
      pp[tid] = o;
      if (tid == 0) {
        pp[HD] = m;
        pp[HD + 1] = l;
      }
    }
  }
  if (nact == 1) return;

  // Publish the partials, then let the last CTA of this kv-head merge.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(&p.counters[kvh], 1u);
    s_last = (prev == nact - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (uint32_t j = 0; j < G; ++j) {
    const uint32_t qh = kvh * G + j;
    const float *base = p.part + static_cast<size_t>(qh) * p.max_splits * (HD + 2);
    float M = -INFINITY;
    for (uint32_t s = 0; s < nact; ++s) M = fmaxf(M, __ldcg(base + s * (HD + 2) + HD));
    float L = 0.f, O = 0.f;
    for (uint32_t s = 0; s < nact; ++s) {
      const float ms = __ldcg(base + s * (HD + 2) + HD);
      const float ls = __ldcg(base + s * (HD + 2) + HD + 1);
      const float f = expf(ms - M);
      L = __fmaf_rn(f, ls, L);
      O = __fmaf_rn(f, __ldcg(base + s * (HD + 2) + tid), O);
    }
    if (!(M > -INFINITY && M < INFINITY) || !(L > 0.f) || !(L < INFINITY)) {
      if (tid == 0) atomicOr(p.status, ZDEV_ERR_NUMERICAL);
    }
    p.out[qh * HD + tid] = __fdiv_rn(O, L);
  }
  if (tid == 0) p.counters[kvh] = 0u;
}

}  // namespace

cudaError_t launch_attention(const AttnParams &ap, const LaunchCfg &lc) {
  if (ap.n_q % ap.n_kv != 0 || ap.n_q / ap.n_kv > kMaxGqa) return cudaErrorInvalidValue;
  if (ap.max_splits == 0 || (ap.max_tokens + ap.max_splits - 1) / ap.max_splits > kMaxSplitTokens)
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ap.n_kv, ap.max_splits);
  cfg.blockDim = dim3(HD);
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
