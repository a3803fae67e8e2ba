// mha.cu — decode attention of the DeepSeek2 layers that use standard
// multi-head attention instead of MLA (mha_attention_single_token,
// crates/zero-llm-inference/src/mla.rs:449-618), between the fused q|k|v
// projection and the output projection:
//
//   mha_prep   one CTA: RoPE (the NeoX half split of the rope part, angle
//              pos * powf(base, -2 i / rope), as mla.rs:491-530) on every q
//              head in place and on the new k, then the cache append of k and
//              v at pos (MhaKvCache::store_kv, kv_cache.rs:487-531; the cache
//              keeps the reference's layout: per MHA layer a K block of
//              [max_tokens][n_kv * (nope + rope)] and a V block of
//              [max_tokens][n_kv * v]).
//   mha_attn   CTA (q head h, split s): tokens [64 s, 64 s + 64) of [0, pos];
//              a warp per token computes q . k_t over nope + rope (kv head
//              h / (n_heads / n_kv)), times 1 / sqrt(nope + rope); the CTA's
//              max, exp weights and their sum, and the thread-per-column sum
//              of p_t v_t, written as the split's partial (m, l, o).
//   mha_merge  CTA per q head: the splits merged in split order into
//              out_h = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s; a non-finite
//              max or a sum <= 0 raises NumericalInstability (attention.rs:48-84).
// The sums are grouped differently from the reference's sequential ones:
// results agree to f32 rounding, not bit for bit.
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "mla.h"
#include "ops.h"

namespace zgpu {

namespace {

__device__ __forceinline__ uint32_t mha_pos(const MhaParams &p) { return p.pos_ptr ? *p.pos_ptr : p.pos_value; }

__device__ __forceinline__ void mha_rope_pair(float x0, float x1, float theta, float *o0, float *o1) {
  float s, c;
  sincosf(theta, &s, &c);
  *o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
  *o1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void __launch_bounds__(256) mha_prep_kernel(const MhaParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = mha_pos(p);
  if (pos >= p.max_tokens) {
    if (threadIdx.x == 0) atomicOr(p.status, ZDEV_ERR_BOUNDS);
    return;
  }
  const uint32_t hq = p.nope + p.rope, half = p.rope / 2;
  const uint32_t qd = p.n_heads * hq, kd = p.n_kv * hq, vd = p.n_kv * p.v;
  const float fpos = static_cast<float>(pos);
  for (uint32_t i = threadIdx.x; i < p.n_heads * half; i += blockDim.x) {
    const uint32_t h = i / half, j = i % half;
    float *x = p.qkv + h * hq + p.nope;
    float a, b;
    mha_rope_pair(x[j], x[j + half], __fmul_rn(fpos, p.inv_freqs[j]), &a, &b);
    x[j] = a;
    x[j + half] = b;
  }
  const float *k = p.qkv + qd, *v = p.qkv + qd + kd;
  float *kc = p.k_cache + static_cast<size_t>(pos) * kd, *vc = p.v_cache + static_cast<size_t>(pos) * vd;
  for (uint32_t i = threadIdx.x; i < kd; i += blockDim.x) {
    const uint32_t j = i % hq;
    if (j < p.nope) {
      kc[i] = k[i];
    } else if (j - p.nope < half) {
      float a, b;
      mha_rope_pair(k[i], k[i + half], __fmul_rn(fpos, p.inv_freqs[j - p.nope]), &a, &b);
      kc[i] = a;
      kc[i + half] = b;
    }
  }
  for (uint32_t i = threadIdx.x; i < vd; i += blockDim.x) vc[i] = v[i];
}

__global__ void __launch_bounds__(kMhaThreads) mha_attn_kernel(const MhaParams p) {
  __shared__ float qs[kMhaMaxHead];
  __shared__ float sc[kMhaSplitTokens];
  __shared__ float mred;
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = mha_pos(p);
  if (pos >= p.max_tokens) return;   // mha_prep has raised the bounds status
  const uint32_t total = pos + 1, split = blockIdx.y, h = blockIdx.x;
  const uint32_t t0 = split * kMhaSplitTokens;
  if (t0 >= total) return;
  const uint32_t t1 = min(t0 + kMhaSplitTokens, total), n = t1 - t0;
  const uint32_t hq = p.nope + p.rope, kd = p.n_kv * hq, vd = p.n_kv * p.v;
  const uint32_t kvh = h / (p.n_heads / p.n_kv);
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (uint32_t i = tid; i < hq; i += kMhaThreads) qs[i] = __ldcg(p.qkv + h * hq + i);
  __syncthreads();
  // the cache rows of this step were appended by mha_prep, an earlier launch
  for (uint32_t t = t0 + warp; t < t1; t += kMhaThreads / 32) {
    const float *kt = p.k_cache + static_cast<size_t>(t) * kd + kvh * hq;
    float d = 0.f;
    for (uint32_t i = lane; i < hq; i += 32) d = fmaf(qs[i], __ldcg(kt + i), d);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    if (lane == 0) sc[t - t0] = __fmul_rn(d, p.scale);
  }
  __syncthreads();
  if (tid == 0) {
    float m = -INFINITY;
    for (uint32_t t = 0; t < n; ++t) m = fmaxf(m, sc[t]);
    mred = m;
  }
  __syncthreads();
  const float m = mred;
  __syncthreads();
  if (tid < n) sc[tid] = (m == -INFINITY) ? 0.f : expf(sc[tid] - m);
  __syncthreads();
  float *pp = p.part + (static_cast<size_t>(h) * p.max_splits + split) * (p.v + 2);
  for (uint32_t j = tid; j < p.v; j += kMhaThreads) {
    const float *vt = p.v_cache + static_cast<size_t>(t0) * vd + kvh * p.v + j;
    float o = 0.f;
    for (uint32_t t = 0; t < n; ++t) o = fmaf(sc[t], __ldcg(vt + static_cast<size_t>(t) * vd), o);
    pp[j] = o;
  }
  if (tid == 0) {
    float l = 0.f;
    for (uint32_t t = 0; t < n; ++t) l = __fadd_rn(l, sc[t]);
    pp[p.v] = m;
    pp[p.v + 1] = l;
  }
}

__global__ void __launch_bounds__(kMhaThreads) mha_merge_kernel(const MhaParams p) {
  __shared__ float wf[256];   // e^(m_s - M) per split (first 256 splits; more are folded below)
  __shared__ float tot[2];
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t pos = mha_pos(p);
  if (pos >= p.max_tokens) return;
  const uint32_t h = blockIdx.x, nact = (pos + 1 + kMhaSplitTokens - 1) / kMhaSplitTokens;
  const float *base = p.part + static_cast<size_t>(h) * p.max_splits * (p.v + 2);
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (uint32_t s = 0; s < nact; ++s) M = fmaxf(M, base[static_cast<size_t>(s) * (p.v + 2) + p.v]);
    float L = 0.f;
    for (uint32_t s = 0; s < nact; ++s) {
      const float ms = base[static_cast<size_t>(s) * (p.v + 2) + p.v];
      const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
      if (s < 256) wf[s] = w;
      L = fmaf(w, base[static_cast<size_t>(s) * (p.v + 2) + p.v + 1], L);
    }
    tot[0] = M;
    tot[1] = L;
    if (!(M > -INFINITY && M < INFINITY) || !(L > 0.f) || !(L < INFINITY)) atomicOr(p.status, ZDEV_ERR_NUMERICAL);
  }
  __syncthreads();
  const float M = tot[0], L = tot[1];
  for (uint32_t j = threadIdx.x; j < p.v; j += kMhaThreads) {
    float acc = 0.f;
    for (uint32_t s = 0; s < nact; ++s) {
      const float *ps = base + static_cast<size_t>(s) * (p.v + 2);
      const float w = s < 256 ? wf[s] : ((ps[p.v] == -INFINITY) ? 0.f : expf(ps[p.v] - M));
      acc = fmaf(w, ps[j], acc);
    }
    p.out[h * p.v + j] = __fdiv_rn(acc, L);
  }
}

bool mha_geometry_ok(const MhaParams &p) {
  return p.n_heads > 0 && p.n_kv > 0 && p.n_heads % p.n_kv == 0 && p.rope % 2 == 0 &&
         p.nope + p.rope > 0 && p.nope + p.rope <= kMhaMaxHead && p.v > 0 && p.v <= kMhaMaxV &&
         p.max_splits >= mha_max_splits(p.max_tokens);
}

}  // namespace

cudaError_t mha_setup() { return cudaSuccess; }

cudaError_t launch_mha_prep(const MhaParams &p, const LaunchCfg &lc) {
  if (!mha_geometry_ok(p)) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(1), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, mha_prep_kernel, p);
}

cudaError_t launch_mha_attention(const MhaParams &p, const LaunchCfg &lc) {
  if (!mha_geometry_ok(p)) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(p.n_heads, p.max_splits), dim3(kMhaThreads), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  cudaError_t e = cudaLaunchKernelEx(&cfg, mha_attn_kernel, p);
  if (e != cudaSuccess) return e;
  cfg = make_launch_cfg(dim3(p.n_heads), dim3(kMhaThreads), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, mha_merge_kernel, p);
}

}  // namespace zgpu
