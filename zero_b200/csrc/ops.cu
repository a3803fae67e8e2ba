// ops.cu — small kernels of the decode step and the unit-op entry points.
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "internal.h"
#include "layout.h"
#include "ops.h"

namespace zgpu {

namespace {

// embed_lookup_dispatch (crates/zero-llm-inference/src/forward_pass.rs:311-370):
// dequantise one embedding row.  The table lives on the device in the group
// layout of layout.h, so row r is row r%4 of group r/4.  Also selects the step's
// token (prompt id or the previous step's argmax) and publishes position.
__global__ void embed_kernel(const EmbedParams p) {
  pdl_launch_dependents();
  pdl_wait();
  StepState *st = p.state;
  const uint32_t step = st->step;
  uint32_t token = (step < st->n_prompt) ? p.prompt[step] : st->next_token;
  if (token >= p.vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(p.status, ZDEV_ERR_BOUNDS);
    token = 0;
  }
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    st->token = token;
    st->pos = st->pos_base + step;
  }
  const uint32_t g = token >> 2, l = token & 3;
  if (!ZDEV_CHECK(g < (p.vocab + 3) / 4, p.status, 20, token, p.vocab)) return;
  const uint8_t *grp = p.emb + static_cast<uint64_t>(g) * p.gstride;
  const uint32_t bpr = p.hidden / 32;
  for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < p.hidden;
       e += gridDim.x * blockDim.x) {
    const uint32_t b = e >> 5, j = e & 31;
    const uint8_t *sc = grp + scale_entry(p.quant, bpr, b) + 2 * l;
    const float d = h2f(static_cast<uint16_t>(sc[0] | (sc[1] << 8)));
    if (p.quant == ZGPU_Q8_0) {
      const int8_t q = static_cast<int8_t>(grp[plane_entry(p.quant, bpr, b, 2 * l + (j >> 4)) + (j & 15)]);
      p.hidden_out[e] = __fmul_rn(static_cast<float>(q), d);
    } else {
      const uint8_t byte = grp[plane_entry(p.quant, bpr, b, l) + (j & 15)];
      const int n = (j < 16) ? (byte & 0x0F) : (byte >> 4);
      p.hidden_out[e] = __fmul_rn(static_cast<float>(n - 8), d);
    }
  }
}

// End of an LM-head step: decode the argmax key, apply the non-finite and
// padding checks of lm_head.rs:157-163, record the generated token, reset the
// argmax slot and advance the step.
__global__ void finalize_kernel(const FinalizeParams p) {
  pdl_launch_dependents();
  pdl_wait();
  StepState *st = p.state;
  const unsigned long long key = *p.argmax;
  const uint32_t idx = argmax_key_index(key);
  const float val = argmax_key_value(key);
  uint32_t err = 0;
  if (!(val > -INFINITY && val < INFINITY)) err |= ZDEV_ERR_LM_NONFINITE;
  else if (idx >= st->vocab_real) err |= ZDEV_ERR_LM_PADDING;
  const uint32_t step = st->step;
  if (err) {
    atomicOr(p.status, err);
    if (st->first_err_step == 0xFFFFFFFFu) st->first_err_step = step;
  }
  if (step + 1 >= st->n_prompt) {
    const uint32_t gi = step + 1 - st->n_prompt;
    if (gi < st->n_gen_cap && ZDEV_CHECK(gi < st->n_gen_cap, p.status, 21, gi, st->n_gen_cap))
      p.tokens_out[gi] = idx;
  }
  st->next_token = idx;
  st->last_max = val;
  *p.argmax = kArgmaxInitKey;
  st->step = step + 1;
}

__device__ __forceinline__ float block_sum_fixed(float v, float *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (uint32_t w = 0; w < (blockDim.x + 31) / 32; ++w) s += red[w];
  return s;
}

// rmsnorm (ops.rs:29-52), one CTA, fixed-order reduction.
__global__ void rmsnorm_kernel(const float *x, const float *w, float *out, uint32_t n, float eps) {
  __shared__ float red[32];
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  const float tot = block_sum_fixed(ss, red);
  const float inv =
      __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(n)), eps)));
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
}

// rope_sincos_lut_avx512 + rope_apply_avx512 (trig.rs:148-216), one CTA per head.
__global__ void rope_kernel(float *qk, const float *inv_freqs, uint32_t head_dim, uint32_t pos) {
  extern __shared__ float lut[];
  const uint32_t half = head_dim / 2;
  float *cs = lut, *sn = lut + half;
  for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
    float s, c;
    ref_sincos(__fmul_rn(static_cast<float>(pos), inv_freqs[i]), &s, &c);
    cs[i] = c;
    sn[i] = s;
  }
  __syncthreads();
  float *h = qk + static_cast<size_t>(blockIdx.x) * head_dim;
  for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = h[i], b = h[i + half];
    h[i] = __fmaf_rn(a, cs[i], -__fmul_rn(b, sn[i]));
    h[i + half] = __fmaf_rn(a, sn[i], __fmul_rn(b, cs[i]));
  }
}

__global__ void silu_mul_kernel(const float *g, const float *u, float *out, uint64_t n) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    out[i] = ref_silu_mul(g[i], u[i]);
}


// Q8_0 activation quantiser with the packer's rule (tools/silicatepack.py:
// 893-907): double-precision d = max|x| / 127, q = round-half-even(x / d)
// clamped to +-127, d stored as binary16 rounded to nearest-even from the
// double (after the packer's +-65504 clamp).  One warp per block of 32.
__global__ void quantize_q8_0_kernel(const float *x, uint8_t *out, uint64_t nblocks,
                                     uint32_t *status) {
  const uint64_t warp = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (warp >= nblocks) return;
  const float v = x[warp * 32 + lane];
  if (!(fabsf(v) < INFINITY)) atomicOr(status, ZDEV_ERR_NUMERICAL);
  double a = fabs(static_cast<double>(v));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = fmax(a, __shfl_xor_sync(0xffffffffu, a, off));
  uint8_t *blk = out + warp * 34;
  if (a == 0.0 || !(a < INFINITY)) {
    blk[2 + lane] = 0;
    if (lane < 2) blk[lane] = 0;
    return;
  }
  const double d = a / 127.0;
  const double inv = 1.0 / d;
  double r = rint(static_cast<double>(v) * inv);
  r = fmin(fmax(r, -127.0), 127.0);
  blk[2 + lane] = static_cast<uint8_t>(static_cast<int8_t>(r));
  if (lane == 0) {
    const uint16_t h = f64_to_f16_rne(fmin(d, 65504.0));
    blk[0] = static_cast<uint8_t>(h & 0xFF);
    blk[1] = static_cast<uint8_t>(h >> 8);
  }
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, const LaunchCfg &lc,
                            cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lc.stream;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  return cfg;
}

}  // namespace

cudaError_t ops_setup() {
  cudaError_t e = cudaFuncSetAttribute(embed_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared);
}

cudaError_t launch_embed(const EmbedParams &p, const LaunchCfg &lc) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(4), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, embed_kernel, p);
}

cudaError_t launch_finalize(const FinalizeParams &p, const LaunchCfg &lc) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(1), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, finalize_kernel, p);
}

cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, uint32_t n, float eps,
                           cudaStream_t s) {
  rmsnorm_kernel<<<1, 256, 0, s>>>(x, w, out, n, eps);
  return cudaGetLastError();
}

cudaError_t launch_rope(float *qk, const float *inv_freqs, uint32_t n_heads, uint32_t head_dim,
                        uint32_t pos, cudaStream_t s) {
  rope_kernel<<<n_heads, 64, head_dim * sizeof(float), s>>>(qk, inv_freqs, head_dim, pos);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float *g, const float *u, float *out, uint64_t n,
                            cudaStream_t s) {
  const uint64_t blocks = (n + 255) / 256;
  silu_mul_kernel<<<static_cast<unsigned>(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(g, u, out, n);
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0(const float *x, uint8_t *out, uint64_t n, uint32_t *status,
                                 cudaStream_t s) {
  const uint64_t nb = n / 32;
  const uint64_t threads = nb * 32;
  quantize_q8_0_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(x, out, nb,
                                                                                     status);
  return cudaGetLastError();
}

}  // namespace zgpu
