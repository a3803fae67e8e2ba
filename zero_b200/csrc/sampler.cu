// sampler.cu — top-K + temperature sampling of the next token
// (lm_head_sample, kernel/src/sampler.rs:41-163; xorshift64, rng.rs:23-46).
//
// The reference keeps the top 40 logits of [0, vocab_real) in 40 slots by
// replacing the current minimum whenever a value exceeds it (strict >), the
// new minimum being the first slot holding the smallest value; the slots'
// order then decides the cumulative draw.  One warp reproduces that scan
// exactly: it reads the logits 32 at a time (eight loads in flight per
// lane), a ballot marks the values above the running minimum, and those are
// taken in index order, each re-tested against the minimum as it stands
// (a replacement raises it) and, when it enters, followed by a warp-wide
// first-minimum search over the slots.  Lane 0 then scales by
// 1 / temperature, takes the softmax with the reference's own exp
// approximation (exp_approx, sampler.rs:123-163) and draws
// r = next_u32 / u32::MAX against the cumulative sum, every multiply and add
// rounded on its own as in the reference's scalar Rust.
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>

#include "common.cuh"
#include "ops.h"

namespace zgpu {

namespace {

constexpr int kTopK = 40;
constexpr int kAhead = 8;   // 32-wide chunks in flight per lane

__device__ __forceinline__ float exp_approx(float x) {
  if (x < -87.0f) x = -87.0f;
  else if (x > 88.0f) x = 88.0f;
  const float a = __fmul_rn(x, 1.44269504f);
  const int ai = (a != a) ? 0 : static_cast<int>(a);   // Rust `as i32`: truncation, NaN -> 0
  const float af = __fsub_rn(a, static_cast<float>(ai));
  const float c1 = 0.69314718f, c2 = 0.2402265f, c3 = 0.0555041f;
  const float frac = __fadd_rn(1.0f, __fmul_rn(af, __fadd_rn(c1, __fmul_rn(af, __fadd_rn(c2, __fmul_rn(af, c3))))));
  return __fmul_rn(__uint_as_float(static_cast<uint32_t>(127 + ai) << 23), frac);
}

__device__ __forceinline__ uint32_t rng_next_u32(unsigned long long *state) {
  unsigned long long x = *state;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *state = x;
  return static_cast<uint32_t>(x >> 32);
}

__global__ void __launch_bounds__(32) sample_topk_kernel(const float *logits, uint32_t n, float temperature,
                                                         unsigned long long *rng, uint32_t *out) {
  __shared__ float vals[kTopK];
  __shared__ uint32_t idxs[kTopK];
  const uint32_t lane = threadIdx.x;
  for (uint32_t k = lane; k < kTopK; k += 32) {
    vals[k] = -INFINITY;
    idxs[k] = 0;
  }
  __syncwarp();
  float min_val = -INFINITY;
  uint32_t min_pos = 0;
  float buf[kAhead];
#pragma unroll
  for (int d = 0; d < kAhead; ++d) {
    const uint32_t i = d * 32 + lane;
    buf[d] = i < n ? __ldg(logits + i) : -INFINITY;   // past the end: never above the minimum
  }
  for (uint32_t base = 0; base < n; base += 32 * kAhead) {
#pragma unroll
    for (int d = 0; d < kAhead; ++d) {
      const float v = buf[d];
      const uint32_t cur = base + d * 32;
      const uint32_t ni = base + (kAhead + d) * 32 + lane;
      buf[d] = ni < n ? __ldg(logits + ni) : -INFINITY;
      unsigned mask = __ballot_sync(0xffffffffu, v > min_val);
      while (mask) {   // warp-uniform
        const int j = __ffs(mask) - 1;
        mask &= mask - 1;
        const float vj = __shfl_sync(0xffffffffu, v, j);
        if (vj > min_val) {
          if (lane == 0) {
            vals[min_pos] = vj;
            idxs[min_pos] = cur + j;
          }
          __syncwarp();
          // first slot holding the smallest value (slots 32..39 folded into lanes 0..7)
          float a = vals[lane];
          uint32_t ia = lane;
          if (lane < kTopK - 32 && vals[32 + lane] < a) {
            a = vals[32 + lane];
            ia = 32 + lane;
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, a, off);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, ia, off);
            if (ob < a || (ob == a && oi < ia)) {
              a = ob;
              ia = oi;
            }
          }
          if (a < INFINITY) {   // no slot below +inf: the reference keeps the old position
            min_val = a;
            min_pos = ia;
          } else {
            min_val = INFINITY;
          }
          __syncwarp();
        }
      }
    }
  }
  if (lane != 0) return;
  float p[kTopK];
  const float inv_temp = __fdiv_rn(1.0f, temperature);
  float max_logit = -INFINITY;
  for (int k = 0; k < kTopK; ++k) {
    p[k] = __fmul_rn(vals[k], inv_temp);
    if (p[k] > max_logit) max_logit = p[k];
  }
  float sum = 0.0f;
  for (int k = 0; k < kTopK; ++k) {
    p[k] = exp_approx(__fsub_rn(p[k], max_logit));
    sum = __fadd_rn(sum, p[k]);
  }
  const float inv_sum = __fdiv_rn(1.0f, sum);
  unsigned long long st = *rng;
  const float r = __fdiv_rn(__uint2float_rn(rng_next_u32(&st)), 4294967296.0f);
  *rng = st;
  float cum = 0.0f;
  uint32_t tok = idxs[kTopK - 1];
  for (int k = 0; k < kTopK; ++k) {
    cum = __fadd_rn(cum, __fmul_rn(p[k], inv_sum));
    if (r < cum) {
      tok = idxs[k];
      break;
    }
  }
  *out = tok;
}

}  // namespace

cudaError_t launch_sample_topk(const float *logits, uint32_t len, uint32_t vocab_real, float temperature,
                               unsigned long long *rng, uint32_t *out, cudaStream_t s) {
  if (len == 0) return cudaErrorInvalidValue;
  sample_topk_kernel<<<1, 32, 0, s>>>(logits, len < vocab_real ? len : vocab_real, temperature, rng, out);
  return cudaGetLastError();
}

}  // namespace zgpu
