// kquant.cu — batch-1 GEMV over GGUF K-quant weights (the GGUF-compat path):
// Q4_K (144-byte, 256-element super-blocks) and Q6_K (210-byte), as
// linear_q4k / linear_q6k read them (crates/zero-llm-inference/src/
// ops.rs:179-292; block formats zero-gguf-parser/src/dequant.rs:75-138 and
// 328-360).
//
// Device layout: Q4_K rows as registered (144 bytes is a multiple of 16);
// Q6_K super-blocks padded to kQ6kStride = 224 bytes at registration, so that
// every field starts on an 8-byte boundary.
//
// One to eight warps per output row (more for matrices with few rows),
// eight warps per CTA.  Per super-block, lane l owns
// eight consecutive elements that share one sub-block scale:
//   Q4_K  sub-block j = l / 4 (32 elements), elements 32 j + 8 (l % 4) + i:
//         the low (j even) or high (j odd) nibbles of qs[32 (j / 2) + 8 (l % 4) + i];
//   Q6_K  half h = l / 16, k = (l / 4) % 4, elements 128 h + 32 k + 8 (l % 4) + i
//         (scale sc[8 h + 2 k + (l % 4) / 2]), ql[64 h + 32 (k % 2) + 8 (l % 4) + i]
//         nibble k / 2 and qh[32 h + 8 (l % 4) + i] bits 2 k.
// The eight quant bytes come in one 8-byte load and become floats exactly
// (magic-number add).  The scale is applied once per lane and sub-block:
//   Q6_K  (d * sc) * sum_i x_i (q_i - 32)
//   Q4_K  (d * sc) * sum_i x_i q_i - (dmin * m) * sum_i x_i
// with every scale product rounded as the reference rounds it, so a one-hot
// input returns the reference's dequantised weight bit for bit; other inputs
// sum in another order than the reference's sequential dot (held to the GEMV
// tolerance).  The per-lane sums of x (eight elements each) are computed once
// per CTA into shared memory.
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"
#include "ops.h"

namespace zgpu {

namespace {

constexpr uint32_t kRowsPerCta = 8;
constexpr uint32_t kMaxKquantIn = 65536;   // in_dim limit (shared memory of the x sums: 32 KB)

// float(b) - bias for a byte b, exactly (b + 2^23 has the byte as its low mantissa bits)
__device__ __forceinline__ float byte_to_float(uint32_t b, float bias) {
  return __fsub_rn(__uint_as_float(0x4B000000u | b), bias);
}

// sum_i x_i * (byte_i(q) - bias) over the 4 bytes of q, in byte order
__device__ __forceinline__ float dot4(uint32_t q, float4 x, float bias, float s) {
  s = fmaf(x.x, byte_to_float(q & 0xFFu, bias), s);
  s = fmaf(x.y, byte_to_float((q >> 8) & 0xFFu, bias), s);
  s = fmaf(x.z, byte_to_float((q >> 16) & 0xFFu, bias), s);
  return fmaf(x.w, byte_to_float(q >> 24, bias), s);
}

// WPR warps share a row (a matrix with few rows would leave most warp slots
// empty): warp k of a row takes super-blocks k, k + WPR, ...; the partial
// sums are added in warp order through shared memory.
template <uint32_t QT, uint32_t WPR>
__global__ void __launch_bounds__(32 * kRowsPerCta) gemv_kquant_kernel(const uint8_t *__restrict__ w, uint32_t rows,
                                                                     uint32_t spr, const float *__restrict__ x,
                                                                     float *__restrict__ y) {
  extern __shared__ float xs8[];   // [in_dim / 8]: sums of x over 8-element runs (Q4_K)
  __shared__ float wpart[kRowsPerCta];
  constexpr uint32_t kRows = kRowsPerCta / WPR;
  const uint32_t lane = threadIdx.x & 31, wk = (threadIdx.x >> 5) % WPR;
  const uint32_t row = blockIdx.x * kRows + (threadIdx.x >> 5) / WPR;
  if (QT == ZGPU_Q4_K) {
    for (uint32_t r = threadIdx.x; r < spr * 32; r += blockDim.x) {
      const float4 a = *reinterpret_cast<const float4 *>(x + 8 * r);
      const float4 b = *reinterpret_cast<const float4 *>(x + 8 * r + 4);
      xs8[r] = ((((((a.x + a.y) + a.z) + a.w) + b.x) + b.y) + b.z) + b.w;
    }
    __syncthreads();
  }
  float acc = 0.f;
  if (row < rows) {
  if (QT == ZGPU_Q4_K) {
    const uint32_t j = lane >> 2, p = lane & 3, sh = (j & 1) * 4;
    const uint8_t *wr = w + static_cast<size_t>(row) * spr * 144;
#pragma unroll 4
    for (uint32_t b = wk; b < spr; b += WPR) {
      const uint8_t *blk = wr + static_cast<size_t>(b) * 144;
      const uint32_t dm = *reinterpret_cast<const uint32_t *>(blk);
      const uint32_t s0 = *reinterpret_cast<const uint32_t *>(blk + 4);
      const uint32_t s1 = *reinterpret_cast<const uint32_t *>(blk + 8);
      const uint32_t s2 = *reinterpret_cast<const uint32_t *>(blk + 12);
      const uint2 qv = *reinterpret_cast<const uint2 *>(blk + 16 + 32 * (j >> 1) + 8 * p);
      const float *xb = x + 256 * b + 32 * j + 8 * p;
      const float4 xa = *reinterpret_cast<const float4 *>(xb);
      const float4 xc = *reinterpret_cast<const float4 *>(xb + 4);
      // get_scale_min_k4 (dequant.rs:75-85) for sub-block j: bytes 0-3 in s0,
      // 4-7 in s1, 8-11 in s2
      const uint32_t bs = 8 * (j & 3);
      const uint32_t b0 = (s0 >> bs) & 0xFFu, b1 = (s1 >> bs) & 0xFFu, b2 = (s2 >> bs) & 0xFFu;
      uint32_t sv, mv;
      if (j < 4) {
        sv = b0 & 0x3F;
        mv = b1 & 0x3F;
      } else {
        sv = (b2 & 0x0F) | ((b0 >> 6) << 4);
        mv = (b2 >> 4) | ((b1 >> 6) << 4);
      }
      const float d = h2f(static_cast<uint16_t>(dm & 0xFFFF)), dmin = h2f(static_cast<uint16_t>(dm >> 16));
      const float d1 = __fmul_rn(d, static_cast<float>(sv)), mn1 = __fmul_rn(dmin, static_cast<float>(mv));
      float s = dot4((qv.x >> sh) & 0x0F0F0F0Fu, xa, 8388608.0f, 0.f);
      s = dot4((qv.y >> sh) & 0x0F0F0F0Fu, xc, 8388608.0f, s);
      acc = __fadd_rn(acc, __fsub_rn(__fmul_rn(d1, s), __fmul_rn(mn1, xs8[32 * b + 4 * j + p])));
    }
  } else {
    const uint32_t h = lane >> 4, k = (lane >> 2) & 3, l0 = (lane & 3) * 8;
    const uint8_t *wr = w + static_cast<size_t>(row) * spr * kQ6kStride;
#pragma unroll 4
    for (uint32_t b = wk; b < spr; b += WPR) {
      const uint8_t *blk = wr + static_cast<size_t>(b) * kQ6kStride;
      const uint2 ql = *reinterpret_cast<const uint2 *>(blk + 64 * h + 32 * (k & 1) + l0);
      const uint2 qh = *reinterpret_cast<const uint2 *>(blk + 128 + 32 * h + l0);
      const int8_t scv = static_cast<int8_t>(blk[192 + 8 * h + 2 * k + (l0 >> 4)]);
      const uint32_t dw = *reinterpret_cast<const uint32_t *>(blk + 208);
      const float *xb = x + 256 * b + 128 * h + 32 * k + l0;
      const float4 xa = *reinterpret_cast<const float4 *>(xb);
      const float4 xc = *reinterpret_cast<const float4 *>(xb + 4);
      const uint32_t nsh = 4 * (k >> 1), hsh = 2 * k;
      const uint32_t q0 = ((ql.x >> nsh) & 0x0F0F0F0Fu) | (((qh.x >> hsh) & 0x03030303u) << 4);
      const uint32_t q1 = ((ql.y >> nsh) & 0x0F0F0F0Fu) | (((qh.y >> hsh) & 0x03030303u) << 4);
      float s = dot4(q0, xa, 8388640.0f, 0.f);   // bias 2^23 + 32: q - 32
      s = dot4(q1, xc, 8388640.0f, s);
      const float dsc = __fmul_rn(h2f(static_cast<uint16_t>(dw & 0xFFFF)), static_cast<float>(scv));
      acc = fmaf(dsc, s, acc);
    }
  }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (WPR == 1) {
    if (lane == 0 && row < rows) y[row] = acc;
    return;
  }
  if (lane == 0) wpart[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (lane == 0 && wk == 0 && row < rows) {
    float t = wpart[threadIdx.x >> 5];
    for (uint32_t k = 1; k < WPR; ++k) t += wpart[(threadIdx.x >> 5) + k];
    y[row] = t;
  }
}

}  // namespace

cudaError_t launch_gemv_kquant(const uint8_t *w, uint32_t quant, uint32_t rows, uint32_t in_dim, const float *x,
                               float *y, cudaStream_t s) {
  // x is read as float4 and the weight fields as 4- and 8-byte words
  if (rows == 0 || in_dim == 0 || in_dim % 256 || in_dim > kMaxKquantIn ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return cudaErrorInvalidValue;
  if (quant != ZGPU_Q4_K && quant != ZGPU_Q6_K) return cudaErrorInvalidValue;
  const uint32_t spr = in_dim / 256;
  // warps per row: enough warps in flight (rows x WPR >= 8192), at most one super-block each
  uint32_t wpr = 1;
  while (wpr < kRowsPerCta && static_cast<uint64_t>(rows) * wpr < 8192 && 2 * wpr <= spr) wpr *= 2;
  const dim3 grid((rows + kRowsPerCta / wpr - 1) / (kRowsPerCta / wpr)), block(32 * kRowsPerCta);
  const size_t smem = quant == ZGPU_Q4_K ? in_dim / 8 * sizeof(float) : 0;
  auto go = [&](auto qt, auto wp) {
    gemv_kquant_kernel<decltype(qt)::value, decltype(wp)::value><<<grid, block, smem, s>>>(w, rows, spr, x, y);
  };
  using Q4 = std::integral_constant<uint32_t, ZGPU_Q4_K>;
  using Q6 = std::integral_constant<uint32_t, ZGPU_Q6_K>;
  auto by_wpr = [&](auto qt) {
    switch (wpr) {
      case 1: go(qt, std::integral_constant<uint32_t, 1>()); break;
      case 2: go(qt, std::integral_constant<uint32_t, 2>()); break;
      case 4: go(qt, std::integral_constant<uint32_t, 4>()); break;
      default: go(qt, std::integral_constant<uint32_t, 8>()); break;
    }
  };
  if (quant == ZGPU_Q4_K)
    by_wpr(Q4());
  else
    by_wpr(Q6());
  return cudaGetLastError();
}

}  // namespace zgpu
