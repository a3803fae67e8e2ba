// kquant.cu — batch-1 GEMV over GGUF K-quant weights (the GGUF-compat path):
// Q4_K (144-byte, 256-element super-blocks) and Q6_K (210-byte), plain rows
// as linear_q4k / linear_q6k read them (crates/zero-llm-inference/src/
// ops.rs:179-292; block formats dequant.rs:63-138 and 286-356).
//
// One warp per output row, eight rows per CTA.  Per super-block, lane l owns
// eight elements:
//   Q4_K  the four bytes qs[32 g + 4 (l % 8) ..] of group g = l / 8: their
//         low nibbles (elements 64 g + 4 (l % 8) ..) with sub-block 2 g's
//         scale / min, the high nibbles (32 further) with 2 g + 1's;
//   Q6_K  element l + 32 k of both 128-element halves (k < 4), from
//         ql[64 h + l], ql[64 h + l + 32] and qh[32 h + l].
// The super-block loop is unrolled four deep so that a warp has four
// blocks' loads in flight (a 2048-wide row is only eight super-blocks).
// Every weight is rebuilt exactly as the reference dequantises it (each
// product rounded on its own); the dot product accumulates with fmaf per
// lane and a warp tree, another order than the reference's sequential sum
// (held to the GEMV tolerance).
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "ops.h"

namespace zgpu {

namespace {

constexpr uint32_t kRowsPerCta = 8;

__device__ __forceinline__ void q4k_scale_min(const uint8_t *sc, int j, float *d, float *m) {
  uint32_t a, b;
  if (j < 4) {
    a = sc[j] & 0x3F;
    b = sc[j + 4] & 0x3F;
  } else {
    a = (sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4);
    b = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
  *d = static_cast<float>(a);
  *m = static_cast<float>(b);
}

template <uint32_t QT>
__global__ void __launch_bounds__(32 * kRowsPerCta) gemv_kquant_kernel(const uint8_t *__restrict__ w, uint32_t rows,
                                                                     uint32_t spr, const float *__restrict__ x,
                                                                     float *__restrict__ y) {
  const uint32_t row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float acc = 0.f;
  if (QT == ZGPU_Q4_K) {
    const uint8_t *wr = w + static_cast<size_t>(row) * spr * 144;
    const uint32_t g = lane >> 3, p = (lane & 7) * 4;
#pragma unroll 4
    for (uint32_t b = 0; b < spr; ++b) {
      const uint8_t *blk = wr + static_cast<size_t>(b) * 144;
      const float d = h2f(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
      const float dmin = h2f(static_cast<uint16_t>(blk[2] | (blk[3] << 8)));
      float s0, m0, s1, m1;
      q4k_scale_min(blk + 4, 2 * g, &s0, &m0);
      q4k_scale_min(blk + 4, 2 * g + 1, &s1, &m1);
      const float d1 = __fmul_rn(d, s0), mn1 = __fmul_rn(dmin, m0);
      const float d2 = __fmul_rn(d, s1), mn2 = __fmul_rn(dmin, m1);
      const uint32_t q = *reinterpret_cast<const uint32_t *>(blk + 16 + 32 * g + p);
      const float4 xl = *reinterpret_cast<const float4 *>(x + 256 * b + 64 * g + p);
      const float4 xh = *reinterpret_cast<const float4 *>(x + 256 * b + 64 * g + 32 + p);
      const float xlv[4] = {xl.x, xl.y, xl.z, xl.w}, xhv[4] = {xh.x, xh.y, xh.z, xh.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float lo = static_cast<float>((q >> (8 * i)) & 0xF), hi = static_cast<float>((q >> (8 * i + 4)) & 0xF);
        acc = fmaf(xlv[i], __fsub_rn(__fmul_rn(d1, lo), mn1), acc);
        acc = fmaf(xhv[i], __fsub_rn(__fmul_rn(d2, hi), mn2), acc);
      }
    }
  } else {
    const uint8_t *wr = w + static_cast<size_t>(row) * spr * 210;
#pragma unroll 4
    for (uint32_t b = 0; b < spr; ++b) {
      const uint8_t *blk = wr + static_cast<size_t>(b) * 210;
      const float d = h2f(static_cast<uint16_t>(blk[208] | (blk[209] << 8)));
      const int is = lane / 16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t ql0 = blk[64 * h + lane], ql1 = blk[64 * h + lane + 32], qh = blk[128 + 32 * h + lane];
        const int8_t *sc = reinterpret_cast<const int8_t *>(blk + 192 + 8 * h + is);
        const int qv[4] = {static_cast<int>((ql0 & 0xF) | ((qh & 3) << 4)) - 32,
                           static_cast<int>((ql1 & 0xF) | (((qh >> 2) & 3) << 4)) - 32,
                           static_cast<int>((ql0 >> 4) | (((qh >> 4) & 3) << 4)) - 32,
                           static_cast<int>((ql1 >> 4) | (((qh >> 6) & 3) << 4)) - 32};
        const float *xb = x + 256 * b + 128 * h + lane;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float wv = __fmul_rn(__fmul_rn(d, static_cast<float>(sc[2 * k])), static_cast<float>(qv[k]));
          acc = fmaf(xb[32 * k], wv, acc);
        }
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) y[row] = acc;
}

}  // namespace

cudaError_t launch_gemv_kquant(const uint8_t *w, uint32_t quant, uint32_t rows, uint32_t in_dim, const float *x,
                               float *y, cudaStream_t s) {
  // x is read as float4 and the weight bytes as u32 words
  if (rows == 0 || in_dim == 0 || in_dim % 256 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return cudaErrorInvalidValue;
  const dim3 grid((rows + kRowsPerCta - 1) / kRowsPerCta), block(32 * kRowsPerCta);
  if (quant == ZGPU_Q4_K)
    gemv_kquant_kernel<ZGPU_Q4_K><<<grid, block, 0, s>>>(w, rows, in_dim / 256, x, y);
  else if (quant == ZGPU_Q6_K)
    gemv_kquant_kernel<ZGPU_Q6_K><<<grid, block, 0, s>>>(w, rows, in_dim / 256, x, y);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace zgpu
