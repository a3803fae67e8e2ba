// gemv_body.cuh — device code shared by the standalone GEMV kernel (gemv.cu)
// and the persistent step kernel (step.cu): the integer activation image,
// the dp4a row-block dot products and the warp reduce-scatter.
//
// Activation image.  Each 32-element block of x (after RMSNorm when asked)
// becomes integers N_i = rint(x_i * 2^-E), 2^E a power of two that puts the
// block maximum in [2^22, 2^23); the three bytes of N_i (two unsigned, the
// top one signed) are packed into int8 digit words.  A block occupies 32
// words in 16-byte chunks
//   0-1: digit-0 words, 2-3: digit-1 words, 4-5: digit-2 words,
//   6: (offset0, offset1, offset2, 2^E as f32 bits), 7: unused,
// digit word k holding the digits of elements 4k..4k+3 (for Q4_0 words 0-3
// meet the low nibbles of qs word k, words 4-7 the high nibbles of qs word
// k-4; for Q8_0 word k meets qs word k).  The offsets (Q4_0 only) are
// -8 * sum_i digit_i and remove the nibble bias inside the integer chains.
// Chunk c of block b is stored at chunk position c ^ (b & 7), so lanes that
// read different blocks hit different banks.  The image carries x to 2^-23
// of its block maximum: a row's error stays a few 1e-7 of sum |x w|.
#pragma once

#include <cfloat>

#include "common.cuh"
#include "layout.h"

namespace zgpu {

__device__ __forceinline__ uint32_t x_word(uint32_t b, uint32_t chunk, uint32_t w) {
  return b * 32 + ((chunk ^ (b & 7)) << 2) + w;
}

// dp4a with the byte signedness of each operand (PTX dp4a.atype.btype).
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// R row sums spread over the 32 lanes -> lane l holds the total of row
// l / (32 / R) (every lane of that row's group of 32/R lanes).
template <int R>
__device__ __forceinline__ float reduce_scatter(float (&v)[R], uint32_t lane) {
#pragma unroll
  for (int lvl = 0; lvl < 5; ++lvl) {
    const int off = 16 >> lvl;
    const int n = R >> lvl;
    if (n >= 2) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int k = 0; k < n / 2; ++k) {
        float send = upper ? v[k] : v[k + n / 2];
        float keep = upper ? v[k + n / 2] : v[k];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
  return v[0];
}

// sum_j (n_j - 8) * N_j of one Q4_0 row-block from its 16 nibble bytes: the
// digit offsets start each chain at -8 * sum_j digit_j.
__device__ __forceinline__ float q4_dot(const uint4 q, const uint32_t (&D)[3][8], const int (&I)[3]) {
  int s0 = I[0], s1 = I[1], s2 = I[2];
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t lo = w[m] & 0x0F0F0F0Fu, hi = (w[m] >> 4) & 0x0F0F0F0Fu;
    s0 = dp4a_uu(lo, D[0][m], s0);
    s1 = dp4a_uu(lo, D[1][m], s1);
    s2 = dp4a_us(lo, D[2][m], s2);
    s0 = dp4a_uu(hi, D[0][m + 4], s0);
    s1 = dp4a_uu(hi, D[1][m + 4], s1);
    s2 = dp4a_us(hi, D[2][m + 4], s2);
  }
  // |s0 + 256 s1| < 2^24: exact in int32 and in f32
  return fmaf(static_cast<float>(s2), 65536.0f, static_cast<float>(s0 + (s1 << 8)));
}

// sum_j q_j * N_j of one Q8_0 row-block from its two 16-byte halves.
__device__ __forceinline__ float q8_dot(const uint4 qa, const uint4 qb, const uint32_t (&D)[3][8]) {
  int s0 = 0, s1 = 0, s2 = 0;
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    s0 = dp4a_su(w[k], D[0][k], s0);
    s1 = dp4a_su(w[k], D[1][k], s1);
    s2 = dp4a_ss(w[k], D[2][k], s2);
  }
  return fmaf(static_cast<float>(s2), 65536.0f, static_cast<float>(s0 + (s1 << 8)));
}

// 1 / sqrt(mean(x^2) + eps) of x[n] (rmsnorm, ops.rs:29-52) with a fixed
// summation order: per thread over its float4s in order, xor-tree in the
// warp, warps in order.  `red` holds NW floats; every one of the NW*32
// consumer threads calls this; bar_id names their barrier.
template <int NW>
__device__ __forceinline__ float rms_inv(const float *x, uint32_t n, float eps, float *red,
                                         uint32_t tid, uint32_t bar_id) {
  const uint32_t warp = tid >> 5, lane = tid & 31;
  float ss = 0.f;
  for (uint32_t f = tid; f < n / 4; f += NW * 32) {
    const float4 t = __ldcg(reinterpret_cast<const float4 *>(x) + f);
    ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(t.x, t.x), __fmul_rn(t.y, t.y)),
                                 __fadd_rn(__fmul_rn(t.z, t.z), __fmul_rn(t.w, t.w))));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if (lane == 0) red[warp] = ss;
  named_bar_sync(bar_id, NW * 32);
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) tot = __fadd_rn(tot, red[w]);
  // every thread has read red[] before anyone can overwrite it: the caller
  // passes another barrier before the next use
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(n)), eps)));
}

// The integers of one block (see the file header): n_k = rint(t_k * 2^(22-e))
// (at most 2^23 - 1) for the float4 t = x[4f..4f+3], and the block's scale
// 2^(e-22) (0 for an all-zero or negligible block, NaN for a non-finite
// one).  Called by all 32 lanes of a warp for 32 consecutive float4s (8
// blocks): the statistics shuffle across the 8 lanes of each block.  The
// GEMV image (digitise_f4) and the batched tensor-core image (digit_mma.cu)
// both take their digits from here.
__device__ __forceinline__ float block_ints(float4 t, int (&n)[4]) {
  // block maximum and non-finite flag over the block's 8 lanes
  float am = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
  uint32_t bad = (fabsf(t.x) <= FLT_MAX && fabsf(t.y) <= FLT_MAX && fabsf(t.z) <= FLT_MAX &&
                  fabsf(t.w) <= FLT_MAX) ? 0u : 1u;
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) {
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    bad |= __shfl_xor_sync(0xffffffffu, bad, off);
  }
  n[0] = n[1] = n[2] = n[3] = 0;
  float bscale = 0.0f;                              // all-zero (or negligible) block
  if (bad) {
    bscale = __uint_as_float(0x7fc00000u);          // NaN: the rows' sums become NaN
  } else if (am >= 7.888609052e-31f) {              // 2^-100
    const int e = static_cast<int>(__float_as_uint(am) >> 23) - 127;   // am in [2^e, 2^(e+1))
    const float up = __uint_as_float(static_cast<uint32_t>(149 - e) << 23);   // 2^(22-e)
    bscale = __uint_as_float(static_cast<uint32_t>(105 + e) << 23);          // 2^(e-22)
    const float v[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) n[k] = min(__float2int_rn(v[k] * up), 0x7FFFFF);
  }
  return bscale;
}

// Digitise the float4 t = x[4f..4f+3] into the image (see the file header).
// Called by all 32 lanes of a warp for 32 consecutive float4s (8 blocks):
// the block statistics shuffle across the 8 lanes of each block, so lanes
// with valid == false must still call it.
template <int QT>
__device__ __forceinline__ void digitise_f4(float4 t, uint32_t f, bool valid, uint32_t *xsm,
                                            uint32_t bpr, uint32_t xbytes, uint32_t *status) {
  const uint32_t b = f >> 3, k4 = f & 7;
  // a failed check only suppresses the writes: every lane still reaches the
  // shuffles below
  const bool in_range = valid && ZDEV_CHECK(b < bpr && b * 128 + 128 <= xbytes, status, 3, b, xbytes);
  int n[4];
  const float bscale = block_ints(t, n);
  const uint32_t w0 = __byte_perm(__byte_perm(n[0], n[1], 0x0040), __byte_perm(n[2], n[3], 0x0040), 0x5410);
  const uint32_t w1 = __byte_perm(__byte_perm(n[0], n[1], 0x0051), __byte_perm(n[2], n[3], 0x0051), 0x5410);
  const uint32_t w2 = __byte_perm(__byte_perm(n[0], n[1], 0x0062), __byte_perm(n[2], n[3], 0x0062), 0x5410);
  int ds[3] = {0, 0, 0};
  if (QT == ZGPU_Q4_0) {
    ds[0] = dp4a_uu(w0, 0x01010101u, 0);
    ds[1] = dp4a_uu(w1, 0x01010101u, 0);
    ds[2] = dp4a_us(0x01010101u, w2, 0);
#pragma unroll
    for (int off = 1; off < 8; off <<= 1)
#pragma unroll
      for (int d = 0; d < 3; ++d) ds[d] += __shfl_xor_sync(0xffffffffu, ds[d], off);
  }
  if (in_range) {
    xsm[x_word(b, 0 + (k4 >> 2), k4 & 3)] = w0;
    xsm[x_word(b, 2 + (k4 >> 2), k4 & 3)] = w1;
    xsm[x_word(b, 4 + (k4 >> 2), k4 & 3)] = w2;
    if (k4 == 0) {
      xsm[x_word(b, 6, 0)] = static_cast<uint32_t>(-8 * ds[0]);
      xsm[x_word(b, 6, 1)] = static_cast<uint32_t>(-8 * ds[1]);
      xsm[x_word(b, 6, 2)] = static_cast<uint32_t>(-8 * ds[2]);
      xsm[x_word(b, 6, 3)] = __float_as_uint(bscale);
    }
  }
}

// Row sums of one item for the lane's block: G groups (4G rows) of the slot
// at `sbase` (group g's chunk at sbase + g * group_bytes, a chunk of nb
// blocks in the plane layout), against the image of block b.
template <int QT, int G>
__device__ __forceinline__ void item_rows(const uint8_t *sbase, uint32_t group_bytes, uint32_t nb,
                                          uint32_t lane, uint32_t b, const uint32_t *xsm,
                                          float (&acc)[4 * G]) {
  constexpr uint32_t P = (QT == ZGPU_Q4_0) ? 4 : 8;
  const uint4 *xb = reinterpret_cast<const uint4 *>(xsm + b * 32);
  const uint32_t sw = b & 7;
  uint32_t D[3][8];
#pragma unroll
  for (int c = 0; c < 6; ++c) {
    const uint4 v = xb[c ^ sw];
    D[c >> 1][4 * (c & 1) + 0] = v.x;
    D[c >> 1][4 * (c & 1) + 1] = v.y;
    D[c >> 1][4 * (c & 1) + 2] = v.z;
    D[c >> 1][4 * (c & 1) + 3] = v.w;
  }
  const uint4 meta = xb[6 ^ sw];
  const int I[3] = {static_cast<int>(meta.x), static_cast<int>(meta.y), static_cast<int>(meta.z)};
  const float bscale = __uint_as_float(meta.w);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint8_t *cb = sbase + g * group_bytes;
    const uint2 sc = *reinterpret_cast<const uint2 *>(cb + P * nb * 16 + lane * 8);
    const float d[4] = {h2f(sc.x & 0xFFFF), h2f(sc.x >> 16), h2f(sc.y & 0xFFFF), h2f(sc.y >> 16)};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float t;
      if (QT == ZGPU_Q4_0) {
        t = q4_dot(*reinterpret_cast<const uint4 *>(cb + r * nb * 16 + lane * 16), D, I);
      } else {
        t = q8_dot(*reinterpret_cast<const uint4 *>(cb + (2 * r) * nb * 16 + lane * 16),
                   *reinterpret_cast<const uint4 *>(cb + (2 * r + 1) * nb * 16 + lane * 16), D);
      }
      acc[4 * g + r] = __fmul_rn(__fmul_rn(d[r], bscale), t);
    }
  }
}

// Image of a Q8_0-quantised activation block (the config-1 Q4_0 x Q8_0
// GEMV): one digit.  Chunks 0-1 hold the block's 32 int8 quants as words
// (word k: elements 4k..4k+3), chunk 6 holds (-8 * sum_j q_j, 0, 0, d_x as
// f32 bits), in the same swizzled 128-byte slot as the three-digit image.
// Called by one thread per block: the 34-byte block at xb (2-byte aligned).
__device__ __forceinline__ void q8_block_image(const uint8_t *xb, uint32_t b, uint32_t *xsm) {
  // all 17 halfwords are loaded before any is used, so that the loads are in
  // flight together (the block is read once, after the launch's dependency
  // wait: plain loads)
  const uint16_t *h = reinterpret_cast<const uint16_t *>(xb);
  uint16_t hw[17];
#pragma unroll
  for (int k = 0; k < 17; ++k) hw[k] = h[k];
  const float d = h2f(hw[0]);
  uint32_t w[8];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    w[k] = static_cast<uint32_t>(hw[1 + 2 * k]) | (static_cast<uint32_t>(hw[2 + 2 * k]) << 16);
    sum = dp4a_ss(0x01010101u, w[k], sum);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) xsm[x_word(b, k >> 2, k & 3)] = w[k];
  xsm[x_word(b, 6, 0)] = static_cast<uint32_t>(-8 * sum);
  xsm[x_word(b, 6, 1)] = 0u;
  xsm[x_word(b, 6, 2)] = 0u;
  xsm[x_word(b, 6, 3)] = __float_as_uint(d);
}

// Row sums of one item against a Q8_0 activation image (q8_block_image):
// sum_j (n_j - 8) * q_j exactly in int32 (one dp4a chain), times d_w * d_x.
template <int G>
__device__ __forceinline__ void item_rows_q8act(const uint8_t *sbase, uint32_t group_bytes, uint32_t nb,
                                                uint32_t lane, uint32_t b, const uint32_t *xsm,
                                                float (&acc)[4 * G]) {
  const uint4 *xb = reinterpret_cast<const uint4 *>(xsm + b * 32);
  const uint32_t sw = b & 7;
  const uint4 v0 = xb[0 ^ sw], v1 = xb[1 ^ sw], meta = xb[6 ^ sw];
  const uint32_t D[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  const int off = static_cast<int>(meta.x);
  const float dx = __uint_as_float(meta.w);
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint8_t *cb = sbase + g * group_bytes;
    const uint2 sc = *reinterpret_cast<const uint2 *>(cb + 4 * nb * 16 + lane * 8);
    const float d[4] = {h2f(sc.x & 0xFFFF), h2f(sc.x >> 16), h2f(sc.y & 0xFFFF), h2f(sc.y >> 16)};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint4 q = *reinterpret_cast<const uint4 *>(cb + r * nb * 16 + lane * 16);
      const uint32_t wq[4] = {q.x, q.y, q.z, q.w};
      int s = off;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        s = dp4a_us(wq[m] & 0x0F0F0F0Fu, D[m], s);
        s = dp4a_us((wq[m] >> 4) & 0x0F0F0F0Fu, D[m + 4], s);
      }
      acc[4 * g + r] = __fmul_rn(__fmul_rn(d[r], dx), static_cast<float>(s));
    }
  }
}

}  // namespace zgpu
