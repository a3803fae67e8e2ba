// gemv.cu — batch-1 dequant GEMV over the .smodel-v2 4-row-interleaved layout.
//
// Replaces linear_q4_0x4_avx512_range / linear_q8_0x4_avx512_range
// (kernel/src/arch/x86_64/math/linear.rs:909, :1096) and the fused
// multi-projection / LM-head-argmax dispatches built on them
// (kernel/src/inference_avx512.rs:826-945, :1061-1118).
//
// Work decomposition.  A unit is two consecutive 4-row groups (8 output rows;
// for the SwiGLU epilogue the device layout pairs gate group g with up group
// g).  An item is one unit restricted to one K-chunk of 32 blocks (1024
// inputs), so every lane of a warp handles exactly one 32-element block of
// the 8 rows.  CTA c owns a contiguous range of units and all their chunks.
//
// Data path (2 CTAs per SM):
//   * prologue: the consumer threads build the activation image once per CTA
//     in shared memory.  Each 32-element block of x (RMSNorm applied for
//     PRO_RMSNORM, with a fixed-order sum of squares identical in every CTA)
//     becomes integers N_i = rint(x_i * 2^-E) with 2^E a power of two that
//     puts the block maximum in [2^22, 2^23); the three bytes of each N_i
//     (two unsigned, the top one signed) are stored as packed int8 digit
//     words, with the block scale 2^E and, for Q4_0, the per-digit offset
//     -8 * sum_i byte_i that removes the nibble bias.  16-byte chunks are
//     XOR-swizzled by block so that lanes reading different blocks hit
//     different banks;
//   * consumer warp w takes items w, w+8, ... of the CTA; it owns ring slots
//     [w*S, (w+1)*S), fed by lane w of the producer warp with two 1-D TMA bulk
//     copies per item (the chunk of each group stream; cp.async.bulk, L2
//     evict-first).  One producer lane and one consumer warp per slot keep
//     every slot's mbarrier phases strictly in order.  The producer starts
//     before the programmatic-dependent-launch wait, so weights stream while
//     the previous kernel finishes;
//   * each lane takes one block of the item's 8 rows: per row one 16-byte
//     plane load (two for Q8_0), three dp4a chains (one per digit, exact
//     int32), then t = (s0 + 256 s1) + 65536 s2 and acc = (d * 2^E) * t.  The
//     digit image carries x to 2^-23 of its block maximum, so a row's error
//     stays a few 1e-7 of sum |x w|, like a reordered f32 sum;
//   * a warp reduce-scatter leaves the item's 8 row sums in lanes 4r, which
//     store them to shared memory; after all items the K-chunks of each row
//     are added in chunk order and the epilogue stores / adds the residual /
//     applies SiLU(gate)*up / tracks the LM-head argmax.
// Every reduction has a fixed order, so results are bitwise reproducible from
// run to run and independent of the grid size.
#include <cfloat>

#include "common.cuh"
#include "internal.h"
#include "layout.h"

namespace zgpu {

namespace {

constexpr int kWarps = 8;                      // consumer warps per CTA
constexpr int kThreads = 32 * (kWarps + 1);
constexpr int kConsumers = 32 * kWarps;
constexpr int kRows = 8;                       // output rows per unit
constexpr size_t kSmemBudget = 110 * 1024;     // two CTAs per SM
constexpr int kCtasPerSm = 2;
constexpr uint32_t kMaxSlotsPerWarp = 4;

struct KParams {
  const uint8_t *w;
  uint64_t gstride;          // bytes per group stream (multiple of 16)
  uint64_t wbytes;           // bytes of the weight buffer
  uint32_t rows;             // valid output rows (SwiGLU: output length)
  uint32_t units;            // total units
  uint32_t units_per_cta;
  uint32_t bpr;              // 32-element blocks per row
  uint32_t ks;               // K-chunks per unit
  uint32_t in_dim;
  uint32_t spw;              // ring slots per consumer warp
  uint32_t half_bytes;       // bytes of one group's chunk in a slot (multiple of 16)
  uint32_t xbytes;           // shared bytes of the prepared activation image
  uint32_t ring_off;         // offset of the ring (after the image and the partials)
  uint32_t smem_bytes;       // dynamic shared bytes of the launch
  const float *x;
  const float *norm_w;
  float eps;
  float *out;
  unsigned long long *argmax;
  uint32_t *status;
};

// Activation image: 32 words per block, in 16-byte chunks
//   0-1: digit-0 words, 2-3: digit-1 words, 4-5: digit-2 words,
//   6: (offset0, offset1, offset2, 2^E as f32 bits), 7: unused;
// digit word k packs the digit bytes of elements 4k..4k+3 (for Q4_0 words
// 0-3 meet the low nibbles of qs word k, words 4-7 the high nibbles of qs
// word k-4; for Q8_0 word k meets qs word k).  Chunk c of block b sits at
// chunk position c ^ (b & 7).
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

template <int QT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_x4_kernel(const KParams p) {
  constexpr uint32_t P = (QT == ZGPU_Q4_0) ? 4 : 8;   // planes per chunk (layout.h)
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[kWarps];
  __shared__ unsigned long long best_w[kWarps];

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t S = p.spw;
  const uint32_t slot_bytes = 2 * p.half_bytes;
  uint32_t *xsm = reinterpret_cast<uint32_t *>(smem);                 // bpr * 32 words
  float *part = reinterpret_cast<float *>(smem + p.xbytes);           // [items][8]
  uint8_t *ring = smem + p.ring_off;
  uint64_t *full = reinterpret_cast<uint64_t *>(ring + static_cast<size_t>(kWarps) * S * slot_bytes);
  uint64_t *empty = full + kWarps * S;

  const uint32_t u0 = blockIdx.x * p.units_per_cta;
  const uint32_t u1 = min(u0 + p.units_per_cta, p.units);
  const uint32_t nloc = u1 > u0 ? u1 - u0 : 0;
  const uint32_t nitems = nloc * p.ks;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kWarps * S; ++i) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kWarps) {
    // ---------------- producer: lane w feeds consumer warp w's slots ----------
    if (lane < kWarps) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t issued = 0;
      for (uint32_t k = lane, j = 0; k < nitems; k += kWarps, ++j) {
        const uint32_t slot = lane * S + (j % S);
        if (j >= S && !mbar_wait(smem_addr(&empty[slot]), ((j / S) - 1) & 1, p.status)) break;
        const uint32_t unit = u0 + k / p.ks, chunk = k % p.ks;
        const uint32_t bytes = static_cast<uint32_t>(chunk_bytes(QT, chunk_blocks(p.bpr, chunk)));
        const uint64_t src = (2ull * unit) * p.gstride + chunk_offset(QT, chunk);
        if (!ZDEV_CHECK(src + p.gstride + bytes <= p.wbytes && bytes <= p.half_bytes, p.status, 1,
                        unit, chunk))
          break;
        if (!ZDEV_CHECK(p.ring_off + (slot + 1) * slot_bytes <= p.smem_bytes, p.status, 2, slot,
                        p.smem_bytes))
          break;
        const uint32_t fb = smem_addr(&full[slot]);
        const uint32_t dst = smem_addr(ring + static_cast<size_t>(slot) * slot_bytes);
        mbar_arrive_expect_tx(fb, 2 * bytes);
        tma_bulk_g2s(dst, p.w + src, bytes, fb, pol);
        tma_bulk_g2s(dst + p.half_bytes, p.w + src + p.gstride, bytes, fb, pol);
        ++issued;
      }
      // Drain: never leave a copy in flight when the CTA may exit.
      for (uint32_t s = 0; s < S && s < issued; ++s) {
        const uint32_t last = s + ((issued - 1 - s) / S) * S;
        mbar_wait(smem_addr(&full[lane * S + s]), (last / S) & 1, p.status);
      }
    }
    return;
  }

  // ---------------- consumers: prepare the activation image ----------------
  pdl_wait();   // the activations are the previous kernel's output
  const uint32_t tid = threadIdx.x;
  const uint32_t nf4 = p.in_dim / 4;
  float inv = 1.0f;
  if (PRO == PRO_RMSNORM) {
    // rmsnorm (ops.rs:29-52): fixed-order sum of squares (per thread over its
    // float4s in order, xor-tree in the warp, warps in order).
    float ss = 0.f;
    for (uint32_t f = tid; f < nf4; f += kConsumers) {
      const float4 t = reinterpret_cast<const float4 *>(p.x)[f];
      ss = __fadd_rn(ss, __fadd_rn(__fadd_rn(__fmul_rn(t.x, t.x), __fmul_rn(t.y, t.y)),
                                   __fadd_rn(__fmul_rn(t.z, t.z), __fmul_rn(t.w, t.w))));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) red[warp] = ss;
    named_bar_sync(1, kConsumers);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot = __fadd_rn(tot, red[w]);
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(p.in_dim)), p.eps)));
  }
  // Warp-uniform trip count: the per-block sum below shuffles across the 8
  // lanes of a block, and nf4 is a multiple of 8, so a block's lanes are
  // either all in range or all out of range.
  for (uint32_t f0 = warp * 32; f0 < nf4; f0 += kConsumers) {
    const uint32_t f = f0 + lane;
    const bool valid = f < nf4;
    float4 t = valid ? reinterpret_cast<const float4 *>(p.x)[f] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (PRO == PRO_RMSNORM && valid) {
      const float4 g = reinterpret_cast<const float4 *>(p.norm_w)[f];
      t.x = __fmul_rn(__fmul_rn(t.x, inv), g.x);
      t.y = __fmul_rn(__fmul_rn(t.y, inv), g.y);
      t.z = __fmul_rn(__fmul_rn(t.z, inv), g.z);
      t.w = __fmul_rn(__fmul_rn(t.w, inv), g.w);
    }
    const uint32_t b = f >> 3, k4 = f & 7;
    // a failed check only suppresses the writes: every lane still reaches the
    // shuffles below
    const bool in_range =
        valid && ZDEV_CHECK(b < p.bpr && b * 128 + 128 <= p.xbytes, p.status, 3, b, p.xbytes);
    // block maximum and non-finite flag over the block's 8 lanes
    float am = fmaxf(fmaxf(fabsf(t.x), fabsf(t.y)), fmaxf(fabsf(t.z), fabsf(t.w)));
    uint32_t bad = (fabsf(t.x) <= FLT_MAX && fabsf(t.y) <= FLT_MAX && fabsf(t.z) <= FLT_MAX &&
                    fabsf(t.w) <= FLT_MAX) ? 0u : 1u;
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
      bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    int n[4] = {0, 0, 0, 0};
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
  named_bar_sync(1, kConsumers);

  // ---------------- consumers: items ----------------
  bool failed = false;
  for (uint32_t k = warp, j = 0; k < nitems; k += kWarps, ++j) {
    const uint32_t slot = warp * S + (j % S);
    if (!failed && !mbar_wait(smem_addr(&full[slot]), (j / S) & 1, p.status)) failed = true;
    const uint32_t chunk = k % p.ks;
    const uint32_t b = chunk * kChunkBlocks + lane;
    float acc[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
    if (!failed && b < p.bpr) {
      const uint8_t *sbase = ring + static_cast<size_t>(slot) * slot_bytes;
      const uint32_t nb = chunk_blocks(p.bpr, chunk);
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
      for (int g = 0; g < 2; ++g) {
        const uint8_t *cb = sbase + g * p.half_bytes;
        const uint2 sc = *reinterpret_cast<const uint2 *>(cb + P * nb * 16 + lane * 8);
        const float d[4] = {h2f(sc.x & 0xFFFF), h2f(sc.x >> 16), h2f(sc.y & 0xFFFF),
                            h2f(sc.y >> 16)};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float t;
          if (QT == ZGPU_Q4_0) {
            t = q4_dot(*reinterpret_cast<const uint4 *>(cb + r * nb * 16 + lane * 16), D, I);
          } else {
            t = q8_dot(*reinterpret_cast<const uint4 *>(cb + (2 * r) * nb * 16 + lane * 16),
                       *reinterpret_cast<const uint4 *>(cb + (2 * r + 1) * nb * 16 + lane * 16), D);
          }
          acc[4 * g + r] = __fmul_rn(d[r], bscale) * t;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));
    const float v = reduce_scatter<kRows>(acc, lane);        // lane holds row lane >> 2
    if ((lane & 3) == 0) part[k * kRows + (lane >> 2)] = v;
  }
  named_bar_sync(1, kConsumers);

  // ---------------- epilogue: K-chunks in order, then per row ---------------
  unsigned long long best = kArgmaxInitKey;
  if (EPI == EPI_SWIGLU) {
    // unit = {gate rows 4u..4u+3, up rows 4u..4u+3}
    for (uint32_t t = tid; t < nloc * 4; t += kConsumers) {
      const uint32_t ul = t >> 2, r = t & 3;
      float yg = 0.f, yu = 0.f;
      for (uint32_t c = 0; c < p.ks; ++c) {
        yg += part[(ul * p.ks + c) * kRows + r];
        yu += part[(ul * p.ks + c) * kRows + 4 + r];
      }
      const uint32_t row = (u0 + ul) * 4 + r;
      if (row < p.rows) p.out[row] = ref_silu_mul(yg, yu);
    }
  } else {
    for (uint32_t t = tid; t < nloc * kRows; t += kConsumers) {
      const uint32_t ul = t / kRows, r = t % kRows;
      float y = 0.f;
      for (uint32_t c = 0; c < p.ks; ++c) y += part[(ul * p.ks + c) * kRows + r];
      const uint32_t row = (u0 + ul) * kRows + r;
      if (row < p.rows) {
        if (EPI == EPI_STORE) {
          p.out[row] = y;
        } else if (EPI == EPI_RESADD) {
          p.out[row] = p.out[row] + y;
        } else {
          p.out[row] = y;
          const unsigned long long key = argmax_key(y, row);
          best = key > best ? key : best;
        }
      }
    }
  }

  if (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0) best_w[warp] = best;
    named_bar_sync(1, kConsumers);
    if (threadIdx.x == 0) {
      unsigned long long b = kArgmaxInitKey;
      for (int w = 0; w < kWarps; ++w) b = best_w[w] > b ? best_w[w] : b;
      if (b != kArgmaxInitKey) atomicMax(p.argmax, b);
    }
  }
}

// Every kernel of the step asks for the maximum shared-memory carveout: an SM
// only hosts CTAs of kernels with one carveout at a time, so a uniform
// carveout is what lets the next kernel's CTAs become resident (and start
// their weight prefetch) while the current kernel drains.
template <int QT, int PRO, int EPI>
cudaError_t configure_one() {
  cudaError_t e = cudaFuncSetAttribute(gemv_x4_kernel<QT, PRO, EPI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kSmemBudget));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemv_x4_kernel<QT, PRO, EPI>,
                              cudaFuncAttributePreferredSharedMemoryCarveout,
                              cudaSharedmemCarveoutMaxShared);
}

template <int QT, int PRO>
cudaError_t configure_pro() {
  cudaError_t e;
  if ((e = configure_one<QT, PRO, EPI_STORE>()) != cudaSuccess) return e;
  if ((e = configure_one<QT, PRO, EPI_RESADD>()) != cudaSuccess) return e;
  if ((e = configure_one<QT, PRO, EPI_SWIGLU>()) != cudaSuccess) return e;
  return configure_one<QT, PRO, EPI_ARGMAX>();
}

template <int QT, int PRO, int EPI>
cudaError_t launch_one(const KParams &kp, uint32_t grid, size_t smem, const LaunchCfg &lc) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lc.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, gemv_x4_kernel<QT, PRO, EPI>, kp);
}

template <int QT, int PRO>
cudaError_t dispatch_epi(GemvEpi epi, const KParams &kp, uint32_t grid, size_t smem,
                         const LaunchCfg &lc) {
  switch (epi) {
    case EPI_STORE: return launch_one<QT, PRO, EPI_STORE>(kp, grid, smem, lc);
    case EPI_RESADD: return launch_one<QT, PRO, EPI_RESADD>(kp, grid, smem, lc);
    case EPI_SWIGLU: return launch_one<QT, PRO, EPI_SWIGLU>(kp, grid, smem, lc);
    case EPI_ARGMAX: return launch_one<QT, PRO, EPI_ARGMAX>(kp, grid, smem, lc);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t gemv_setup() {
  cudaError_t e;
  if ((e = configure_pro<ZGPU_Q4_0, PRO_PLAIN>()) != cudaSuccess) return e;
  if ((e = configure_pro<ZGPU_Q4_0, PRO_RMSNORM>()) != cudaSuccess) return e;
  if ((e = configure_pro<ZGPU_Q8_0, PRO_PLAIN>()) != cudaSuccess) return e;
  return configure_pro<ZGPU_Q8_0, PRO_RMSNORM>();
}

cudaError_t launch_gemv(const GemvDesc &g, GemvPro pro, GemvEpi epi, const GemvIo &io,
                        const LaunchCfg &lc) {
  if (g.in_dim == 0 || g.in_dim % 32 != 0 || g.groups == 0 || g.groups % 2 != 0)
    return cudaErrorInvalidValue;
  if (g.gstride % 16 != 0) return cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && g.quant != ZGPU_Q4_0) return cudaErrorInvalidValue;
  KParams kp = {};
  kp.w = g.w;
  kp.gstride = g.gstride;
  kp.wbytes = g.wbytes ? g.wbytes : static_cast<uint64_t>(g.groups) * g.gstride;
  kp.rows = g.rows;
  kp.bpr = g.in_dim / 32;
  kp.ks = (kp.bpr + kChunkBlocks - 1) / kChunkBlocks;
  kp.in_dim = g.in_dim;
  kp.units = g.groups / 2;
  const uint32_t ctas = static_cast<uint32_t>((lc.sm_count > 0 ? lc.sm_count : 148) * kCtasPerSm);
  kp.units_per_cta = (kp.units + ctas - 1) / ctas;
  const uint32_t grid = (kp.units + kp.units_per_cta - 1) / kp.units_per_cta;
  kp.half_bytes = static_cast<uint32_t>(chunk_bytes(g.quant, min(kChunkBlocks, kp.bpr)));
  const size_t slot = 2 * static_cast<size_t>(kp.half_bytes);
  // activation image: 128 B per block
  kp.xbytes = static_cast<uint32_t>(static_cast<size_t>(kp.bpr) * 128);
  const size_t part_bytes =
      (static_cast<size_t>(kp.units_per_cta) * kp.ks * kRows * sizeof(float) + 127) & ~size_t(127);
  kp.ring_off = static_cast<uint32_t>(kp.xbytes + part_bytes);
  const size_t fixed = kp.ring_off + 1024;
  if (fixed + kWarps * slot > kSmemBudget) return cudaErrorInvalidValue;
  uint32_t spw = static_cast<uint32_t>((kSmemBudget - fixed) / (kWarps * slot));
  const uint32_t items_per_warp = (kp.units_per_cta * kp.ks + kWarps - 1) / kWarps;
  if (spw > items_per_warp) spw = items_per_warp;
  if (spw > kMaxSlotsPerWarp) spw = kMaxSlotsPerWarp;
  if (spw < 1) spw = 1;
  kp.spw = spw;
  kp.x = io.x;
  kp.norm_w = io.norm_w;
  kp.eps = io.eps;
  kp.out = io.out;
  kp.argmax = io.argmax;
  kp.status = io.status;
  const size_t smem = kp.ring_off + static_cast<size_t>(kWarps) * spw * slot + 16 * kWarps * spw;
  kp.smem_bytes = static_cast<uint32_t>(smem);
  if (g.quant == ZGPU_Q4_0) {
    return pro == PRO_RMSNORM ? dispatch_epi<ZGPU_Q4_0, PRO_RMSNORM>(epi, kp, grid, smem, lc)
                              : dispatch_epi<ZGPU_Q4_0, PRO_PLAIN>(epi, kp, grid, smem, lc);
  }
  if (g.quant == ZGPU_Q8_0) {
    return pro == PRO_RMSNORM ? dispatch_epi<ZGPU_Q8_0, PRO_RMSNORM>(epi, kp, grid, smem, lc)
                              : dispatch_epi<ZGPU_Q8_0, PRO_PLAIN>(epi, kp, grid, smem, lc);
  }
  return cudaErrorInvalidValue;
}

}  // namespace zgpu
