// prefill.cu — the token-parallel kernels of a Qwen3 prompt prefill: all
// prompt tokens go through a layer at once, so the projections are batched
// matmuls on the tensor cores (mma_gemm.cu) and the rest are these row-wise
// kernels.  The reference has no prefill of its own: it runs
// forward_single_token once per prompt token (inference.rs:1188-1320); this
// path produces the same KV cache and LM-head token to the tolerance that the
// Q8_0 activation quantisation allows.
//
//   rows_embed        embed_lookup_dispatch (forward_pass.rs:311-370) per token
//   rows_rmsnorm_quant rmsnorm (ops.rs:29-52) of each row, then the Q8_0
//                     activation rule (the planar form the matmul reads)
//   qk_rope_kv        per token: QK RMSNorm + RoPE of every head (the
//                     reference's sincos polynomial, trig.rs:60-127) and the
//                     KV-cache append of k and v (kv_cache.rs:139)
//   causal_attn       softmax(q.k / sqrt(hd)) . V over keys 0..pos: the
//                     register-tiled kernel (a CTA per kv head x 128 query
//                     rows of its GQA group, 64-key tiles) for power-of-two
//                     groups, else a warp-per-row kernel over 32-key tiles;
//                     NumericalInstability as attention.rs:48
//   swiglu_rows       SiLU(gate) * up on the gate/up matmul's unit layout
//                     (silu_mul_avx512, activation.rs:115-148); the prefill
//                     uses swiglu_quant_tiles, the same product quantised
//                     straight into the down projection's Q8_0 tiles
#include <cfloat>
#include <cmath>

#include "attn_body.cuh"
#include "common.cuh"
#include "internal.h"
#include "layout.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr uint32_t kRowThreads = 256;

__device__ __forceinline__ float row_block_sum(float v, float *red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (uint32_t w = 0; w < kRowThreads / 32; ++w) s = __fadd_rn(s, red[w]);
  return s;
}

// Q8_0 rule of one 32-element block held by the 32 lanes of a warp.
// CTA per row of the padded row count (a multiple of 128): RMSNorm, then the
// Q8_0 rule into the matmul's activation tiles (ops.h); rows past T are zero.
__global__ void __launch_bounds__(kRowThreads) rows_rmsnorm_quant_kernel(const float *x, const float *g, float eps,
                                                                         uint32_t T, uint32_t n, int8_t *xt,
                                                                         float *xs, uint32_t *status) {
  __shared__ float red[kRowThreads / 32];
  const uint32_t t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bpr = n / 32;
  if (t >= T) {
    for (uint32_t b = warp; b < bpr; b += kRowThreads / 32) {
      xt[mma_tile_off(t, b, bpr, lane >> 4) + (lane & 15)] = 0;
      if (lane == 0) xs[mma_scale_off(t, b, bpr)] = 0.f;
    }
    return;
  }
  const float *xr = x + static_cast<size_t>(t) * n;
  float ss = 0.f;
  for (uint32_t i = tid; i < n; i += kRowThreads) ss = __fadd_rn(ss, __fmul_rn(xr[i], xr[i]));
  const float tot = row_block_sum(ss, red);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(n)), eps)));
  for (uint32_t b = warp; b < bpr; b += kRowThreads / 32) {
    const uint32_t i = 32 * b + lane;
    const float y = __fmul_rn(__fmul_rn(xr[i], inv), g[i]);
    quant_lane_q8_0(y, xt + mma_tile_off(t, b, bpr, lane >> 4) + (lane & 15), xs + mma_scale_off(t, b, bpr), lane,
                    status);
  }
}

__global__ void rows_embed_kernel(const uint8_t *emb, uint64_t gstride, uint32_t quant, uint32_t hidden,
                                  uint32_t vocab, const uint32_t *tokens, float *out, uint32_t *status) {
  const uint32_t t = blockIdx.x;
  uint32_t token = tokens[t];
  if (token >= vocab) {
    if (threadIdx.x == 0) atomicOr(status, ZDEV_ERR_BOUNDS);
    token = 0;
  }
  const uint8_t *grp = emb + static_cast<uint64_t>(token >> 2) * gstride;
  const uint32_t l = token & 3, bpr = hidden / 32;
  for (uint32_t e = threadIdx.x; e < hidden; e += blockDim.x) {
    const uint32_t b = e >> 5, j = e & 31;
    const uint8_t *sc = grp + scale_entry(quant, bpr, b) + 2 * l;
    const float dsc = h2f(static_cast<uint16_t>(sc[0] | (sc[1] << 8)));
    float v;
    if (quant == ZGPU_Q8_0) {
      v = __fmul_rn(static_cast<float>(static_cast<int8_t>(grp[plane_entry(quant, bpr, b, 2 * l + (j >> 4)) + (j & 15)])),
                    dsc);
    } else {
      const uint8_t byte = grp[plane_entry(quant, bpr, b, l) + (j & 15)];
      v = __fmul_rn(static_cast<float>(((j < 16) ? (byte & 0x0F) : (byte >> 4)) - 8), dsc);
    }
    out[static_cast<size_t>(t) * hidden + e] = v;
  }
}

// One CTA per token, one warp per head (q heads, then k heads, then v heads).
__global__ void qk_rope_kv_kernel(const float *qkv, const float *q_norm, const float *k_norm,
                                  const float *inv_freqs, float *kv_layer, uint64_t kv_block, uint32_t n_q,
                                  uint32_t n_kv, uint32_t pos0, float eps, float *q_out) {
  __shared__ float cs[kAttnHd / 2], sn[kAttnHd / 2];
  const uint32_t t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t pos = pos0 + t;
  if (threadIdx.x < kAttnHd / 2) {
    float s, c;
    ref_sincos(__fmul_rn(static_cast<float>(pos), inv_freqs[threadIdx.x]), &s, &c);
    cs[threadIdx.x] = c;
    sn[threadIdx.x] = s;
  }
  __syncthreads();
  const uint32_t qd = n_q * kAttnHd, kvd = n_kv * kAttnHd;
  const float *row = qkv + static_cast<size_t>(t) * (qd + 2 * kvd);
  for (uint32_t h = warp; h < n_q + 2 * n_kv; h += blockDim.x >> 5) {
    const float4 x = reinterpret_cast<const float4 *>(row + h * kAttnHd)[lane];
    if (h < n_q) {
      const float4 w = reinterpret_cast<const float4 *>(q_norm)[lane];
      reinterpret_cast<float4 *>(q_out + static_cast<size_t>(t) * qd + h * kAttnHd)[lane] =
          attn_norm_rope_lane(x, w, eps, cs, sn, lane);
    } else if (h < n_q + n_kv) {
      const float4 w = reinterpret_cast<const float4 *>(k_norm)[lane];
      reinterpret_cast<float4 *>(kv_layer + static_cast<size_t>(pos) * kvd + (h - n_q) * kAttnHd)[lane] =
          attn_norm_rope_lane(x, w, eps, cs, sn, lane);
    } else {
      reinterpret_cast<float4 *>(kv_layer + kv_block + static_cast<size_t>(pos) * kvd +
                                 (h - n_q - n_kv) * kAttnHd)[lane] = x;
    }
  }
}

constexpr uint32_t kQTile = 64;            // query rows per CTA
constexpr uint32_t kKTile = 32;            // keys per staged tile
constexpr uint32_t kAttnRowsPerWarp = 16;  // 4 warps x 16 rows
constexpr uint32_t kKPad = kAttnHd + 1;    // padded K rows: lane j reads row j conflict-free

// Causal attention of one (query tile, q head).  Lane j of a warp scores key
// j of the staged tile against the warp's current query row; the row's
// running max / sum / output (4 dims per lane) stay in registers for the
// warp's 16 rows.
__global__ void __launch_bounds__(128) causal_attn_kernel(const float *q, const float *kv_layer, uint64_t kv_block,
                                                          uint32_t n_q, uint32_t n_kv, uint32_t pos0, uint32_t T,
                                                          float scale, float *out, uint32_t *status) {
  extern __shared__ __align__(16) float asmem[];
  float *qs = asmem;                                   // [kQTile][128]
  float *ks = qs + kQTile * kAttnHd;                   // [kKTile][129]
  float *vs = ks + kKTile * kKPad;                     // [kKTile][128]
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t h = blockIdx.y, kvh = h / (n_q / n_kv);
  const uint32_t i0 = blockIdx.x * kQTile;             // first query row (token index)
  const uint32_t qd = n_q * kAttnHd, kvd = n_kv * kAttnHd;
  const uint32_t rows = min(kQTile, T - i0);
  for (uint32_t e = tid; e < kQTile * kAttnHd / 4; e += blockDim.x) {
    const uint32_t r = e / (kAttnHd / 4), c4 = e % (kAttnHd / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) v = reinterpret_cast<const float4 *>(q + static_cast<size_t>(i0 + r) * qd + h * kAttnHd)[c4];
    reinterpret_cast<float4 *>(qs + r * kAttnHd)[c4] = v;
  }
  float m[kAttnRowsPerWarp], l[kAttnRowsPerWarp];
  float4 o[kAttnRowsPerWarp];
#pragma unroll
  for (int r = 0; r < static_cast<int>(kAttnRowsPerWarp); ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
    o[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const uint32_t last_key = pos0 + i0 + rows - 1;      // keys 0..last_key are needed
  for (uint32_t k0 = 0; k0 <= last_key; k0 += kKTile) {
    __syncthreads();   // previous tile consumed (and the Q tile written, first time)
    for (uint32_t e = tid; e < kKTile * kAttnHd / 4; e += blockDim.x) {
      const uint32_t r = e / (kAttnHd / 4), c4 = e % (kAttnHd / 4);
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (k0 + r <= last_key) {
        const size_t off = static_cast<size_t>(k0 + r) * kvd + kvh * kAttnHd;
        kv4 = reinterpret_cast<const float4 *>(kv_layer + off)[c4];
        vv4 = reinterpret_cast<const float4 *>(kv_layer + kv_block + off)[c4];
      }
      float *kr = ks + r * kKPad + 4 * c4;
      kr[0] = kv4.x;
      kr[1] = kv4.y;
      kr[2] = kv4.z;
      kr[3] = kv4.w;
      reinterpret_cast<float4 *>(vs + r * kAttnHd)[c4] = vv4;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < static_cast<int>(kAttnRowsPerWarp); ++rr) {
      const uint32_t r = warp * kAttnRowsPerWarp + rr;
      if (r >= rows) break;   // warp-uniform
      const uint32_t pos_i = pos0 + i0 + r;
      if (k0 > pos_i) continue;
      const float *qr = qs + r * kAttnHd;
      const float *kr = ks + lane * kKPad;
      float s = 0.f;
#pragma unroll 8
      for (uint32_t c = 0; c < kAttnHd; ++c) s = fmaf(qr[c], kr[c], s);
      s = (k0 + lane <= pos_i) ? __fmul_rn(s, scale) : -INFINITY;
      float mx = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[rr], mx);
      const float corr = (m[rr] == mn) ? 1.0f : expf(m[rr] - mn);
      const float p = (s == -INFINITY) ? 0.0f : expf(s - mn);
      float psum = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l[rr] = fmaf(l[rr], corr, psum);
      float4 acc = make_float4(o[rr].x * corr, o[rr].y * corr, o[rr].z * corr, o[rr].w * corr);
#pragma unroll 8
      for (uint32_t j = 0; j < kKTile; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const float4 v = reinterpret_cast<const float4 *>(vs + j * kAttnHd)[lane];
        acc.x = fmaf(pj, v.x, acc.x);
        acc.y = fmaf(pj, v.y, acc.y);
        acc.z = fmaf(pj, v.z, acc.z);
        acc.w = fmaf(pj, v.w, acc.w);
      }
      m[rr] = mn;
      o[rr] = acc;
    }
  }
#pragma unroll
  for (int k = 0; k < static_cast<int>(kAttnRowsPerWarp); ++k) {
    const uint32_t r = warp * kAttnRowsPerWarp + k;
    if (r >= rows) break;
    if (!(m[k] > -INFINITY && m[k] < INFINITY) || !(l[k] > 0.f) || !(l[k] < INFINITY)) {
      if (lane == 0) atomicOr(status, ZDEV_ERR_NUMERICAL);
    }
    const float inv = __fdiv_rn(1.0f, l[k]);
    reinterpret_cast<float4 *>(out + static_cast<size_t>(i0 + r) * qd + h * kAttnHd)[lane] =
        make_float4(o[k].x * inv, o[k].y * inv, o[k].z * inv, o[k].w * inv);
  }
}

// Register-tiled causal attention: one CTA per (kv head, 128 query rows),
// the rows being the G = n_q / n_kv query heads of the group times 128 / G
// tokens, so the group shares every staged K/V tile.  Keys go in tiles of
// 64, double-buffered by cp.async.  Thread (rg, cg) of 16 x 16:
//   S phase   rows 8rg..8rg+7 x keys cg + 16j (j < 4): per 4 dims three
//             shared loads feed 32 FMAs (the 8 Q rows broadcast, the 4 K
//             rows conflict-free on the padded stride);
//   softmax   online, per row: the tile max over the 16 lanes of the row
//             group (4 shuffles), running max m, partial sum l per thread
//             (reduced once at the end), O rescaled by exp(m_old - m_new);
//   PV phase  P^T is written over the consumed K buffer; rows 8rg.. x dims
//             4cg..4cg+3 and 64+4cg..: per key four shared loads feed 64 FMAs.
// Query tiles are launched heaviest (latest) first.  f32 throughout, the
// reference's scaled dot / max-trick softmax (attention.rs:48-84,278-433)
// in another summation order; NumericalInstability as attention.rs:48.
constexpr uint32_t kFaRows = 128;
constexpr uint32_t kFaKeys = 64;
constexpr uint32_t kFaStride = kAttnHd + 4;   // padded Q / K / P^T rows
constexpr uint32_t kFaThreads = 256;
constexpr size_t kFaSmemBytes =
    (static_cast<size_t>(kFaRows) * kFaStride + 2 * kFaKeys * kFaStride + 2 * kFaKeys * kAttnHd) * sizeof(float);
static_assert(kFaRows == kFaKeys * 2, "P^T [keys][rows] must fit a K buffer [keys][stride]");

__global__ void __launch_bounds__(kFaThreads, 1)
    causal_attn_tiled_kernel(const float *q, const float *kv_layer, uint64_t kv_block, uint32_t n_q, uint32_t n_kv,
                             uint32_t pos0, uint32_t T, float scale, float *out, uint32_t *status) {
  extern __shared__ __align__(16) float fsm[];
  float *Qs = fsm;                                   // [kFaRows][kFaStride]
  float *KP = Qs + kFaRows * kFaStride;              // 2 x [kFaKeys][kFaStride]: K, then P^T
  float *Vs = KP + 2 * kFaKeys * kFaStride;          // 2 x [kFaKeys][kAttnHd]
  const uint32_t tid = threadIdx.x, rg = tid >> 4, cg = tid & 15;
  const uint32_t G = n_q / n_kv, TQ = kFaRows / G;
  const uint32_t kvh = blockIdx.x;
  const uint32_t n_qt = (T + TQ - 1) / TQ;
  const uint32_t i0 = (n_qt - 1 - blockIdx.y) * TQ;  // heaviest query tiles first
  const uint32_t rows_tok = min(TQ, T - i0);
  const uint32_t qd = n_q * kAttnHd, kvd = n_kv * kAttnHd;
  const uint32_t last_key = pos0 + i0 + rows_tok - 1;
  const uint32_t n_tiles = last_key / kFaKeys + 1;

  for (uint32_t e = tid; e < kFaRows * (kAttnHd / 4); e += kFaThreads) {
    const uint32_t r = e >> 5, c = e & 31;
    const uint32_t hl = r / TQ, tk = r % TQ;
    const bool ok = tk < rows_tok;
    const float *src = q + static_cast<size_t>(i0 + (ok ? tk : 0u)) * qd + (kvh * G + hl) * kAttnHd + 4 * c;
    cp_async16(smem_addr(Qs + r * kFaStride + 4 * c), src, ok ? 16u : 0u);
  }
  auto load_kv = [&](uint32_t t, uint32_t b) {
    const uint32_t k0 = t * kFaKeys;
    float *Kb = KP + b * kFaKeys * kFaStride;
    float *Vb = Vs + b * kFaKeys * kAttnHd;
    for (uint32_t e = tid; e < kFaKeys * (kAttnHd / 4); e += kFaThreads) {
      const uint32_t r = e >> 5, c = e & 31;
      const bool ok = k0 + r <= last_key;
      const size_t off = static_cast<size_t>(ok ? k0 + r : 0u) * kvd + kvh * kAttnHd + 4 * c;
      cp_async16(smem_addr(Kb + r * kFaStride + 4 * c), kv_layer + off, ok ? 16u : 0u);
      cp_async16(smem_addr(Vb + r * kAttnHd + 4 * c), kv_layer + kv_block + off, ok ? 16u : 0u);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const uint32_t pos_r0 = pos0 + i0 + (rg * 8) % TQ;   // position of row 8rg (TQ is a multiple of 8)
  float m[8], l[8], o[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) o[i][c] = 0.f;
  }
  for (uint32_t t = 0; t < n_tiles; ++t) {
    const uint32_t b = t & 1, k0 = t * kFaKeys;
    __syncthreads();                       // tile t-1's P^T and V are consumed
    if (t + 1 < n_tiles) load_kv(t + 1, b ^ 1u);
    cp_async_commit();
    cp_async_wait<1>();                    // tile t (and Q) have landed
    __syncthreads();
    float *Kb = KP + b * kFaKeys * kFaStride;
    const float *Vb = Vs + b * kFaKeys * kAttnHd;
    float sc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[i][j] = 0.f;
#pragma unroll 2
    for (uint32_t d4 = 0; d4 < kAttnHd / 4; ++d4) {
      float4 kk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) kk[j] = *reinterpret_cast<const float4 *>(Kb + (cg + 16 * j) * kFaStride + 4 * d4);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 qq = *reinterpret_cast<const float4 *>(Qs + (rg * 8 + i) * kFaStride + 4 * d4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          sc[i][j] = fmaf(qq.x, kk[j].x, sc[i][j]);
          sc[i][j] = fmaf(qq.y, kk[j].y, sc[i][j]);
          sc[i][j] = fmaf(qq.z, kk[j].z, sc[i][j]);
          sc[i][j] = fmaf(qq.w, kk[j].w, sc[i][j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t pos_i = pos_r0 + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float v = (k0 + cg + 16 * j <= pos_i) ? __fmul_rn(sc[i][j], scale) : -INFINITY;
        sc[i][j] = v;
        mx = fmaxf(mx, v);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mn = fmaxf(m[i], mx);
      const float corr = (m[i] == mn) ? 1.0f : expf(m[i] - mn);
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = (sc[i][j] == -INFINITY) ? 0.0f : expf(sc[i][j] - mn);
        sc[i][j] = p;
        ps += p;
      }
      l[i] = fmaf(l[i], corr, ps);
      m[i] = mn;
#pragma unroll
      for (int c = 0; c < 8; ++c) o[i][c] *= corr;
    }
    __syncthreads();                       // every thread is done reading K of tile t
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float *pr = Kb + (cg + 16 * j) * kFaStride + rg * 8;
      *reinterpret_cast<float4 *>(pr) = make_float4(sc[0][j], sc[1][j], sc[2][j], sc[3][j]);
      *reinterpret_cast<float4 *>(pr + 4) = make_float4(sc[4][j], sc[5][j], sc[6][j], sc[7][j]);
    }
    __syncthreads();
#pragma unroll 4
    for (uint32_t key = 0; key < kFaKeys; ++key) {
      const float4 p0 = *reinterpret_cast<const float4 *>(Kb + key * kFaStride + rg * 8);
      const float4 p1 = *reinterpret_cast<const float4 *>(Kb + key * kFaStride + rg * 8 + 4);
      const float4 v0 = *reinterpret_cast<const float4 *>(Vb + key * kAttnHd + 4 * cg);
      const float4 v1 = *reinterpret_cast<const float4 *>(Vb + key * kAttnHd + 64 + 4 * cg);
      const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] = fmaf(pv[i], v0.x, o[i][0]);
        o[i][1] = fmaf(pv[i], v0.y, o[i][1]);
        o[i][2] = fmaf(pv[i], v0.z, o[i][2]);
        o[i][3] = fmaf(pv[i], v0.w, o[i][3]);
        o[i][4] = fmaf(pv[i], v1.x, o[i][4]);
        o[i][5] = fmaf(pv[i], v1.y, o[i][5]);
        o[i][6] = fmaf(pv[i], v1.z, o[i][6]);
        o[i][7] = fmaf(pv[i], v1.w, o[i][7]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float L = l[i];
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    const uint32_t r = rg * 8 + i, hl = r / TQ, tk = r % TQ;
    if (tk >= rows_tok) continue;
    if (!(m[i] > -INFINITY && m[i] < INFINITY) || !(L > 0.f) || !(L < INFINITY)) {
      if (cg == 0) atomicOr(status, ZDEV_ERR_NUMERICAL);
    }
    const float inv = __fdiv_rn(1.0f, L);
    float *dst = out + static_cast<size_t>(i0 + tk) * qd + (kvh * G + hl) * kAttnHd;
    *reinterpret_cast<float4 *>(dst + 4 * cg) = make_float4(o[i][0] * inv, o[i][1] * inv, o[i][2] * inv, o[i][3] * inv);
    *reinterpret_cast<float4 *>(dst + 64 + 4 * cg) =
        make_float4(o[i][4] * inv, o[i][5] * inv, o[i][6] * inv, o[i][7] * inv);
  }
}

// act[t][4u + r] = silu(y[t][8u + r]) * y[t][8u + 4 + r]: the gate/up stream
// interleaves gate group u and up group u (layout of the fused gate/up).
__global__ void swiglu_rows_kernel(const float *y, float *act, uint32_t ffn, uint64_t n) {
  const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  const uint64_t t = i / ffn, f = i % ffn;
  const uint64_t u = f >> 2, r = f & 3;
  const float *yr = y + t * 2 * ffn;
  act[i] = ref_silu_mul(yr[8 * u + r], yr[8 * u + 4 + r]);
}

// SwiGLU fused with the Q8_0 rule into the down projection's activation
// tiles: warp (row t, block b) of the padded row count; lane j is feature
// f = 32b + j = 4u + r of the gate/up unit layout, act = silu(y[8u + r]) *
// y[8u + 4 + r], then quantised as quantize_q8_0_tiles does (rows past T:
// zero digits, scale 0).
__global__ void swiglu_quant_tiles_kernel(const float *y, int8_t *xt, float *xs, uint32_t T, uint32_t ffn,
                                          uint64_t nwarps, uint32_t *status) {
  const uint64_t wb = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (wb >= nwarps) return;
  const uint32_t bpr = ffn / 32;
  const uint32_t t = static_cast<uint32_t>(wb / bpr), b = static_cast<uint32_t>(wb % bpr);
  int8_t *qa = xt + mma_tile_off(t, b, bpr, lane >> 4) + (lane & 15);
  float *da = xs + mma_scale_off(t, b, bpr);
  if (t >= T) {
    *qa = 0;
    if (lane == 0) *da = 0.f;
    return;
  }
  const uint32_t f = 32 * b + lane, u = f >> 2, r = f & 3;
  const float *yr = y + static_cast<uint64_t>(t) * 2 * ffn;
  quant_lane_q8_0(ref_silu_mul(yr[8 * u + r], yr[8 * u + 4 + r]), qa, da, lane, status);
}

// Greedy pick per row of n logits (lm_head_argmax_dynamic, lm_head.rs:98-166,
// applied to each sequence of a batch): the first index holding the largest
// value (a NaN never wins; a row of -inf / NaN keeps index 0), then a
// non-finite maximum is ZGPU_ERR_LM_NON_FINITE_LOGITS and an index at or past
// vocab_real ZGPU_ERR_LM_ARGMAX_IN_PADDING, recorded in codes[row] and in the
// status bits.  One CTA per row: strided first-max per thread, then a tree
// in which the larger value wins and equal values go to the smaller index,
// the same pick as the sequential scan.
constexpr uint32_t kArgmaxThreads = 512;

__global__ void __launch_bounds__(kArgmaxThreads)
    rows_argmax_kernel(const float *logits, uint32_t n, uint32_t vocab_real, uint32_t *tok, uint32_t *codes,
                       uint32_t *status) {
  __shared__ float bv[kArgmaxThreads / 32];
  __shared__ uint32_t bi[kArgmaxThreads / 32];
  const float *row = logits + static_cast<size_t>(blockIdx.x) * n;
  float v = -INFINITY;
  uint32_t idx = 0xFFFFFFFFu;
  for (uint32_t i = threadIdx.x; i < n; i += kArgmaxThreads) {
    const float x = row[i];
    if (x > v) {
      v = x;
      idx = i;
    }
  }
  auto better = [](float a, uint32_t ia, float b, uint32_t ib) { return b > a || (b == a && ib < ia); };
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, off);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, off);
    if (better(v, idx, ov, oi)) {
      v = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = v;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (uint32_t w = 1; w < kArgmaxThreads / 32; ++w)
    if (better(v, idx, bv[w], bi[w])) {
      v = bv[w];
      idx = bi[w];
    }
  if (idx == 0xFFFFFFFFu) idx = 0;
  uint32_t code = 0;
  if (!(fabsf(v) < INFINITY)) {
    code = ZGPU_ERR_LM_NON_FINITE_LOGITS;
    atomicOr(status, ZDEV_ERR_LM_NONFINITE);
  } else if (idx >= vocab_real) {
    code = ZGPU_ERR_LM_ARGMAX_IN_PADDING;
    atomicOr(status, ZDEV_ERR_LM_PADDING);
  }
  tok[blockIdx.x] = idx;
  codes[blockIdx.x] = code;
}

}  // namespace

cudaError_t launch_rows_argmax(const float *logits, uint32_t rows, uint32_t n, uint32_t vocab_real, uint32_t *tok,
                               uint32_t *codes, uint32_t *status, cudaStream_t s) {
  if (rows == 0 || n == 0) return cudaErrorInvalidValue;
  rows_argmax_kernel<<<rows, kArgmaxThreads, 0, s>>>(logits, n, vocab_real, tok, codes, status);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_quant_tiles(const float *y, int8_t *xt, float *xs, uint32_t T, uint32_t ffn,
                                      uint32_t *status, cudaStream_t s) {
  if (T == 0 || ffn == 0 || ffn % 32) return cudaErrorInvalidValue;
  const uint64_t rows = (static_cast<uint64_t>(T) + kMmaTile - 1) / kMmaTile * kMmaTile;
  const uint64_t nwarps = rows * (ffn / 32);
  swiglu_quant_tiles_kernel<<<static_cast<unsigned>((nwarps * 32 + 255) / 256), 256, 0, s>>>(y, xt, xs, T, ffn,
                                                                                           nwarps, status);
  return cudaGetLastError();
}

cudaError_t launch_rows_rmsnorm_quant(const float *x, const float *g, float eps, uint32_t T, uint32_t n, int8_t *xt,
                                      float *xs, uint32_t *status, cudaStream_t s) {
  if (n % 32 || T == 0) return cudaErrorInvalidValue;
  const uint32_t rows = (T + kMmaTile - 1) / kMmaTile * kMmaTile;
  rows_rmsnorm_quant_kernel<<<rows, kRowThreads, 0, s>>>(x, g, eps, T, n, xt, xs, status);
  return cudaGetLastError();
}

cudaError_t launch_rows_embed(const uint8_t *emb, uint64_t gstride, uint32_t quant, uint32_t hidden, uint32_t vocab,
                              const uint32_t *tokens, uint32_t T, float *out, uint32_t *status, cudaStream_t s) {
  rows_embed_kernel<<<T, 256, 0, s>>>(emb, gstride, quant, hidden, vocab, tokens, out, status);
  return cudaGetLastError();
}

cudaError_t launch_qk_rope_kv(const float *qkv, const float *q_norm, const float *k_norm, const float *inv_freqs,
                              float *kv_layer, uint64_t kv_block, uint32_t n_q, uint32_t n_kv, uint32_t pos0,
                              uint32_t T, float eps, float *q_out, cudaStream_t s) {
  qk_rope_kv_kernel<<<T, 32 * (n_q + 2 * n_kv) > 1024 ? 1024 : 32 * (n_q + 2 * n_kv), 0, s>>>(
      qkv, q_norm, k_norm, inv_freqs, kv_layer, kv_block, n_q, n_kv, pos0, eps, q_out);
  return cudaGetLastError();
}

size_t causal_attn_smem() {
  return (static_cast<size_t>(kQTile) * kAttnHd + kKTile * kKPad + kKTile * kAttnHd) * sizeof(float);
}

cudaError_t prefill_setup() {
  cudaError_t e = cudaFuncSetAttribute(causal_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(causal_attn_smem()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(causal_attn_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kFaSmemBytes));
  return e;
}

cudaError_t launch_causal_attn(const float *q, const float *kv_layer, uint64_t kv_block, uint32_t n_q, uint32_t n_kv,
                               uint32_t pos0, uint32_t T, float scale, float *out, uint32_t *status,
                               cudaStream_t s) {
  if (!n_kv || n_q % n_kv || T == 0) return cudaErrorInvalidValue;
  const uint32_t G = n_q / n_kv;
  if (G <= 16 && (G & (G - 1)) == 0) {   // 128 / G query tokens per CTA, a multiple of 8
    const uint32_t TQ = kFaRows / G;
    dim3 grid(n_kv, (T + TQ - 1) / TQ);
    causal_attn_tiled_kernel<<<grid, kFaThreads, kFaSmemBytes, s>>>(q, kv_layer, kv_block, n_q, n_kv, pos0, T, scale,
                                                                     out, status);
    return cudaGetLastError();
  }
  dim3 grid((T + kQTile - 1) / kQTile, n_q);
  causal_attn_kernel<<<grid, 128, causal_attn_smem(), s>>>(q, kv_layer, kv_block, n_q, n_kv, pos0, T, scale, out,
                                                           status);
  return cudaGetLastError();
}

cudaError_t launch_swiglu_rows(const float *y, float *act, uint32_t T, uint32_t ffn, cudaStream_t s) {
  const uint64_t n = static_cast<uint64_t>(T) * ffn;
  swiglu_rows_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(y, act, ffn, n);
  return cudaGetLastError();
}

}  // namespace zgpu
