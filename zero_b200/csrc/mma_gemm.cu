// mma_gemm.cu — batched Q4_0 weight x Q8_0 activation matmul on the 5th-gen
// tensor cores (tcgen05, int8), for prefill and multi-token decode.
//
// Y[t][m] = sum_b d_w[m,b] * d_x[t,b] * sum_{j<32} (n[m,b,j] - 8) * q[t,b,j]
//
// Both operands carry one scale per 32-element block, so a block's integer
// dot product must be scaled before it is added to the next block's.  Each
// block is therefore one tcgen05.mma.kind::i8 of M = 128 weight rows x N = 128
// tokens x K = 32 into a TMEM accumulator, read back with tcgen05.ld and added
// as (sumi * d_w) * d_x in block order: the order of the CPU restatement of
// the Q4_0 x Q8_0 product (ggml's vec_dot_q4_0_q8_0 loop), bit for bit.
//
// Operands come pre-tiled (ops.h): weights as int8 (n - 8) tiles built once
// per tensor (build_w8_tiles), activations as Q8_0 tiles written by the
// quantisers, each 128 x 32 block a contiguous 4 KB in the MMA's canonical
// layout, plus f32 scale vectors.  One CTA per SM, warp-specialised, no
// CTA-wide barrier inside the block loop:
//   warp 0      producer: per block, one 1-D bulk copy of the weight tile
//               with its scales and one of the token tile with its scales
//               (two for a 32-wide token tile) into one of 4 shared-memory
//               stages, completion on full[s];
//   warp 1      MMA issuer: waits full[s], one tcgen05.mma into accumulator
//               s (4 x 128 TMEM columns), tcgen05.commit to done[s];
//   warps 2-17  epilogue: warp w reads TMEM lanes 32 (w % 4).. (weight rows)
//               x columns 32 ((w - 2) / 4).. (tokens) of accumulator s, scales
//               and accumulates in f32 registers, then arrives on empty[s],
//               which frees stage s and accumulator s for block b + 4.
// For a few tokens (T <= 32, batched decode) the token tile is 32 wide and
// two CTAs share an SM, each with 8 stages / accumulators of 32 TMEM columns
// (half of TMEM), a 1 KB activation copy per block and 4 epilogue warps, so
// that 16 blocks of weights are in flight per SM instead of 4 on two
// independent pipelines.  A weight with few 128-row tiles can also be split
// along K (MmaGemmParams::ksplit): each split sums its block range in order
// into a partial, and a reduce kernel adds the partials in split order.  The
// split count depends on the weight's shape alone, so a token's result does
// not depend on how many tokens share the launch; with a split the block sum
// is regrouped (no longer the CPU restatement's order bit for bit).
// Every wait is bounded (status ZDEV_ERR_TIMEOUT); on an expired wait each
// role stops, the producer drains its copies in flight and the MMA issuer its
// MMAs before TMEM is freed.  The launch asks for more than half an SM's
// shared memory so that two CTAs never meet on one SM: the second CTA's
// 512-column TMEM allocation would wait for the first.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "common.cuh"
#include "tcgen05.cuh"
#include "internal.h"
#include "layout.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr uint32_t kTileM = 128;
constexpr uint32_t kTmemCols = 512;              // the whole TMEM of the SM
constexpr uint32_t kDynSmem = 120 * 1024;        // > half of an SM: one CTA per SM

// Geometry of the kernel for a token tile of NT columns: 128 for many tokens
// (prefill), 32 for a few (batched decode), where a 32-wide tile leaves TMEM
// room for 16 block accumulators in flight instead of 4.  A stage holds one
// 32-element block: the weight tile (128 rows), the first NT rows of the
// activation tile, and both tiles' block scales.
// The 32-wide tile runs two CTAs per SM, each on half of TMEM (8 stages, 4
// epilogue warps of all 32 columns): two independent producer / MMA /
// epilogue chains per SM.
template <uint32_t NT>
struct MmaCfg {
  static constexpr uint32_t kTileN = NT;
  static constexpr uint32_t kCtasPerSm = NT == 128 ? 1 : 2;
  static constexpr uint32_t kTmem = kTmemCols / kCtasPerSm;     // TMEM columns of one CTA
  static constexpr uint32_t kStages = kTmem / NT;               // = TMEM accumulators
  static constexpr uint32_t kEpiWarps = NT == 128 ? 16 : 4;     // 4 lane quarters x NT / kCols column groups
  static constexpr uint32_t kCols = NT * 4 / kEpiWarps;         // token columns per epilogue warp
  static constexpr uint32_t kThreads = 32 * (2 + kEpiWarps);
  // dynamic shared memory: more than a third of the SM for two CTAs per SM,
  // more than half for one (a further CTA would wait on its TMEM allocation)
  static constexpr uint32_t kDyn = NT == 128 ? kDynSmem : 80 * 1024;
  // A tile + its scales (one 4608-byte copy), then the NT token rows
  // (1024-aligned) and their scales (one copy with them when NT = 128)
  static constexpr uint32_t kStA = 0, kStW = 4096, kStB = 5120;
  static constexpr uint32_t kStX = NT == 128 ? kStB + 4096 : kStB + NT * 32;
  static constexpr uint32_t kStageLoad = kMmaBlockBytes + NT * 32 + NT * 4;   // bytes copied per stage
  static constexpr uint32_t kStageBytes = (kStX + NT * 4 + 1023) / 1024 * 1024;
  // instruction descriptor of kind::i8: D s32, A and B signed int8, both
  // K-major, N = NT, M = 128, dense
  static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((NT >> 3) << 17) | ((kTileM >> 4) << 24);
  static_assert(kStages * kStageBytes <= kDyn, "stages fit the dynamic shared memory");
};
}

namespace {




template <uint32_t NT>
__global__ void __launch_bounds__(MmaCfg<NT>::kThreads, MmaCfg<NT>::kCtasPerSm) q4q8_mma_kernel(const MmaGemmParams p) {
  using Cfg = MmaCfg<NT>;
  constexpr uint32_t kTileN = Cfg::kTileN, kStages = Cfg::kStages, kEpiWarps = Cfg::kEpiWarps;
  constexpr uint32_t kStA = Cfg::kStA, kStB = Cfg::kStB, kStW = Cfg::kStW, kStX = Cfg::kStX;
  constexpr uint32_t kStageBytes = Cfg::kStageBytes, kIdesc = Cfg::kIdesc;
  extern __shared__ __align__(1024) uint8_t ring[];
  __shared__ __align__(8) uint64_t full[MmaCfg<NT>::kStages], done[MmaCfg<NT>::kStages],
      empty[MmaCfg<NT>::kStages], drain;
  __shared__ uint32_t tmem_base;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bpr = p.bpr;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(Cfg::kTmem)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (uint32_t s = 0; s < kStages; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&done[s]), 1);
      mbar_init(smem_addr(&empty[s]), kEpiWarps);
    }
    mbar_init(smem_addr(&drain), 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  // Persistent tile loop: CTA c takes tiles c, c + gridDim.x, ...; tile i is
  // (weight tile i % n_mt, token tile i / n_mt), so the CTAs of one wave share
  // their token tile through L2.  gb counts this CTA's blocks over all its
  // tiles and drives every stage / phase, so one tile's epilogue overlaps
  // the next tile's copies and MMAs.
  // With a K split, tile i also names its block range: (weight tile, token
  // tile, split); split ks covers blocks [ks * bpr / S, (ks + 1) * bpr / S).
  const uint32_t S = p.ksplit > 1 ? p.ksplit : 1u;
  const uint32_t n_mt = p.rows / kTileM, n_nt = (p.T + kTileN - 1) / kTileN, n_tiles = n_mt * n_nt * S;
  auto tile_of = [&](uint32_t tix, uint32_t &mt, uint32_t &nt, uint32_t &b0, uint32_t &b1) {
    mt = tix % n_mt;
    const uint32_t r = tix / n_mt, ks = r / n_nt;
    nt = r % n_nt;
    b0 = static_cast<uint32_t>(static_cast<uint64_t>(ks) * bpr / S);
    b1 = static_cast<uint32_t>(static_cast<uint64_t>(ks + 1) * bpr / S);
  };
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t gb = 0;
      bool stop = false;
      for (uint32_t tix = blockIdx.x; tix < n_tiles && !stop; tix += gridDim.x) {
        uint32_t mt, nt, b0, b1;
        tile_of(tix, mt, nt, b0, b1);
        // token tile nt: rows [nt NT, nt NT + NT) of the 128-row activation
        // tiles, which in the canonical layout are NT * 32 contiguous bytes
        const uint32_t tt = nt * kTileN / kMmaTile, r0 = nt * kTileN % kMmaTile;
        // block b of a tile: kMmaBlockBytes at b * kMmaBlockBytes, its 4 KB
        // of digits then the 128 rows' scales (ops.h)
        const int8_t *wa = p.wt + static_cast<size_t>(mt) * bpr * kMmaBlockBytes;
        const int8_t *xa = p.xt + static_cast<size_t>(tt) * bpr * kMmaBlockBytes;
        for (uint32_t b = b0; b < b1; ++b, ++gb) {
          const uint32_t s = gb % kStages;
          if (gb >= kStages && !mbar_wait(smem_addr(&empty[s]), ((gb / kStages) - 1) & 1, p.status)) {
            stop = true;
            break;
          }
          const uint32_t st = smem_addr(ring + s * kStageBytes), fb = smem_addr(&full[s]);
          mbar_arrive_expect_tx(fb, Cfg::kStageLoad);
          const int8_t *xb = xa + static_cast<size_t>(b) * kMmaBlockBytes;
          bulk_copy_g2s(st + kStA, wa + static_cast<size_t>(b) * kMmaBlockBytes, kMmaBlockBytes, fb);
          if (kTileN == kMmaTile) {
            bulk_copy_g2s(st + kStB, xb, kMmaBlockBytes, fb);
          } else {
            bulk_copy_g2s(st + kStB, xb + r0 * 32u, kTileN * 32, fb);
            bulk_copy_g2s(st + kStX, xb + 4096u + r0 * 4u, kTileN * 4, fb);
          }
        }
      }
      // never leave a copy in flight when the CTA may exit
      for (uint32_t j = gb > kStages ? gb - kStages : 0; j < gb; ++j)
        mbar_wait(smem_addr(&full[j % kStages]), (j / kStages) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t gb = 0;
      bool stop = false;
      for (uint32_t tix = blockIdx.x; tix < n_tiles && !stop; tix += gridDim.x) {
        uint32_t mt, nt, b0, b1;
        tile_of(tix, mt, nt, b0, b1);
        for (uint32_t b = b0; b < b1; ++b, ++gb) {
          const uint32_t s = gb % kStages;
          if (!mbar_wait(smem_addr(&full[s]), (gb / kStages) & 1, p.status)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_addr(ring + s * kStageBytes);
          umma_i8(tmem + s * kTileN, umma_desc(st + kStA, 128, 256), umma_desc(st + kStB, 128, 256), kIdesc, 0u);
          umma_commit(smem_addr(&done[s]));
        }
      }
      // every MMA of this thread has completed before TMEM is freed
      umma_commit(smem_addr(&drain));
      mbar_wait(smem_addr(&drain), 0, p.status);
    }
  } else {
    // ---------------- epilogue ----------------
    // TMEM lane quarter (a warp reads the quarter warp % 4) and group of CW token columns
    constexpr uint32_t CW = Cfg::kCols;
    const uint32_t q = warp & 3, c = kEpiWarps == 16 ? (warp - 2) >> 2 : 0;
    uint32_t gb = 0;
    bool ok = true;
    for (uint32_t tix = blockIdx.x; tix < n_tiles; tix += gridDim.x) {
      uint32_t mt, nt, b0, b1;
      tile_of(tix, mt, nt, b0, b1);
      float acc[CW];
#pragma unroll
      for (int j = 0; j < static_cast<int>(CW); ++j) acc[j] = 0.f;
      // wait for block gbk's accumulator and start its TMEM load
      auto tmem_ld = [&](uint32_t gbk, uint32_t (&v)[CW]) -> bool {
        const uint32_t sk = gbk % kStages, park = (gbk / kStages) & 1;
        if (!mbar_wait(smem_addr(&done[sk]), park, p.status) || !mbar_wait(smem_addr(&full[sk]), park, p.status))
          return false;
        tc_fence_after();
        tmem_ld32(tmem + ((32u * q) << 16) + sk * kTileN + CW * c, v);
        return true;
      };
      // block b (its load issued, global block count gb):
      // acc += (sumi * d_w) * d_x, two columns per packed instruction.  sumi
      // -> f32 exactly: |sumi| <= 32 * 8 * 127 < 2^22, so sumi + 1.5 * 2^23
      // taken as float bits, minus 1.5 * 2^23, is sumi
      auto step = [&](uint32_t (&v)[CW]) {
        tmem_ld_wait();
        const uint32_t s = gb % kStages;
        const uint8_t *st = ring + s * kStageBytes;
        const float dw = reinterpret_cast<const float *>(st + kStW)[32 * q + lane];
        const float4 *dx4 = reinterpret_cast<const float4 *>(st + kStX) + (CW / 4) * c;
        const float2 dw2 = make_float2(dw, dw), magic = make_float2(-12582912.0f, -12582912.0f);
#pragma unroll
        for (int j4 = 0; j4 < static_cast<int>(CW / 4); ++j4) {
          const float4 d4 = dx4[j4];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int j = 4 * j4 + 2 * k;
            float2 f = make_float2(__int_as_float(static_cast<int>(v[j]) + 0x4B400000),
                                   __int_as_float(static_cast<int>(v[j + 1]) + 0x4B400000));
            f = mul2_rn(mul2_rn(add2_rn(f, magic), dw2), k ? make_float2(d4.z, d4.w) : make_float2(d4.x, d4.y));
            acc[j] = __fadd_rn(acc[j], f.x);
            acc[j + 1] = __fadd_rn(acc[j + 1], f.y);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&empty[s]));
        ++gb;
      };
      uint32_t va[CW];
      for (uint32_t b = b0; b < b1 && ok; ++b) {
        ok = tmem_ld(gb, va);
        if (ok) step(va);
      }
      tmem_ld_wait();
      const uint32_t row = mt * kTileM + 32 * q + lane;
#pragma unroll
      for (int j = 0; j < static_cast<int>(CW); ++j) {
        const uint32_t t = nt * kTileN + CW * c + j;
        if (t < p.T) {
          const float val = ok ? acc[j] : __uint_as_float(0x7fc00000u);
          if (S > 1) {   // this split's partial; the reduce kernel adds the splits in order
            const uint32_t ks = tix / (n_mt * n_nt);
            p.part[(static_cast<uint64_t>(ks) * p.T + t) * p.rows + row] = val;
          } else {
            float *dst = p.y + static_cast<uint64_t>(t) * p.ldy + row;
            *dst = p.resadd ? __fadd_rn(*dst, val) : val;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::kTmem) : "memory");
}

// y[t][r] = (resadd ? y[t][r] : 0) + sum over splits, added in split order.
__global__ void mma_split_reduce_kernel(const float *part, float *y, uint32_t rows, uint32_t T, uint32_t ldy,
                                        uint32_t S, uint32_t resadd) {
  const uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<uint64_t>(rows) * T) return;
  const uint32_t t = static_cast<uint32_t>(i / rows), r = static_cast<uint32_t>(i % rows);
  float acc = part[i];
  for (uint32_t ks = 1; ks < S; ++ks) acc = __fadd_rn(acc, part[static_cast<uint64_t>(ks) * rows * T + i]);
  float *dst = y + static_cast<uint64_t>(t) * ldy + r;
  *dst = resadd ? __fadd_rn(*dst, acc) : acc;
}

// Q4_0 or Q8_0 group streams -> weight tiles: CTA (row tile, block), thread
// = row.  Q4_0 nibbles become q - 8 (elements 0..15 from the low nibbles,
// 16..31 from the high); Q8_0's two 16-byte planes of a row are its halves.
template <uint32_t QT>
__global__ void build_w8_tiles_kernel(const uint8_t *w, uint64_t gstride, uint32_t bpr, int8_t *wt, float *ws) {
  const uint32_t row = blockIdx.x * kTileM + threadIdx.x, b = blockIdx.y;
  const uint8_t *grp = w + static_cast<uint64_t>(row >> 2) * gstride;
  const uint8_t *sc = grp + scale_entry(QT, bpr, b) + 2 * (row & 3);
  uint4 lo, hi;
  if (QT == ZGPU_Q4_0) {
    const uint4 qv = *reinterpret_cast<const uint4 *>(grp + plane_entry(QT, bpr, b, row & 3));
    lo.x = nib_to_s8(qv.x & 0x0F0F0F0Fu);
    lo.y = nib_to_s8(qv.y & 0x0F0F0F0Fu);
    lo.z = nib_to_s8(qv.z & 0x0F0F0F0Fu);
    lo.w = nib_to_s8(qv.w & 0x0F0F0F0Fu);
    hi.x = nib_to_s8((qv.x >> 4) & 0x0F0F0F0Fu);
    hi.y = nib_to_s8((qv.y >> 4) & 0x0F0F0F0Fu);
    hi.z = nib_to_s8((qv.z >> 4) & 0x0F0F0F0Fu);
    hi.w = nib_to_s8((qv.w >> 4) & 0x0F0F0F0Fu);
  } else {
    lo = *reinterpret_cast<const uint4 *>(grp + plane_entry(QT, bpr, b, 2 * (row & 3)));
    hi = *reinterpret_cast<const uint4 *>(grp + plane_entry(QT, bpr, b, 2 * (row & 3) + 1));
  }
  *reinterpret_cast<uint4 *>(wt + mma_tile_off(row, b, bpr, 0)) = lo;
  *reinterpret_cast<uint4 *>(wt + mma_tile_off(row, b, bpr, 1)) = hi;
  ws[mma_scale_off(row, b, bpr)] = h2f(static_cast<uint16_t>(sc[0] | (sc[1] << 8)));
}

// Q8_0 activation tiles: one warp per (row, block) of the padded row count;
// rows past T become zero digits and scale 0.  The packer's rule, as
// quantize_q8_0_kernel.
__global__ void quantize_q8_0_tiles_kernel(const float *x, int8_t *xt, float *xs, uint32_t T, uint32_t bpr,
                                           uint64_t nwarps, uint32_t *status) {
  const uint64_t wb = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (wb >= nwarps) return;
  const uint32_t t = static_cast<uint32_t>(wb / bpr), b = static_cast<uint32_t>(wb % bpr);
  int8_t *qa = xt + mma_tile_off(t, b, bpr, lane >> 4) + (lane & 15);
  float *da = xs + mma_scale_off(t, b, bpr);
  if (t >= T) {
    *qa = 0;
    if (lane == 0) *da = 0.f;
    return;
  }
  quant_lane_q8_0(x[static_cast<uint64_t>(t) * bpr * 32 + 32 * b + lane], qa, da, lane, status);
}

}  // namespace

namespace {
int g_sm_count = 0;   // SMs of the device (one resident CTA each)
}

cudaError_t mma_setup() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(q4q8_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmaCfg<128>::kDyn);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(q4q8_mma_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, MmaCfg<32>::kDyn);
  return e;
}

cudaError_t launch_q4q8_mma(const MmaGemmParams &p, cudaStream_t s) {
  if (p.rows == 0 || p.rows % kTileM || p.bpr == 0 || p.T == 0 || !p.wt || !p.ws || !p.xt || !p.xs ||
      g_sm_count <= 0)
    return cudaErrorInvalidValue;
  const uint32_t S = p.ksplit > 1 ? p.ksplit : 1u;
  if (S > p.bpr || (S > 1 && !p.part)) return cudaErrorInvalidValue;
  // a few tokens (batched decode): 32-token tiles, 16 blocks in flight; the
  // per-row arithmetic is the same for both widths
  const uint32_t nt_w = p.T <= 32 ? 32u : 128u;
  const uint64_t tiles = static_cast<uint64_t>(p.rows / kTileM) * ((p.T + nt_w - 1) / nt_w) * S;
  const uint64_t slots = static_cast<uint64_t>(g_sm_count) * (nt_w == 32 ? MmaCfg<32>::kCtasPerSm : 1u);
  const unsigned grid = static_cast<unsigned>(tiles < slots ? tiles : slots);
  if (nt_w == 32)
    q4q8_mma_kernel<32><<<grid, MmaCfg<32>::kThreads, MmaCfg<32>::kDyn, s>>>(p);
  else
    q4q8_mma_kernel<128><<<grid, MmaCfg<128>::kThreads, MmaCfg<128>::kDyn, s>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || S == 1) return e;
  const uint64_t n = static_cast<uint64_t>(p.rows) * p.T;
  mma_split_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(p.part, p.y, p.rows, p.T, p.ldy, S,
                                                                              p.resadd);
  return cudaGetLastError();
}

uint32_t mma_ksplit(uint32_t rows, uint32_t bpr) {
  // The split that minimises the blocks the busiest CTA streams: waves of
  // (weight tile, split) pairs over the SMs times the blocks of one split,
  // plus a few blocks' worth of per-tile start-up; at least 4 blocks a split.
  // CTA slots of the 32-wide tile (the split serves few tokens): two per SM
  const uint32_t n_mt = rows / kTileM,
                 sms = (g_sm_count > 0 ? static_cast<uint32_t>(g_sm_count) : 148u) * MmaCfg<32>::kCtasPerSm;
  if (n_mt == 0) return 1;
  const uint32_t s_max = std::min(kMmaMaxSplit, std::max(1u, bpr / 4));
  uint32_t best = 1;
  uint64_t best_cost = ~0ull;
  for (uint32_t S = 1; S <= s_max; ++S) {
    const uint64_t waves = (static_cast<uint64_t>(n_mt) * S + sms - 1) / sms;
    const uint64_t cost = waves * ((bpr + S - 1) / S + 4);
    if (cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

cudaError_t launch_build_w8_tiles(const uint8_t *w, uint64_t gstride, uint32_t rows, uint32_t bpr, uint32_t quant,
                                  int8_t *wt, float *ws, cudaStream_t s) {
  if (rows == 0 || rows % kTileM || bpr == 0 || gstride % 16) return cudaErrorInvalidValue;
  if (quant == ZGPU_Q4_0)
    build_w8_tiles_kernel<ZGPU_Q4_0><<<dim3(rows / kTileM, bpr), kTileM, 0, s>>>(w, gstride, bpr, wt, ws);
  else if (quant == ZGPU_Q8_0)
    build_w8_tiles_kernel<ZGPU_Q8_0><<<dim3(rows / kTileM, bpr), kTileM, 0, s>>>(w, gstride, bpr, wt, ws);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0_tiles(const float *x, int8_t *xt, float *xs, uint32_t T, uint32_t K,
                                       uint32_t *status, cudaStream_t s) {
  if (T == 0 || K == 0 || K % 32) return cudaErrorInvalidValue;
  const uint32_t bpr = K / 32;
  const uint64_t rows = (static_cast<uint64_t>(T) + kMmaTile - 1) / kMmaTile * kMmaTile;
  const uint64_t nwarps = rows * bpr;
  quantize_q8_0_tiles_kernel<<<static_cast<unsigned>((nwarps * 32 + 255) / 256), 256, 0, s>>>(x, xt, xs, T, bpr,
                                                                                            nwarps, status);
  return cudaGetLastError();
}

}  // namespace zgpu
