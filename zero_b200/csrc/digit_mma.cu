// digit_mma.cu — batched matvec of Q4_0 / Q8_0 weights with up to 32 f32
// vectors on the tensor cores (tcgen05.mma.kind::i8), equal for every vector
// to the single-vector GEMV (gemv.cu) bit for bit.
//
// The GEMV turns each 32-element block of x into integers N_j (block_ints,
// gemv_body.cuh) split into three bytes d0, d1 (unsigned) and d2 (signed),
// forms the exact integer chains s_d = sum_j w_j d_dj (w_j = n_j - 8 for
// Q4_0, q_j for Q8_0), takes t = fma(s2, 65536, s0 + 256 s1) and adds
// (d_w * 2^(e-22)) * t over the 32 blocks of a chunk in the xor-butterfly
// tree of its warp reduce (pairs 16 apart first, then 8, 4, 2, 1), and the
// chunks in order from 0.  Here the same integer chains come out of one MMA
// per block: A = the block's 128 weight rows as int8 w_j, B = 48 digit rows
// (3 digits x 16 vectors; d0 and d1 stored minus 128 so that B is signed,
// s_d = sum w (d - 128) + 128 sum w restores them exactly), D = 128 x 48 s32
// in TMEM.  The epilogue forms t and the block term with the GEMV's
// operations and folds the blocks of a chunk in bit-reversed order with a
// five-level stack, which is the butterfly's tree; the chunk partials are
// added in order by dm_combine.  Only integer sums are reassociated, so the
// result is the GEMV's for any number of vectors.
//
// The weights are pre-tiled once per tensor (launch_build_dm_tiles: int8
// rows in the MMA layout with their f32 scales and row sums), so a block is
// two bulk copies.  One CTA per SM, persistent over units (segment, 128-row
// tile, chunk of 32 blocks, vector group), all roles walking the same
// sequence of present blocks (a chunk's blocks in bit-reversed order; the
// missing blocks of a short last chunk count as +0 in the tree, as the
// GEMV's idle lanes):
//   warp 0      producer: the weight tile block (5 KB) and the digit image
//               block (1600 B) into stage k % 8;
//   warp 1      MMA issuer: one tcgen05.mma (M 128, N 48, K 32) into
//               accumulator k % 8 once the epilogue has read block k - 8
//               out of it, commit;
//   warps 2-9   epilogue: TMEM lane quarter (warp % 4) x 8 of the 16
//               vectors (vq, vq + 2, ..., vq + 14: few vectors still use
//               every warp); the block terms folded into the chunk's tree.
// Every wait is bounded; an expired wait stops that role, which drains what
// it has in flight, and raises ZDEV_ERR_TIMEOUT.
#include <cuda_runtime.h>

#include <cfloat>
#include <stdint.h>

#include "common.cuh"
#include "digit_mma.h"
#include "gemv_body.cuh"
#include "internal.h"
#include "layout.h"
#include "ops.h"
#include "tcgen05.cuh"

namespace zgpu {

namespace {

constexpr uint32_t kDmSlots = 8;                         // shared-memory stages (blocks in flight)
constexpr uint32_t kDmAccs = 8;                          // TMEM accumulators
constexpr uint32_t kDmAccCols = 64;                      // TMEM columns per accumulator (48 used)
constexpr uint32_t kDmTmem = kDmAccs * kDmAccCols;       // 512: the whole TMEM, one CTA per SM
constexpr uint32_t kDmEpiWarps = 8;                      // 4 lane quarters x kDmVq vector sets
constexpr uint32_t kDmVq = kDmEpiWarps / 4;              // epilogue warps per TMEM lane quarter
constexpr uint32_t kDmVpw = kDmVec / kDmVq;              // vectors per epilogue thread
constexpr uint32_t kDmPairs = kDmVpw / 2;                // of them, packed f32x2 pairs
static_assert(kDmEpiWarps % 4 == 0 && kDmVec % (2 * kDmVq) == 0, "epilogue shape");
// Column position of vector v of a group: epilogue warp vq of a lane quarter
// reads positions kDmVpw * vq .. + kDmVpw - 1 = vectors vq, vq + kDmVq, ...,
// so a group with few vectors still spreads them over every warp.
__host__ __device__ __forceinline__ uint32_t dm_pos(uint32_t v) { return (v % kDmVq) * kDmVpw + v / kDmVq; }
constexpr uint32_t kDmThreads = 32 * (2 + kDmEpiWarps);  // producer, MMA, epilogue
constexpr uint32_t kDmSlotBytes = kDmTileBlock + kDmImgBlock;   // weight block, then image block
constexpr uint32_t kDmSmem = kDmSlots * kDmSlotBytes;
// more than half an SM's shared memory: a second CTA on the SM would wait on
// its TMEM allocation
constexpr uint32_t kDmDynSmem = 120 * 1024;
// kind::i8, D s32, A and B signed, K-major, N = 48, M = 128
constexpr uint32_t kDmIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((kDmN >> 3) << 17) | ((128u >> 4) << 24);
static_assert(kDmSmem + 1024 <= kDmDynSmem, "shared memory");
static_assert(kDmSlotBytes % 16 == 0 && kDmTileBlock % 16 == 0 && kDmImgBlock % 16 == 0, "bulk-copy alignment");

// byte offset of (row, K half) in a K-major no-swizzle tile: 8-row core
// matrices of 16-byte rows, K halves 128 B apart, row groups 256 B apart
__host__ __device__ __forceinline__ uint32_t kmaj_off(uint32_t row, uint32_t half) {
  return (row % 8) * 16u + (row / 8) * 256u + half * 128u;
}

__device__ __forceinline__ uint32_t br5(uint32_t i) { return __brev(i) >> 27; }

// ------------------------------------------------------------ digit image
__global__ void __launch_bounds__(256) digit_image_kernel(const DigitImageParams p) {
  __shared__ float red[8];
  pdl_launch_dependents();
  pdl_wait();
  uint32_t v = blockIdx.x, im = blockIdx.y;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t nvi;
  if (p.pairs) {
    if (blockIdx.x >= __ldcg(p.n_pairs)) return;
    const uint32_t iv = __ldcg(p.pairs + blockIdx.x);
    im = iv >> 8;
    v = iv & 0xFFu;
    nvi = v + 1;   // this vector is live
  } else {
    nvi = p.n_vec_of ? min(__ldcg(p.n_vec_of + im), p.n_vec) : p.n_vec;
    // a vector group no unit reads (all past the count) is not written
    if (v >= (nvi + kDmVec - 1) / kDmVec * kDmVec) return;
  }
  const bool live = v < nvi;
  const float *x = p.x;
  if (live)
    x = p.x_rows ? p.x + static_cast<uint64_t>(__ldcg(p.x_rows + im * kDmMaxVec + v)) * p.x_stride
                 : p.x + im * p.x_img_stride + static_cast<uint64_t>(v) * p.x_stride;
  float inv = 1.0f;
  if (p.norm_w && live) inv = rms_inv<8>(x, p.in_dim, p.eps, red, tid, 1);
  const uint32_t bpr = p.in_dim / 32, nf4 = p.in_dim / 4, ng = (p.n_vec + kDmVec - 1) / kDmVec;
  // vector vl of group g sits at column position pv (dm_pos)
  const uint32_t g = v / kDmVec, vl = v % kDmVec, pv = dm_pos(vl);
  uint8_t *img = p.img + (static_cast<uint64_t>(im) * ng + g) * bpr * kDmImgBlock;
  // warp-uniform trip count: a block's 8 lanes are all in range or all out
  for (uint32_t f0 = warp * 32; f0 < nf4; f0 += 256) {
    const uint32_t f = f0 + lane;
    const bool valid = live && f < nf4;
    float4 t = valid ? __ldcg(reinterpret_cast<const float4 *>(x) + f) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (p.norm_w && valid) {
      const float4 gw = reinterpret_cast<const float4 *>(p.norm_w)[f];
      t.x = __fmul_rn(__fmul_rn(t.x, inv), gw.x);
      t.y = __fmul_rn(__fmul_rn(t.y, inv), gw.y);
      t.z = __fmul_rn(__fmul_rn(t.z, inv), gw.z);
      t.w = __fmul_rn(__fmul_rn(t.w, inv), gw.w);
    }
    int n[4];
    const float bs = block_ints(t, n);
    if (f < nf4) {
      const uint32_t b = f >> 3, j = (f & 7) * 4;   // elements j..j+3 of block b
      uint8_t *blk = img + static_cast<uint64_t>(b) * kDmImgBlock;
      const uint32_t w0 = __byte_perm(__byte_perm(n[0], n[1], 0x0040), __byte_perm(n[2], n[3], 0x0040), 0x5410);
      const uint32_t w1 = __byte_perm(__byte_perm(n[0], n[1], 0x0051), __byte_perm(n[2], n[3], 0x0051), 0x5410);
      const uint32_t w2 = __byte_perm(__byte_perm(n[0], n[1], 0x0062), __byte_perm(n[2], n[3], 0x0062), 0x5410);
      const uint32_t dw[3] = {w0 ^ 0x80808080u, w1 ^ 0x80808080u, w2};
#pragma unroll
      for (int d = 0; d < 3; ++d)
        *reinterpret_cast<uint32_t *>(blk + kmaj_off(d * kDmVec + pv, j >> 4) + (j & 15)) = dw[d];
      if ((f & 7) == 0) *reinterpret_cast<float *>(blk + kDmN * 32 + pv * 4) = bs;
    }
  }
}

// ------------------------------------------------------------ weight tiles
// CTA (tile, block), thread = row of the tile.
__global__ void __launch_bounds__(128) build_dm_tiles_kernel(const uint8_t *w, uint64_t gstride, uint32_t quant,
                                                             uint32_t rows, uint32_t bpr, uint8_t *tiles) {
  const uint32_t t = blockIdx.x, b = blockIdx.y, r = threadIdx.x, row = t * 128 + r;
  uint8_t *blk = tiles + (static_cast<uint64_t>(t) * bpr + b) * kDmTileBlock;
  uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
  float dw = 0.f;
  int rs = 0;
  if (row < rows) {
    const uint8_t *grp = w + static_cast<uint64_t>(row >> 2) * gstride;
    if (quant == ZGPU_Q4_0) {
      const uint4 qv = *reinterpret_cast<const uint4 *>(grp + plane_entry(ZGPU_Q4_0, bpr, b, row & 3));
      lo = make_uint4(nib_to_s8(qv.x & 0x0F0F0F0Fu), nib_to_s8(qv.y & 0x0F0F0F0Fu), nib_to_s8(qv.z & 0x0F0F0F0Fu),
                      nib_to_s8(qv.w & 0x0F0F0F0Fu));
      hi = make_uint4(nib_to_s8((qv.x >> 4) & 0x0F0F0F0Fu), nib_to_s8((qv.y >> 4) & 0x0F0F0F0Fu),
                      nib_to_s8((qv.z >> 4) & 0x0F0F0F0Fu), nib_to_s8((qv.w >> 4) & 0x0F0F0F0Fu));
    } else {
      lo = *reinterpret_cast<const uint4 *>(grp + plane_entry(ZGPU_Q8_0, bpr, b, 2 * (row & 3)));
      hi = *reinterpret_cast<const uint4 *>(grp + plane_entry(ZGPU_Q8_0, bpr, b, 2 * (row & 3) + 1));
    }
    const uint32_t ones = 0x01010101u;
    rs = dp4a_ss(lo.x, ones, dp4a_ss(lo.y, ones, dp4a_ss(lo.z, ones, dp4a_ss(lo.w, ones, 0))));
    rs = dp4a_ss(hi.x, ones, dp4a_ss(hi.y, ones, dp4a_ss(hi.z, ones, dp4a_ss(hi.w, ones, rs))));
    const uint8_t *sc = grp + scale_entry(quant, bpr, b) + 2 * (row & 3);
    dw = h2f(static_cast<uint16_t>(sc[0] | (sc[1] << 8)));
  }
  *reinterpret_cast<uint4 *>(blk + kmaj_off(r, 0)) = lo;
  *reinterpret_cast<uint4 *>(blk + kmaj_off(r, 1)) = hi;
  reinterpret_cast<float *>(blk + 4096)[r] = dw;
  reinterpret_cast<int *>(blk + 4096 + 512)[r] = rs;
}

// ------------------------------------------------------------ the MMA kernel
struct DmGeom {
  uint32_t bpr, ks, n_mt, n_vg, n_units;
  // per-segment vector counts and tile bases, copied to shared memory once
  // (null: read from global memory, for launches of many segments)
  const uint32_t *nv_s;
  const unsigned long long *tab_s;
};
constexpr uint32_t kDmSegCache = 256;

__device__ __forceinline__ DmGeom dm_geom(const DmGemmParams &p) {
  DmGeom g;
  g.bpr = p.in_dim / 32;
  g.ks = (g.bpr + kChunkBlocks - 1) / kChunkBlocks;
  g.n_mt = (p.rows + 127) / 128;
  g.n_vg = (p.n_vec + kDmVec - 1) / kDmVec;
  g.n_units = p.n_seg * g.n_mt * g.ks * g.n_vg;
  g.nv_s = nullptr;
  g.tab_s = nullptr;
  return g;
}

struct DmUnit {
  uint32_t seg, mt, c, vg, nb, nv;   // nv: vectors of this unit's group
  const uint8_t *w;                  // the segment's weight tiles
};

// Decode unit u; false when it has no work (a zero table entry, or no
// vector in its group).
__device__ __forceinline__ bool dm_unit(const DmGemmParams &p, const DmGeom &g, uint32_t u, DmUnit &x) {
  x.vg = u % g.n_vg;
  x.c = (u / g.n_vg) % g.ks;
  x.mt = (u / (g.n_vg * g.ks)) % g.n_mt;
  x.seg = u / (g.n_vg * g.ks * g.n_mt);
  x.nb = chunk_blocks(g.bpr, x.c);
  const uint32_t nvs = g.nv_s ? g.nv_s[x.seg] : p.n_vec_of ? min(__ldcg(p.n_vec_of + x.seg), p.n_vec) : p.n_vec;
  if (nvs <= x.vg * kDmVec) return false;
  x.nv = min(nvs - x.vg * kDmVec, kDmVec);
  if (p.w_tab) {
    x.w = reinterpret_cast<const uint8_t *>(g.tab_s ? g.tab_s[x.seg] : __ldcg(p.w_tab + x.seg % p.w_tab_mod));
    if (!x.w) return false;
  } else {
    x.w = p.wt + x.seg * p.wt_seg_stride;
  }
  return true;
}

// A walk over this CTA's present blocks: units blockIdx.x + k gridDim.x,
// each chunk's blocks in bit-reversed order, missing blocks skipped.
struct DmWalk {
  uint32_t u, i;
  DmUnit x;
  bool live;   // x decoded for u
};

__device__ __forceinline__ void walk_start(DmWalk &w) {
  w.u = blockIdx.x;
  w.i = 0;
  w.live = false;
}

// Advance to the next present block at or after the cursor; false at the end.
__device__ __forceinline__ bool walk_next(const DmGemmParams &p, const DmGeom &g, DmWalk &w) {
  while (w.u < g.n_units) {
    if (!w.live) {
      if (!dm_unit(p, g, w.u, w.x)) {
        w.u += gridDim.x;
        w.i = 0;
        continue;
      }
      w.live = true;
    }
    while (w.i < 32 && br5(w.i) >= w.x.nb) ++w.i;
    if (w.i < 32) return true;
    w.u += gridDim.x;
    w.i = 0;
    w.live = false;
  }
  return false;
}

__global__ void __launch_bounds__(kDmThreads, 1) dm_gemm_kernel(const DmGemmParams p) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kDmSlots], eempty[kDmSlots], done[kDmAccs], drain;
  __shared__ uint32_t tmem_base;
  __shared__ uint32_t nv_s[kDmSegCache];
  __shared__ unsigned long long tab_s[kDmSegCache];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  DmGeom g = dm_geom(p);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kDmTmem)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (uint32_t s = 0; s < kDmSlots; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&eempty[s]), kDmEpiWarps);
    }
    for (uint32_t a = 0; a < kDmAccs; ++a) mbar_init(smem_addr(&done[a]), 1);
    mbar_init(smem_addr(&drain), 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch_dependents();
  pdl_wait();   // images and dispatch tables are earlier kernels' outputs
  if (p.n_seg <= kDmSegCache) {
    for (uint32_t sg = tid; sg < p.n_seg; sg += kDmThreads) {
      nv_s[sg] = p.n_vec_of ? min(__ldcg(p.n_vec_of + sg), p.n_vec) : p.n_vec;
      tab_s[sg] = p.w_tab ? __ldcg(p.w_tab + sg % p.w_tab_mod) : 0ull;
    }
    __syncthreads();
    g.nv_s = nv_s;
    g.tab_s = p.w_tab ? tab_s : nullptr;
  }

  const uint64_t img_bytes = static_cast<uint64_t>(g.n_vg) * g.bpr * kDmImgBlock;
  DmWalk wk;
  walk_start(wk);
  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      uint32_t k = 0;
      while (walk_next(p, g, wk)) {
        const uint32_t s = k % kDmSlots;
        if (k >= kDmSlots && !mbar_wait(smem_addr(&eempty[s]), ((k / kDmSlots) - 1) & 1, p.status)) break;
        const uint32_t b = wk.x.c * kChunkBlocks + br5(wk.i);
        const uint8_t *wsrc = wk.x.w + (static_cast<uint64_t>(wk.x.mt) * g.bpr + b) * kDmTileBlock;
        const uint8_t *isrc = p.img + (p.img_seg ? wk.x.seg * img_bytes : 0) +
                              (static_cast<uint64_t>(wk.x.vg) * g.bpr + b) * kDmImgBlock;
        const uint32_t fb = smem_addr(&full[s]), dst = smem_addr(sm + s * kDmSlotBytes);
        mbar_arrive_expect_tx(fb, kDmSlotBytes);
        bulk_copy_g2s(dst, wsrc, kDmTileBlock, fb);
        bulk_copy_g2s(dst + kDmTileBlock, isrc, kDmImgBlock, fb);
        ++k;
        ++wk.i;
      }
      // never leave a copy in flight when the CTA may exit
      for (uint32_t j = k > kDmSlots ? k - kDmSlots : 0; j < k; ++j)
        mbar_wait(smem_addr(&full[j % kDmSlots]), (j / kDmSlots) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t k = 0;
      while (walk_next(p, g, wk)) {
        const uint32_t s = k % kDmSlots, a = k % kDmAccs;
        if (!mbar_wait(smem_addr(&full[s]), (k / kDmSlots) & 1, p.status)) break;
        // accumulator a is free once the epilogue has finished block k - 8
        if (k >= kDmAccs &&
            !mbar_wait(smem_addr(&eempty[(k - kDmAccs) % kDmSlots]), ((k - kDmAccs) / kDmSlots) & 1, p.status))
          break;
        tc_fence_after();
        const uint32_t st = smem_addr(sm + s * kDmSlotBytes);
        umma_i8(tmem + a * kDmAccCols, umma_desc(st, 128, 256), umma_desc(st + kDmTileBlock, 128, 256), kDmIdesc, 0u);
        umma_commit(smem_addr(&done[a]));
        ++k;
        ++wk.i;
      }
      // every MMA of this thread has completed before TMEM is freed
      umma_commit(smem_addr(&drain));
      mbar_wait(smem_addr(&drain), 0, p.status);
    }
  } else {
    // ---------------- epilogue ----------------
    // thread: tile row rt (TMEM lane quarter warp % 4) x vectors vq, vq + kDmVq,
    // ... (column positions kDmVpw * vq .. + kDmVpw - 1, dm_pos)
    const uint32_t q = warp & 3, vq = (warp - 2) >> 2, rt = 32 * q + lane;
    const uint32_t taddr = tmem + ((32u * q) << 16) + kDmVpw * vq;
    const float M = 12582912.0f;   // 1.5 * 2^23: int v, |v| < 2^22, is float(bits(M) + v) - M exactly
    uint32_t k = 0;
    bool ok = true;
    // block terms of leaf i of the chunk for the thread's vectors, as packed
    // pairs (0 for a missing block)
    auto leaf = [&](const DmUnit &x, uint32_t i, float2 (&val)[kDmPairs]) {
#pragma unroll
      for (int h = 0; h < static_cast<int>(kDmPairs); ++h) val[h] = make_float2(0.0f, 0.0f);
      if (!ok || br5(i) >= x.nb) return;
      const uint32_t s = k % kDmSlots, a = k % kDmAccs;
      // the accumulator, and (acquired directly) the stage's scales and row sums
      ok = mbar_wait(smem_addr(&done[a]), (k / kDmAccs) & 1, p.status) &&
           mbar_wait(smem_addr(&full[s]), (k / kDmSlots) & 1, p.status);
      if (!ok) return;
      ++k;
      if (vq >= x.nv) {   // none of this warp's vectors: only release the stage
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&eempty[s]));
        return;
      }
      tc_fence_after();
      uint32_t a0[kDmVpw], a1[kDmVpw], a2[kDmVpw];
      tmem_ld_cols(taddr + a * kDmAccCols, a0);
      tmem_ld_cols(taddr + a * kDmAccCols + kDmVec, a1);
      tmem_ld_cols(taddr + a * kDmAccCols + 2 * kDmVec, a2);
      const uint8_t *slot = sm + s * kDmSlotBytes;
      const float dw = reinterpret_cast<const float *>(slot + 4096)[rt];
      // s_d = a_d + 128 * row sum for the two low digits, folded into the magic constant
      const int kk = reinterpret_cast<const int *>(slot + 4096 + 512)[rt] * 128 + 0x4B400000;
      float bsv[kDmVpw];
      const float4 *bs4 = reinterpret_cast<const float4 *>(slot + kDmTileBlock + kDmN * 32) + vq * (kDmVpw / 4);
#pragma unroll
      for (int c = 0; c < static_cast<int>(kDmVpw / 4); ++c) {
        const float4 b4 = bs4[c];
        bsv[4 * c] = b4.x;
        bsv[4 * c + 1] = b4.y;
        bsv[4 * c + 2] = b4.z;
        bsv[4 * c + 3] = b4.w;
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&eempty[s]));
      const float2 m2 = make_float2(M, M), c256 = make_float2(256.0f, 256.0f), c64k = make_float2(65536.0f, 65536.0f);
      const float2 dw2 = make_float2(dw, dw);
#pragma unroll
      for (int h = 0; h < static_cast<int>(kDmPairs); ++h) {
        // pair h = vectors vq + kDmVq * 2h and vq + kDmVq * (2h + 1)
        if (vq + kDmVq * 2 * h >= x.nv) break;
        // S0, S1, S2 exactly as floats (|S| < 2^22); X = S0 + 256 S1 rounded
        // once, as the GEMV's int-to-float of its s0 + (s1 << 8)
        const float2 f0 = sub2_rn(make_float2(__int_as_float(static_cast<int>(a0[2 * h]) + kk),
                                              __int_as_float(static_cast<int>(a0[2 * h + 1]) + kk)), m2);
        const float2 f1 = sub2_rn(make_float2(__int_as_float(static_cast<int>(a1[2 * h]) + kk),
                                              __int_as_float(static_cast<int>(a1[2 * h + 1]) + kk)), m2);
        const float2 f2 = sub2_rn(make_float2(__int_as_float(static_cast<int>(a2[2 * h]) + 0x4B400000),
                                              __int_as_float(static_cast<int>(a2[2 * h + 1]) + 0x4B400000)), m2);
        const float2 t = fma2_rn(f2, c64k, fma2_rn(f1, c256, f0));
        val[h] = mul2_rn(mul2_rn(dw2, make_float2(bsv[2 * h], bsv[2 * h + 1])), t);
      }
    };
    for (uint32_t u = blockIdx.x; u < g.n_units && ok; u += gridDim.x) {
      DmUnit x;
      if (!dm_unit(p, g, u, x)) continue;
      // the chunk's 32 leaves in bit-reversed block order folded as the
      // GEMV's butterfly: 4-leaf subtrees, then a counter over 8 subtrees
      float2 L2[kDmPairs], L3[kDmPairs], L4[kDmPairs], res[kDmPairs];
      for (uint32_t o = 0; o < 8; ++o) {
        float2 s01[kDmPairs], v2[kDmPairs], v3[kDmPairs], xs[kDmPairs];
        leaf(x, 4 * o, xs);
        leaf(x, 4 * o + 1, v2);
#pragma unroll
        for (int h = 0; h < static_cast<int>(kDmPairs); ++h) s01[h] = add2_rn(xs[h], v2[h]);
        leaf(x, 4 * o + 2, v2);
        leaf(x, 4 * o + 3, v3);
#pragma unroll
        for (int h = 0; h < static_cast<int>(kDmPairs); ++h) xs[h] = add2_rn(s01[h], add2_rn(v2[h], v3[h]));
        if (o & 1) {
#pragma unroll
          for (int h = 0; h < static_cast<int>(kDmPairs); ++h) xs[h] = add2_rn(L2[h], xs[h]);
          if (o & 2) {
#pragma unroll
            for (int h = 0; h < static_cast<int>(kDmPairs); ++h) xs[h] = add2_rn(L3[h], xs[h]);
            if (o & 4) {
#pragma unroll
              for (int h = 0; h < static_cast<int>(kDmPairs); ++h) res[h] = add2_rn(L4[h], xs[h]);
            } else {
#pragma unroll
              for (int h = 0; h < static_cast<int>(kDmPairs); ++h) L4[h] = xs[h];
            }
          } else {
#pragma unroll
            for (int h = 0; h < static_cast<int>(kDmPairs); ++h) L3[h] = xs[h];
          }
        } else {
#pragma unroll
          for (int h = 0; h < static_cast<int>(kDmPairs); ++h) L2[h] = xs[h];
        }
      }
      const uint32_t row = x.mt * 128 + rt;
      if (row < p.rows) {
        float *dst = p.part + (static_cast<uint64_t>(x.seg) * g.ks + x.c) * p.n_vec * p.rows + row;
#pragma unroll
        for (int j = 0; j < static_cast<int>(kDmVpw); ++j) {
          const uint32_t v = vq + kDmVq * j;   // this thread's j-th vector
          const float r = (j & 1) ? res[j / 2].y : res[j / 2].x;
          if (v < x.nv) dst[static_cast<uint64_t>(x.vg * kDmVec + v) * p.rows] = ok ? r : __uint_as_float(0x7fc00000u);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kDmTmem) : "memory");
}

// ------------------------------------------------------------ combine
__global__ void dm_combine_kernel(const DmCombineParams p) {
  pdl_launch_dependents();
  pdl_wait();
  uint32_t seg = blockIdx.z, v = blockIdx.y;
  if (p.pairs) {
    if (blockIdx.y >= __ldcg(p.n_pairs)) return;
    const uint32_t sv = __ldcg(p.pairs + blockIdx.y);
    seg = sv >> 8;
    v = sv & 0xFFu;
  } else {
    const uint32_t nvs = p.n_vec_of ? min(__ldcg(p.n_vec_of + seg), p.n_vec) : p.n_vec;
    if (v >= nvs) return;
  }
  const uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t out_rows = p.epi == EPI_SWIGLU ? p.rows / 2 : p.rows;
  if (j >= out_rows) return;
  const float *pb = p.part + (static_cast<uint64_t>(seg) * p.ks * p.n_vec + v) * p.rows;
  const uint64_t cs = static_cast<uint64_t>(p.n_vec) * p.rows;   // chunk stride
  float *dst = p.out_rows ? p.out_rows[seg * kDmMaxVec + v]
                          : p.out + seg * p.out_seg_stride + static_cast<uint64_t>(v) * p.out_vec_stride;
  if (p.epi == EPI_SWIGLU) {
    const uint32_t r = (j / 4) * 8 + (j % 4);   // gate row; its up row is r + 4
    float yg = 0.f, yu = 0.f;
    for (uint32_t c = 0; c < p.ks; ++c) {
      yg += __ldcg(pb + c * cs + r);
      yu += __ldcg(pb + c * cs + r + 4);
    }
    dst[j] = ref_silu_mul(yg, yu);
    return;
  }
  float y = 0.f;
  for (uint32_t c = 0; c < p.ks; ++c) y += __ldcg(pb + c * cs + j);
  dst[j] = p.epi == EPI_RESADD ? dst[j] + y : y;
}

}  // namespace

cudaError_t dm_setup() {
  return cudaFuncSetAttribute(dm_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kDmDynSmem));
}

cudaError_t launch_build_dm_tiles(const uint8_t *w, uint64_t gstride, uint32_t quant, uint32_t rows, uint32_t bpr,
                                  uint8_t *tiles, cudaStream_t s) {
  if (!w || !tiles || rows == 0 || bpr == 0 || gstride % 16 || (quant != ZGPU_Q4_0 && quant != ZGPU_Q8_0))
    return cudaErrorInvalidValue;
  build_dm_tiles_kernel<<<dim3((rows + 127) / 128, bpr), 128, 0, s>>>(w, gstride, quant, rows, bpr, tiles);
  return cudaGetLastError();
}

cudaError_t launch_digit_image(const DigitImageParams &p, const LaunchCfg &lc) {
  if (p.in_dim == 0 || p.in_dim % 32 || p.n_vec == 0 || p.n_img == 0 || !p.img ||
      p.n_vec > (p.x_rows || p.n_vec_of ? kDmMaxVec : kDmMaxVecPlain))
    return cudaErrorInvalidValue;
  if (p.pairs && (!p.n_pairs || p.max_pairs == 0)) return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  const dim3 grid = p.pairs ? dim3(p.max_pairs) : dim3(dm_groups(p.n_vec) * kDmVec, p.n_img);
  cudaLaunchConfig_t cfg = make_launch_cfg(grid, dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, digit_image_kernel, p);
}

cudaError_t launch_dm_gemm(const DmGemmParams &p, const LaunchCfg &lc) {
  if (p.in_dim == 0 || p.in_dim % 32 || p.rows == 0 || p.n_vec == 0 || p.n_seg == 0 ||
      p.n_vec > (p.n_vec_of ? kDmMaxVec : kDmMaxVecPlain) || !p.part || !p.img || (p.w_tab && p.w_tab_mod == 0) ||
      (!p.w_tab && !p.wt))
    return cudaErrorInvalidValue;
  const uint64_t units = static_cast<uint64_t>(p.n_seg) * ((p.rows + 127) / 128) *
                         ((p.in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks) * dm_groups(p.n_vec);
  const uint32_t sms = lc.sm_count > 0 ? static_cast<uint32_t>(lc.sm_count) : 148u;
  uint32_t grid = static_cast<uint32_t>(units < sms ? units : sms);
  // CTA b takes units b, b + grid, ...: a grid coprime with (vector groups x
  // chunks) gives every CTA a mix of both, whose work differs (empty vector
  // groups, a short last chunk)
  const uint32_t period = dm_groups(p.n_vec) * ((p.in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks);
  auto gcd = [](uint32_t a, uint32_t b) {
    while (b) {
      const uint32_t t = a % b;
      a = b;
      b = t;
    }
    return a;
  };
  while (grid > 1 && units > grid && gcd(grid, period) != 1) --grid;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(grid), dim3(kDmThreads), kDmDynSmem, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, dm_gemm_kernel, p);
}

cudaError_t launch_dm_combine(const DmCombineParams &p, const LaunchCfg &lc) {
  if (p.rows == 0 || p.ks == 0 || p.n_vec == 0 || p.n_vec > (p.out_rows || p.n_vec_of ? kDmMaxVec : kDmMaxVecPlain) ||
      p.n_seg == 0 ||
      (p.epi != EPI_STORE && p.epi != EPI_RESADD && p.epi != EPI_SWIGLU) ||
      (p.epi == EPI_SWIGLU && p.rows % 8) || (!p.out && !p.out_rows))
    return cudaErrorInvalidValue;
  if (p.pairs && (!p.n_pairs || p.max_pairs == 0 || p.max_pairs > 65535)) return cudaErrorInvalidValue;
  const uint32_t out_rows = p.epi == EPI_SWIGLU ? p.rows / 2 : p.rows;
  cudaLaunchAttribute attr[1];
  const dim3 grid = p.pairs ? dim3((out_rows + 255) / 256, p.max_pairs, 1) : dim3((out_rows + 255) / 256, p.n_vec, p.n_seg);
  cudaLaunchConfig_t cfg = make_launch_cfg(grid, dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, dm_combine_kernel, p);
}

}  // namespace zgpu
