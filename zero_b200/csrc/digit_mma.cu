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
// One CTA per SM, persistent over units (segment, 128-row tile, chunk of 32
// blocks, vector group), all roles walking the same sequence of present
// blocks (a chunk's blocks in bit-reversed order; the missing blocks of a
// short last chunk count as +0 in the tree, as the GEMV's idle lanes):
//   warp 0     image producer: the block's 1600-byte digit image (48 rows and
//              16 block scales) by one bulk copy into slot s = k % 4;
//   warp 1     MMA issuer: one tcgen05.mma into accumulator s, commit;
//   warps 2-5  epilogue: TMEM lane quarter (warp % 4), 16 vectors per thread;
//   warps 6-9  weight converters: thread = row; cp.async of the row's 16 (32)
//              bytes and its scale word 7 blocks ahead, then int8 A tile,
//              row sum and f32 scale into slot s.
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

constexpr uint32_t kDmSlots = 4;                         // A / image / scale slots = accumulators
constexpr uint32_t kDmStg = 8;                           // weight staging depth per converter thread
constexpr uint32_t kDmAccCols = 64;                      // TMEM columns per accumulator (48 used)
constexpr uint32_t kDmTmem = kDmSlots * kDmAccCols;      // 256
constexpr uint32_t kDmThreads = 320;
constexpr uint32_t kOffA = 0;                                        // kDmSlots x 4 KB int8 tiles
constexpr uint32_t kOffB = kOffA + kDmSlots * 4096;                  // kDmSlots x image blocks
constexpr uint32_t kOffQ = kOffB + kDmSlots * kDmImgBlock;           // kDmStg x 128 rows x 32 B
constexpr uint32_t kOffS = kOffQ + kDmStg * 128 * 32;                // kDmStg x 128 scale words
constexpr uint32_t kOffDw = kOffS + kDmStg * 128 * 4;                // kDmSlots x 128 f32 d_w
constexpr uint32_t kOffRs = kOffDw + kDmSlots * 128 * 4;             // kDmSlots x 128 s32 row sums
constexpr uint32_t kDmSmem = kOffRs + kDmSlots * 128 * 4;
// kind::i8, D s32, A and B signed, K-major, N = 48, M = 128
constexpr uint32_t kDmIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((kDmN >> 3) << 17) | ((128u >> 4) << 24);
static_assert(kDmSmem + 1024 <= 227 * 1024, "shared memory");
static_assert(kOffB % 16 == 0 && kOffQ % 16 == 0 && kDmImgBlock % 16 == 0, "bulk-copy alignment");

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
  const uint32_t v = blockIdx.x, im = blockIdx.y;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t nvi = p.n_vec_of ? min(__ldcg(p.n_vec_of + im), p.n_vec) : p.n_vec;
  const bool live = v < nvi;
  const float *x = p.x;
  if (live)
    x = p.x_rows ? p.x + static_cast<uint64_t>(__ldcg(p.x_rows + im * kDmMaxVec + v)) * p.x_stride
                 : p.x + im * p.x_img_stride + static_cast<uint64_t>(v) * p.x_stride;
  float inv = 1.0f;
  if (p.norm_w && live) inv = rms_inv<8>(x, p.in_dim, p.eps, red, tid, 1);
  const uint32_t bpr = p.in_dim / 32, nf4 = p.in_dim / 4, ng = (p.n_vec + kDmVec - 1) / kDmVec;
  const uint32_t g = v / kDmVec, vl = v % kDmVec;
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
        *reinterpret_cast<uint32_t *>(blk + kmaj_off(d * kDmVec + vl, j >> 4) + (j & 15)) = dw[d];
      if ((f & 7) == 0) *reinterpret_cast<float *>(blk + kDmN * 32 + vl * 4) = bs;
    }
  }
}

// ------------------------------------------------------------ the MMA kernel
struct DmGeom {
  uint32_t bpr, ks, n_mt, n_vg, n_units;
};

__device__ __forceinline__ DmGeom dm_geom(const DmGemmParams &p) {
  DmGeom g;
  g.bpr = p.in_dim / 32;
  g.ks = (g.bpr + kChunkBlocks - 1) / kChunkBlocks;
  g.n_mt = (p.rows + 127) / 128;
  g.n_vg = (p.n_vec + kDmVec - 1) / kDmVec;
  g.n_units = p.n_seg * g.n_mt * g.ks * g.n_vg;
  return g;
}

struct DmUnit {
  uint32_t seg, mt, c, vg, nb, nv;   // nv: vectors of this unit's group
  const uint8_t *w;                  // the segment's group streams
};

// Decode unit u; false when it has no work (a zero table entry, or no
// vector in its group).
__device__ __forceinline__ bool dm_unit(const DmGemmParams &p, const DmGeom &g, uint32_t u, DmUnit &x) {
  x.vg = u % g.n_vg;
  x.c = (u / g.n_vg) % g.ks;
  x.mt = (u / (g.n_vg * g.ks)) % g.n_mt;
  x.seg = u / (g.n_vg * g.ks * g.n_mt);
  x.nb = chunk_blocks(g.bpr, x.c);
  const uint32_t nvs = p.n_vec_of ? min(__ldcg(p.n_vec_of + x.seg), p.n_vec) : p.n_vec;
  if (nvs <= x.vg * kDmVec) return false;
  x.nv = min(nvs - x.vg * kDmVec, kDmVec);
  if (p.w_tab) {
    x.w = reinterpret_cast<const uint8_t *>(__ldcg(p.w_tab + x.seg % p.w_tab_mod));
    if (!x.w) return false;
  } else {
    x.w = p.w + x.seg * p.w_seg_stride;
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
  __shared__ __align__(8) uint64_t afull[kDmSlots], bfull[kDmSlots], done[kDmSlots], eempty[kDmSlots], drain;
  __shared__ uint32_t tmem_base;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const DmGeom g = dm_geom(p);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kDmTmem)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    for (uint32_t s = 0; s < kDmSlots; ++s) {
      mbar_init(smem_addr(&afull[s]), 4);
      mbar_init(smem_addr(&bfull[s]), 1);
      mbar_init(smem_addr(&done[s]), 1);
      mbar_init(smem_addr(&eempty[s]), 4);
    }
    mbar_init(smem_addr(&drain), 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  pdl_launch_dependents();
  pdl_wait();   // images and dispatch tables are earlier kernels' outputs

  const uint64_t img_bytes = static_cast<uint64_t>(g.n_vg) * g.bpr * kDmImgBlock;
  DmWalk wk;
  walk_start(wk);
  if (warp == 0) {
    // ---------------- image producer ----------------
    if (lane == 0) {
      uint32_t k = 0;
      while (walk_next(p, g, wk)) {
        const uint32_t s = k % kDmSlots;
        if (k >= kDmSlots && !mbar_wait(smem_addr(&eempty[s]), ((k / kDmSlots) - 1) & 1, p.status)) break;
        const uint32_t b = wk.x.c * kChunkBlocks + br5(wk.i);
        const uint8_t *src = p.img + (p.img_seg ? wk.x.seg * img_bytes : 0) +
                             (static_cast<uint64_t>(wk.x.vg) * g.bpr + b) * kDmImgBlock;
        const uint32_t fb = smem_addr(&bfull[s]);
        mbar_arrive_expect_tx(fb, kDmImgBlock);
        bulk_copy_g2s(smem_addr(sm + kOffB + s * kDmImgBlock), src, kDmImgBlock, fb);
        ++k;
        ++wk.i;
      }
      // never leave a copy in flight when the CTA may exit
      for (uint32_t j = k > kDmSlots ? k - kDmSlots : 0; j < k; ++j)
        mbar_wait(smem_addr(&bfull[j % kDmSlots]), (j / kDmSlots) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t k = 0;
      while (walk_next(p, g, wk)) {
        const uint32_t s = k % kDmSlots, ph = (k / kDmSlots) & 1;
        if (!mbar_wait(smem_addr(&afull[s]), ph, p.status) || !mbar_wait(smem_addr(&bfull[s]), ph, p.status)) break;
        tc_fence_after();
        umma_i8(tmem + s * kDmAccCols, umma_desc(smem_addr(sm + kOffA + s * 4096), 128, 256),
                umma_desc(smem_addr(sm + kOffB + s * kDmImgBlock), 128, 256), kDmIdesc, 0u);
        umma_commit(smem_addr(&done[s]));
        ++k;
        ++wk.i;
      }
      // every MMA of this thread has completed before TMEM is freed
      umma_commit(smem_addr(&drain));
      mbar_wait(smem_addr(&drain), 0, p.status);
    }
  } else if (warp >= 6) {
    // ---------------- weight converters ----------------
    const uint32_t cr = tid - 192;   // row of the tile
    const bool q4 = p.quant == ZGPU_Q4_0;
    DmWalk ic = wk;                  // issue cursor, kDmStg - 1 blocks ahead
    uint32_t issued = 0;
    auto issue_next = [&]() {
      if (walk_next(p, g, ic)) {
        const uint32_t row = ic.x.mt * 128 + cr, st = issued % kDmStg;
        if (row < p.rows) {
          const uint32_t b = ic.x.c * kChunkBlocks + br5(ic.i);
          const uint8_t *grp = ic.x.w + static_cast<uint64_t>(row >> 2) * p.gstride;
          const uint32_t dq = smem_addr(sm + kOffQ + st * 4096 + cr * 32);
          if (q4) {
            cp_async16(dq, grp + plane_entry(ZGPU_Q4_0, g.bpr, b, row & 3), 16);
          } else {
            cp_async16(dq, grp + plane_entry(ZGPU_Q8_0, g.bpr, b, 2 * (row & 3)), 16);
            cp_async16(dq + 16, grp + plane_entry(ZGPU_Q8_0, g.bpr, b, 2 * (row & 3) + 1), 16);
          }
          cp_async4(smem_addr(sm + kOffS + st * 512 + cr * 4),
                    grp + scale_entry(p.quant, g.bpr, b) + 4 * ((row & 3) >> 1), 4);
        }
        ++ic.i;
        ++issued;
      }
      cp_async_commit();
    };
    for (uint32_t j = 0; j + 1 < kDmStg; ++j) issue_next();
    uint32_t k = 0;
    while (walk_next(p, g, wk)) {
      issue_next();
      cp_async_wait<kDmStg - 1>();
      const uint32_t s = k % kDmSlots;
      if (k >= kDmSlots && !mbar_wait(smem_addr(&eempty[s]), ((k / kDmSlots) - 1) & 1, p.status)) break;
      const uint32_t row = wk.x.mt * 128 + cr, st = k % kDmStg;
      uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
      int rs = 0;
      float dw = 0.f;
      if (row < p.rows) {
        const uint8_t *q = sm + kOffQ + st * 4096 + cr * 32;
        if (q4) {
          const uint4 qv = *reinterpret_cast<const uint4 *>(q);
          lo = make_uint4(nib_to_s8(qv.x & 0x0F0F0F0Fu), nib_to_s8(qv.y & 0x0F0F0F0Fu),
                          nib_to_s8(qv.z & 0x0F0F0F0Fu), nib_to_s8(qv.w & 0x0F0F0F0Fu));
          hi = make_uint4(nib_to_s8((qv.x >> 4) & 0x0F0F0F0Fu), nib_to_s8((qv.y >> 4) & 0x0F0F0F0Fu),
                          nib_to_s8((qv.z >> 4) & 0x0F0F0F0Fu), nib_to_s8((qv.w >> 4) & 0x0F0F0F0Fu));
        } else {
          lo = *reinterpret_cast<const uint4 *>(q);
          hi = *reinterpret_cast<const uint4 *>(q + 16);
        }
        const uint32_t ones = 0x01010101u;
        rs = dp4a_ss(lo.x, ones, dp4a_ss(lo.y, ones, dp4a_ss(lo.z, ones, dp4a_ss(lo.w, ones, 0))));
        rs = dp4a_ss(hi.x, ones, dp4a_ss(hi.y, ones, dp4a_ss(hi.z, ones, dp4a_ss(hi.w, ones, rs))));
        const uint32_t sw = *reinterpret_cast<const uint32_t *>(sm + kOffS + st * 512 + cr * 4);
        dw = h2f(static_cast<uint16_t>((row & 1) ? (sw >> 16) : (sw & 0xFFFFu)));
      }
      uint8_t *a = sm + kOffA + s * 4096;
      *reinterpret_cast<uint4 *>(a + kmaj_off(cr, 0)) = lo;
      *reinterpret_cast<uint4 *>(a + kmaj_off(cr, 1)) = hi;
      reinterpret_cast<float *>(sm + kOffDw + s * 512)[cr] = dw;
      reinterpret_cast<int *>(sm + kOffRs + s * 512)[cr] = rs;
      // generic-proxy writes, read by the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&afull[s]));
      ++k;
      ++wk.i;
    }
    cp_async_wait<0>();
  } else {
    // ---------------- epilogue ----------------
    const uint32_t q = warp & 3, rt = 32 * q + lane;   // TMEM lane quarter, tile row
    const uint32_t taddr = tmem + ((32u * q) << 16);
    uint32_t k = 0;
    bool ok = true;
    for (uint32_t u = blockIdx.x; u < g.n_units && ok; u += gridDim.x) {
      DmUnit x;
      if (!dm_unit(p, g, u, x)) continue;
      float L[5][kDmVec];
      float res[kDmVec];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float val[kDmVec];
        if (ok && static_cast<uint32_t>(br5(i)) < x.nb) {
          const uint32_t s = k % kDmSlots;
          const uint32_t ph = (k / kDmSlots) & 1;
          // the accumulator, and (acquired directly) the converters' scales
          // and the image's block scales
          ok = mbar_wait(smem_addr(&done[s]), ph, p.status) && mbar_wait(smem_addr(&afull[s]), ph, p.status) &&
               mbar_wait(smem_addr(&bfull[s]), ph, p.status);
          if (ok) {
            tc_fence_after();
            uint32_t d0[16], d1[16], d2[16];
            tmem_ld16(taddr + s * kDmAccCols, d0);
            tmem_ld16(taddr + s * kDmAccCols + 16, d1);
            tmem_ld16(taddr + s * kDmAccCols + 32, d2);
            tmem_ld_wait();
            const float dw = reinterpret_cast<const float *>(sm + kOffDw + s * 512)[rt];
            const int rs128 = reinterpret_cast<const int *>(sm + kOffRs + s * 512)[rt] * 128;
            const float *bsc = reinterpret_cast<const float *>(sm + kOffB + s * kDmImgBlock + kDmN * 32);
#pragma unroll
            for (int v = 0; v < static_cast<int>(kDmVec); ++v) {
              const int s0 = static_cast<int>(d0[v]) + rs128, s1 = static_cast<int>(d1[v]) + rs128;
              const float t = fmaf(static_cast<float>(static_cast<int>(d2[v])), 65536.0f,
                                   static_cast<float>(s0 + (s1 << 8)));
              val[v] = __fmul_rn(__fmul_rn(dw, bsc[v]), t);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_addr(&eempty[s]));
            ++k;
          }
        }
        if (!(ok && static_cast<uint32_t>(br5(i)) < x.nb)) {
#pragma unroll
          for (int v = 0; v < static_cast<int>(kDmVec); ++v) val[v] = 0.0f;
        }
        // leaf i of the chunk's tree: fold equal-sized subtrees (left + right)
#pragma unroll
        for (int lv = 0; lv < 5; ++lv) {
          if ((i >> lv) & 1) {
#pragma unroll
            for (int v = 0; v < static_cast<int>(kDmVec); ++v) val[v] = __fadd_rn(L[lv][v], val[v]);
          } else {
#pragma unroll
            for (int v = 0; v < static_cast<int>(kDmVec); ++v) L[lv][v] = val[v];
            break;
          }
        }
        if (i == 31) {
#pragma unroll
          for (int v = 0; v < static_cast<int>(kDmVec); ++v) res[v] = val[v];
        }
      }
      const uint32_t row = x.mt * 128 + rt;
      if (row < p.rows) {
        float *dst = p.part + (static_cast<uint64_t>(x.seg) * g.ks + x.c) * p.n_vec * p.rows + row;
#pragma unroll
        for (int v = 0; v < static_cast<int>(kDmVec); ++v)
          if (static_cast<uint32_t>(v) < x.nv)
            dst[static_cast<uint64_t>(x.vg * kDmVec + v) * p.rows] = ok ? res[v] : __uint_as_float(0x7fc00000u);
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
  const uint32_t seg = blockIdx.z, v = blockIdx.y;
  const uint32_t nvs = p.n_vec_of ? min(__ldcg(p.n_vec_of + seg), p.n_vec) : p.n_vec;
  if (v >= nvs) return;
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
                              static_cast<int>(kDmSmem + 1024));
}

cudaError_t launch_digit_image(const DigitImageParams &p, const LaunchCfg &lc) {
  if (p.in_dim == 0 || p.in_dim % 32 || p.n_vec == 0 || p.n_vec > kDmMaxVec || p.n_img == 0 || !p.img)
    return cudaErrorInvalidValue;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(dm_groups(p.n_vec) * kDmVec, p.n_img), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, digit_image_kernel, p);
}

cudaError_t launch_dm_gemm(const DmGemmParams &p, const LaunchCfg &lc) {
  if (p.in_dim == 0 || p.in_dim % 32 || p.rows == 0 || p.n_vec == 0 || p.n_vec > kDmMaxVec || p.n_seg == 0 ||
      p.gstride % 16 || (p.quant != ZGPU_Q4_0 && p.quant != ZGPU_Q8_0) || !p.part || !p.img ||
      (p.w_tab && p.w_tab_mod == 0) || (!p.w_tab && !p.w))
    return cudaErrorInvalidValue;
  const uint64_t units = static_cast<uint64_t>(p.n_seg) * ((p.rows + 127) / 128) *
                         ((p.in_dim / 32 + kChunkBlocks - 1) / kChunkBlocks) * dm_groups(p.n_vec);
  const uint32_t sms = lc.sm_count > 0 ? static_cast<uint32_t>(lc.sm_count) : 148u;
  const uint32_t grid = static_cast<uint32_t>(units < sms ? units : sms);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3(grid), dim3(kDmThreads), kDmSmem + 1024, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, dm_gemm_kernel, p);
}

cudaError_t launch_dm_combine(const DmCombineParams &p, const LaunchCfg &lc) {
  if (p.rows == 0 || p.ks == 0 || p.n_vec == 0 || p.n_vec > kDmMaxVec || p.n_seg == 0 ||
      (p.epi != EPI_STORE && p.epi != EPI_RESADD && p.epi != EPI_SWIGLU) ||
      (p.epi == EPI_SWIGLU && p.rows % 8) || (!p.out && !p.out_rows))
    return cudaErrorInvalidValue;
  const uint32_t out_rows = p.epi == EPI_SWIGLU ? p.rows / 2 : p.rows;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_launch_cfg(dim3((out_rows + 255) / 256, p.n_vec, p.n_seg), dim3(256), 0, lc, attr);
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, dm_combine_kernel, p);
}

}  // namespace zgpu
