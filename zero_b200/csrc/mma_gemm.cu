// mma_gemm.cu — batched Q4_0 weight x Q8_0 activation matmul on the 5th-gen
// tensor cores (tcgen05, int8), for prefill and multi-token decode.
//
// Y[t][m] = sum_b d_w[m,b] * d_x[t,b] * sum_{j<32} (n[m,b,j] - 8) * q[t,b,j]
//
// Both operands carry one scale per 32-element block, so a block's integer
// dot product must be scaled before it is added to the next block's.  Each
// block is therefore one tcgen05.mma.kind::i8 of M = 128 weight rows x N = 128
// tokens x K = 32 whose int32 result lands in TMEM; eight warps read it back
// (tcgen05.ld: warp w takes lanes 32(w%4).. = rows, columns 64(w/4)..) and add (sumi * d_w) * d_x to f32
// accumulators in block order.  That is exactly the order of the CPU
// restatement of the Q4_0 x Q8_0 product (ggml's vec_dot_q4_0_q8_0 loop), so
// results are bit-identical to it.
//
// Data path per block, 256 threads:
//   * a cp.async ring of kStages stages (kStages - 2 blocks ahead) holds, per block, the 128 rows' 16
//     nibble bytes (one plane entry of each row's group stream, layout.h), the
//     32 groups' fp16 scales, the 128 tokens' 32 int8 activations (placed
//     directly in the MMA's canonical K-major layout) and their scales;
//   * thread t < 128 unpacks row t's nibbles into int8 (n - 8) in the A tile
//     (canonical K-major layout, no swizzle: 8-row x 16-byte core matrices,
//     SBO = 256 B between row groups, LBO = 128 B between the two K halves);
//   * thread 0 issues the MMA and commits it to an mbarrier; all threads wait
//     (bounded), load their row of D from TMEM and accumulate.  The loop is
//     software-pipelined: block b+1's unpack and MMA (two A buffers, two TMEM
//     accumulators) are issued before block b's accumulator is scaled.
// Requires rows % 128 == 0 and in_dim % 32 == 0; tokens are zero-filled past T.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "internal.h"
#include "layout.h"
#include "ops.h"

namespace zgpu {

namespace {

constexpr uint32_t kTileM = 128;
constexpr uint32_t kTileN = 128;
constexpr uint32_t kGemmThreads = 256;   // 8 warps: (lane quarter, 64-column half) of the accumulator
constexpr uint32_t kStages = 5;
// stage layout (bytes)
constexpr uint32_t kRawA = 0;                    // 128 rows x 16 B nibbles
constexpr uint32_t kScA = 2048;                  // 32 groups x 8 B fp16 scales
constexpr uint32_t kTileB = 2304;                // 128 tokens x 32 B, canonical K-major
constexpr uint32_t kScB = 6400;                  // 128 tokens x f32 scales
constexpr uint32_t kStageBytes = 6912;
constexpr uint32_t kTmemCols = 256;              // two 128 x 128 int32 accumulators

// Byte offset of (row r, K half h) in a canonical K-major no-swizzle tile of
// 32-byte rows: core matrix (r / 8, h) holds rows 8(r/8).. x bytes 16h..16h+15.
__device__ __forceinline__ uint32_t core_off(uint32_t r, uint32_t h) {
  return (r & 7) * 16 + (r >> 3) * 256 + h * 128;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// UMMA shared-memory descriptor: K-major, no swizzle (layout type 0),
// descriptor version 1, LBO / SBO in 16-byte units.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;   // version
  return d;
}

// Instruction descriptor of kind::i8: D s32, A and B signed int8, both
// K-major, N = 64, M = 128, dense.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((kTileN >> 3) << 17) | ((kTileM >> 4) << 24);

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
               : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Exact int32 -> f32 for |v| < 2^22 with two full-rate ops: v + 1.5 * 2^23
// as float bits, minus 1.5 * 2^23 (a block's |sumi| <= 32 * 8 * 127).
__device__ __forceinline__ float small_i2f(uint32_t v) {
  return __fsub_rn(__int_as_float(static_cast<int>(v) + 0x4B400000), 12582912.0f);
}

// Nibbles n (0..15) of four bytes -> four int8 (n - 8): flip bit 3, then
// sign-extend it over the high nibble (0x08 * 0x1E = 0xF0, no carries).
__device__ __forceinline__ uint32_t nib_to_s8(uint32_t n4) {
  const uint32_t m = n4 ^ 0x08080808u;
  return m | ((m & 0x08080808u) * 0x1Eu);
}

__global__ void __launch_bounds__(kGemmThreads, 2) q4q8_mma_kernel(const MmaGemmParams p) {
  __shared__ __align__(128) uint8_t ring[kStages * kStageBytes];
  __shared__ __align__(128) uint8_t tileA[2][kTileM * 32];
  __shared__ __align__(8) uint64_t mbar[2];
  __shared__ uint32_t tmem_base;
  const uint32_t tid = threadIdx.x, warp = tid >> 5;
  const uint32_t m0 = blockIdx.x * kTileM, t0 = blockIdx.y * kTileN;
  const uint32_t bpr = p.bpr, K = bpr * 32;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(smem_addr(&mbar[0]), 1);
    mbar_init(smem_addr(&mbar[1]), 1);
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  // issue the copies of block b into its stage
  // threads 0..127 own a weight row each (copy, unpack, and their rows' scale)
  const uint32_t arow = tid & (kTileM - 1);
  const uint32_t row = m0 + arow;
  const uint8_t *grp_row = p.w + static_cast<uint64_t>(row >> 2) * p.gstride;
  const uint32_t tl = tid >> 1, th = tid & 1;          // token / K half this thread copies
  const bool tok_ok = t0 + tl < p.T;
  const int8_t *xrow = p.xq + static_cast<uint64_t>(tok_ok ? t0 + tl : 0) * K;
  auto issue = [&](uint32_t b) {
    const uint32_t st = smem_addr(ring + (b % kStages) * kStageBytes);
    if (tid < kTileM) cp_async16(st + kRawA + tid * 16, grp_row + plane_entry(ZGPU_Q4_0, bpr, b, row & 3), 16);
    else if (tid < kTileM + 32)
      cp_async8(st + kScA + (tid - kTileM) * 8,
                p.w + static_cast<uint64_t>((m0 >> 2) + tid - kTileM) * p.gstride + scale_entry(ZGPU_Q4_0, bpr, b));
    cp_async16(st + kTileB + core_off(tl, th), xrow + 32 * b + 16 * th, tok_ok ? 16u : 0u);
    if (tid < kTileN) {
      const bool ok = t0 + tid < p.T;
      cp_async4(st + kScB + tid * 4, p.xs + static_cast<uint64_t>(ok ? t0 + tid : 0) * bpr + b, ok ? 4u : 0u);
    }
  };
  // The ring runs kStages - 2 blocks ahead: prepare(c) refills the stage of
  // block c - 2, whose MMA and epilogue are complete by then (block c - 1's
  // MMA and block c - 1's epilogue may still use theirs).
#pragma unroll
  for (uint32_t s = 0; s < kStages - 2; ++s) {
    if (s < bpr) issue(s);
    cp_async_commit();
  }

  constexpr int kCols = 64;   // accumulator columns (tokens) per thread
  const uint32_t chalf = warp >> 2;
  float acc[kCols];
#pragma unroll
  for (int j = 0; j < kCols; ++j) acc[j] = 0.f;

  // Stage b's data is complete (all threads' copies), then row tid's nibbles
  // become int8 (n - 8) in A buffer b % 2; returns this row's scale d_w.
  auto prepare = [&](uint32_t b) -> float {
    if (b + kStages - 2 < bpr) issue(b + kStages - 2);
    cp_async_commit();
    cp_async_wait<kStages - 2>();   // this thread's copies of block b have landed
    __syncthreads();                // ... and everyone's; A buffer b % 2 is free (its MMA completed)
    const uint8_t *st = ring + (b % kStages) * kStageBytes;
    uint8_t *ta = tileA[b & 1];
    const uint16_t hw = *reinterpret_cast<const uint16_t *>(st + kScA + (arow >> 2) * 8 + (arow & 3) * 2);
    if (tid >= kTileM) {
      fence_proxy_async_smem();
      return h2f(hw);
    }
    const uint4 q = *reinterpret_cast<const uint4 *>(st + kRawA + tid * 16);
    uint4 lo, hi;
    lo.x = nib_to_s8(q.x & 0x0F0F0F0Fu);
    lo.y = nib_to_s8(q.y & 0x0F0F0F0Fu);
    lo.z = nib_to_s8(q.z & 0x0F0F0F0Fu);
    lo.w = nib_to_s8(q.w & 0x0F0F0F0Fu);
    hi.x = nib_to_s8((q.x >> 4) & 0x0F0F0F0Fu);
    hi.y = nib_to_s8((q.y >> 4) & 0x0F0F0F0Fu);
    hi.z = nib_to_s8((q.z >> 4) & 0x0F0F0F0Fu);
    hi.w = nib_to_s8((q.w >> 4) & 0x0F0F0F0Fu);
    *reinterpret_cast<uint4 *>(ta + core_off(tid, 0)) = lo;
    *reinterpret_cast<uint4 *>(ta + core_off(tid, 1)) = hi;
    fence_proxy_async_smem();   // generic-proxy writes of A and B -> visible to the tensor core
    return h2f(hw);
  };
  // thread 0: MMA of block b into accumulator b % 2, committed to mbar[b % 2]
  auto mma = [&](uint32_t b) {
    if (tid == 0) {
      tc_fence_after();
      const uint8_t *st = ring + (b % kStages) * kStageBytes;
      umma_i8(tmem + (b & 1) * kTileN, umma_desc(smem_addr(tileA[b & 1]), 128, 256),
              umma_desc(smem_addr(st + kTileB), 128, 256), kIdesc, 0u);
      umma_commit(smem_addr(&mbar[b & 1]));
    }
  };

  // Software pipeline: block b+1 is prepared and its MMA issued before block
  // b's accumulator is read back and scaled, so the tensor core and the
  // copies run under the epilogue's arithmetic.  Two A buffers and two TMEM
  // accumulators; a buffer is reused two blocks later, after the barrier in
  // prepare() that follows everyone's reads of it.
  bool ok = true;
  float dw_cur = prepare(0);
  __syncthreads();
  mma(0);
  for (uint32_t b = 0; b < bpr; ++b) {
    float dw_next = 0.f;
    if (b + 1 < bpr) {
      dw_next = prepare(b + 1);
      __syncthreads();
      mma(b + 1);
    }
    if (ok && !mbar_wait(smem_addr(&mbar[b & 1]), (b >> 1) & 1, p.status)) ok = false;
    tc_fence_after();
    const uint32_t taddr = tmem + (((warp & 3) * 32u) << 16) + (b & 1) * kTileN + chalf * kCols;
    const float4 *dx4 =
        reinterpret_cast<const float4 *>(ring + (b % kStages) * kStageBytes + kScB) + chalf * (kCols / 4);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t v[32];
      tmem_ld32(taddr + 32 * h, v);
      tmem_ld_wait();
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4) {
        const float4 d4 = dx4[8 * h + j4];
        const float dxv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 32 * h + 4 * j4 + k;
          acc[j] = __fadd_rn(acc[j], __fmul_rn(__fmul_rn(small_i2f(v[4 * j4 + k]), dw_cur), dxv[k]));
        }
      }
    }
    tc_fence_before();
    dw_cur = dw_next;
  }
  cp_async_wait<0>();
#pragma unroll
  for (int j = 0; j < kCols; ++j) {
    const uint32_t t = t0 + chalf * kCols + j;
    if (t < p.T) {
      float *dst = p.y + static_cast<uint64_t>(t) * p.ldy + row;
      const float v = ok ? acc[j] : __uint_as_float(0x7fc00000u);
      *dst = p.resadd ? __fadd_rn(*dst, v) : v;
    }
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Q8_0 activation rows in the planar form the MMA reads: q int8 [T][K] and
// the block scale d (fp16-rounded, as f32) [T][K/32].  The packer's rule, as
// quantize_q8_0_kernel.  One warp per block.
__global__ void quantize_q8_0_planar_kernel(const float *x, int8_t *q, float *d, uint64_t nblocks,
                                            uint32_t *status) {
  const uint64_t wb = (blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31;
  if (wb >= nblocks) return;
  const float v = x[wb * 32 + lane];
  if (!(fabsf(v) < INFINITY)) atomicOr(status, ZDEV_ERR_NUMERICAL);
  double a = fabs(static_cast<double>(v));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = fmax(a, __shfl_xor_sync(0xffffffffu, a, off));
  if (a == 0.0 || !(a < INFINITY)) {
    q[wb * 32 + lane] = 0;
    if (lane == 0) d[wb] = 0.f;
    return;
  }
  const double dd = a / 127.0;
  double r = rint(static_cast<double>(v) * (1.0 / dd));
  r = fmin(fmax(r, -127.0), 127.0);
  q[wb * 32 + lane] = static_cast<int8_t>(r);
  if (lane == 0) d[wb] = h2f(f64_to_f16_rne(fmin(dd, 65504.0)));
}

}  // namespace

cudaError_t launch_q4q8_mma(const MmaGemmParams &p, cudaStream_t s) {
  if (p.rows == 0 || p.rows % kTileM || p.bpr == 0 || p.T == 0 || p.gstride % 16) return cudaErrorInvalidValue;
  dim3 grid(p.rows / kTileM, (p.T + kTileN - 1) / kTileN);
  q4q8_mma_kernel<<<grid, kGemmThreads, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0_planar(const float *x, int8_t *q, float *d, uint64_t n, uint32_t *status,
                                        cudaStream_t s) {
  const uint64_t nb = n / 32;
  quantize_q8_0_planar_kernel<<<static_cast<unsigned>((nb * 32 + 255) / 256), 256, 0, s>>>(x, q, d, nb, status);
  return cudaGetLastError();
}

}  // namespace zgpu
