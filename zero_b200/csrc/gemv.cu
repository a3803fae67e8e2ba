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
//
// PRO_Q8ACT (BASELINE config 1's Q4_0 weight x Q8_0 activation GEMV): the
// input is already Q8_0, so the image holds one digit per element (the int8
// quant) with the offset -8 * sum q and the block scale d_x; a row-block is
// one dp4a chain of eight, exact in int32, times d_w * d_x.
#include <cfloat>

#include "common.cuh"
#include "gemv_body.cuh"
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
  // segmented launch (GemvDesc::seg_w or seg_count > 1): units / wbytes are
  // per segment
  const unsigned long long *seg_w;
  uint32_t segmented, ctas_per_seg, seg_x_stride, seg_out_stride, seg_dynamic;
  uint32_t seg_x_group, seg_w_mod;
};

template <int QT, int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_x4_kernel(const KParams p) {
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

  // segment of this CTA (a plain launch is one segment at p.w)
  uint32_t seg = 0, cta = blockIdx.x;
  if (p.segmented) {
    seg = blockIdx.x / p.ctas_per_seg;
    cta = blockIdx.x - seg * p.ctas_per_seg;
  }
  // the segment's weight-table entry and input vector
  const uint32_t wseg = p.seg_w_mod ? seg % p.seg_w_mod : seg;
  const float *xin = p.x + static_cast<size_t>(seg / p.seg_x_group) * p.seg_x_stride;
  float *yout = p.out + static_cast<size_t>(seg) * p.seg_out_stride;
  const uint32_t u0 = cta * p.units_per_cta;
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
      const uint8_t *w = p.w;
      if (p.seg_w) {
        if (p.seg_dynamic) pdl_wait();   // the table is the previous kernel's output
        w = reinterpret_cast<const uint8_t *>(__ldcg(p.seg_w + wseg));
        if (!w) return;   // a segment of no work (another rank's expert)
      }
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
        tma_bulk_g2s(dst, w + src, bytes, fb, pol);
        tma_bulk_g2s(dst + p.half_bytes, w + src + p.gstride, bytes, fb, pol);
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
  // a zero table entry: the segment does nothing (expert parallelism leaves
  // another rank's experts out); uniform over the CTA, before any barrier
  if (p.seg_w && p.seg_dynamic && __ldcg(p.seg_w + wseg) == 0ull) return;
  const uint32_t tid = threadIdx.x;
  const uint32_t nf4 = PRO == PRO_Q8ACT ? 0u : p.in_dim / 4;
  float inv = 1.0f;
  if (PRO == PRO_RMSNORM) inv = rms_inv<kWarps>(xin, p.in_dim, p.eps, red, tid, 1);
  if (PRO == PRO_Q8ACT) {
    // the input is already Q8_0: one thread per 34-byte block
    const uint8_t *xq = reinterpret_cast<const uint8_t *>(xin);
    for (uint32_t b = tid; b < p.bpr; b += kConsumers)
      if (ZDEV_CHECK(b * 128 + 128 <= p.xbytes, p.status, 4, b, p.xbytes)) q8_block_image(xq + b * 34, b, xsm);
  }
  // Warp-uniform trip count: the per-block statistics shuffle across the 8
  // lanes of a block, and nf4 is a multiple of 8, so a block's lanes are
  // either all in range or all out of range.
  for (uint32_t f0 = warp * 32; f0 < nf4; f0 += kConsumers) {
    const uint32_t f = f0 + lane;
    const bool valid = f < nf4;
    float4 t = valid ? __ldcg(reinterpret_cast<const float4 *>(xin) + f) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (PRO == PRO_RMSNORM && valid) {
      const float4 g = reinterpret_cast<const float4 *>(p.norm_w)[f];
      t.x = __fmul_rn(__fmul_rn(t.x, inv), g.x);
      t.y = __fmul_rn(__fmul_rn(t.y, inv), g.y);
      t.z = __fmul_rn(__fmul_rn(t.z, inv), g.z);
      t.w = __fmul_rn(__fmul_rn(t.w, inv), g.w);
    }
    digitise_f4<QT>(t, f, valid, xsm, p.bpr, p.xbytes, p.status);
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
      if (PRO == PRO_Q8ACT) item_rows_q8act<2>(sbase, p.half_bytes, chunk_blocks(p.bpr, chunk), lane, b, xsm, acc);
      else item_rows<QT, 2>(sbase, p.half_bytes, chunk_blocks(p.bpr, chunk), lane, b, xsm, acc);
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
      if (row < p.rows) yout[row] = ref_silu_mul(yg, yu);
    }
  } else {
    for (uint32_t t = tid; t < nloc * kRows; t += kConsumers) {
      const uint32_t ul = t / kRows, r = t % kRows;
      float y = 0.f;
      for (uint32_t c = 0; c < p.ks; ++c) y += part[(ul * p.ks + c) * kRows + r];
      const uint32_t row = (u0 + ul) * kRows + r;
      if (row < p.rows) {
        if (EPI == EPI_STORE) {
          yout[row] = y;
        } else if (EPI == EPI_RESADD) {
          yout[row] = yout[row] + y;
        } else {
          yout[row] = y;
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
  if ((e = configure_one<ZGPU_Q4_0, PRO_Q8ACT, EPI_STORE>()) != cudaSuccess) return e;
  return configure_pro<ZGPU_Q8_0, PRO_RMSNORM>();
}

cudaError_t launch_gemv(const GemvDesc &g, GemvPro pro, GemvEpi epi, const GemvIo &io,
                        const LaunchCfg &lc) {
  if (g.in_dim == 0 || g.in_dim % 32 != 0 || g.groups == 0 || g.groups % 2 != 0)
    return cudaErrorInvalidValue;
  if (g.gstride % 16 != 0) return cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && g.quant != ZGPU_Q4_0) return cudaErrorInvalidValue;
  if (pro == PRO_Q8ACT && (g.quant != ZGPU_Q4_0 || epi != EPI_STORE || g.seg_w)) return cudaErrorInvalidValue;
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
  uint32_t grid = 0;
  kp.seg_x_group = 1;
  if (g.seg_w || g.seg_count > 1) {
    if (g.seg_count == 0 || !g.wbytes || g.seg_x_group == 0) return cudaErrorInvalidValue;
    kp.segmented = 1;
    kp.seg_x_group = g.seg_x_group;
    kp.seg_w_mod = g.seg_w_mod;
    const uint64_t total = static_cast<uint64_t>(kp.units) * g.seg_count;
    kp.units_per_cta = static_cast<uint32_t>((total + ctas - 1) / ctas);
    kp.ctas_per_seg = (kp.units + kp.units_per_cta - 1) / kp.units_per_cta;
    grid = kp.ctas_per_seg * g.seg_count;
    kp.seg_w = g.seg_w;
    kp.seg_x_stride = g.seg_x_stride;
    kp.seg_out_stride = g.seg_out_stride;
    kp.seg_dynamic = g.seg_dynamic ? 1u : 0u;
  } else {
    kp.units_per_cta = (kp.units + ctas - 1) / ctas;
    grid = (kp.units + kp.units_per_cta - 1) / kp.units_per_cta;
  }
  kp.half_bytes = static_cast<uint32_t>(chunk_bytes(g.quant, min(kChunkBlocks, kp.bpr)));
  const size_t slot = 2 * static_cast<size_t>(kp.half_bytes);
  // activation image: 128 B per block
  kp.xbytes = static_cast<uint32_t>(static_cast<size_t>(kp.bpr) * 128);
  // A launch whose per-CTA share of units leaves no room for one ring slot
  // per warp (a batch of many segments) takes fewer units per CTA and more
  // CTAs than one wave.
  const size_t unit_part = static_cast<size_t>(kp.ks) * kRows * sizeof(float);
  const size_t room = kSmemBudget - 1024 - kp.xbytes - kWarps * slot - 127;
  if (kSmemBudget > 1024 + kp.xbytes + kWarps * slot + 127 && kp.units_per_cta * unit_part > room) {
    kp.units_per_cta = static_cast<uint32_t>(room / unit_part);
    if (kp.units_per_cta == 0) return cudaErrorInvalidValue;
    if (kp.segmented) {
      kp.ctas_per_seg = (kp.units + kp.units_per_cta - 1) / kp.units_per_cta;
      grid = kp.ctas_per_seg * g.seg_count;
    } else {
      grid = (kp.units + kp.units_per_cta - 1) / kp.units_per_cta;
    }
  }
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
    if (pro == PRO_Q8ACT) return launch_one<ZGPU_Q4_0, PRO_Q8ACT, EPI_STORE>(kp, grid, smem, lc);
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
