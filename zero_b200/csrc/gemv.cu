// gemv.cu — batch-1 dequant GEMV over the .smodel-v2 4-row-interleaved layout.
//
// Replaces linear_q4_0x4_avx512_range / linear_q8_0x4_avx512_range
// (kernel/src/arch/x86_64/math/linear.rs:909, :1096) and the fused
// multi-projection / LM-head-argmax dispatches built on them
// (kernel/src/inference_avx512.rs:826-945, :1061-1118).
//
// Data path (one CTA per SM, persistent over a contiguous range of "units";
// a unit is U consecutive 4-row groups — U = 2 pairs a gate group with its up
// group for the SwiGLU epilogue):
//   * one producer lane streams each unit's group bytes (contiguous on the
//     device) into a ring of shared-memory slots with 1-D TMA bulk copies
//     (cp.async.bulk, L2 evict-first), signalling an mbarrier per slot;
//   * consumer warps are arranged as KS x GW: warp (ks, team) owns K-slice ks
//     (32 blocks, one per lane) of every unit its team takes, so each lane
//     keeps its block's 32 activations in registers for the whole launch;
//   * the lane dequantises its block for the unit's 4U rows in registers:
//     Q4_0 nibbles become exact floats through the 2^23 exponent trick
//     (bits OR'd into a float whose exponent makes the nibble's place value
//     an integer; one packed f32x2 subtract removes the bias), accumulated
//     with packed f32x2 FMAs against the pre-scaled activations; Q8_0 bytes
//     go through the same trick after a byte permute;
//   * a warp reduce-scatter leaves each row's K-slice sum in a lane, K-slices
//     are combined in fixed order through shared memory, and the epilogue
//     stores / adds the residual / applies SiLU(gate)*up / tracks the argmax.
// Every reduction has a fixed order, so results are bitwise reproducible
// from run to run and independent of the grid size.
#include <cfloat>

#include "common.cuh"
#include "internal.h"

namespace zgpu {

namespace {

constexpr int kMaxConsumerWarps = 8;
constexpr int kThreads = 32 * (kMaxConsumerWarps + 1);
constexpr uint32_t kMagic = 0x4B000000u;       // 2^23 as f32 bits
constexpr float kTwo23 = 8388608.0f;
constexpr size_t kRingBudget = 100 * 1024;     // two CTAs (two kernels) fit per SM

struct KParams {
  const uint8_t *w;
  uint64_t gstride;          // bytes per group stream (multiple of 16)
  uint32_t rows;             // valid output rows
  uint32_t units;            // total units
  uint32_t units_per_cta;
  uint32_t bpr;              // 32-element blocks per row
  uint32_t in_dim;
  uint32_t ks, gw, ns;
  const float *x;
  const float *norm_w;
  float eps;
  float *out;
  unsigned long long *argmax;
  uint32_t *status;
};

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

template <int R>
struct RowShift {
  static constexpr int value = (R == 4) ? 3 : (R == 8) ? 2 : 0;
};

// One Q4_0 row of one block: sum_j x_j * n_j (x pre-scaled per bit class),
// returned as d * (sum - 8 * sum_j x_j).
__device__ __forceinline__ float q4_row(const uint32_t (&q)[4], const float2 (&xs)[16], float d,
                                        float x8) {
  const float2 bias = make_float2(-kTwo23, -kTwo23);
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t w = q[m], w12 = w >> 12;
    // element 4m (bits 0-3, class 0) and 4m+16 (bits 4-7, class 4)
    float2 f0 = make_float2(__uint_as_float((w & 0x0000000Fu) | kMagic),
                            __uint_as_float((w & 0x000000F0u) | kMagic));
    // element 4m+1 (bits 8-11, class 8) and 4m+17 (bits 12-15, class 12)
    float2 f1 = make_float2(__uint_as_float((w & 0x00000F00u) | kMagic),
                            __uint_as_float((w & 0x0000F000u) | kMagic));
    // element 4m+2 (bits 16-19, class 16) and 4m+18 (bits 20-23 -> 8-11, class 8)
    float2 f2 = make_float2(__uint_as_float((w & 0x000F0000u) | kMagic),
                            __uint_as_float((w12 & 0x00000F00u) | kMagic));
    // element 4m+3 (bits 24-27 -> 12-15, class 12) and 4m+19 (bits 28-31 -> 16-19, class 16)
    float2 f3 = make_float2(__uint_as_float((w12 & 0x0000F000u) | kMagic),
                            __uint_as_float((w12 & 0x000F0000u) | kMagic));
    acc0 = __ffma2_rn(xs[4 * m + 0], __fadd2_rn(f0, bias), acc0);
    acc1 = __ffma2_rn(xs[4 * m + 1], __fadd2_rn(f1, bias), acc1);
    acc0 = __ffma2_rn(xs[4 * m + 2], __fadd2_rn(f2, bias), acc0);
    acc1 = __ffma2_rn(xs[4 * m + 3], __fadd2_rn(f3, bias), acc1);
  }
  float s = (acc0.x + acc0.y) + (acc1.x + acc1.y);
  return d * (s - x8);
}

// One Q8_0 row of one block: d * sum_j x_j * q_j.
__device__ __forceinline__ float q8_row(const uint32_t (&q)[8], const float2 (&xp)[16], float d) {
  const float2 bias = make_float2(-(kTwo23 + 128.f), -(kTwo23 + 128.f));
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t w = q[k] ^ 0x80808080u;   // i8 -> u8 + 128
    float2 f0 = make_float2(__uint_as_float(__byte_perm(w, kMagic, 0x7540)),
                            __uint_as_float(__byte_perm(w, kMagic, 0x7541)));
    float2 f1 = make_float2(__uint_as_float(__byte_perm(w, kMagic, 0x7542)),
                            __uint_as_float(__byte_perm(w, kMagic, 0x7543)));
    acc0 = __ffma2_rn(xp[2 * k + 0], __fadd2_rn(f0, bias), acc0);
    acc1 = __ffma2_rn(xp[2 * k + 1], __fadd2_rn(f1, bias), acc1);
  }
  float s = (acc0.x + acc0.y) + (acc1.x + acc1.y);
  return d * s;
}

template <int QT, int PRO, int EPI, int U>
__global__ void __launch_bounds__(kThreads, 2) gemv_x4_kernel(const KParams p) {
  constexpr int GB = (QT == ZGPU_Q4_0) ? 72 : 136;
  constexpr int R = 4 * U;
  constexpr int SH = RowShift<R>::value;
  extern __shared__ __align__(128) uint8_t smem[];

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t KS = p.ks, GW = p.gw, NW = KS * GW, NS = p.ns;
  const uint32_t slot_bytes = U * static_cast<uint32_t>(p.gstride);
  uint8_t *ring = smem;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + static_cast<size_t>(NS) * slot_bytes);
  uint64_t *empty = full + NS;
  float *red = reinterpret_cast<float *>(empty + NS);      // [GW][2][KS][R]
  float *ssq_part = red + GW * 2 * KS * R;                  // [KS]

  const uint32_t u0 = blockIdx.x * p.units_per_cta;
  const uint32_t u1 = min(u0 + p.units_per_cta, p.units);
  const uint32_t nloc = u1 > u0 ? u1 - u0 : 0;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < NS; ++i) {
      mbar_init(smem_addr(&full[i]), 1);
      mbar_init(smem_addr(&empty[i]), KS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp >= NW) {
    // ---------------- producer ----------------
    if (warp == NW && lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t issued = 0;
      for (uint32_t i = 0; i < nloc; ++i) {
        const uint32_t slot = i % NS;
        if (i >= NS && !mbar_wait(smem_addr(&empty[slot]), ((i / NS) - 1) & 1, p.status)) break;
        const uint32_t fb = smem_addr(&full[slot]);
        mbar_arrive_expect_tx(fb, slot_bytes);
        tma_bulk_g2s(smem_addr(ring + static_cast<size_t>(slot) * slot_bytes),
                     p.w + static_cast<uint64_t>(u0 + i) * slot_bytes, slot_bytes, fb, pol);
        ++issued;
      }
      // Drain: never leave a copy in flight when the CTA may exit.
      for (uint32_t s = 0; s < NS && s < issued; ++s) {
        const uint32_t last = s + ((issued - 1 - s) / NS) * NS;
        mbar_wait(smem_addr(&full[s]), (last / NS) & 1, p.status);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const uint32_t ks = warp % KS, team = warp / KS;
  const uint32_t b = ks * 32 + lane;
  const bool has_b = b < p.bpr;

  pdl_wait();   // the activations are the previous kernel's output

  float xv[32];
  if (has_b) {
    const float4 *src = reinterpret_cast<const float4 *>(p.x + static_cast<size_t>(b) * 32);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float4 t = src[k];
      xv[4 * k] = t.x; xv[4 * k + 1] = t.y; xv[4 * k + 2] = t.z; xv[4 * k + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) xv[k] = 0.f;
  }

  if (PRO == PRO_RMSNORM) {
    // rmsnorm (ops.rs:29-52) with a fixed-order parallel sum of squares:
    // lane-sequential over its 32 values, xor-tree over lanes, then the
    // K-slices in order.  Every CTA computes the identical value.
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) ss = __fadd_rn(ss, __fmul_rn(xv[k], xv[k]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (team == 0 && lane == 0) ssq_part[ks] = ss;
    named_bar_sync(1, NW * 32);
    float tot = 0.f;
    for (uint32_t k = 0; k < KS; ++k) tot = __fadd_rn(tot, ssq_part[k]);
    const float mean = __fdiv_rn(tot, static_cast<float>(p.in_dim));
    const float rms = __fsqrt_rn(__fadd_rn(mean, p.eps));
    const float inv = __fdiv_rn(1.0f, rms);
    if (has_b) {
      const float4 *wsrc = reinterpret_cast<const float4 *>(p.norm_w + static_cast<size_t>(b) * 32);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float4 t = wsrc[k];
        xv[4 * k] = __fmul_rn(__fmul_rn(xv[4 * k], inv), t.x);
        xv[4 * k + 1] = __fmul_rn(__fmul_rn(xv[4 * k + 1], inv), t.y);
        xv[4 * k + 2] = __fmul_rn(__fmul_rn(xv[4 * k + 2], inv), t.z);
        xv[4 * k + 3] = __fmul_rn(__fmul_rn(xv[4 * k + 3], inv), t.w);
      }
    }
  }

  // Per-lane activation operands.
  float2 xs[16];
  float x8 = 0.f;
  if (QT == ZGPU_Q4_0) {
    // element -> bit class (see q4_row): x scaled by 2^-class so that the
    // product with (n << class) is exactly x * n.
    float sx = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) sx += xv[k];
    x8 = 8.0f * sx;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      xs[4 * m + 0] = make_float2(xv[4 * m], xv[4 * m + 16] * 0.0625f);
      xs[4 * m + 1] = make_float2(xv[4 * m + 1] * 0.00390625f, xv[4 * m + 17] * 0.000244140625f);
      xs[4 * m + 2] = make_float2(xv[4 * m + 2] * 1.52587890625e-05f, xv[4 * m + 18] * 0.00390625f);
      xs[4 * m + 3] = make_float2(xv[4 * m + 3] * 0.000244140625f, xv[4 * m + 19] * 1.52587890625e-05f);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) xs[k] = make_float2(xv[2 * k], xv[2 * k + 1]);
  }

  bool failed = false;
  unsigned long long best = kArgmaxInitKey;
  uint32_t it = 0;
  for (uint32_t i = team; i < nloc; i += GW, ++it) {
    const uint32_t slot = i % NS;
    if (!failed && !mbar_wait(smem_addr(&full[slot]), (i / NS) & 1, p.status)) failed = true;
    float part[R];
    const uint8_t *ubase = ring + static_cast<size_t>(slot) * slot_bytes;
#pragma unroll
    for (int g = 0; g < U; ++g) {
      const uint8_t *blk = ubase + g * p.gstride + static_cast<size_t>(b) * GB;
      if (has_b && !failed) {
        const uint2 sc = *reinterpret_cast<const uint2 *>(blk);
        const float d[4] = {h2f(sc.x & 0xFFFF), h2f(sc.x >> 16), h2f(sc.y & 0xFFFF),
                            h2f(sc.y >> 16)};
        if (QT == ZGPU_Q4_0) {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint2 a = *reinterpret_cast<const uint2 *>(blk + 8 + 16 * r);
            const uint2 c = *reinterpret_cast<const uint2 *>(blk + 16 + 16 * r);
            const uint32_t q[4] = {a.x, a.y, c.x, c.y};
            part[4 * g + r] = q4_row(q, xs, d[r], x8);
          }
        } else {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            uint32_t q[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint2 a = *reinterpret_cast<const uint2 *>(blk + 8 + 32 * r + 8 * k);
              q[2 * k] = a.x;
              q[2 * k + 1] = a.y;
            }
            part[4 * g + r] = q8_row(q, xs, d[r]);
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r) part[4 * g + r] = 0.f;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));

    float v = reduce_scatter<R>(part, lane);
    float y = 0.f;
    if (KS > 1) {
      float *rb = red + (static_cast<size_t>(team) * 2 + (it & 1)) * KS * R;
      if ((lane & ((1u << SH) - 1)) == 0) rb[ks * R + (lane >> SH)] = v;
      named_bar_sync(2 + team, KS * 32);
      if (ks == 0 && lane < R) {
        for (uint32_t k = 0; k < KS; ++k) y += rb[k * R + lane];
      }
    } else {
      y = __shfl_sync(0xffffffffu, v, (lane & (R - 1)) << SH);
    }
    if (ks != 0) continue;

    const uint32_t unit = u0 + i;
    if (EPI == EPI_SWIGLU) {
      // unit = {gate rows 4u..4u+3, up rows 4u..4u+3}
      const float yu = __shfl_down_sync(0xffffffffu, y, 4);
      const uint32_t row = unit * 4 + lane;
      if (lane < 4 && row < p.rows) p.out[row] = ref_silu_mul(y, yu);
    } else if (lane < R) {
      const uint32_t row = unit * R + lane;
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

  if (EPI == EPI_ARGMAX && ks == 0) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    if (lane == 0 && best != kArgmaxInitKey) atomicMax(p.argmax, best);
  }
}

template <int QT, int PRO, int EPI, int U>
cudaError_t configure_one() {
  return cudaFuncSetAttribute(gemv_x4_kernel<QT, PRO, EPI, U>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kRingBudget + 16 * 1024));
}

template <int QT, int PRO>
cudaError_t configure_pro() {
  cudaError_t e;
  if ((e = configure_one<QT, PRO, EPI_STORE, 1>()) != cudaSuccess) return e;
  if ((e = configure_one<QT, PRO, EPI_RESADD, 1>()) != cudaSuccess) return e;
  if ((e = configure_one<QT, PRO, EPI_SWIGLU, 2>()) != cudaSuccess) return e;
  return configure_one<QT, PRO, EPI_ARGMAX, 1>();
}

template <int QT, int PRO, int EPI, int U>
cudaError_t launch_one(const KParams &kp, uint32_t grid, size_t smem, const LaunchCfg &lc) {
  auto fn = gemv_x4_kernel<QT, PRO, EPI, U>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(32 * (kp.ks * kp.gw + 1));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = lc.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = lc.pdl ? 1 : 0;
  if (lc.launch_counter) ++*lc.launch_counter;
  return cudaLaunchKernelEx(&cfg, fn, kp);
}

template <int QT, int PRO>
cudaError_t dispatch_epi(GemvEpi epi, const KParams &kp, uint32_t grid, size_t smem,
                         const LaunchCfg &lc) {
  switch (epi) {
    case EPI_STORE: return launch_one<QT, PRO, EPI_STORE, 1>(kp, grid, smem, lc);
    case EPI_RESADD: return launch_one<QT, PRO, EPI_RESADD, 1>(kp, grid, smem, lc);
    case EPI_SWIGLU: return launch_one<QT, PRO, EPI_SWIGLU, 2>(kp, grid, smem, lc);
    case EPI_ARGMAX: return launch_one<QT, PRO, EPI_ARGMAX, 1>(kp, grid, smem, lc);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

// Raise the dynamic shared-memory limit of every GEMV instantiation on the
// current device (called once per context, outside any stream capture).
cudaError_t gemv_setup() {
  cudaError_t e;
  if ((e = configure_pro<ZGPU_Q4_0, PRO_PLAIN>()) != cudaSuccess) return e;
  if ((e = configure_pro<ZGPU_Q4_0, PRO_RMSNORM>()) != cudaSuccess) return e;
  if ((e = configure_pro<ZGPU_Q8_0, PRO_PLAIN>()) != cudaSuccess) return e;
  return configure_pro<ZGPU_Q8_0, PRO_RMSNORM>();
}

cudaError_t launch_gemv(const GemvDesc &g, GemvPro pro, GemvEpi epi, const GemvIo &io,
                        const LaunchCfg &lc) {
  if (g.in_dim == 0 || g.in_dim % 32 != 0 || g.groups == 0) return cudaErrorInvalidValue;
  if (g.gstride % 16 != 0) return cudaErrorInvalidValue;
  if (epi == EPI_SWIGLU && (g.groups % 2 != 0 || g.quant != ZGPU_Q4_0))
    return cudaErrorInvalidValue;
  KParams kp = {};
  kp.w = g.w;
  kp.gstride = g.gstride;
  kp.rows = g.rows;
  kp.bpr = g.in_dim / 32;
  kp.in_dim = g.in_dim;
  kp.ks = (kp.bpr + 31) / 32;
  if (kp.ks > static_cast<uint32_t>(kMaxConsumerWarps)) return cudaErrorInvalidValue;
  kp.gw = kMaxConsumerWarps / kp.ks;
  const uint32_t U = (epi == EPI_SWIGLU) ? 2 : 1;
  kp.units = g.groups / U;
  const uint32_t ctas = static_cast<uint32_t>(lc.sm_count > 0 ? lc.sm_count : 148);
  kp.units_per_cta = (kp.units + ctas - 1) / ctas;
  const uint32_t grid = (kp.units + kp.units_per_cta - 1) / kp.units_per_cta;
  const size_t slot = static_cast<size_t>(U) * g.gstride;
  if (slot * 2 > kRingBudget) return cudaErrorInvalidValue;
  uint32_t ns = static_cast<uint32_t>(kRingBudget / slot);
  if (ns > kp.units_per_cta) ns = kp.units_per_cta;
  if (ns > 32) ns = 32;
  if (ns < 1) ns = 1;
  kp.ns = ns;
  kp.x = io.x;
  kp.norm_w = io.norm_w;
  kp.eps = io.eps;
  kp.out = io.out;
  kp.argmax = io.argmax;
  kp.status = io.status;
  const size_t R = 4 * U;
  const size_t smem = slot * ns + 16 * ns + sizeof(float) * (kp.gw * 2 * kp.ks * R + kp.ks) + 16;
  if (g.quant == ZGPU_Q4_0) {
    return pro == PRO_RMSNORM ? dispatch_epi<ZGPU_Q4_0, PRO_RMSNORM>(epi, kp, grid, smem, lc)
                              : dispatch_epi<ZGPU_Q4_0, PRO_PLAIN>(epi, kp, grid, smem, lc);
  }
  if (g.quant == ZGPU_Q8_0) {
    if (epi == EPI_SWIGLU) return cudaErrorInvalidValue;
    return pro == PRO_RMSNORM ? dispatch_epi<ZGPU_Q8_0, PRO_RMSNORM>(epi, kp, grid, smem, lc)
                              : dispatch_epi<ZGPU_Q8_0, PRO_PLAIN>(epi, kp, grid, smem, lc);
  }
  return cudaErrorInvalidValue;
}

}  // namespace zgpu
