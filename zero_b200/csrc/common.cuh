// common.cuh — shared device helpers for the zero-b200 sm_100a kernels.
//
// PTX wrappers for the Blackwell features the decode path uses: mbarrier
// phases, the 1-D TMA bulk copy (cp.async.bulk, no multicast), programmatic
// dependent launch (griddepcontrol) and named barriers.  Every spin on an
// mbarrier is bounded by a wall-clock limit read from %globaltimer; on expiry
// the waiter records ZDEV_ERR_TIMEOUT in the kernel's status word and returns
// false so the caller can skip its remaining work instead of hanging.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace zgpu {

// Device status word bits (read back by the host after a step).
enum : uint32_t {
  ZDEV_ERR_TIMEOUT = 1u << 0,
  ZDEV_ERR_NUMERICAL = 1u << 1,   // softmax max non-finite or sum <= 0
  ZDEV_ERR_LM_NONFINITE = 1u << 2,
  ZDEV_ERR_LM_PADDING = 1u << 3,
  ZDEV_ERR_BOUNDS = 1u << 4,      // a token / position outside the cache
};

// The status block is kStatusWords uint32: word 0 holds the ZDEV_ERR_* bits;
// builds with ZGPU_DEVICE_CHECKS record the first failed bounds check in
// words 1..3 (check code, two values) and skip the offending access.
constexpr int kStatusWords = 8;

__device__ __forceinline__ void dev_check_fail(uint32_t *status, uint32_t code, uint32_t a,
                                               uint32_t b) {
  if (atomicCAS(&status[1], 0u, code) == 0u) {
    status[2] = a;
    status[3] = b;
  }
  atomicOr(&status[0], ZDEV_ERR_BOUNDS);
}

#ifdef ZGPU_DEVICE_CHECKS
#define ZDEV_CHECK(cond, status, code, a, b) \
  ((cond) ? true : (::zgpu::dev_check_fail((status), (code), (a), (b)), false))
#else
#define ZDEV_CHECK(cond, status, code, a, b) true
#endif

// 1 s bound on any device-side wait.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t *status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicOr(status, ZDEV_ERR_TIMEOUT);
      return false;
    }
  }
}

// 1-D bulk copy global -> this CTA's shared memory, completion signalled on
// the mbarrier as transaction bytes.  dst, src and bytes must be multiples
// of 16.  No multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void tma_bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                             uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory without a cache hint
// (same alignment rules; no multicast).
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// cp.async copies global -> shared (Ampere form, no mbarrier).  src_bytes <
// the copy size zero-fills the rest (0: a pure zero fill, src unread).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// L2 policy for weights streamed exactly once per step: evict first, so the
// KV cache and activations keep their L2 residency.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Programmatic dependent launch.  Both are no-ops when the kernel was not
// launched with the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Packed f32x2 add / multiply, each lane rounded to nearest.  The explicit
// .rn keeps every one a separate rounding (PTX never contracts an add or mul
// that carries a rounding modifier into an fma), so two columns at a time
// follow the scalar order exactly: the exact magic-number subtract, then
// (x * d_w) * d_x.  The accumulation itself stays scalar: a packed add did
// not reproduce the scalar sums bit for bit.
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  uint64_t r;
  asm("{\n\t.reg .b64 pa, pb;\n\tmov.b64 pa, {%1, %2};\n\tmov.b64 pb, {%3, %4};\n\t"
      "add.rn.f32x2 %0, pa, pb;\n\t}"
      : "=l"(r)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  uint64_t r;
  asm("{\n\t.reg .b64 pa, pb;\n\tmov.b64 pa, {%1, %2};\n\tmov.b64 pb, {%3, %4};\n\t"
      "mul.rn.f32x2 %0, pa, pb;\n\t}"
      : "=l"(r)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}
__device__ __forceinline__ float2 sub2_rn(float2 a, float2 b) {
  uint64_t r;
  asm("{\n\t.reg .b64 pa, pb;\n\tmov.b64 pa, {%1, %2};\n\tmov.b64 pb, {%3, %4};\n\t"
      "sub.rn.f32x2 %0, pa, pb;\n\t}"
      : "=l"(r)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}
// Packed fused multiply-add a * b + c, each lane rounded once.
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  uint64_t r;
  asm("{\n\t.reg .b64 pa, pb, pc;\n\tmov.b64 pa, {%1, %2};\n\tmov.b64 pb, {%3, %4};\n\tmov.b64 pc, {%5, %6};\n\t"
      "fma.rn.f32x2 %0, pa, pb, pc;\n\t}"
      : "=l"(r)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}

// Nibbles n (0..15) of four bytes -> four int8 (n - 8): flip bit 3, then
// sign-extend it over the high nibble (0x08 * 0x1E = 0xF0, no carries).
__device__ __forceinline__ uint32_t nib_to_s8(uint32_t n4) {
  const uint32_t m = n4 ^ 0x08080808u;
  return m | ((m & 0x08080808u) * 0x1Eu);
}

__device__ __forceinline__ float h2f(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

// ---------------------------------------------------------------------------
// Restatements of the reference's own AVX-512 polynomials (activation.rs:56-97
// and trig.rs:60-127), written with explicitly rounded operations so that no
// contraction changes them; they reproduce the reference lane values bit for
// bit given the same inputs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ref_exp(float x) {
  const float log2e = 1.44269504f, ln2_hi = 0.6933594f, ln2_lo = -2.1219444e-4f;
  // _mm512_min_ps / _mm512_max_ps return the second operand on NaN.
  x = (x < 88.37625f) ? x : 88.37625f;
  x = (x > -88.37625f) ? x : -88.37625f;
  float kf = rintf(__fmul_rn(x, log2e));
  int k = __float2int_rn(kf);
  float r = __fmaf_rn(-kf, ln2_lo, __fmaf_rn(-kf, ln2_hi, x));
  float p = __fmaf_rn(r, 8.3333333e-3f, 4.1666667e-2f);
  p = __fmaf_rn(r, p, 0.16666667f);
  p = __fmaf_rn(r, p, 0.5f);
  p = __fmaf_rn(r, p, 1.0f);
  p = __fmaf_rn(r, p, 1.0f);
  float two_k = __uint_as_float(static_cast<uint32_t>(k + 127) << 23);
  return __fmul_rn(p, two_k);
}

// silu_mul_avx512 (activation.rs:115-148): (g / (1 + exp(0 - g))) * u.
__device__ __forceinline__ float ref_silu_mul(float g, float u) {
  float e = ref_exp(__fsub_rn(0.0f, g));
  float silu = __fdiv_rn(g, __fadd_rn(1.0f, e));
  return __fmul_rn(silu, u);
}

// sincos_f32_avx512 (trig.rs:60-127).
__device__ __forceinline__ void ref_sincos(float x, float *s_out, float *c_out) {
  float kf = rintf(__fmul_rn(x, 0.63661977f));
  int k = __float2int_rn(kf);
  float r = __fmaf_rn(-kf, 7.5497903e-8f, __fmaf_rn(-kf, 1.57079625f, x));
  float r2 = __fmul_rn(r, r);
  float sp = __fmaf_rn(r2, -1.98412698e-4f, 8.3333333e-3f);
  sp = __fmaf_rn(r2, sp, -0.16666667f);
  sp = __fmaf_rn(r2, sp, 1.0f);
  float sin_r = __fmul_rn(r, sp);
  float cp = __fmaf_rn(r2, 2.4801587e-5f, -1.3888889e-3f);
  cp = __fmaf_rn(r2, cp, 4.1666667e-2f);
  cp = __fmaf_rn(r2, cp, -0.5f);
  float cos_r = __fmaf_rn(r2, cp, 1.0f);
  int q = k & 3, b0 = q & 1, b1 = (q >> 1) & 1;
  float s = b0 ? cos_r : sin_r;
  float c = b0 ? sin_r : cos_r;
  *s_out = b1 ? -s : s;
  *c_out = (b0 ^ b1) ? -c : c;
}

// binary16 bits of a finite double with |v| <= 65504, rounded to nearest-even
// straight from the double (struct.pack('<e') semantics): scale the value
// exactly onto the binary16 grid of its binade (a power-of-two ldexp), round
// with rint, re-encode.  Subnormal results and the carry into the next binade
// fall out of the continuous encoding.
__device__ __forceinline__ uint16_t f64_to_f16_rne(double v) {
  const uint16_t sign = signbit(v) ? 0x8000u : 0u;
  const double a = fabs(v);
  if (a == 0.0) return sign;
  const int e = ilogb(a);
  const int qe = (e < -14 ? -14 : e) - 10;
  const double r = rint(ldexp(a, -qe));
  if (e < -14) return static_cast<uint16_t>(sign | static_cast<uint16_t>(r));
  if (r >= 2048.0) return static_cast<uint16_t>(sign | ((e + 16) << 10));
  return static_cast<uint16_t>(sign | ((e + 15) << 10) | static_cast<uint16_t>(r - 1024.0));
}

// Tagged activation words (the persistent step kernel's inter-stage
// vectors): element i is (version << 32) | f32 bits, written with one 64-bit
// store, so a reader that sees the expected version also sees its value.
// The packer's Q8_0 rule for one 32-element block (silicatepack.py:893-907),
// one lane per element: d = amax / 127 in f64, q = rint(x / d) clamped to
// +-127, d stored as fp16 (read back as f32).  Lane j writes its digit to
// *qa; lane 0 writes the scale to *da.  An all-zero block gives zeros.
__device__ __forceinline__ void quant_lane_q8_0(float v, int8_t *qa, float *da, uint32_t lane, uint32_t *status) {
  if (!(fabsf(v) < INFINITY)) atomicOr(status, ZDEV_ERR_NUMERICAL);
  double a = fabs(static_cast<double>(v));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) a = fmax(a, __shfl_xor_sync(0xffffffffu, a, off));
  if (a == 0.0 || !(a < INFINITY)) {
    *qa = 0;
    if (lane == 0) *da = 0.f;
    return;
  }
  const double dd = a / 127.0;
  double r = rint(static_cast<double>(v) * (1.0 / dd));
  r = fmin(fmax(r, -127.0), 127.0);
  *qa = static_cast<int8_t>(r);
  if (lane == 0) *da = h2f(f64_to_f16_rne(fmin(dd, 65504.0)));
}

__device__ __forceinline__ unsigned long long tag_word(float x, uint32_t ver) {
  return (static_cast<unsigned long long>(ver) << 32) | __float_as_uint(x);
}

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until the four words at p (16-byte aligned) carry `ver`, then return
// their values.  Bounded: gives up (false) when this CTA or the launch is
// aborting, or after kWaitLimitNs, which also sets ZDEV_ERR_TIMEOUT and the
// abort flags.
__device__ __forceinline__ bool tag_wait4(const unsigned long long *p, uint32_t ver, float4 *out,
                                          uint32_t *status, volatile uint32_t *abort,
                                          uint32_t *gabort) {
  const ulonglong2 *q = reinterpret_cast<const ulonglong2 *>(p);
  ulonglong2 a = __ldcg(q), b = __ldcg(q + 1);
  auto ready = [&]() {
    return static_cast<uint32_t>(a.x >> 32) == ver && static_cast<uint32_t>(a.y >> 32) == ver &&
           static_cast<uint32_t>(b.x >> 32) == ver && static_cast<uint32_t>(b.y >> 32) == ver;
  };
  if (!ready()) {
    const uint64_t t0 = globaltimer_ns();
    while (true) {
      a = __ldcg(q);
      b = __ldcg(q + 1);
      if (ready()) break;
      if (*abort || ld_relaxed_u32(gabort)) {
        *abort = 1;
        *out = make_float4(0.f, 0.f, 0.f, 0.f);
        return false;
      }
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(status, ZDEV_ERR_TIMEOUT);
        atomicExch(gabort, 1u);
        *abort = 1;
        *out = make_float4(0.f, 0.f, 0.f, 0.f);
        return false;
      }
    }
  }
  *out = make_float4(__uint_as_float(static_cast<uint32_t>(a.x)), __uint_as_float(static_cast<uint32_t>(a.y)),
                     __uint_as_float(static_cast<uint32_t>(b.x)), __uint_as_float(static_cast<uint32_t>(b.y)));
  return true;
}

// Orderable key for the LM-head argmax: larger value wins, then the smaller
// index (inference_avx512.rs:1027-1044 merge rule).  NaN never wins (it is
// mapped to the initial key); -0 is folded onto +0 so ties behave like the
// reference's `>` comparison.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  if (v != v) v = -INFINITY;
  v = v + 0.0f;
  uint32_t b = __float_as_uint(v);
  uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | (0xFFFFFFFFu - idx);
}
__device__ __forceinline__ float argmax_key_value(unsigned long long key) {
  uint32_t ord = static_cast<uint32_t>(key >> 32);
  uint32_t b = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
  return __uint_as_float(b);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long key) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull);
}
// Key of (-inf, index 0): what the reference returns when every logit is NaN.
constexpr unsigned long long kArgmaxInitKey = 0x007FFFFFFFFFFFFFull;

}  // namespace zgpu
