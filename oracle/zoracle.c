/*
 * zoracle.c — CPU parity oracle for the zero-llm-inference decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see zoracle.h).  Every function cites the
 * reference file:line whose behaviour it restates.  Compile with
 * -ffp-contract=off: the reference's scalar Rust performs every multiply and
 * add with its own rounding, and the AVX-512 path's fused operations are
 * written out here explicitly with fmaf().
 */
#define _GNU_SOURCE
#include "zoracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdio.h>
#include <time.h>
#include <unistd.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif

/* ======================================================================
 * fp16 <-> float
 * ====================================================================== */

/* dequant.rs:28-61 (fp16_to_f32): normals by exponent rebias, denormals as
 * mant * 2^-10 * 2^-14 in f32, +-0, +-inf, NaN payload kept. */
float zo_fp16_to_f32(uint16_t bits) {
  uint32_t sign = (bits >> 15) & 1u, exp = (bits >> 10) & 0x1Fu, mant = bits & 0x3FFu;
  uint32_t out;
  float f;
  if (exp == 0) {
    if (mant == 0) {
      out = sign << 31;
      memcpy(&f, &out, 4);
      return f;
    }
    float val = ((float)mant * (1.0f / 1024.0f)) * (1.0f / 16384.0f);
    return sign ? -val : val;
  } else if (exp == 31) {
    out = (sign << 31) | (0xFFu << 23) | (mant << 13);
  } else {
    out = (sign << 31) | ((exp + 112u) << 23) | (mant << 13);
  }
  memcpy(&f, &out, 4);
  return f;
}

/* tools/silicatepack.py float_to_fp16_bytes: non-finite -> 0.0, clamp to
 * +-65504, then struct.pack('<e') which rounds the double to binary16 with
 * round-half-to-even directly (no intermediate f32 rounding). */
uint16_t zo_f64_to_fp16(double v) {
  if (!isfinite(v)) v = 0.0;
  if (v > 65504.0) v = 65504.0;
  if (v < -65504.0) v = -65504.0;
  uint16_t sign = signbit(v) ? 0x8000u : 0u;
  double a = fabs(v);
  if (a == 0.0) return sign;
  int e;
  (void)frexp(a, &e);          /* a = m * 2^e, m in [0.5, 1) */
  int unbiased = e - 1;        /* a in [2^unbiased, 2^(unbiased+1)) */
  double q;                    /* quantum of the binary16 grid at this magnitude */
  if (unbiased < -14) q = ldexp(1.0, -24);      /* subnormal grid */
  else q = ldexp(1.0, unbiased - 10);
  double n = a / q;            /* exact: q is a power of two */
  double r = nearbyint(n);     /* default rounding mode: half-to-even */
  double res = r * q;
  /* re-encode */
  if (res >= 65520.0) return (uint16_t)(sign | 0x7C00u); /* not reachable after clamp */
  if (res < ldexp(1.0, -14)) {
    uint16_t m = (uint16_t)(res / ldexp(1.0, -24));
    return (uint16_t)(sign | m);  /* may carry into exponent 1: encoding is continuous */
  }
  int e2;
  double m2 = frexp(res, &e2);   /* res = m2 * 2^e2 */
  int ub = e2 - 1;
  uint16_t mant = (uint16_t)((m2 * 2.0 - 1.0) * 1024.0);
  return (uint16_t)(sign | (uint16_t)((ub + 15) << 10) | mant);
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* dequant.rs:186-198: byte j -> low nibble out[j], high nibble out[j+16],
 * value = (nibble - 8) * d. */
void zo_dequant_q4_0_block(const uint8_t *blk, float *out) {
  float d = zo_fp16_to_f32(rd16(blk));
  for (int j = 0; j < 16; ++j) {
    uint8_t b = blk[2 + j];
    out[j] = (float)((int)(b & 0x0F) - 8) * d;
    out[j + 16] = (float)((int)((b >> 4) & 0x0F) - 8) * d;
  }
}

/* dequant.rs:247-257: out[k] = (i8)qs[k] * d. */
void zo_dequant_q8_0_block(const uint8_t *blk, float *out) {
  float d = zo_fp16_to_f32(rd16(blk));
  for (int k = 0; k < 32; ++k) out[k] = (float)(int8_t)blk[2 + k] * d;
}

/* silicatepack.py:910-941 (quantize_q4_0_block): d = max_signed / -8 in
 * double, q = trunc(v * (1/d) + 8.5) clamped to [0, 15], byte j packs
 * q[j] | q[j+16] << 4, fp16(d) stored first.  All-zero block -> 18 zero bytes. */
void zo_quantize_q4_0_block(const float *v, uint8_t *out) {
  double max_abs = 0.0, max_signed = 0.0;
  for (int i = 0; i < 32; ++i) {
    double a = fabs((double)v[i]);
    if (a > max_abs) { max_abs = a; max_signed = (double)v[i]; }
  }
  if (max_abs == 0.0) { memset(out, 0, 18); return; }
  double d = max_signed / -8.0;
  double inv_d = 1.0 / d;
  int q[32];
  for (int i = 0; i < 32; ++i) {
    double t = (double)v[i] * inv_d + 8.5;
    long qi = (long)t;            /* Python int(): truncation toward zero */
    if (qi < 0) qi = 0;
    if (qi > 15) qi = 15;
    q[i] = (int)qi;
  }
  uint16_t h = zo_f64_to_fp16(d);
  out[0] = (uint8_t)(h & 0xFF);
  out[1] = (uint8_t)(h >> 8);
  for (int j = 0; j < 16; ++j) out[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

/* silicatepack.py:893-907 (quantize_q8_0_block): d = max_abs / 127 in
 * double, q = round-half-even(v * (1/d)) clamped to [-127, 127]. */
void zo_quantize_q8_0_block(const float *v, uint8_t *out) {
  double max_abs = 0.0;
  for (int i = 0; i < 32; ++i) {
    double a = fabs((double)v[i]);
    if (a > max_abs) max_abs = a;
  }
  if (max_abs == 0.0) { memset(out, 0, 34); return; }
  double d = max_abs / 127.0;
  double inv_d = 1.0 / d;
  uint16_t h = zo_f64_to_fp16(d);
  out[0] = (uint8_t)(h & 0xFF);
  out[1] = (uint8_t)(h >> 8);
  for (int i = 0; i < 32; ++i) {
    double r = nearbyint((double)v[i] * inv_d);   /* Python round(): half-even */
    if (r < -127.0) r = -127.0;
    if (r > 127.0) r = 127.0;
    out[2 + i] = (uint8_t)(int8_t)r;
  }
}

void zo_quantize_row_q8_0(const float *x, uint8_t *out, size_t n) {
  for (size_t b = 0; b < n / 32; ++b) zo_quantize_q8_0_block(x + 32 * b, out + 34 * b);
}

/* silicatepack.py:982-1022: for each group of 4 rows and each K-block b,
 * emit the 4 fp16 scales then the 4 quant bodies (rows in lane order). */
int zo_interleave_x4(const uint8_t *plain, uint8_t *x4, size_t rows, size_t cols, int quant) {
  size_t bb = (quant == ZO_Q4_0) ? 18 : (quant == ZO_Q8_0) ? 34 : 0;
  if (!bb || cols % 32 || rows % 4) return ZO_ERR_ARG;
  size_t bpr = cols / 32, body = bb - 2;
  uint8_t *dst = x4;
  for (size_t g = 0; g < rows; g += 4) {
    for (size_t b = 0; b < bpr; ++b) {
      for (size_t l = 0; l < 4; ++l) {
        const uint8_t *src = plain + ((g + l) * bpr + b) * bb;
        *dst++ = src[0];
        *dst++ = src[1];
      }
      for (size_t l = 0; l < 4; ++l) {
        const uint8_t *src = plain + ((g + l) * bpr + b) * bb;
        memcpy(dst, src + 2, body);
        dst += body;
      }
    }
  }
  return ZO_OK;
}

void zo_linear_q4_0_q8act(const uint8_t *xq, const uint8_t *w, float *out, size_t in_dim,
                          size_t out_dim) {
  size_t bpr = in_dim / 32;
  for (size_t i = 0; i < out_dim; ++i) {
    float acc = 0.0f;
    for (size_t b = 0; b < bpr; ++b) {
      const uint8_t *wb = w + (i * bpr + b) * 18;
      const uint8_t *xb = xq + b * 34;
      int sumi = 0;
      for (int j = 0; j < 16; ++j) {
        int lo = (wb[2 + j] & 0x0F) - 8, hi = (wb[2 + j] >> 4) - 8;
        sumi += lo * (int8_t)xb[2 + j] + hi * (int8_t)xb[2 + 16 + j];
      }
      acc += ((float)sumi * zo_fp16_to_f32(rd16(wb))) * zo_fp16_to_f32(rd16(xb));
    }
    out[i] = acc;
  }
}

/* Q8_0 weights on Q8_0-quantised inputs, the batched path's LM head: per
 * block the exact integer dot, then (sumi * d_w) * d_x added in block order
 * (the arithmetic of zo_linear_q4_0_q8act with int8 weights). */
void zo_linear_q8_0_q8act(const uint8_t *xq, const uint8_t *w, float *out, size_t in_dim,
                          size_t out_dim) {
  size_t bpr = in_dim / 32;
  for (size_t i = 0; i < out_dim; ++i) {
    float acc = 0.0f;
    for (size_t b = 0; b < bpr; ++b) {
      const uint8_t *wb = w + (i * bpr + b) * 34;
      const uint8_t *xb = xq + b * 34;
      int sumi = 0;
      for (int j = 0; j < 32; ++j) sumi += (int8_t)wb[2 + j] * (int8_t)xb[2 + j];
      acc += ((float)sumi * zo_fp16_to_f32(rd16(wb))) * zo_fp16_to_f32(rd16(xb));
    }
    out[i] = acc;
  }
}

/* ======================================================================
 * Scalar crate ops (crates/zero-llm-inference/src)
 * ====================================================================== */

/* ops.rs:29-52: sequential sum of squares, mean, sqrtf(mean + eps), 1/rms,
 * out = x * rms_inv * w (left to right, each product rounded). */
void zo_rmsnorm(const float *x, const float *w, float *out, size_t n, float eps) {
  float ssq = 0.0f;
  for (size_t i = 0; i < n; ++i) ssq += x[i] * x[i];
  float mean_sq = ssq / (float)n;
  float rms = sqrtf(mean_sq + eps);
  float rms_inv = 1.0f / rms;
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * rms_inv * w[i];
}

/* ops.rs:79-93: inv_freq[i] = powf(base, -2*i / head_dim) in f32. */
void zo_rope_ctx(float base, size_t half, float *inv) {
  float head_dim_f = (float)(half * 2);
  for (size_t i = 0; i < half; ++i) {
    float exponent = -2.0f * (float)i / head_dim_f;
    inv[i] = powf(base, exponent);
  }
}

/* ops.rs:111-132: NeoX half-split rotation with libm cosf/sinf. */
void zo_rope(float *qk, const float *inv, size_t half, size_t pos) {
  float pos_f = (float)pos;
  for (size_t i = 0; i < half; ++i) {
    float theta = pos_f * inv[i];
    float c = cosf(theta), s = sinf(theta);
    float x = qk[i], y = qk[i + half];
    qk[i] = x * c - y * s;
    qk[i + half] = x * s + y * c;
  }
}

/* ops.rs:318-378 (linear_q4_0): per row, per block: dequantise 32 values,
 * then acc += x * w sequentially (unfused). */
void zo_linear_q4_0(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim) {
  size_t bpr = in_dim / 32;
  float buf[32];
  for (size_t i = 0; i < out_dim; ++i) {
    float acc = 0.0f;
    for (size_t b = 0; b < bpr; ++b) {
      zo_dequant_q4_0_block(w + (i * bpr + b) * 18, buf);
      for (int k = 0; k < 32; ++k) acc += x[b * 32 + k] * buf[k];
    }
    out[i] = acc;
  }
}

/* ops.rs:403-457 (linear_q8_0). */
void zo_linear_q8_0(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim) {
  size_t bpr = in_dim / 32;
  float buf[32];
  for (size_t i = 0; i < out_dim; ++i) {
    float acc = 0.0f;
    for (size_t b = 0; b < bpr; ++b) {
      zo_dequant_q8_0_block(w + (i * bpr + b) * 34, buf);
      for (int k = 0; k < 32; ++k) acc += x[b * 32 + k] * buf[k];
    }
    out[i] = acc;
  }
}

/* ops.rs:486-523 (linear_dispatch).  The reference panics on an
 * unsupported quant; the oracle returns ZO_ERR_UNSUPPORTED_QUANT. */
/* dequant.rs:75-85 get_scale_min_k4: 6-bit sub-block scale and min j of
 * the 12 packed bytes. */
static void q4k_scale_min(const uint8_t *sc, int j, uint8_t *d, uint8_t *m) {
  if (j < 4) {
    *d = sc[j] & 0x3F;
    *m = sc[j + 4] & 0x3F;
  } else {
    *d = (uint8_t)((sc[j + 4] & 0x0F) | ((sc[j - 4] >> 6) << 4));
    *m = (uint8_t)((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
  }
}

/* dequant_q4k_block (zero-gguf-parser/src/dequant.rs:98-138, scales by
 * get_scale_min_k4 at :75-85): d, dmin fp16; four 64-element groups, the low nibbles
 * of qs[32 g ..] with sub-block 2g's scale / min, the high nibbles with 2g+1's;
 * out = (d * sc) * q - dmin * mn, each product rounded on its own. */
void zo_dequant_q4_k_block(const uint8_t *blk, float *out) {
  const float d = zo_fp16_to_f32(rd16(blk)), dmin = zo_fp16_to_f32(rd16(blk + 2));
  const uint8_t *sc = blk + 4, *qs = blk + 16;
  for (int g = 0; g < 4; ++g) {
    uint8_t s0, m0, s1, m1;
    q4k_scale_min(sc, 2 * g, &s0, &m0);
    q4k_scale_min(sc, 2 * g + 1, &s1, &m1);
    const float d1 = d * (float)s0, mn1 = dmin * (float)m0;
    const float d2 = d * (float)s1, mn2 = dmin * (float)m1;
    for (int l = 0; l < 32; ++l) out[64 * g + l] = d1 * (float)(qs[32 * g + l] & 0xF) - mn1;
    for (int l = 0; l < 32; ++l) out[64 * g + 32 + l] = d2 * (float)(qs[32 * g + l] >> 4) - mn2;
  }
}

/* dequant_q6k_block (zero-gguf-parser/src/dequant.rs:328-360, the ggml
 * dequantize_row_q6_K order): two 128-element halves; element 128 h + l + 32 k
 * takes a 4-bit part of ql and a 2-bit part of qh, minus 32, times
 * d * scale (left to right) with scale = int8 sc[8 h + l / 16 + 2 k]. */
void zo_dequant_q6_k_block(const uint8_t *blk, float *out) {
  const float d = zo_fp16_to_f32(rd16(blk + 208));
  const uint8_t *ql = blk, *qh = blk + 128, *sc = blk + 192;
  for (int h = 0; h < 2; ++h) {
    const uint8_t *l0 = ql + 64 * h, *h0 = qh + 32 * h;
    const int8_t *s0 = (const int8_t *)sc + 8 * h;
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = ((l0[l] & 0xF) | ((h0[l] & 3) << 4)) - 32;
      const int q2 = ((l0[l + 32] & 0xF) | (((h0[l] >> 2) & 3) << 4)) - 32;
      const int q3 = ((l0[l] >> 4) | (((h0[l] >> 4) & 3) << 4)) - 32;
      const int q4 = ((l0[l + 32] >> 4) | (((h0[l] >> 6) & 3) << 4)) - 32;
      out[128 * h + l] = d * (float)s0[is] * (float)q1;
      out[128 * h + l + 32] = d * (float)s0[is + 2] * (float)q2;
      out[128 * h + l + 64] = d * (float)s0[is + 4] * (float)q3;
      out[128 * h + l + 96] = d * (float)s0[is + 6] * (float)q4;
    }
  }
}

/* ops.rs:179-292: per row, per super-block dequantise, then acc += x * w
 * over its 256 elements in order. */
static void linear_kquant(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim, size_t bb,
                          void (*deq)(const uint8_t *, float *)) {
  const size_t bpr = in_dim / 256;
  float buf[256];
  for (size_t i = 0; i < out_dim; ++i) {
    float acc = 0.0f;
    for (size_t b = 0; b < bpr; ++b) {
      deq(w + (i * bpr + b) * bb, buf);
      for (int k = 0; k < 256; ++k) acc += x[b * 256 + k] * buf[k];
    }
    out[i] = acc;
  }
}
void zo_linear_q4_k(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim) {
  linear_kquant(x, w, out, in_dim, out_dim, 144, zo_dequant_q4_k_block);
}
void zo_linear_q6_k(const float *x, const uint8_t *w, float *out, size_t in_dim, size_t out_dim) {
  linear_kquant(x, w, out, in_dim, out_dim, 210, zo_dequant_q6_k_block);
}

int zo_linear_dispatch(const float *x, const uint8_t *w, float *out, size_t in_dim,
                       size_t out_dim, int quant) {
  if (quant == ZO_Q4_0) { zo_linear_q4_0(x, w, out, in_dim, out_dim); return ZO_OK; }
  if (quant == ZO_Q8_0) { zo_linear_q8_0(x, w, out, in_dim, out_dim); return ZO_OK; }
  if (quant == ZO_Q4_K) { zo_linear_q4_k(x, w, out, in_dim, out_dim); return ZO_OK; }
  if (quant == ZO_Q6_K) { zo_linear_q6_k(x, w, out, in_dim, out_dim); return ZO_OK; }
  return ZO_ERR_UNSUPPORTED_QUANT;
}

/* attention.rs:48-84 (softmax): max-trick with libm expf; errors when the
 * max is non-finite or the sum is <= 0 or non-finite. */
int zo_softmax(float *s, size_t len) {
  if (len == 0) return ZO_OK;
  float mx = -INFINITY;
  for (size_t i = 0; i < len; ++i) if (s[i] > mx) mx = s[i];
  if (!isfinite(mx)) return ZO_ERR_NUMERICAL_INSTABILITY;
  float sum = 0.0f;
  for (size_t i = 0; i < len; ++i) {
    float e = expf(s[i] - mx);
    s[i] = e;
    sum += e;
  }
  if (sum <= 0.0f || !isfinite(sum)) return ZO_ERR_NUMERICAL_INSTABILITY;
  float inv = 1.0f / sum;
  for (size_t i = 0; i < len; ++i) s[i] *= inv;
  return ZO_OK;
}

/* ======================================================================
 * AVX-512-order ops (kernel/src/arch/x86_64/math)
 * ====================================================================== */

/* _mm512_reduce_add_ps as lowered for the reference (halving tree):
 * t8[i] = v[i] + v[i+8]; t4[i] = t8[i] + t8[i+4]; t2[i] = t4[i] + t4[i+2];
 * result = t2[0] + t2[1]. */
static inline float reduce16(const float *v) {
  float t8[8], t4[4], t2[2];
  for (int i = 0; i < 8; ++i) t8[i] = v[i] + v[i + 8];
  for (int i = 0; i < 4; ++i) t4[i] = t8[i] + t8[i + 4];
  for (int i = 0; i < 2; ++i) t2[i] = t4[i] + t4[i + 2];
  return t2[0] + t2[1];
}

/* Per-row body shared by linear.rs:909-1072 (Q4_0X4) and the plain
 * single-row body linear.rs:710-859: for each block in K order,
 * acc_lo[l] = fma(x[32b+l], d * (lo_l - 8), acc_lo[l]) and
 * acc_hi[l] = fma(x[32b+16+l], d * (hi_l - 8), acc_hi[l]); finally
 * reduce_add(acc_lo + acc_hi).  `scale_at(b)` / `qs_at(b)` locate the
 * block's fp16 scale and 16 nibble bytes in either layout. */
static float row_q4_emul(const float *x, size_t bpr, const uint8_t *base, size_t stride,
                         size_t d_off, size_t qs_off) {
  float lo[16] = {0}, hi[16] = {0};
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = base + b * stride;
    float d = zo_fp16_to_f32(rd16(blk + d_off));
    const uint8_t *qs = blk + qs_off;
    for (int l = 0; l < 16; ++l) {
      float wl = d * ((float)(qs[l] & 0x0F) - 8.0f);
      float wh = d * ((float)((qs[l] >> 4) & 0x0F) - 8.0f);
      lo[l] = fmaf(x[b * 32 + l], wl, lo[l]);
      hi[l] = fmaf(x[b * 32 + 16 + l], wh, hi[l]);
    }
  }
  float s[16];
  for (int l = 0; l < 16; ++l) s[l] = lo[l] + hi[l];
  return reduce16(s);
}

/* linear.rs:1096-1213 (Q8_0X4) / :1271-1402 (plain): same accumulator
 * structure with sign-extended i8 and w = d * q. */
static float row_q8_emul(const float *x, size_t bpr, const uint8_t *base, size_t stride,
                         size_t d_off, size_t qs_off) {
  float lo[16] = {0}, hi[16] = {0};
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = base + b * stride;
    float d = zo_fp16_to_f32(rd16(blk + d_off));
    const int8_t *qs = (const int8_t *)(blk + qs_off);
    for (int l = 0; l < 16; ++l) {
      lo[l] = fmaf(x[b * 32 + l], d * (float)qs[l], lo[l]);
      hi[l] = fmaf(x[b * 32 + 16 + l], d * (float)qs[16 + l], hi[l]);
    }
  }
  float s[16];
  for (int l = 0; l < 16; ++l) s[l] = lo[l] + hi[l];
  return reduce16(s);
}

#if defined(__x86_64__)
/* Real AVX-512 forms of the same per-row bodies (used for the timed
 * baseline; bit-identical to the emulation by construction, tested). */
__attribute__((target("avx512f,fma"))) static inline float hsum512(__m512 v) {
  __m256 a = _mm256_add_ps(_mm512_castps512_ps256(v),
                           _mm256_castpd_ps(_mm512_extractf64x4_pd(_mm512_castps_pd(v), 1)));
  __m128 b = _mm_add_ps(_mm256_castps256_ps128(a), _mm256_extractf128_ps(a, 1));
  __m128 c = _mm_add_ps(b, _mm_shuffle_ps(b, b, _MM_SHUFFLE(1, 0, 3, 2)));
  return _mm_cvtss_f32(c) + _mm_cvtss_f32(_mm_shuffle_ps(c, c, 1));
}

__attribute__((target("avx512f,fma"))) static void rows4_q4_avx512(
    const float *x, size_t bpr, const uint8_t *grp, float *out4) {
  const __m512i m = _mm512_set1_epi32(0x0F);
  const __m512 b8 = _mm512_set1_ps(8.0f);
  __m512 lo[4], hi[4];
  for (int r = 0; r < 4; ++r) { lo[r] = _mm512_setzero_ps(); hi[r] = _mm512_setzero_ps(); }
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = grp + b * 72;
    __m512 xl = _mm512_loadu_ps(x + b * 32), xh = _mm512_loadu_ps(x + b * 32 + 16);
    for (int r = 0; r < 4; ++r) {
      __m512 d = _mm512_set1_ps(zo_fp16_to_f32(rd16(blk + 2 * r)));
      __m512i by = _mm512_cvtepu8_epi32(_mm_loadu_si128((const __m128i *)(blk + 8 + 16 * r)));
      __m512 l = _mm512_cvtepi32_ps(_mm512_and_epi32(by, m));
      __m512 h = _mm512_cvtepi32_ps(_mm512_and_epi32(_mm512_srli_epi32(by, 4), m));
      lo[r] = _mm512_fmadd_ps(xl, _mm512_mul_ps(d, _mm512_sub_ps(l, b8)), lo[r]);
      hi[r] = _mm512_fmadd_ps(xh, _mm512_mul_ps(d, _mm512_sub_ps(h, b8)), hi[r]);
    }
  }
  for (int r = 0; r < 4; ++r) out4[r] = hsum512(_mm512_add_ps(lo[r], hi[r]));
}

__attribute__((target("avx512f,fma"))) static void rows4_q8_avx512(
    const float *x, size_t bpr, const uint8_t *grp, float *out4) {
  __m512 lo[4], hi[4];
  for (int r = 0; r < 4; ++r) { lo[r] = _mm512_setzero_ps(); hi[r] = _mm512_setzero_ps(); }
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = grp + b * 136;
    __m512 xl = _mm512_loadu_ps(x + b * 32), xh = _mm512_loadu_ps(x + b * 32 + 16);
    for (int r = 0; r < 4; ++r) {
      __m512 d = _mm512_set1_ps(zo_fp16_to_f32(rd16(blk + 2 * r)));
      const uint8_t *q = blk + 8 + 32 * r;
      __m512 l = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i *)q)));
      __m512 h =
          _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i *)(q + 16))));
      lo[r] = _mm512_fmadd_ps(xl, _mm512_mul_ps(d, l), lo[r]);
      hi[r] = _mm512_fmadd_ps(xh, _mm512_mul_ps(d, h), hi[r]);
    }
  }
  for (int r = 0; r < 4; ++r) out4[r] = hsum512(_mm512_add_ps(lo[r], hi[r]));
}

/* The plain-layout single-row bodies (linear.rs:710-859 / :1271-1402) as
 * real AVX-512: one row of 18- (Q4_0) or 34-byte (Q8_0) blocks, the same
 * lane sequence as row_q4_emul / row_q8_emul. */
__attribute__((target("avx512f,fma"))) static float row_q4_plain_avx512(const float *x, size_t bpr,
                                                                        const uint8_t *row) {
  const __m512i m = _mm512_set1_epi32(0x0F);
  const __m512 b8 = _mm512_set1_ps(8.0f);
  __m512 lo = _mm512_setzero_ps(), hi = _mm512_setzero_ps();
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = row + b * 18;
    __m512 xl = _mm512_loadu_ps(x + b * 32), xh = _mm512_loadu_ps(x + b * 32 + 16);
    __m512 d = _mm512_set1_ps(zo_fp16_to_f32(rd16(blk)));
    __m512i by = _mm512_cvtepu8_epi32(_mm_loadu_si128((const __m128i *)(blk + 2)));
    __m512 l = _mm512_cvtepi32_ps(_mm512_and_epi32(by, m));
    __m512 h = _mm512_cvtepi32_ps(_mm512_and_epi32(_mm512_srli_epi32(by, 4), m));
    lo = _mm512_fmadd_ps(xl, _mm512_mul_ps(d, _mm512_sub_ps(l, b8)), lo);
    hi = _mm512_fmadd_ps(xh, _mm512_mul_ps(d, _mm512_sub_ps(h, b8)), hi);
  }
  return hsum512(_mm512_add_ps(lo, hi));
}

__attribute__((target("avx512f,fma"))) static float row_q8_plain_avx512(const float *x, size_t bpr,
                                                                        const uint8_t *row) {
  __m512 lo = _mm512_setzero_ps(), hi = _mm512_setzero_ps();
  for (size_t b = 0; b < bpr; ++b) {
    const uint8_t *blk = row + b * 34;
    __m512 xl = _mm512_loadu_ps(x + b * 32), xh = _mm512_loadu_ps(x + b * 32 + 16);
    __m512 d = _mm512_set1_ps(zo_fp16_to_f32(rd16(blk)));
    __m512 l = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i *)(blk + 2))));
    __m512 h = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i *)(blk + 18))));
    lo = _mm512_fmadd_ps(xl, _mm512_mul_ps(d, l), lo);
    hi = _mm512_fmadd_ps(xh, _mm512_mul_ps(d, h), hi);
  }
  return hsum512(_mm512_add_ps(lo, hi));
}
#endif

int zo_have_avx512(void) {
#if defined(__x86_64__)
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx512f") ? 1 : 0;
#else
  return 0;
#endif
}

/* Row split across host threads in whole 4-row groups, as the reference's
 * SMP dispatcher aligns ranges to the interleave group (smp_partition.rs:143):
 * participant i takes units [i*base + min(i, extra), ...). */
typedef struct {
  void (*fn)(void *ctx, size_t u0, size_t u1);
  void *ctx;
  size_t u0, u1;
} zo_task;

static void *zo_task_main(void *p) {
  zo_task *t = (zo_task *)p;
  if (t->u0 < t->u1) t->fn(t->ctx, t->u0, t->u1);
  return NULL;
}

static int zo_ncores(int threads) {
  if (threads > 0) return threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void parallel_units(size_t units, int threads, void (*fn)(void *, size_t, size_t), void *ctx) {
  int n = zo_ncores(threads);
  if (n > 256) n = 256;
  if ((size_t)n > units) n = (int)(units ? units : 1);
  if (n <= 1) { fn(ctx, 0, units); return; }
  pthread_t tid[256];
  zo_task task[256];
  size_t base = units / (size_t)n, extra = units % (size_t)n;
  for (int i = 0; i < n; ++i) {
    size_t s = (size_t)i * base + ((size_t)i < extra ? (size_t)i : extra);
    size_t e = s + base + ((size_t)i < extra ? 1 : 0);
    task[i].fn = fn; task[i].ctx = ctx; task[i].u0 = s; task[i].u1 = e;
  }
  for (int i = 1; i < n; ++i) pthread_create(&tid[i], NULL, zo_task_main, &task[i]);
  zo_task_main(&task[0]);
  for (int i = 1; i < n; ++i) pthread_join(tid[i], NULL);
}


/* ----------------------------------------------------------------------
 * Persistent dispatcher for the timed CPU baseline, after the reference's
 * SMP matmul dispatch (smp.rs:1559-1700): the worker threads are created
 * once per run, each pinned to its own physical core, and park on a shared
 * epoch word.  A dispatch publishes (fn, ctx, units), bumps the epoch with
 * release semantics (the wake signal), runs participant 0's range on the
 * calling thread and waits until every worker has arrived.  Ranges are the
 * reference's closed-form even split in whole units (row_range_for,
 * smp_partition.rs:143-167), so each row is computed exactly as the
 * single-threaded kernel computes it.
 * ---------------------------------------------------------------------- */
#define ZO_POOL_MAX 256

typedef void (*zo_part_fn)(void *ctx, size_t u0, size_t u1, int part);

struct zo_pool {
  int n;                                 /* participants, the caller is 0 */
  pthread_t tid[ZO_POOL_MAX];
  int cpu[ZO_POOL_MAX];                  /* pinned logical CPU (-1: not pinned) */
  _Atomic unsigned long long epoch;
  _Atomic int arrived;
  _Atomic int quit;
  zo_part_fn fn;
  void *ctx;
  size_t units;
  int caller_cpu;                        /* participant 0's core (-1: not pinned) */
};

typedef struct {
  struct zo_pool *p;
  int part;
} zo_worker_arg;

static void zo_range_for(size_t units, int n, int i, size_t *u0, size_t *u1) {
  size_t base = units / (size_t)n, extra = units % (size_t)n;
  size_t s = (size_t)i * base + ((size_t)i < extra ? (size_t)i : extra);
  *u0 = s;
  *u1 = s + base + ((size_t)i < extra ? 1 : 0);
}

static int zo_read_int(const char *path) {
  FILE *f = fopen(path, "r");
  int v = -1;
  if (f) {
    if (fscanf(f, "%d", &v) != 1) v = -1;
    fclose(f);
  }
  return v;
}

/* One logical CPU per physical core (the lowest-numbered sibling) among the
 * CPUs this process may run on; returns how many were found. */
static int zo_physical_cpus(int *out, int cap) {
  cpu_set_t allowed;
  if (sched_getaffinity(0, sizeof(allowed), &allowed) != 0) return 0;
  int n = 0;
  int keys[4096];
  for (int c = 0; c < CPU_SETSIZE && n < cap; ++c) {
    if (!CPU_ISSET(c, &allowed)) continue;
    char path[128];
    snprintf(path, sizeof path, "/sys/devices/system/cpu/cpu%d/topology/core_id", c);
    int core = zo_read_int(path);
    snprintf(path, sizeof path, "/sys/devices/system/cpu/cpu%d/topology/physical_package_id", c);
    int pkg = zo_read_int(path);
    int key = (core < 0 || pkg < 0) ? -1 - c : pkg * 65536 + core;
    int seen = 0;
    for (int k = 0; k < n; ++k) seen |= keys[k] == key;
    if (!seen) {
      keys[n] = key;
      out[n++] = c;
    }
  }
  return n;
}

/* The calling thread runs participant 0 on the first physical core while a
 * forward or LM-head call is in flight, and gets its own affinity back at
 * the end of the call (threads it creates later must not inherit the pin). */
typedef struct {
  cpu_set_t saved;
  int active;
} zo_caller_pin;

static void zo_caller_pin_begin(const struct zo_pool *p, zo_caller_pin *cp);
static void zo_caller_pin_end(zo_caller_pin *cp);

static void zo_pin(int cpu) {
  if (cpu < 0) return;
  cpu_set_t m;
  CPU_ZERO(&m);
  CPU_SET(cpu, &m);
  pthread_setaffinity_np(pthread_self(), sizeof(m), &m);
}

static void *zo_worker_main(void *a) {
  zo_worker_arg *wa = (zo_worker_arg *)a;
  struct zo_pool *p = wa->p;
  const int part = wa->part;
  free(wa);
  zo_pin(p->cpu[part]);
  unsigned long long seen = 0;
  for (;;) {
    unsigned long long e;
    unsigned spins = 0;
    while ((e = atomic_load_explicit(&p->epoch, memory_order_acquire)) == seen) {
      if (atomic_load_explicit(&p->quit, memory_order_acquire)) return NULL;
      _mm_pause();
      if (++spins > (1u << 20)) {          /* parked for a while: stop burning the core */
        struct timespec ts = {0, 20000};
        nanosleep(&ts, NULL);
        spins = 1u << 19;
      }
    }
    seen = e;
    size_t u0, u1;
    zo_range_for(p->units, p->n, part, &u0, &u1);
    if (u0 < u1) p->fn(p->ctx, u0, u1, part);
    atomic_fetch_add_explicit(&p->arrived, 1, memory_order_acq_rel);
  }
}

zo_pool *zo_pool_create(int threads) {
  struct zo_pool *p = (struct zo_pool *)calloc(1, sizeof(struct zo_pool));
  if (!p) return NULL;
  int cpus[ZO_POOL_MAX];
  int ncpu = zo_physical_cpus(cpus, ZO_POOL_MAX);
  int n = threads > 0 ? threads : (ncpu > 0 ? ncpu : zo_ncores(0));
  if (n > ZO_POOL_MAX) n = ZO_POOL_MAX;
  if (n < 1) n = 1;
  p->n = n;
  /* workers take the physical cores after the first, which the calling
   * thread takes during a call (zo_caller_pin_begin) */
  for (int i = 0; i < n; ++i) p->cpu[i] = (ncpu >= n && i > 0) ? cpus[i] : -1;
  p->caller_cpu = ncpu >= n ? cpus[0] : -1;
  for (int i = 1; i < n; ++i) {
    zo_worker_arg *wa = (zo_worker_arg *)malloc(sizeof(zo_worker_arg));
    wa->p = p;
    wa->part = i;
    if (pthread_create(&p->tid[i], NULL, zo_worker_main, wa) != 0) {
      free(wa);
      p->n = i;                              /* run with the workers that started */
      break;
    }
  }
  return p;
}

static void zo_caller_pin_begin(const struct zo_pool *p, zo_caller_pin *cp) {
  cp->active = 0;
  if (!p || p->n <= 1 || p->caller_cpu < 0) return;
  if (pthread_getaffinity_np(pthread_self(), sizeof(cp->saved), &cp->saved) != 0) return;
  zo_pin(p->caller_cpu);
  cp->active = 1;
}

static void zo_caller_pin_end(zo_caller_pin *cp) {
  if (cp->active) pthread_setaffinity_np(pthread_self(), sizeof(cp->saved), &cp->saved);
}

void zo_pool_destroy(zo_pool *p) {
  if (!p) return;
  atomic_store_explicit(&p->quit, 1, memory_order_release);
  for (int i = 1; i < p->n; ++i) pthread_join(p->tid[i], NULL);
  free(p);
}

int zo_pool_size(const zo_pool *p) { return p ? p->n : 1; }

/* One dispatch: fn over [0, units) split across the participants; returns
 * once every participant has finished its range. */
static void zo_pool_run(struct zo_pool *p, size_t units, zo_part_fn fn, void *ctx) {
  if (!p || p->n <= 1) {
    if (units) fn(ctx, 0, units, 0);
    return;
  }
  p->fn = fn;
  p->ctx = ctx;
  p->units = units;
  atomic_store_explicit(&p->arrived, 0, memory_order_relaxed);
  atomic_fetch_add_explicit(&p->epoch, 1, memory_order_release);
  size_t u0, u1;
  zo_range_for(units, p->n, 0, &u0, &u1);
  if (u0 < u1) fn(ctx, u0, u1, 0);
  while (atomic_load_explicit(&p->arrived, memory_order_acquire) < p->n - 1) _mm_pause();
}

typedef struct {
  const float *x;
  const uint8_t *w;
  float *out;
  size_t bpr;
  int quant, simd;
} zo_plain_ctx;

static void plain_rows_part(void *p, size_t i0, size_t i1, int part) {
  (void)part;
  const zo_plain_ctx *c = (const zo_plain_ctx *)p;
  const size_t rb = c->bpr * (c->quant == ZO_Q4_0 ? 18 : 34);
  for (size_t i = i0; i < i1; ++i) {
    const uint8_t *row = c->w + i * rb;
#if defined(__x86_64__)
    if (c->simd) {
      c->out[i] = c->quant == ZO_Q4_0 ? row_q4_plain_avx512(c->x, c->bpr, row)
                                      : row_q8_plain_avx512(c->x, c->bpr, row);
      continue;
    }
#endif
    c->out[i] = c->quant == ZO_Q4_0 ? row_q4_emul(c->x, c->bpr, row, 18, 0, 2)
                                    : row_q8_emul(c->x, c->bpr, row, 34, 0, 2);
  }
}

/* linear_dispatch_avx512 (inference_avx512.rs:1147) on plain Q4_0 / Q8_0
 * rows (the DeepSeek2 tensors): rows split over the pool's participants
 * (a null pool: the calling thread alone); each row's arithmetic is the
 * single-row AVX-512 body, so the split does not change any bit. */
int zo_linear_plain_pool(zo_pool *p, const float *x, const uint8_t *w, float *out, size_t in_dim,
                         size_t out_dim, int quant, int simd) {
  if (quant != ZO_Q4_0 && quant != ZO_Q8_0) return ZO_ERR_UNSUPPORTED_QUANT;
  if (in_dim % 32) return ZO_ERR_ARG;
  zo_plain_ctx c = {x, w, out, in_dim / 32, quant, simd && zo_have_avx512()};
  zo_pool_run(p, out_dim, plain_rows_part, &c);
  return ZO_OK;
}

typedef struct {
  const float *x;
  const uint8_t *w;
  float *out;
  size_t bpr;
  int use;
} zo_lin_ctx;

static void q4x4_units(void *p, size_t g0, size_t g1) {
  zo_lin_ctx *c = (zo_lin_ctx *)p;
  for (size_t g = g0; g < g1; ++g) {
    const uint8_t *grp = c->w + g * c->bpr * 72;
#if defined(__x86_64__)
    if (c->use) { rows4_q4_avx512(c->x, c->bpr, grp, c->out + 4 * g); continue; }
#endif
    for (int r = 0; r < 4; ++r) c->out[4 * g + r] = row_q4_emul(c->x, c->bpr, grp, 72, 2 * r, 8 + 16 * r);
  }
}

static void q8x4_units(void *p, size_t g0, size_t g1) {
  zo_lin_ctx *c = (zo_lin_ctx *)p;
  for (size_t g = g0; g < g1; ++g) {
    const uint8_t *grp = c->w + g * c->bpr * 136;
#if defined(__x86_64__)
    if (c->use) { rows4_q8_avx512(c->x, c->bpr, grp, c->out + 4 * g); continue; }
#endif
    for (int r = 0; r < 4; ++r) c->out[4 * g + r] = row_q8_emul(c->x, c->bpr, grp, 136, 2 * r, 8 + 32 * r);
  }
}

static void q4_units(void *p, size_t i0, size_t i1) {
  zo_lin_ctx *c = (zo_lin_ctx *)p;
  for (size_t i = i0; i < i1; ++i) c->out[i] = row_q4_emul(c->x, c->bpr, c->w + i * c->bpr * 18, 18, 0, 2);
}

static void q8_units(void *p, size_t i0, size_t i1) {
  zo_lin_ctx *c = (zo_lin_ctx *)p;
  for (size_t i = i0; i < i1; ++i) c->out[i] = row_q8_emul(c->x, c->bpr, c->w + i * c->bpr * 34, 34, 0, 2);
}

/* linear_q4_0x4_avx512_range (linear.rs:909) over all groups. */
void zo_linear_q4_0x4_avx512(const float *x, const uint8_t *w, float *out, size_t in_dim,
                             size_t out_dim, int threads, int simd) {
  zo_lin_ctx c = {x, w, out, in_dim / 32, simd && zo_have_avx512()};
  parallel_units(out_dim / 4, threads, q4x4_units, &c);
}

/* linear_q8_0x4_avx512_range (linear.rs:1096). */
void zo_linear_q8_0x4_avx512(const float *x, const uint8_t *w, float *out, size_t in_dim,
                             size_t out_dim, int threads, int simd) {
  zo_lin_ctx c = {x, w, out, in_dim / 32, simd && zo_have_avx512()};
  parallel_units(out_dim / 4, threads, q8x4_units, &c);
}

/* linear_q4_0_avx512_range (linear.rs:710-859) on the plain layout: the
 * per-row FP sequence equals the X4 kernel's (linear.rs:886-895). */
void zo_linear_q4_0_avx512(const float *x, const uint8_t *w, float *out, size_t in_dim,
                           size_t out_dim, int threads, int simd) {
  zo_lin_ctx c = {x, w, out, in_dim / 32, simd};
  parallel_units(out_dim, threads, q4_units, &c);
}

/* linear_q8_0_avx512_range (linear.rs:1271-1402) on the plain layout. */
void zo_linear_q8_0_avx512(const float *x, const uint8_t *w, float *out, size_t in_dim,
                           size_t out_dim, int threads, int simd) {
  zo_lin_ctx c = {x, w, out, in_dim / 32, simd};
  parallel_units(out_dim, threads, q8_units, &c);
}

/* linear.rs:515-536 (dot_product_f32_avx512): 16-lane FMA chain,
 * reduce_add, then a scalar tail with unfused multiply-add. */
float zo_dot_product_avx512(const float *a, const float *b, size_t len) {
  float acc[16] = {0};
  size_t chunks = len / 16;
  for (size_t c = 0; c < chunks; ++c)
    for (int l = 0; l < 16; ++l) acc[l] = fmaf(a[c * 16 + l], b[c * 16 + l], acc[l]);
  float r = reduce16(acc);
  for (size_t j = chunks * 16; j < len; ++j) r += a[j] * b[j];
  return r;
}

/* linear.rs:616-639 (weighted_add_f32_avx512): out = fma(w, v, out). */
void zo_weighted_add_avx512(float weight, const float *v, float *out, size_t len) {
  size_t chunks = len / 16;
  for (size_t i = 0; i < chunks * 16; ++i) out[i] = fmaf(weight, v[i], out[i]);
  for (size_t j = chunks * 16; j < len; ++j) out[j] += weight * v[j];
}

/* linear.rs:558-609 (argmax_f32_avx512): NaN-suppressed max, then the
 * first index holding it; all-NaN -> (0, -inf). */
size_t zo_argmax_avx512(const float *v, size_t n, float *max_out) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) if (v[i] > mx) mx = v[i];
  if (max_out) *max_out = mx;
  for (size_t i = 0; i < n; ++i) if (v[i] == mx) return i;
  return 0;
}

/* AVX-512 min/max semantics: the second operand is returned when either
 * input is NaN. */
static inline float mm_min(float a, float b) { return a < b ? a : b; }
static inline float mm_max(float a, float b) { return a > b ? a : b; }

/* activation.rs:56-97 (exp_f32_avx512): clamp to +-88.37625, k =
 * round-to-nearest-even(x * log2e), two-part Cody-Waite reduction with fused
 * negated multiply-adds, degree-5 Horner polynomial with fma, times 2^k built
 * from the exponent field.  Constants are the reference's own. */
static inline float exp_avx512_lane(float x) {
  const float log2e = 1.44269504f, ln2_hi = 0.6933594f, ln2_lo = -2.1219444e-4f;
  x = mm_max(mm_min(x, 88.37625f), -88.37625f);
  float kf = nearbyintf(x * log2e);
  int32_t k = (int32_t)kf;
  float r = fmaf(-kf, ln2_lo, fmaf(-kf, ln2_hi, x));
  float p = fmaf(r, 8.3333333e-3f, 4.1666667e-2f);
  p = fmaf(r, p, 0.16666667f);
  p = fmaf(r, p, 0.5f);
  p = fmaf(r, p, 1.0f);
  p = fmaf(r, p, 1.0f);
  uint32_t bits = (uint32_t)(k + 127) << 23;
  float two_k;
  memcpy(&two_k, &bits, 4);
  return p * two_k;
}

void zo_exp_avx512(const float *x, float *y, size_t n) {
  for (size_t i = 0; i < n; ++i) y[i] = exp_avx512_lane(x[i]);
}

/* activation.rs:115-148 (silu_mul_avx512): silu = g / (1 + exp(0 - g)),
 * out = silu * u. */
void zo_silu_mul_avx512(const float *g, const float *u, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    float e = exp_avx512_lane(0.0f - g[i]);
    float silu = g[i] / (1.0f + e);
    out[i] = silu * u[i];
  }
}

/* trig.rs:60-127 (sincos_f32_avx512): k = rne(x * 2/pi), two-part
 * Cody-Waite reduction, odd/even polynomials with fma, quadrant fix-up by
 * swap and sign flips.  Constants are the reference's own. */
static inline void sincos_avx512_lane(float x, float *s_out, float *c_out) {
  float kf = nearbyintf(x * 0.63661977f);
  int32_t k = (int32_t)kf;
  float r = fmaf(-kf, 7.5497903e-8f, fmaf(-kf, 1.57079625f, x));
  float r2 = r * r;
  float sp = fmaf(r2, -1.98412698e-4f, 8.3333333e-3f);
  sp = fmaf(r2, sp, -0.16666667f);
  sp = fmaf(r2, sp, 1.0f);
  float sin_r = r * sp;
  float cp = fmaf(r2, 2.4801587e-5f, -1.3888889e-3f);
  cp = fmaf(r2, cp, 4.1666667e-2f);
  cp = fmaf(r2, cp, -0.5f);
  float cos_r = fmaf(r2, cp, 1.0f);
  int q = k & 3;
  int bit0 = q & 1, bit1 = (q >> 1) & 1;
  float s = bit0 ? cos_r : sin_r;
  float c = bit0 ? sin_r : cos_r;
  if (bit1) s = -s;
  if (bit0 ^ bit1) c = -c;
  *s_out = s;
  *c_out = c;
}

/* trig.rs:148-170 (rope_sincos_lut_avx512): theta = pos * inv_freq. */
void zo_rope_sincos_lut_avx512(size_t pos, const float *inv, float *cos_out, float *sin_out,
                               size_t len) {
  float p = (float)pos;
  for (size_t i = 0; i < len; ++i) sincos_avx512_lane(p * inv[i], &sin_out[i], &cos_out[i]);
}

/* trig.rs:192-216 (rope_apply_avx512): x' = fmsub(x, c, y*s),
 * y' = fmadd(x, s, y*c). */
void zo_rope_apply_avx512(float *qk, const float *c, const float *s, size_t half) {
  for (size_t i = 0; i < half; ++i) {
    float x = qk[i], y = qk[i + half];
    qk[i] = fmaf(x, c[i], -(y * s[i]));
    qk[i + half] = fmaf(x, s[i], y * c[i]);
  }
}

/* ======================================================================
 * Qwen3-shaped forward pass
 * ====================================================================== */

/* Steps 2-5 of gqa_attention_single_token_dispatch (attention.rs:344-425;
 * order 0) and of gqa_attention_single_token_avx512 (inference_avx512.rs:
 * 1612-1800; order 1) for one layer: per-head QK RMSNorm (ops.rs:29), RoPE at
 * pos (ops.rs:111 / trig.rs:148,192), KvCache::store_kv (kv_cache.rs:139),
 * then per q head scores q.k * (1/sqrt(hd)), softmax (attention.rs:48) and
 * sum_t p_t v_t.  k_block / v_block are this layer's K and V blocks
 * [max_tokens][n_kv*hd]; work holds (n_q + n_kv + 1)*hd + max_tokens floats. */
/* Steps 2-3 (QK RMSNorm, RoPE at pos, store_kv) of the decode attention
 * below; qo / ko receive the rotated q and k. */
static void attn_prepare(const float *q, const float *k, const float *v, const float *q_norm,
                         const float *k_norm, const float *inv_freqs, float *k_block, float *v_block,
                         uint32_t pos, uint32_t n_q, uint32_t n_kv, uint32_t hd, float eps, int order,
                         float *qo, float *ko) {
  const size_t half = hd / 2, kvd = (size_t)n_kv * hd;
  float cos_lut[256], sin_lut[256];
  if (order == 1) zo_rope_sincos_lut_avx512(pos, inv_freqs, cos_lut, sin_lut, half);
  for (size_t h = 0; h < n_q; ++h) zo_rmsnorm(q + h * hd, q_norm, qo + h * hd, hd, eps);
  for (size_t h = 0; h < n_kv; ++h) zo_rmsnorm(k + h * hd, k_norm, ko + h * hd, hd, eps);
  for (size_t h = 0; h < n_q; ++h) {
    if (order == 1) zo_rope_apply_avx512(qo + h * hd, cos_lut, sin_lut, half);
    else zo_rope(qo + h * hd, inv_freqs, half, pos);
  }
  for (size_t h = 0; h < n_kv; ++h) {
    if (order == 1) zo_rope_apply_avx512(ko + h * hd, cos_lut, sin_lut, half);
    else zo_rope(ko + h * hd, inv_freqs, half, pos);
  }
  memcpy(k_block + (size_t)pos * kvd, ko, kvd * 4);
  memcpy(v_block + (size_t)pos * kvd, v, kvd * 4);
}

/* Steps 4-5 for q head qh (attn_heads_kernel, inference_avx512.rs:1459-1512):
 * scores into sb, softmax, then sum_t p_t v_t accumulated into out_head. */
static int attn_head(const float *qo, const float *k_block, const float *v_block, size_t qh, size_t total,
                     uint32_t n_q, uint32_t n_kv, uint32_t hd, int order, float *sb, float *out_head) {
  const size_t kvd = (size_t)n_kv * hd, kh = qh / (n_q / n_kv);
  const float scale = 1.0f / sqrtf((float)hd);
  const float *qv = qo + qh * hd;
  for (size_t t = 0; t < total; ++t) {
    const float *kt = k_block + t * kvd + kh * hd;
    if (order == 1) {
      sb[t] = zo_dot_product_avx512(qv, kt, hd) * scale;
    } else {
      float dot = 0.0f;
      for (size_t i = 0; i < hd; ++i) dot += qv[i] * kt[i];
      sb[t] = dot * scale;
    }
  }
  int st = zo_softmax(sb, total);
  if (st) return st;
  memset(out_head, 0, hd * 4);
  for (size_t t = 0; t < total; ++t) {
    const float *vt = v_block + t * kvd + kh * hd;
    if (order == 1) zo_weighted_add_avx512(sb[t], vt, out_head, hd);
    else for (size_t i = 0; i < hd; ++i) out_head[i] += sb[t] * vt[i];
  }
  return ZO_OK;
}

int zo_gqa_attention_decode(const float *q, const float *k, const float *v, const float *q_norm,
                            const float *k_norm, const float *inv_freqs, float *k_block,
                            float *v_block, uint32_t pos, uint32_t max_tokens, uint32_t n_q,
                            uint32_t n_kv, uint32_t hd, float eps, int order, float *work,
                            float *out) {
  if (pos >= max_tokens) return ZO_ERR_KV_TOKEN_OUT_OF_RANGE;
  if (n_kv == 0 || n_q % n_kv || hd % 2 || hd > 512) return ZO_ERR_ARG;
  const size_t kvd = (size_t)n_kv * hd, total = (size_t)pos + 1;
  float *qo = work, *ko = qo + (size_t)n_q * hd, *head = ko + kvd, *sb = head + hd;
  attn_prepare(q, k, v, q_norm, k_norm, inv_freqs, k_block, v_block, pos, n_q, n_kv, hd, eps, order, qo, ko);
  for (size_t qh = 0; qh < n_q; ++qh) {
    int st = attn_head(qo, k_block, v_block, qh, total, n_q, n_kv, hd, order, sb, head);
    if (st) return st;
    memcpy(out + qh * hd, head, hd * 4);
  }
  return ZO_OK;
}

struct zo_run {
  const zo_qwen3 *m;
  int order, threads, simd;
  int q8act;                                   /* Q4_0 matmuls on Q8_0-quantised inputs */
  uint8_t *xq;                                 /* their Q8_0 blocks */
  uint32_t max_tokens;
  float *kv;                                   /* kv_cache.rs:100 layout */
  float *inv_freqs;
  float *hidden, *norm, *attn_out, *mlp_out, *q, *k, *v, *qo, *ko, *score, *head, *concat;
  float *gate, *up, *hmlp, *logits;
  float *attn_work;                            /* zo_gqa_attention_decode workspace */
  uint8_t **x4;                                /* per-layer X4 copies for the AVX path */
  uint8_t *out_x4;
  zo_pool *pool;                               /* persistent workers (AVX order, threads != 1) */
};

static uint8_t *make_x4(const uint8_t *plain, size_t rows, size_t cols, int q) {
  size_t bb = q == ZO_Q4_0 ? 18 : 34;
  uint8_t *p = (uint8_t *)malloc(rows * (cols / 32) * bb);
  if (p) zo_interleave_x4(plain, p, rows, cols, q);
  return p;
}

zo_run *zo_run_create(const zo_qwen3 *m, uint32_t max_tokens, int order, int threads, int simd) {
  zo_run *r = (zo_run *)calloc(1, sizeof(zo_run));
  if (!r) return NULL;
  r->m = m;
  r->order = order;
  r->threads = threads;
  r->simd = simd;
  r->max_tokens = max_tokens;
  size_t H = m->hidden, F = m->ffn, qd = (size_t)m->n_q_heads * m->head_dim,
         kvd = (size_t)m->n_kv_heads * m->head_dim;
  r->kv = (float *)calloc((size_t)2 * m->n_layers * max_tokens * kvd, sizeof(float));
  r->inv_freqs = (float *)calloc(m->head_dim / 2, sizeof(float));
  r->hidden = calloc(H, 4); r->norm = calloc(H, 4); r->attn_out = calloc(H, 4);
  r->mlp_out = calloc(H, 4); r->q = calloc(qd, 4); r->k = calloc(kvd, 4); r->v = calloc(kvd, 4);
  r->qo = calloc(qd, 4); r->ko = calloc(kvd, 4);
  r->score = calloc((size_t)max_tokens * m->n_q_heads, 4);
  r->head = calloc(m->head_dim, 4); r->concat = calloc(qd, 4);
  r->gate = calloc(F, 4); r->up = calloc(F, 4); r->hmlp = calloc(F, 4);
  r->logits = calloc(m->vocab_padded, 4);
  r->attn_work = calloc((size_t)(m->n_q_heads + m->n_kv_heads + 1) * m->head_dim + max_tokens, 4);
  {
    size_t mx = H > F ? H : F;
    if (qd > mx) mx = qd;
    r->xq = (uint8_t *)calloc(mx / 32 * 34, 1);
  }
  zo_rope_ctx(m->rope_theta, m->head_dim / 2, r->inv_freqs);
  if (order == 1) {
    r->x4 = (uint8_t **)calloc((size_t)m->n_layers * 7, sizeof(uint8_t *));
    for (uint32_t l = 0; l < m->n_layers; ++l) {
      const zo_qwen3_layer *L = &m->layers[l];
      uint8_t **x = r->x4 + 7 * l;
      x[0] = make_x4(L->attn_q, qd, H, ZO_Q4_0);
      x[1] = make_x4(L->attn_k, kvd, H, ZO_Q4_0);
      x[2] = make_x4(L->attn_v, kvd, H, ZO_Q4_0);
      x[3] = make_x4(L->attn_o, H, qd, ZO_Q4_0);
      x[4] = make_x4(L->ffn_gate, F, H, ZO_Q4_0);
      x[5] = make_x4(L->ffn_up, F, H, ZO_Q4_0);
      x[6] = make_x4(L->ffn_down, H, F, ZO_Q4_0);
    }
    r->out_x4 = make_x4(m->output, m->vocab_padded, H, m->output_quant);
    if (threads != 1) r->pool = zo_pool_create(threads);
  }
  return r;
}

void zo_run_destroy(zo_run *r) {
  if (!r) return;
  zo_pool_destroy(r->pool);
  if (r->x4) {
    for (uint32_t i = 0; i < r->m->n_layers * 7; ++i) free(r->x4[i]);
    free(r->x4);
  }
  free(r->out_x4);
  free(r->kv); free(r->inv_freqs); free(r->hidden); free(r->norm); free(r->attn_out);
  free(r->mlp_out); free(r->q); free(r->k); free(r->v); free(r->qo); free(r->ko);
  free(r->score); free(r->head); free(r->concat); free(r->gate); free(r->up); free(r->hmlp);
  free(r->logits); free(r->attn_work); free(r->xq);
  free(r);
}

const float *zo_run_kv(const zo_run *r) { return r->kv; }

/* mode 1: the Q4_0 matmuls of the run take Q8_0-quantised inputs
 * (zo_quantize_row_q8_0, then zo_linear_q4_0_q8act), the arithmetic of the
 * prefill path, whose batched matmuls quantise their activations; mode 2:
 * the Q8_0 LM head too (zo_linear_q8_0_q8act), the batched decode path. */
void zo_run_set_q8act(zo_run *r, int on) { r->q8act = on; }

/* ----------------------------------------------------------------------
 * Fused dispatches of the AVX-512 step on the persistent workers.
 *   linear_fused_dispatch (inference_avx512.rs:890-945): several X4 tensors
 *     that read the same input (Q|K|V, gate|up) as one virtual row space of
 *     4-row groups, split once across the participants;
 *   lm_head_linear_argmax_dispatch (:1093-1118): the LM-head rows and, per
 *     participant, the first maximum of the rows it wrote, merged with the
 *     reference's rule (lm_argmax_propose, :1027-1044: the larger value
 *     wins, equal values go to the smaller index);
 *   attn_heads_kernel (:1459-1512): q heads split across the participants.
 * Every row and head is computed by the same code as the single-threaded
 * path, so the results are identical whatever the thread count.
 * ---------------------------------------------------------------------- */
typedef struct {
  const uint8_t *x4;
  float *out;
  size_t groups;
} zo_seg;

typedef struct {
  const float *x;
  size_t bpr;
  int quant, simd, argmax;
  int nseg;
  zo_seg seg[4];
  float best_v[ZO_POOL_MAX];
  size_t best_i[ZO_POOL_MAX];
} zo_fused_ctx;

static void fused_groups(void *p, size_t g0, size_t g1, int part) {
  zo_fused_ctx *c = (zo_fused_ctx *)p;
  const size_t gb = (c->quant == ZO_Q4_0 ? 72 : 136) * c->bpr;
  size_t base = 0;
  for (int s = 0; s < c->nseg; ++s) {
    const zo_seg *sg = &c->seg[s];
    size_t lo = g0 > base ? g0 : base, hi = g1 < base + sg->groups ? g1 : base + sg->groups;
    for (size_t g = lo; g < hi; ++g) {
      const size_t lg = g - base;
      const uint8_t *grp = sg->x4 + lg * gb;
      float *o = sg->out + 4 * lg;
#if defined(__x86_64__)
      if (c->simd) {
        if (c->quant == ZO_Q4_0) rows4_q4_avx512(c->x, c->bpr, grp, o);
        else rows4_q8_avx512(c->x, c->bpr, grp, o);
        continue;
      }
#endif
      for (int r = 0; r < 4; ++r)
        o[r] = c->quant == ZO_Q4_0 ? row_q4_emul(c->x, c->bpr, grp, 72, 2 * r, 8 + 16 * r)
                                   : row_q8_emul(c->x, c->bpr, grp, 136, 2 * r, 8 + 32 * r);
    }
    base += sg->groups;
  }
  if (c->argmax) {   /* first maximum of this participant's rows of segment 0 */
    const float *v = c->seg[0].out;
    float mx = -INFINITY;
    size_t idx = 4 * g0;
    for (size_t i = 4 * g0; i < 4 * g1; ++i)
      if (v[i] > mx) { mx = v[i]; idx = i; }
    c->best_v[part] = mx;
    c->best_i[part] = idx;
  }
}

static void fused_dispatch(zo_run *r, zo_fused_ctx *c) {
  size_t groups = 0;
  for (int s = 0; s < c->nseg; ++s) groups += c->seg[s].groups;
  c->simd = r->simd && zo_have_avx512();
  if (c->argmax)
    for (int i = 0; i < ZO_POOL_MAX; ++i) { c->best_v[i] = -INFINITY; c->best_i[i] = (size_t)-1; }
  zo_pool_run(r->pool, groups, fused_groups, c);
}

typedef struct {
  const float *qo, *k_block, *v_block;
  size_t total, max_tokens;
  uint32_t n_q, n_kv, hd;
  float *score, *out;
  int err[ZO_POOL_MAX];
} zo_heads_ctx;

static void heads_part(void *p, size_t h0, size_t h1, int part) {
  zo_heads_ctx *c = (zo_heads_ctx *)p;
  for (size_t h = h0; h < h1; ++h) {
    int st = attn_head(c->qo, c->k_block, c->v_block, h, c->total, c->n_q, c->n_kv, c->hd, 1,
                       c->score + h * c->max_tokens, c->out + h * c->hd);
    if (st && !c->err[part]) c->err[part] = st;
  }
}

static void lin(zo_run *r, const float *x, const uint8_t *plain, const uint8_t *x4, float *out,
                size_t in, size_t outd, int quant) {
  if (r->q8act && quant == ZO_Q4_0) {
    zo_quantize_row_q8_0(x, r->xq, in);
    zo_linear_q4_0_q8act(r->xq, plain, out, in, outd);
    return;
  }
  if (r->q8act == 2 && quant == ZO_Q8_0) {
    zo_quantize_row_q8_0(x, r->xq, in);
    zo_linear_q8_0_q8act(r->xq, plain, out, in, outd);
    return;
  }
  if (r->order == 0) {
    zo_linear_dispatch(x, plain, out, in, outd, quant);
  } else if (r->pool && outd % 4 == 0) {
    /* the persistent workers (linear_dispatch_avx512 through the SMP
     * dispatcher, inference_avx512.rs:1147) */
    zo_fused_ctx c = {.x = x, .bpr = in / 32, .quant = quant, .nseg = 1, .seg = {{x4, out, outd / 4}}};
    fused_dispatch(r, &c);
  } else if (quant == ZO_Q4_0) {
    zo_linear_q4_0x4_avx512(x, x4, out, in, outd, r->threads, r->simd);
  } else {
    zo_linear_q8_0x4_avx512(x, x4, out, in, outd, r->threads, r->simd);
  }
}

/* forward_pass.rs:515-631 (order 0) and inference_avx512.rs:1826-1987 with
 * gqa_attention_single_token_avx512 :1527-1810 and mlp_swiglu_avx512
 * :1280-1340 (order 1). */
static int run_forward(zo_run *r, uint32_t token, uint32_t pos, float *hidden_out);
static int run_lm_head(zo_run *r, uint32_t *token_out, float *logits_out);

int zo_run_forward(zo_run *r, uint32_t token, uint32_t pos, float *hidden_out) {
  zo_caller_pin cp;
  zo_caller_pin_begin(r->pool, &cp);
  int st = run_forward(r, token, pos, hidden_out);
  zo_caller_pin_end(&cp);
  return st;
}

int zo_run_lm_head(zo_run *r, uint32_t *token_out, float *logits_out) {
  zo_caller_pin cp;
  zo_caller_pin_begin(r->pool, &cp);
  int st = run_lm_head(r, token_out, logits_out);
  zo_caller_pin_end(&cp);
  return st;
}

static int run_forward(zo_run *r, uint32_t token, uint32_t pos, float *hidden_out) {
  const zo_qwen3 *m = r->m;
  size_t H = m->hidden, F = m->ffn, hd = m->head_dim;
  size_t nq = m->n_q_heads, nkv = m->n_kv_heads, qd = nq * hd, kvd = nkv * hd;
  if (pos >= r->max_tokens) return ZO_ERR_KV_TOKEN_OUT_OF_RANGE;
  if (token >= m->vocab_padded) return ZO_ERR_ARG;
  /* embed_lookup_dispatch (forward_pass.rs:311-370): dequantise one row. */
  {
    size_t bpr = H / 32;
    if (m->token_embd_quant == ZO_Q8_0) {
      for (size_t b = 0; b < bpr; ++b)
        zo_dequant_q8_0_block(m->token_embd + ((size_t)token * bpr + b) * 34, r->hidden + 32 * b);
    } else if (m->token_embd_quant == ZO_Q4_0) {
      for (size_t b = 0; b < bpr; ++b)
        zo_dequant_q4_0_block(m->token_embd + ((size_t)token * bpr + b) * 18, r->hidden + 32 * b);
    } else {
      return ZO_ERR_UNSUPPORTED_QUANT;
    }
  }
  size_t block = (size_t)r->max_tokens * kvd, layer_stride = 2 * block;

  for (uint32_t li = 0; li < m->n_layers; ++li) {
    const zo_qwen3_layer *L = &m->layers[li];
    uint8_t **x4 = r->order == 1 ? r->x4 + 7 * li : NULL;
    const int fused = r->pool && x4 && !r->q8act;
    zo_rmsnorm(r->hidden, L->attn_norm, r->norm, H, m->rms_eps);
    if (fused) {
      zo_fused_ctx c = {.x = r->norm, .bpr = H / 32, .quant = ZO_Q4_0, .nseg = 3,
                        .seg = {{x4[0], r->q, qd / 4}, {x4[1], r->k, kvd / 4}, {x4[2], r->v, kvd / 4}}};
      fused_dispatch(r, &c);
    } else {
      lin(r, r->norm, L->attn_q, x4 ? x4[0] : NULL, r->q, H, qd, ZO_Q4_0);
      lin(r, r->norm, L->attn_k, x4 ? x4[1] : NULL, r->k, H, kvd, ZO_Q4_0);
      lin(r, r->norm, L->attn_v, x4 ? x4[2] : NULL, r->v, H, kvd, ZO_Q4_0);
    }
    {
      float *kbase = r->kv + li * layer_stride;
      if (fused) {
        attn_prepare(r->q, r->k, r->v, L->q_norm, L->k_norm, r->inv_freqs, kbase, kbase + block, pos,
                     (uint32_t)nq, (uint32_t)nkv, (uint32_t)hd, m->rms_eps, 1, r->qo, r->ko);
        zo_heads_ctx hc = {.qo = r->qo, .k_block = kbase, .v_block = kbase + block, .total = (size_t)pos + 1,
                           .max_tokens = r->max_tokens, .n_q = (uint32_t)nq, .n_kv = (uint32_t)nkv,
                           .hd = (uint32_t)hd, .score = r->score, .out = r->concat};
        zo_pool_run(r->pool, nq, heads_part, &hc);
        for (int i = 0; i < ZO_POOL_MAX; ++i)
          if (hc.err[i]) return hc.err[i];
      } else {
        int st = zo_gqa_attention_decode(r->q, r->k, r->v, L->q_norm, L->k_norm, r->inv_freqs, kbase,
                                         kbase + block, pos, r->max_tokens, (uint32_t)nq, (uint32_t)nkv,
                                         (uint32_t)hd, m->rms_eps, r->order, r->attn_work, r->concat);
        if (st) return st;
      }
    }
    lin(r, r->concat, L->attn_o, x4 ? x4[3] : NULL, r->attn_out, qd, H, ZO_Q4_0);
    for (size_t i = 0; i < H; ++i) r->hidden[i] += r->attn_out[i];
    zo_rmsnorm(r->hidden, L->ffn_norm, r->norm, H, m->rms_eps);
    if (fused) {
      zo_fused_ctx c = {.x = r->norm, .bpr = H / 32, .quant = ZO_Q4_0, .nseg = 2,
                        .seg = {{x4[4], r->gate, F / 4}, {x4[5], r->up, F / 4}}};
      fused_dispatch(r, &c);
    } else {
      lin(r, r->norm, L->ffn_gate, x4 ? x4[4] : NULL, r->gate, H, F, ZO_Q4_0);
      lin(r, r->norm, L->ffn_up, x4 ? x4[5] : NULL, r->up, H, F, ZO_Q4_0);
    }
    if (r->order == 1) {
      zo_silu_mul_avx512(r->gate, r->up, r->hmlp, F);
    } else {
      /* forward_pass.rs:493-498: gate = gate / (1 + expf(-gate)); h = gate * up. */
      for (size_t i = 0; i < F; ++i) r->gate[i] = r->gate[i] / (1.0f + expf(-r->gate[i]));
      for (size_t i = 0; i < F; ++i) r->hmlp[i] = r->gate[i] * r->up[i];
    }
    lin(r, r->hmlp, L->ffn_down, x4 ? x4[6] : NULL, r->mlp_out, F, H, ZO_Q4_0);
    for (size_t i = 0; i < H; ++i) r->hidden[i] += r->mlp_out[i];
  }
  if (hidden_out) memcpy(hidden_out, r->hidden, H * 4);
  return ZO_OK;
}

/* lm_head.rs:98-166 (order 0) / inference_avx512.rs:1200-1270 (order 1):
 * final RMSNorm, logits over the padded vocab, first-max argmax, then the
 * non-finite and padding-region checks. */
static int run_lm_head(zo_run *r, uint32_t *token_out, float *logits_out) {
  const zo_qwen3 *m = r->m;
  size_t H = m->hidden, V = m->vocab_padded;
  zo_rmsnorm(r->hidden, m->output_norm, r->norm, H, m->rms_eps);
  float mx = -INFINITY;
  size_t idx = 0;
  if (r->pool && r->out_x4 && !r->q8act && V % 4 == 0) {
    zo_fused_ctx c = {.x = r->norm, .bpr = H / 32, .quant = m->output_quant, .argmax = 1, .nseg = 1,
                      .seg = {{r->out_x4, r->logits, V / 4}}};
    fused_dispatch(r, &c);
    mx = -INFINITY;
    idx = (size_t)-1;
    for (int i = 0; i < zo_pool_size(r->pool); ++i)
      if (c.best_v[i] > mx || (c.best_v[i] == mx && c.best_i[i] < idx)) { mx = c.best_v[i]; idx = c.best_i[i]; }
    if (idx == (size_t)-1) idx = 0;
  } else if (r->order == 1) {
    lin(r, r->norm, m->output, r->out_x4, r->logits, H, V, m->output_quant);
    idx = zo_argmax_avx512(r->logits, V, &mx);
  } else {
    lin(r, r->norm, m->output, r->out_x4, r->logits, H, V, m->output_quant);
    for (size_t i = 0; i < V; ++i) if (r->logits[i] > mx) { mx = r->logits[i]; idx = i; }
  }
  if (logits_out) memcpy(logits_out, r->logits, V * 4);
  if (!isfinite(mx)) return ZO_ERR_LM_NON_FINITE;
  if (idx >= m->vocab_real) return ZO_ERR_LM_PADDING;
  *token_out = (uint32_t)idx;
  return ZO_OK;
}

static float top2_gap(const float *v, size_t n) {
  float a = -INFINITY, b = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    if (v[i] > a) { b = a; a = v[i]; }
    else if (v[i] > b) b = v[i];
  }
  return a - b;
}

int zo_run_generate(zo_run *r, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen,
                    uint32_t *tokens_out, float *margins_out, float *logits_all) {
  int st;
  uint32_t tok = 0;
  size_t V = r->m->vocab_padded;
  for (uint32_t i = 0; i < n_prompt; ++i)
    if ((st = zo_run_forward(r, prompt[i], i, NULL))) return st;
  /* first generated token: LM head after the last prompt token */
  if ((st = zo_run_lm_head(r, &tok, logits_all))) return st;
  if (margins_out) margins_out[0] = top2_gap(r->logits, V);
  if (n_gen) tokens_out[0] = tok;
  for (uint32_t s = 1; s < n_gen; ++s) {
    if ((st = zo_run_forward(r, tok, n_prompt + s - 1, NULL))) return st;
    if ((st = zo_run_lm_head(r, &tok, logits_all ? logits_all + (size_t)s * V : NULL))) return st;
    if (margins_out) margins_out[s] = top2_gap(r->logits, V);
    tokens_out[s] = tok;
  }
  return ZO_OK;
}


/* ------------------------------------------------------------ sampler */
/* rng.rs:23-46 (Marsaglia xorshift64; a zero seed is replaced by
 * 0x853c49e6748fea9b in Rng::new, which the caller applies). */
uint32_t zo_rng_next_u32(uint64_t *state) {
  uint64_t x = *state;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *state = x;
  return (uint32_t)(x >> 32);
}

/* sampler.rs:123-163, operation by operation (every multiply and add
 * rounded on its own: the Makefile turns contraction off). */
float zo_exp_approx(float x) {
  if (x < -87.0f) x = -87.0f;
  else if (x > 88.0f) x = 88.0f;
  const float log2e = 1.44269504f;
  const float a = x * log2e;
  const int32_t ai = (a != a) ? 0 : (int32_t)a;   /* Rust `as i32`: truncation, NaN -> 0 */
  const float af = a - (float)ai;
  const float c1 = 0.69314718f, c2 = 0.2402265f, c3 = 0.0555041f;
  const float frac = 1.0f + af * (c1 + af * (c2 + af * c3));
  const uint32_t exp_bits = ((uint32_t)(127 + ai)) << 23;
  float pow2_int;
  memcpy(&pow2_int, &exp_bits, 4);
  return pow2_int * frac;
}

uint32_t zo_lm_head_sample(const float *logits, uint32_t len, uint64_t *rng_state, float temperature,
                           uint32_t vocab_real) {
  enum { K = 40 };
  const uint32_t vocab_len = len < vocab_real ? len : vocab_real;
  float top_vals[K];
  uint32_t top_idxs[K];
  for (int k = 0; k < K; ++k) {
    top_vals[k] = -INFINITY;
    top_idxs[k] = 0;
  }
  float min_val = -INFINITY;
  int min_pos = 0;
  for (uint32_t i = 0; i < vocab_len; ++i) {
    const float v = logits[i];
    if (v > min_val) {
      top_vals[min_pos] = v;
      top_idxs[min_pos] = i;
      min_val = INFINITY;
      for (int k = 0; k < K; ++k)
        if (top_vals[k] < min_val) {
          min_val = top_vals[k];
          min_pos = k;
        }
    }
  }
  const float inv_temp = 1.0f / temperature;
  for (int k = 0; k < K; ++k) top_vals[k] *= inv_temp;
  float max_logit = -INFINITY;
  for (int k = 0; k < K; ++k)
    if (top_vals[k] > max_logit) max_logit = top_vals[k];
  float exp_sum = 0.0f;
  for (int k = 0; k < K; ++k) {
    const float e = zo_exp_approx(top_vals[k] - max_logit);
    top_vals[k] = e;
    exp_sum += e;
  }
  const float inv_sum = 1.0f / exp_sum;
  for (int k = 0; k < K; ++k) top_vals[k] *= inv_sum;
  const float r = (float)zo_rng_next_u32(rng_state) / (float)UINT32_MAX;
  float cumulative = 0.0f;
  for (int k = 0; k < K; ++k) {
    cumulative += top_vals[k];
    if (r < cumulative) return top_idxs[k];
  }
  return top_idxs[K - 1];
}
