/*
 * zoracle_ds2.c — CPU parity oracle for the DeepSeek2 (MLA + MoE) decode
 * step of zero-llm-inference.
 *
 * TEST INFRASTRUCTURE ONLY (see zoracle.h).  Scalar crate order: every
 * multiply and add separately rounded (compiled with -ffp-contract=off),
 * sequential loops exactly as the Rust source writes them, libm
 * expf/sinf/cosf/powf/sqrtf through glibc.  Each function cites the
 * reference lines it restates.  A run can instead take the crate's AVX-512
 * kernel order (inference_avx512.rs:2141-2825), the path the reference
 * times: see ds2_ops below.
 */
#define _GNU_SOURCE
#include "zoracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* The two arithmetic orders of the DeepSeek2 step.  NULL / avx == 0: the
 * scalar crate path (mla.rs, moe.rs, forward_pass.rs:703-909).  avx == 1:
 * forward_single_token_deepseek2_avx512 (inference_avx512.rs:2611-2825),
 * which differs in exactly these places: every matmul is
 * linear_dispatch_avx512 (16-lane accumulators, rows split over the SMP
 * pool), mla_attention_avx512 (:2301-2577) scores each cached token as
 * dot_product_f32_avx512(q_nope, k_nope) + dot_product_f32_avx512(q_rope,
 * k_rope) and accumulates the context with weighted_add_f32_avx512,
 * moe_ffn_avx512 (:2195-2290) adds each routed expert with
 * weighted_add_f32_avx512, and the SwiGLU activations (expert_swiglu_avx512
 * :2141-2186, the dense FFN) run silu_mul_avx512.  RMSNorm, RoPE, softmax,
 * routing and the MHA layers stay scalar there too. */
typedef struct {
  int avx, simd;
  zo_pool *pool;
} ds2_ops;

static int ops_lin(const ds2_ops *o, const float *x, const uint8_t *w, float *out, size_t in_dim,
                   size_t out_dim, int quant) {
  if (o && o->avx) return zo_linear_plain_pool(o->pool, x, w, out, in_dim, out_dim, quant, o->simd);
  return zo_linear_dispatch(x, w, out, in_dim, out_dim, quant);
}

/* moe.rs:65-85 (normalised_expert_weight_scale / apply_expert_weight_scale):
 * a non-finite or non-positive scale means 1.0; a scale of exactly 1.0 is
 * not applied at all. */
static void apply_scale(float *w, size_t k, float scale) {
  float s = (isfinite(scale) && scale > 0.0f) ? scale : 1.0f;
  if (s != 1.0f)
    for (size_t i = 0; i < k; ++i) w[i] *= s;
}

static void uniform_fallback(float *w, size_t k, float scale) {
  float u = 1.0f / (float)k;
  for (size_t i = 0; i < k; ++i) w[i] = u;
  apply_scale(w, k, scale);
}

/* moe.rs:132-317 (moe_route_f32).
 *   scores: s_e = sequential unfused dot(hidden, row_e), + bias (Softmax mode)
 *           or sigmoid 1/(1+expf(-dot)) (SigmoidNormalize);
 *   selection key: the score, + bias in SigmoidNormalize mode;
 *   top-k: seed slots 0..k-1 with experts 0..k-1, then every later expert
 *          whose key is strictly greater than the current minimum replaces
 *          it (the minimum is the FIRST smallest slot, rescanned after each
 *          replacement); the slot order is the output order (not sorted);
 *   weights: the selected raw scores, then softmax over the k (max-trick,
 *          libm expf) or plain normalisation; a non-finite max, or a sum that
 *          is non-finite or <= 0, gives the uniform 1/k; finally the
 *          expert_weight_scale.
 * The reference panics on top_k == 0 or top_k > n_experts; the oracle
 * returns ZO_ERR_ARG. */
int zo_moe_route_f32(const float *hidden, size_t dim, const float *router_w,
                     const float *router_bias, size_t n_experts, size_t top_k, float *score_buf,
                     uint32_t *indices, float *weights, int mode, float expert_weight_scale) {
  if (top_k == 0 || top_k > n_experts) return ZO_ERR_ARG;
  int use_bias = router_bias != NULL;
  for (size_t e = 0; e < n_experts; ++e) {
    const float *row = router_w + e * dim;
    float dot = 0.0f;
    for (size_t i = 0; i < dim; ++i) dot += hidden[i] * row[i];
    if (mode == ZO_ROUTE_SOFTMAX)
      score_buf[e] = use_bias ? dot + router_bias[e] : dot;
    else
      score_buf[e] = 1.0f / (1.0f + expf(-dot));
  }
#define SEL_BIAS(e) ((use_bias && mode == ZO_ROUTE_SIGMOID_NORMALIZE) ? router_bias[(e)] : 0.0f)
  for (size_t i = 0; i < top_k; ++i) {
    indices[i] = (uint32_t)i;
    weights[i] = score_buf[i] + SEL_BIAS(i);
  }
  size_t min_idx = 0;
  float min_val = weights[0];
  for (size_t i = 1; i < top_k; ++i)
    if (weights[i] < min_val) { min_val = weights[i]; min_idx = i; }
  for (size_t e = top_k; e < n_experts; ++e) {
    float key = score_buf[e] + SEL_BIAS(e);
    if (key > min_val) {
      indices[min_idx] = (uint32_t)e;
      weights[min_idx] = key;
      min_val = weights[0];
      min_idx = 0;
      for (size_t i = 1; i < top_k; ++i)
        if (weights[i] < min_val) { min_val = weights[i]; min_idx = i; }
    }
  }
#undef SEL_BIAS
  for (size_t i = 0; i < top_k; ++i) weights[i] = score_buf[indices[i]];
  float mx = weights[0];
  for (size_t i = 1; i < top_k; ++i)
    if (weights[i] > mx) mx = weights[i];
  if (!isfinite(mx)) {
    uniform_fallback(weights, top_k, expert_weight_scale);
    return ZO_OK;
  }
  if (mode == ZO_ROUTE_SOFTMAX) {
    float sum = 0.0f;
    for (size_t i = 0; i < top_k; ++i) {
      weights[i] = expf(weights[i] - mx);
      sum += weights[i];
    }
    if (!isfinite(sum) || sum <= 0.0f) {
      uniform_fallback(weights, top_k, expert_weight_scale);
      return ZO_OK;
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < top_k; ++i) weights[i] *= inv;
  } else {
    float sum = 0.0f;
    for (size_t i = 0; i < top_k; ++i) sum += weights[i];
    if (!isfinite(sum) || sum <= 0.0f) {
      uniform_fallback(weights, top_k, expert_weight_scale);
      return ZO_OK;
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < top_k; ++i) weights[i] *= inv;
  }
  apply_scale(weights, top_k, expert_weight_scale);
  return ZO_OK;
}

/* moe.rs:345-397 (expert_swiglu): gate and up projections, silu(g) =
 * g / (1 + expf(-g)), h = silu * up, then the down projection.
 * work: 3 * inter floats. */
static int expert_swiglu_ops(const ds2_ops *o, const float *x, const uint8_t *gate_w,
                             const uint8_t *up_w, const uint8_t *down_w, size_t dim, size_t inter,
                             int quant, float *work, float *out) {
  float *g = work, *u = work + inter, *h = work + 2 * inter;
  int st;
  if ((st = ops_lin(o, x, gate_w, g, dim, inter, quant))) return st;
  if ((st = ops_lin(o, x, up_w, u, dim, inter, quant))) return st;
  if (o && o->avx) {
    zo_silu_mul_avx512(g, u, h, inter);
  } else {
    for (size_t i = 0; i < inter; ++i) {
      float silu = g[i] / (1.0f + expf(-g[i]));
      h[i] = silu * u[i];
    }
  }
  return ops_lin(o, h, down_w, out, inter, dim, quant);
}

int zo_expert_swiglu(const float *x, const uint8_t *gate_w, const uint8_t *up_w,
                     const uint8_t *down_w, size_t dim, size_t inter, int quant, float *work,
                     float *out) {
  return expert_swiglu_ops(NULL, x, gate_w, up_w, down_w, dim, inter, quant, work, out);
}

static size_t quant_row_bytes(size_t cols, int quant) {
  return quant == ZO_Q4_0 ? cols / 32 * 18 : cols / 32 * 34;
}

/* moe.rs:486-590 (moe_ffn): route, then the shared expert written straight
 * into `out`, then for k in selection order out[i] += w_k * expert_k(x)[i]
 * (multiply, then add).  Experts are slices of the stacked rank-3 tensors
 * (moe.rs:427-466 expert_quant_bytes / slice_expert_weight).
 *
 * n_shared > 1 extends the reference, whose moe_ffn runs exactly one shared
 * expert of width `inter`: shared expert 0 is written into `out` as there,
 * each further one (a slice of the stacked shared tensors, like the routed
 * ones) is computed into the expert buffer and added (out[i] += s[i]) before
 * the routed experts.  A shared FFN of width n_shared * inter is the sum of
 * n_shared SwiGLUs of width inter, so this is DeepSeek-V2-Lite's "2 shared
 * experts".  n_shared == 0 starts from out = 0.
 * work: n_experts + 3 * inter + dim floats. */
static int moe_ffn_ops(const ds2_ops *o, const float *x, const float *router_w,
                       const float *router_bias, const uint8_t *gate_exps, const uint8_t *up_exps,
                       const uint8_t *down_exps, const uint8_t *gate_sh, const uint8_t *up_sh,
                       const uint8_t *down_sh, size_t n_shared, size_t n_experts, size_t top_k,
                       size_t dim, size_t inter, int quant, int mode, float expert_weight_scale,
                       float *work, uint32_t *ids_out, float *weights_out, float *out) {
  if (top_k == 0 || top_k > n_experts) return ZO_ERR_ARG;
  if (quant != ZO_Q4_0 && quant != ZO_Q8_0) return ZO_ERR_UNSUPPORTED_QUANT;
  float *scores = work, *sw = work + n_experts, *eo = sw + 3 * inter;
  int st = zo_moe_route_f32(x, dim, router_w, router_bias, n_experts, top_k, scores, ids_out,
                            weights_out, mode, expert_weight_scale);
  if (st) return st;
  size_t gu_bytes = quant_row_bytes(dim, quant) * inter;     /* one expert's gate (or up) */
  size_t dn_bytes = quant_row_bytes(inter, quant) * dim;     /* one expert's down */
  if (n_shared == 0) memset(out, 0, dim * sizeof(float));
  for (size_t s = 0; s < n_shared; ++s) {
    float *dst = s == 0 ? out : eo;
    if ((st = expert_swiglu_ops(o, x, gate_sh + s * gu_bytes, up_sh + s * gu_bytes,
                                down_sh + s * dn_bytes, dim, inter, quant, sw, dst)))
      return st;
    if (s > 0)
      for (size_t i = 0; i < dim; ++i) out[i] += eo[i];
  }
  for (size_t k = 0; k < top_k; ++k) {
    size_t e = ids_out[k];
    float w = weights_out[k];
    if ((st = expert_swiglu_ops(o, x, gate_exps + e * gu_bytes, up_exps + e * gu_bytes,
                                down_exps + e * dn_bytes, dim, inter, quant, sw, eo)))
      return st;
    if (o && o->avx)
      zo_weighted_add_avx512(w, eo, out, dim);
    else
      for (size_t i = 0; i < dim; ++i) out[i] += w * eo[i];
  }
  return ZO_OK;
}

int zo_moe_ffn(const float *x, const float *router_w, const float *router_bias,
               const uint8_t *gate_exps, const uint8_t *up_exps, const uint8_t *down_exps,
               const uint8_t *gate_sh, const uint8_t *up_sh, const uint8_t *down_sh,
               size_t n_shared, size_t n_experts, size_t top_k, size_t dim, size_t inter,
               int quant, int mode, float expert_weight_scale, float *work, uint32_t *ids_out,
               float *weights_out, float *out) {
  return moe_ffn_ops(NULL, x, router_w, router_bias, gate_exps, up_exps, down_exps, gate_sh, up_sh,
                     down_sh, n_shared, n_experts, top_k, dim, inter, quant, mode,
                     expert_weight_scale, work, ids_out, weights_out, out);
}

/* mla.rs:169-171 / :199-213: NeoX half-split rotation of one rope slice,
 * inv-freq recomputed per pair with powf(base, -2 i / rope_dim) and the
 * angle pos * freq through libm cosf/sinf. */
static void mla_rope(float *v, size_t rope_dim, uint32_t pos, float base) {
  size_t half = rope_dim / 2;
  for (size_t i = 0; i < half; ++i) {
    float freq = powf(base, -2.0f * (float)i / (float)rope_dim);
    float theta = (float)pos * freq;
    float c = cosf(theta), s = sinf(theta);
    float x0 = v[i], x1 = v[i + half];
    v[i] = x0 * c - x1 * s;
    v[i + half] = x0 * s + x1 * c;
  }
}

size_t zo_mla_work_floats(const zo_mla_dims *d, uint32_t max_tokens) {
  size_t kv_a = d->kv_lora_rank + d->rope_dim;
  size_t kvb = (size_t)d->n_heads * (d->nope_dim + d->v_dim);
  size_t qd = (size_t)d->n_heads * (d->nope_dim + d->rope_dim);
  return kv_a + d->kv_lora_rank + kvb + 2 * (size_t)d->q_lora_rank + qd +
         (size_t)d->n_heads * max_tokens + (size_t)d->n_heads * d->v_dim;
}

/* mla.rs:122-414 (mla_attention_single_token), compressed-latent cache
 * (kv_cache.rs:257-407: per layer [max_tokens][kv_lora_rank | rope_dim]):
 *   kv_a = W_kv_a_mqa . x;  c_kv = rmsnorm(kv_a[:r], kv_a_norm);
 *   k_rope = kv_a[r:]: optional RMS norm with k_norm (sqrtf(ssq/n + eps),
 *            1/rms, x * inv * w), then RoPE at `pos`; store [c_kv | k_rope];
 *   q = W_q_b . rmsnorm(W_q_a . x, q_a_norm); RoPE on each head's rope part;
 *   for every cached token t: re-expand kv_b . c_kv_t, score_h,t =
 *            (sum q_nope.k_nope, continued over q_rope.k_rope_t) * scale,
 *            scale = 1/sqrtf(nope + rope);
 *   softmax per head (attention.rs:48, NumericalInstability on failure);
 *   second pass: re-expand again, concat_h += p_h,t * v_h,t;
 *   out = W_o . concat.
 * With w->k_b and w->v_b both set, the split projections are used instead
 * of kv_b (mla.rs:251-275).  cache_layer is this layer's slice of the
 * cache; work: zo_mla_work_floats floats. */
static int mla_attention_ops(const ds2_ops *o, const float *x, const zo_mla_weights *w,
                             const zo_mla_dims *d, float *cache_layer, uint32_t pos,
                             uint32_t max_tokens, float *work, float *out) {
  const size_t H = d->hidden, R = d->kv_lora_rank, RD = d->rope_dim, NH = d->n_heads;
  const size_t NO = d->nope_dim, VD = d->v_dim, QL = d->q_lora_rank;
  const size_t kv_a_out = R + RD, nv = NO + VD, tk = NO + RD;
  const size_t kvb_out = NH * nv, qb_out = NH * tk, kn_out = NH * NO, v_out = NH * VD;
  const int quant = d->quant;
  const int split = w->k_b && w->v_b;
  if (pos >= max_tokens) return ZO_ERR_KV_TOKEN_OUT_OF_RANGE;
  float *kv_a = work, *c_kv = kv_a + kv_a_out, *kvd = c_kv + R, *c_q = kvd + kvb_out,
        *c_qn = c_q + QL, *q = c_qn + QL, *score = q + qb_out, *concat = score + NH * max_tokens;
  const size_t tstride = R + RD, total = (size_t)pos + 1;
  int st;
  if ((st = ops_lin(o, x, w->kv_a_mqa, kv_a, H, kv_a_out, quant))) return st;
  zo_rmsnorm(kv_a, w->kv_a_norm, c_kv, R, d->eps);
  {
    float *kr = kv_a + R;
    if (w->k_norm) {
      float ssq = 0.0f;
      for (size_t i = 0; i < RD; ++i) ssq += kr[i] * kr[i];
      float rms = sqrtf(ssq / (float)RD + d->eps);
      float inv = 1.0f / rms;
      for (size_t i = 0; i < RD; ++i) kr[i] = kr[i] * inv * w->k_norm[i];
    }
    mla_rope(kr, RD, pos, d->rope_base);
  }
  memcpy(cache_layer + (size_t)pos * tstride, c_kv, R * sizeof(float));
  memcpy(cache_layer + (size_t)pos * tstride + R, kv_a + R, RD * sizeof(float));
  if ((st = ops_lin(o, x, w->q_a, c_q, H, QL, quant))) return st;
  zo_rmsnorm(c_q, w->q_a_norm, c_qn, QL, d->eps);
  if ((st = ops_lin(o, c_qn, w->q_b, q, QL, qb_out, quant))) return st;
  for (size_t h = 0; h < NH; ++h) mla_rope(q + h * tk + NO, RD, pos, d->rope_base);
  const float scale = 1.0f / sqrtf((float)tk);
  for (size_t t = 0; t < total; ++t) {
    const float *ct = cache_layer + t * tstride, *krt = ct + R;
    if (split) {
      if ((st = ops_lin(o, ct, w->k_b, kvd, R, kn_out, quant))) return st;
      if ((st = ops_lin(o, ct, w->v_b, kvd + kn_out, R, v_out, quant))) return st;
    } else if ((st = ops_lin(o, ct, w->kv_b, kvd, R, kvb_out, quant))) {
      return st;
    }
    for (size_t h = 0; h < NH; ++h) {
      const float *qn = q + h * tk, *qr = qn + NO;
      const float *kn = split ? kvd + h * NO : kvd + h * nv;
      float dot;
      if (o && o->avx) {
        dot = zo_dot_product_avx512(qn, kn, NO) + zo_dot_product_avx512(qr, krt, RD);
      } else {
        dot = 0.0f;
        for (size_t i = 0; i < NO; ++i) dot += qn[i] * kn[i];
        for (size_t i = 0; i < RD; ++i) dot += qr[i] * krt[i];
      }
      score[h * max_tokens + t] = dot * scale;
    }
  }
  for (size_t h = 0; h < NH; ++h)
    if (zo_softmax(score + h * max_tokens, total)) return ZO_ERR_NUMERICAL_INSTABILITY;
  memset(concat, 0, v_out * sizeof(float));
  for (size_t t = 0; t < total; ++t) {
    const float *ct = cache_layer + t * tstride;
    if (split) {
      if ((st = ops_lin(o, ct, w->k_b, kvd, R, kn_out, quant))) return st;
      if ((st = ops_lin(o, ct, w->v_b, kvd + kn_out, R, v_out, quant))) return st;
    } else if ((st = ops_lin(o, ct, w->kv_b, kvd, R, kvb_out, quant))) {
      return st;
    }
    for (size_t h = 0; h < NH; ++h) {
      const float *vh = split ? kvd + kn_out + h * VD : kvd + h * nv + NO;
      float p = score[h * max_tokens + t];
      if (o && o->avx)
        zo_weighted_add_avx512(p, vh, concat + h * VD, VD);
      else
        for (size_t i = 0; i < VD; ++i) concat[h * VD + i] += p * vh[i];
    }
  }
  return ops_lin(o, concat, w->output, out, v_out, H, quant);
}

int zo_mla_attention(const float *x, const zo_mla_weights *w, const zo_mla_dims *d,
                     float *cache_layer, uint32_t pos, uint32_t max_tokens, float *work,
                     float *out) {
  return mla_attention_ops(NULL, x, w, d, cache_layer, pos, max_tokens, work, out);
}

size_t zo_mha_work_floats(const zo_mla_dims *d, uint32_t n_kv, uint32_t max_tokens) {
  size_t hq = d->nope_dim + d->rope_dim;
  return (size_t)d->n_heads * hq + (size_t)n_kv * hq + (size_t)n_kv * d->v_dim +
         (size_t)d->n_heads * max_tokens + (size_t)d->n_heads * d->v_dim;
}

/* mla.rs:449-618 (mha_attention_single_token):
 *   q = W_q . x, k = W_k . x, v = W_v . x (head width nope + rope for q / k);
 *   RoPE (mla_rope above) on the rope part of every q head and k head;
 *   store k, v at pos (MhaKvCache::store_kv, kv_cache.rs:487-531);
 *   per q head h (kv head h / (n_heads / n_kv)): scores over [0, pos] as the
 *   sequential dot q . k_t times 1 / sqrtf(nope + rope), softmax
 *   (attention.rs:48), concat_h = sum_t p_t v_t in token order;
 *   out = W_o . concat. */
int zo_mha_attention(const float *x, const uint8_t *wq, const uint8_t *wk, const uint8_t *wv,
                     const uint8_t *wo, const zo_mla_dims *d, uint32_t n_kv, float *k_cache,
                     float *v_cache, uint32_t pos, uint32_t max_tokens, float *work, float *out) {
  const size_t H = d->hidden, NH = d->n_heads, NO = d->nope_dim, RD = d->rope_dim, VD = d->v_dim;
  const size_t hq = NO + RD, q_out = NH * hq, k_out = (size_t)n_kv * hq, v_out = (size_t)n_kv * VD;
  const size_t total = (size_t)pos + 1, G = n_kv ? NH / n_kv : 1;
  const int quant = d->quant;
  int st;
  if (pos >= max_tokens) return ZO_ERR_KV_TOKEN_OUT_OF_RANGE;
  float *q = work, *k = q + q_out, *v = k + k_out, *score = v + v_out, *concat = score + NH * max_tokens;
  if ((st = zo_linear_dispatch(x, wq, q, H, q_out, quant))) return st;
  if ((st = zo_linear_dispatch(x, wk, k, H, k_out, quant))) return st;
  if ((st = zo_linear_dispatch(x, wv, v, H, v_out, quant))) return st;
  for (size_t h = 0; h < NH; ++h) mla_rope(q + h * hq + NO, RD, pos, d->rope_base);
  for (size_t h = 0; h < n_kv; ++h) mla_rope(k + h * hq + NO, RD, pos, d->rope_base);
  memcpy(k_cache + (size_t)pos * k_out, k, k_out * sizeof(float));
  memcpy(v_cache + (size_t)pos * v_out, v, v_out * sizeof(float));
  const float scale = 1.0f / sqrtf((float)hq);
  for (size_t qh = 0; qh < NH; ++qh) {
    const size_t kvh = G ? qh / G : 0;
    const float *qv = q + qh * hq;
    float *sc = score + qh * max_tokens;
    for (size_t t = 0; t < total; ++t) {
      const float *kt = k_cache + t * k_out + kvh * hq;
      float dot = 0.0f;
      for (size_t i = 0; i < hq; ++i) dot += qv[i] * kt[i];
      sc[t] = dot * scale;
    }
    if (zo_softmax(sc, total)) return ZO_ERR_NUMERICAL_INSTABILITY;
    float *o = concat + qh * VD;
    memset(o, 0, VD * sizeof(float));
    for (size_t t = 0; t < total; ++t) {
      const float *vt = v_cache + t * v_out + kvh * VD;
      const float w = sc[t];
      for (size_t i = 0; i < VD; ++i) o[i] += w * vt[i];
    }
  }
  return zo_linear_dispatch(concat, wo, out, NH * VD, H, quant);
}

/* ======================================================================
 * DeepSeek2 decode step (forward_pass.rs:703-909) + LM head (lm_head.rs:98)
 * ====================================================================== */

struct zo_ds2_run {
  const zo_ds2 *m;
  uint32_t max_tokens;
  float *cache;          /* [L][max_tokens][kv_lora | rope] */
  float *hidden, *norm, *attn_out, *mlp_out, *logits;
  float *mla_work, *ffn_work;
  float *mha_cache;      /* per MHA layer: K block [max_tokens][n_kv*hq] | V block [max_tokens][n_kv*v] */
  float *mha_work;
  uint32_t n_kv;
  size_t mha_k_block, mha_v_block;
  uint32_t *ids;         /* [L][top_k] experts of the last forward (0 for dense layers) */
  float *wts;            /* [L][top_k] */
  ds2_ops ops;           /* arithmetic order (and the AVX-512 order's pool) */
};

zo_ds2_run *zo_ds2_run_create_order(const zo_ds2 *m, uint32_t max_tokens, int order, int threads,
                                    int simd) {
  zo_ds2_run *r = (zo_ds2_run *)calloc(1, sizeof(zo_ds2_run));
  if (!r) return NULL;
  r->m = m;
  r->max_tokens = max_tokens;
  r->ops.avx = order == 1;
  r->ops.simd = simd;
  if (r->ops.avx) {
    r->ops.pool = zo_pool_create(threads);
    if (!r->ops.pool) {
      free(r);
      return NULL;
    }
  }
  const zo_mla_dims *d = &m->mla;
  size_t H = d->hidden;
  size_t inter = m->ffn > m->expert_ffn ? m->ffn : m->expert_ffn;
  r->cache = (float *)calloc((size_t)m->n_layers * max_tokens * (d->kv_lora_rank + d->rope_dim), 4);
  r->hidden = calloc(H, 4);
  r->norm = calloc(H, 4);
  r->attn_out = calloc(H, 4);
  r->mlp_out = calloc(H, 4);
  r->logits = calloc(m->vocab_padded, 4);
  r->mla_work = calloc(zo_mla_work_floats(d, max_tokens), 4);
  r->ffn_work = calloc(m->n_experts + 3 * inter + H, 4);
  r->ids = calloc((size_t)m->n_layers * (m->top_k ? m->top_k : 1), 4);
  r->wts = calloc((size_t)m->n_layers * (m->top_k ? m->top_k : 1), 4);
  {
    size_t n_mha = 0;
    for (uint32_t li = 0; li < m->n_layers; ++li) n_mha += m->layers[li].mha ? 1 : 0;
    r->n_kv = m->n_kv_heads ? m->n_kv_heads : d->n_heads;
    r->mha_k_block = (size_t)max_tokens * r->n_kv * (d->nope_dim + d->rope_dim);
    r->mha_v_block = (size_t)max_tokens * r->n_kv * d->v_dim;
    r->mha_cache = calloc(n_mha ? n_mha * (r->mha_k_block + r->mha_v_block) : 1, 4);
    r->mha_work = calloc(zo_mha_work_floats(d, r->n_kv, max_tokens), 4);
  }
  if (!r->cache || !r->hidden || !r->norm || !r->attn_out || !r->mlp_out || !r->logits ||
      !r->mla_work || !r->ffn_work || !r->ids || !r->wts || !r->mha_cache || !r->mha_work) {
    zo_ds2_run_destroy(r);
    return NULL;
  }
  return r;
}

zo_ds2_run *zo_ds2_run_create(const zo_ds2 *m, uint32_t max_tokens) {
  return zo_ds2_run_create_order(m, max_tokens, 0, 1, 0);
}

void zo_ds2_run_destroy(zo_ds2_run *r) {
  if (!r) return;
  free(r->cache); free(r->hidden); free(r->norm); free(r->attn_out); free(r->mlp_out);
  free(r->logits); free(r->mla_work); free(r->ffn_work); free(r->ids); free(r->wts);
  free(r->mha_cache); free(r->mha_work);
  zo_pool_destroy(r->ops.pool);
  free(r);
}

int zo_ds2_run_threads(const zo_ds2_run *r) { return r->ops.avx ? zo_pool_size(r->ops.pool) : 1; }

/* Overwrite cached latent rows [t0, t0 + n) of one MLA layer with `rows`
 * ([n][kv_lora | rope]): a cache at a given context without decoding every
 * token first (what a step costs depends on the context, not the values). */
int zo_ds2_run_set_cache_rows(zo_ds2_run *r, uint32_t layer, uint32_t t0, uint32_t n, const float *rows) {
  const zo_mla_dims *d = &r->m->mla;
  const size_t ts = d->kv_lora_rank + d->rope_dim;
  if (layer >= r->m->n_layers || (uint64_t)t0 + n > r->max_tokens) return ZO_ERR_ARG;
  memcpy(r->cache + ((size_t)layer * r->max_tokens + t0) * ts, rows, (size_t)n * ts * sizeof(float));
  return ZO_OK;
}

const float *zo_ds2_run_cache(const zo_ds2_run *r) { return r->cache; }
const float *zo_ds2_run_mha_cache(const zo_ds2_run *r) { return r->mha_cache; }
const uint32_t *zo_ds2_run_expert_ids(const zo_ds2_run *r) { return r->ids; }
const float *zo_ds2_run_expert_weights(const zo_ds2_run *r) { return r->wts; }

/* forward_pass.rs:703-909 (forward_single_token_deepseek2): embed, then per
 * layer rmsnorm -> MLA -> hidden += attn_out -> rmsnorm -> dense SwiGLU
 * (forward_pass.rs:459-508) or moe_ffn over a zeroed mlp_out -> hidden +=
 * mlp_out.  A layer flagged mha runs mha_attention_single_token on its slot
 * of the MHA cache (the n-th MHA layer takes slot n, as mha_layer_idx). */
int zo_ds2_run_forward(zo_ds2_run *r, uint32_t token, uint32_t pos, float *hidden_out) {
  const zo_ds2 *m = r->m;
  const zo_mla_dims *d = &m->mla;
  size_t H = d->hidden, F = m->ffn, tstride = d->kv_lora_rank + d->rope_dim;
  if (pos >= r->max_tokens) return ZO_ERR_KV_TOKEN_OUT_OF_RANGE;
  if (token >= m->vocab_padded) return ZO_ERR_ARG;
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
  int st;
  size_t mha_slot = 0;
  for (uint32_t li = 0; li < m->n_layers; ++li) {
    const zo_ds2_layer *L = &m->layers[li];
    zo_rmsnorm(r->hidden, L->attn_norm, r->norm, H, d->eps);
    if (L->mha) {
      float *kc = r->mha_cache + mha_slot * (r->mha_k_block + r->mha_v_block), *vc = kc + r->mha_k_block;
      ++mha_slot;
      if ((st = zo_mha_attention(r->norm, L->q_mha, L->k_mha, L->v_mha, L->mla.output, d, r->n_kv, kc, vc,
                                 pos, r->max_tokens, r->mha_work, r->attn_out)))
        return st;
    } else {
      float *cl = r->cache + (size_t)li * r->max_tokens * tstride;
      if ((st = mla_attention_ops(&r->ops, r->norm, &L->mla, d, cl, pos, r->max_tokens, r->mla_work,
                                  r->attn_out)))
        return st;
    }
    for (size_t i = 0; i < H; ++i) r->hidden[i] += r->attn_out[i];
    zo_rmsnorm(r->hidden, L->ffn_norm, r->norm, H, d->eps);
    if (!L->moe) {
      float *g = r->ffn_work, *u = g + F, *h = u + F;
      /* mlp_swiglu_dispatch needs 3 * ffn floats: ffn_work holds
       * n_experts + 3 * max(ffn, expert_ffn) + H */
      if ((st = ops_lin(&r->ops, r->norm, L->ffn_gate, g, H, F, d->quant))) return st;
      if ((st = ops_lin(&r->ops, r->norm, L->ffn_up, u, H, F, d->quant))) return st;
      if (r->ops.avx) {
        zo_silu_mul_avx512(g, u, h, F);
      } else {
        for (size_t i = 0; i < F; ++i) g[i] = g[i] / (1.0f + expf(-g[i]));
        for (size_t i = 0; i < F; ++i) h[i] = g[i] * u[i];
      }
      if ((st = ops_lin(&r->ops, h, L->ffn_down, r->mlp_out, F, H, d->quant))) return st;
      for (size_t k = 0; k < m->top_k; ++k) {
        r->ids[(size_t)li * m->top_k + k] = 0;
        r->wts[(size_t)li * m->top_k + k] = 0.0f;
      }
    } else {
      memset(r->mlp_out, 0, H * sizeof(float));
      if ((st = moe_ffn_ops(&r->ops, r->norm, L->router_w, L->router_b, L->gate_exps, L->up_exps,
                            L->down_exps, L->gate_shexp, L->up_shexp, L->down_shexp, m->n_shared,
                            m->n_experts, m->top_k, H, m->expert_ffn, d->quant, m->route_mode,
                            m->expert_weight_scale, r->ffn_work, r->ids + (size_t)li * m->top_k,
                            r->wts + (size_t)li * m->top_k, r->mlp_out)))
        return st;
    }
    for (size_t i = 0; i < H; ++i) r->hidden[i] += r->mlp_out[i];
  }
  if (hidden_out) memcpy(hidden_out, r->hidden, H * 4);
  return ZO_OK;
}

/* lm_head.rs:98-166 (lm_head_argmax_dynamic), as zo_run_lm_head. */
int zo_ds2_run_lm_head(zo_ds2_run *r, uint32_t *token_out, float *logits_out) {
  const zo_ds2 *m = r->m;
  size_t H = m->mla.hidden, V = m->vocab_padded;
  zo_rmsnorm(r->hidden, m->output_norm, r->norm, H, m->mla.eps);
  int st = ops_lin(&r->ops, r->norm, m->output, r->logits, H, V, m->output_quant);
  if (st) return st;
  float mx = -INFINITY;
  size_t idx = 0;
  for (size_t i = 0; i < V; ++i)
    if (r->logits[i] > mx) { mx = r->logits[i]; idx = i; }
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

int zo_ds2_run_generate(zo_ds2_run *r, const uint32_t *prompt, uint32_t n_prompt, uint32_t n_gen,
                        uint32_t *tokens_out, float *margins_out, float *logits_all) {
  int st;
  uint32_t tok = 0;
  size_t V = r->m->vocab_padded;
  for (uint32_t i = 0; i < n_prompt; ++i)
    if ((st = zo_ds2_run_forward(r, prompt[i], i, NULL))) return st;
  if ((st = zo_ds2_run_lm_head(r, &tok, logits_all))) return st;
  if (margins_out) margins_out[0] = top2_gap(r->logits, V);
  if (n_gen) tokens_out[0] = tok;
  for (uint32_t s = 1; s < n_gen; ++s) {
    if ((st = zo_ds2_run_forward(r, tok, n_prompt + s - 1, NULL))) return st;
    if ((st = zo_ds2_run_lm_head(r, &tok, logits_all ? logits_all + (size_t)s * V : NULL))) return st;
    if (margins_out) margins_out[s] = top2_gap(r->logits, V);
    tokens_out[s] = tok;
  }
  return ZO_OK;
}
