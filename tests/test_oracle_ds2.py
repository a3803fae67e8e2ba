"""CPU oracle of the DeepSeek2 (MLA + MoE) rows, pinned before it is trusted.

Routing is pinned by the reference's own contract tests
(crates/zero-llm-inference/tests/deepseek2_moe_pipeline.rs:405-723, same
inputs and assertions) and, bit for bit, by a pure-Python float32 restatement
of moe.rs:132-317.  expert_swiglu / moe_ffn / mla_attention_single_token have
no value-level golden vectors in the reference (its pipeline test uses Q4_K
weights and only checks finiteness and determinism), so they are pinned
against an independent float64 numpy restatement of the same mathematics.
"""
import numpy as np
import pytest

import oracle as O
from zero_b200 import synth

# ---------------------------------------------------------------- helpers


def deq_q4_0(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Plain Q4_0 blocks -> float64 [rows, cols] (dequant.rs:186-232)."""
    b = blocks.reshape(rows, cols // 32, 18)
    d = b[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    qs = b[:, :, 2:]
    lo = (qs & 15).astype(np.int32) - 8
    hi = (qs >> 4).astype(np.int32) - 8
    return (np.concatenate([lo, hi], axis=2) * d[..., None]).reshape(rows, cols)


def rms64(x, w, eps):
    x = x.astype(np.float64)
    return x / np.sqrt(np.mean(x * x) + eps) * w


def rope64(v, pos, base):
    v = v.astype(np.float64).copy()
    half = v.size // 2
    i = np.arange(half)
    theta = pos * base ** (-2.0 * i / v.size)
    x0, x1 = v[:half].copy(), v[half:].copy()
    v[:half] = x0 * np.cos(theta) - x1 * np.sin(theta)
    v[half:] = x0 * np.sin(theta) + x1 * np.cos(theta)
    return v


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


# ------------------------------------------- routing: the reference's contract tests

HIDDEN, N_EXPERTS, TOP_K = 256, 4, 2


def skewed_router():
    # deepseek2_moe_pipeline.rs:178-190: expert 0 cold, expert 3 hot
    e = np.arange(N_EXPERTS, dtype=np.float32)[:, None]
    i = np.arange(HIDDEN)[None, :]
    return (np.float32(0.001) * e + np.float32(0.0001) * (i % 8).astype(np.float32)).astype(np.float32).ravel()


def ramp_hidden():
    return (np.float32(0.1) + np.float32(0.01) * np.arange(HIDDEN, dtype=np.float32)).astype(np.float32)


def test_route_skewed_router_picks_hot_experts():
    rc, ids, w, _ = O.moe_route_f32(ramp_hidden(), skewed_router(), N_EXPERTS, TOP_K, O.ROUTE_SOFTMAX, 1.0)
    assert rc == 0
    assert {2, 3} <= set(ids.tolist())
    assert abs(float(w.sum()) - 1.0) < 1e-5


def test_route_top_k_preconditions():
    h = np.full(HIDDEN, 0.5, np.float32)
    r = np.zeros(N_EXPERTS * HIDDEN, np.float32)
    assert O.moe_route_f32(h, r, N_EXPERTS, 0)[0] == 1          # top_k must be > 0
    assert O.moe_route_f32(h, r, N_EXPERTS, N_EXPERTS + 1)[0] == 1   # top_k must be <= n_experts


def test_route_nan_router_falls_back_to_uniform():
    h = np.ones(HIDDEN, np.float32)
    r = np.zeros(N_EXPERTS * HIDDEN, np.float32)
    r[0] = np.nan
    rc, ids, w, _ = O.moe_route_f32(h, r, N_EXPERTS, TOP_K)
    assert rc == 0
    assert np.all(np.isfinite(w)) and abs(float(w.sum()) - 1.0) < 1e-6
    assert np.all(np.abs(w - 1.0 / TOP_K) < 1e-6)


def test_route_identical_scores_uniform_softmax():
    rc, ids, w, _ = O.moe_route_f32(np.ones(HIDDEN, np.float32), np.zeros(N_EXPERTS * HIDDEN, np.float32),
                                    N_EXPERTS, TOP_K)
    assert rc == 0 and np.all(np.abs(w - 1.0 / TOP_K) < 1e-6)
    assert ids.tolist() == [0, 1]    # nothing beats the seeded slots under a strict `>`


def test_route_sigmoid_normalize_sums_to_one():
    rc, _, w, _ = O.moe_route_f32(ramp_hidden(), skewed_router(), N_EXPERTS, TOP_K, O.ROUTE_SIGMOID_NORMALIZE)
    assert rc == 0 and abs(float(w.sum()) - 1.0) < 1e-5
    assert np.all((w > 0) & (w < 1))


def test_route_sigmoid_normalize_applies_scale():
    rc, _, w, _ = O.moe_route_f32(ramp_hidden(), skewed_router(), N_EXPERTS, TOP_K, O.ROUTE_SIGMOID_NORMALIZE,
                                  2.5)
    assert rc == 0 and abs(float(w.sum()) - 2.5) < 1e-5


def test_route_uniform_fallback_preserves_scale():
    r = np.full(N_EXPERTS * HIDDEN, np.nan, np.float32)
    rc, _, w, _ = O.moe_route_f32(np.ones(HIDDEN, np.float32), r, N_EXPERTS, TOP_K, O.ROUTE_SIGMOID_NORMALIZE,
                                  2.5)
    assert rc == 0 and abs(float(w.sum()) - 2.5) < 1e-5 and np.all(np.abs(w - 1.25) < 1e-5)


def test_route_bias_shifts_selection_not_weights():
    h = np.full(HIDDEN, 0.5, np.float32)
    r = np.zeros(N_EXPERTS * HIDDEN, np.float32)
    bias = np.zeros(N_EXPERTS, np.float32)
    bias[-1] = 10.0
    rc, ids, w, _ = O.moe_route_f32(h, r, N_EXPERTS, TOP_K, O.ROUTE_SIGMOID_NORMALIZE, 1.0, router_bias=bias)
    assert rc == 0 and N_EXPERTS - 1 in ids.tolist()
    assert np.all(np.abs(w - 1.0 / TOP_K) < 1e-6)


# ------------------------------------------- routing: bit-exact against a Python restatement


def route_py(h, r, n_experts, top_k, mode, scale, bias=None):
    """moe.rs:132-317 in float32 scalar steps (each op rounded, like the Rust)."""
    f = np.float32
    dim = h.size
    scores = []
    for e in range(n_experts):
        dot = f(0.0)
        for i in range(dim):
            dot = f(dot + f(h[i] * r[e * dim + i]))
        if mode == 0:
            scores.append(f(dot + bias[e]) if bias is not None else dot)
        else:
            scores.append(f(f(1.0) / f(f(1.0) + np.exp(-dot, dtype=np.float32))))
    sel = (lambda e: bias[e]) if (bias is not None and mode == 1) else (lambda e: f(0.0))
    idx = list(range(top_k))
    wts = [f(scores[i] + sel(i)) for i in range(top_k)]
    mi, mv = 0, wts[0]
    for i in range(1, top_k):
        if wts[i] < mv:
            mv, mi = wts[i], i
    for e in range(top_k, n_experts):
        key = f(scores[e] + sel(e))
        if key > mv:
            idx[mi], wts[mi] = e, key
            mi, mv = 0, wts[0]
            for i in range(1, top_k):
                if wts[i] < mv:
                    mv, mi = wts[i], i
    return np.array(idx, np.uint32), np.array(scores, np.float32)


@pytest.mark.parametrize("mode", [O.ROUTE_SOFTMAX, O.ROUTE_SIGMOID_NORMALIZE])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_route_bit_exact_python(mode, seed):
    rng = np.random.default_rng(seed)
    dim, E, K = 96, 24, 5
    h = rng.standard_normal(dim).astype(np.float32)
    r = rng.standard_normal(E * dim).astype(np.float32)
    bias = rng.standard_normal(E).astype(np.float32) if seed == 3 else None
    rc, ids, w, scores = O.moe_route_f32(h, r, E, K, mode, 1.0, router_bias=bias)
    ref_ids, ref_scores = route_py(h, r, E, K, mode, 1.0, bias)
    assert rc == 0
    if mode == O.ROUTE_SOFTMAX:
        assert np.array_equal(scores.view(np.uint32), ref_scores.view(np.uint32))
    else:   # libm expf vs numpy's float32 exp: a few ulp at most
        np.testing.assert_allclose(scores, ref_scores, rtol=3e-7)
    assert np.array_equal(ids, ref_ids)
    raw = scores[ids].astype(np.float64)
    ref_w = np.exp(raw - raw.max()) / np.exp(raw - raw.max()).sum() if mode == 0 else raw / raw.sum()
    np.testing.assert_allclose(w, ref_w, rtol=2e-6, atol=1e-7)


# ------------------------------------------- experts / MoE FFN against float64


def small_cfg(**kw):
    return synth.ds2_small_config(n_layers=2, hidden=256, ffn=512, n_heads=2, n_experts=8, top_k=3,
                                  expert_ffn=128, n_shared=2, vocab=256, **kw)


def swiglu64(x, g, u, d, H, F):
    a = deq_q4_0(g, F, H) @ x
    b = deq_q4_0(u, F, H) @ x
    return deq_q4_0(d, H, F) @ (a / (1 + np.exp(-a)) * b)


@pytest.mark.parametrize("n_shared", [0, 1, 2])
def test_moe_ffn_against_float64(n_shared):
    cfg = small_cfg()
    cfg = synth.Ds2Config(**{**cfg.__dict__, "n_shared": n_shared})
    w = synth.ds2_weights(cfg, seed=4)
    lw = w["layers"][1]
    x = synth.f32(4, 77, cfg.hidden, 0.0, 1.0)
    rc, out, ids, wts = O.moe_ffn(x, lw, cfg)
    assert rc == 0
    H, EF = cfg.hidden, cfg.expert_ffn
    x64 = x.astype(np.float64)
    gu, dn = EF * H // 32 * 18, H * EF // 32 * 18
    ref = np.zeros(H)
    for s in range(n_shared):
        ref += swiglu64(x64, lw["gate_shexp"][s * gu:(s + 1) * gu], lw["up_shexp"][s * gu:(s + 1) * gu],
                        lw["down_shexp"][s * dn:(s + 1) * dn], H, EF)
    scores = lw["router_w"].reshape(cfg.n_experts, H).astype(np.float64) @ x64
    assert set(ids.tolist()) == set(np.argsort(-scores)[:cfg.top_k].tolist())
    for e, wk in zip(ids, wts):
        ref += float(wk) * swiglu64(x64, lw["gate_exps"][e * gu:(e + 1) * gu], lw["up_exps"][e * gu:(e + 1) * gu],
                                    lw["down_exps"][e * dn:(e + 1) * dn], H, EF)
    assert rel_l2(out, ref) < 1e-5


def test_expert_swiglu_against_float64():
    cfg = small_cfg()
    w = synth.ds2_weights(cfg, seed=5)
    lw = w["layers"][1]
    H, EF = cfg.hidden, cfg.expert_ffn
    gu, dn = EF * H // 32 * 18, H * EF // 32 * 18
    x = synth.f32(5, 78, H, 0.0, 1.0)
    out = O.expert_swiglu(x, lw["gate_exps"][:gu], lw["up_exps"][:gu], lw["down_exps"][:dn], H, EF)
    ref = swiglu64(x.astype(np.float64), lw["gate_exps"][:gu], lw["up_exps"][:gu], lw["down_exps"][:dn], H, EF)
    assert rel_l2(out, ref) < 1e-5


# ------------------------------------------- MLA against float64


def mla64(x, lw, cfg, cache64, pos):
    """mla.rs:122-414 in float64 (reference order is irrelevant here)."""
    H, R, RD, NH, NO, VD, QL = (cfg.hidden, cfg.kv_lora_rank, cfg.rope_dim, cfg.n_heads, cfg.nope_dim,
                                cfg.v_dim, cfg.q_lora_rank)
    x = x.astype(np.float64)
    kv_a = deq_q4_0(lw["kv_a_mqa"], R + RD, H) @ x
    c = rms64(kv_a[:R], lw["kv_a_norm"], cfg.rms_eps)
    kr = kv_a[R:]
    if "k_norm" in lw:
        kr = rms64(kr, lw["k_norm"], cfg.rms_eps)
    kr = rope64(kr, pos, cfg.rope_theta)
    cache64[pos, :R], cache64[pos, R:] = c, kr
    cq = rms64(deq_q4_0(lw["q_a"], QL, H) @ x, lw["q_a_norm"], cfg.rms_eps)
    q = (deq_q4_0(lw["q_b"], NH * (NO + RD), QL) @ cq).reshape(NH, NO + RD)
    for h in range(NH):
        q[h, NO:] = rope64(q[h, NO:], pos, cfg.rope_theta)
    if "kv_b" in lw:
        kvb = deq_q4_0(lw["kv_b"], NH * (NO + VD), R).reshape(NH, NO + VD, R)
        kb, vb = kvb[:, :NO], kvb[:, NO:]
    else:
        kb = deq_q4_0(lw["k_b"], NH * NO, R).reshape(NH, NO, R)
        vb = deq_q4_0(lw["v_b"], NH * VD, R).reshape(NH, VD, R)
    C = cache64[:pos + 1]
    out = np.zeros(NH * VD)
    for h in range(NH):
        s = (C[:, :R] @ kb[h].T @ q[h, :NO] + C[:, R:] @ q[h, NO:]) / np.sqrt(NO + RD)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * VD:(h + 1) * VD] = vb[h] @ (C[:, :R].T @ p)
    return deq_q4_0(lw["attn_output"], H, NH * VD) @ out


@pytest.mark.parametrize("variant", ["kv_b", "split", "k_norm"])
def test_mla_against_float64(variant):
    cfg = small_cfg(split_kv_b=variant == "split", k_norm=variant == "k_norm")
    w = synth.ds2_weights(cfg, seed=6, norm_sigma=0.1)
    lw = w["layers"][0]
    T = 12
    cache = np.zeros((T, cfg.kv_lora_rank + cfg.rope_dim), np.float32)
    cache64 = np.zeros(cache.shape)
    for pos in range(T):
        x = synth.f32(6, 200 + pos, cfg.hidden, 0.0, 1.0)
        rc, out = O.mla_attention(x, lw, cfg, cache, pos)
        assert rc == 0
        ref = mla64(x, lw, cfg, cache64, pos)
        assert rel_l2(out, ref) < 2e-5, pos
        assert rel_l2(cache[:pos + 1], cache64[:pos + 1]) < 1e-6


def test_mla_errors():
    cfg = small_cfg()
    w = synth.ds2_weights(cfg, seed=7)
    lw = w["layers"][0]
    cache = np.zeros((4, cfg.kv_lora_rank + cfg.rope_dim), np.float32)
    x = synth.f32(7, 1, cfg.hidden, 0.0, 1.0)
    assert O.mla_attention(x, lw, cfg, cache, 4)[0] == 10        # TokenIndexOutOfRange
    bad = x.copy()
    bad[3] = np.inf
    assert O.mla_attention(bad, lw, cfg, cache, 0)[0] == 20      # NumericalInstability


# ------------------------------------------- MHA layers against float64


def mha64(x, lw, cfg, k64, v64, pos):
    """mla.rs:449-618 in float64."""
    H, NH, NKV, NO, RD, VD = cfg.hidden, cfg.n_heads, cfg.kv_heads, cfg.nope_dim, cfg.rope_dim, cfg.v_dim
    hq = NO + RD
    x = x.astype(np.float64)
    q = (deq_q4_0(lw["q_mha"], NH * hq, H) @ x).reshape(NH, hq)
    k = (deq_q4_0(lw["k_mha"], NKV * hq, H) @ x).reshape(NKV, hq)
    v = deq_q4_0(lw["v_mha"], NKV * VD, H) @ x
    for h in range(NH):
        q[h, NO:] = rope64(q[h, NO:], pos, cfg.rope_theta)
    for h in range(NKV):
        k[h, NO:] = rope64(k[h, NO:], pos, cfg.rope_theta)
    k64[pos], v64[pos] = k.ravel(), v
    out = np.zeros(NH * VD)
    G = NH // NKV
    for h in range(NH):
        kv = h // G
        K = k64[:pos + 1, kv * hq:(kv + 1) * hq]
        Vv = v64[:pos + 1, kv * VD:(kv + 1) * VD]
        s = K @ q[h] / np.sqrt(hq)
        p = np.exp(s - s.max())
        out[h * VD:(h + 1) * VD] = Vv.T @ (p / p.sum())
    return deq_q4_0(lw["attn_output"], H, NH * VD) @ out


@pytest.mark.parametrize("n_kv", [2, 1])
def test_mha_against_float64(n_kv):
    cfg = small_cfg(mha_layers=(0,), n_kv_heads=n_kv)
    w = synth.ds2_weights(cfg, seed=16, norm_sigma=0.1)
    lw = w["layers"][0]
    T = 12
    kc = np.zeros((T, cfg.kv_heads * cfg.q_head), np.float32)
    vc = np.zeros((T, cfg.kv_heads * cfg.v_dim), np.float32)
    k64, v64 = np.zeros(kc.shape), np.zeros(vc.shape)
    for pos in range(T):
        x = synth.f32(16, 300 + pos, cfg.hidden, 0.0, 1.0)
        rc, out = O.mha_attention(x, lw, cfg, kc, vc, pos)
        assert rc == 0
        ref = mha64(x, lw, cfg, k64, v64, pos)
        assert rel_l2(out, ref) < 2e-5, pos
        assert rel_l2(kc[:pos + 1], k64[:pos + 1]) < 1e-6 and rel_l2(vc[:pos + 1], v64[:pos + 1]) < 1e-6


def test_mha_errors():
    cfg = small_cfg(mha_layers=(0,))
    w = synth.ds2_weights(cfg, seed=17)
    lw = w["layers"][0]
    kc = np.zeros((4, cfg.kv_heads * cfg.q_head), np.float32)
    vc = np.zeros((4, cfg.kv_heads * cfg.v_dim), np.float32)
    x = synth.f32(17, 1, cfg.hidden, 0.0, 1.0)
    assert O.mha_attention(x, lw, cfg, kc, vc, 4)[0] == 10      # TokenIndexOutOfRange
    bad = x.copy()
    bad[3] = np.inf
    assert O.mha_attention(bad, lw, cfg, kc, vc, 0)[0] == 20    # NumericalInstability


def test_ds2_forward_with_an_mha_layer():
    """Layer 0 as standard attention (AttnType::Mha) inside the step: the run
    equals the per-layer restatements composed on the residual stream."""
    cfg = small_cfg(mha_layers=(0,), n_kv_heads=1)
    w = synth.ds2_weights(cfg, seed=18, norm_sigma=0.1)
    r = O.OracleDs2Run(cfg, w, 8)
    H = cfg.hidden
    kc = np.zeros((8, cfg.kv_heads * cfg.q_head), np.float32)
    vc = np.zeros((8, cfg.kv_heads * cfg.v_dim), np.float32)
    cache = np.zeros((cfg.n_layers, 8, cfg.kv_lora_rank + cfg.rope_dim), np.float32)
    for pos, tok in enumerate([5, 9, 2]):
        hidden = r.forward(tok, pos)
        emb = w["token_embd"].reshape(cfg.vocab_padded, H // 32, 34)[tok]
        h = (emb[:, 2:].view(np.int8).astype(np.float32) * emb[:, :2].copy().view(np.float16).astype(np.float32))
        h = h.ravel().astype(np.float32)
        for li, lw in enumerate(w["layers"]):
            x = O.rmsnorm(h, lw["attn_norm"], cfg.rms_eps)
            rc, a = (O.mha_attention(x, lw, cfg, kc, vc, pos) if li == 0
                     else O.mla_attention(x, lw, cfg, cache[li], pos))
            assert rc == 0
            h = (h + a).astype(np.float32)
            x = O.rmsnorm(h, lw["ffn_norm"], cfg.rms_eps)
            if cfg.is_moe(li):
                rc, m, _, _ = O.moe_ffn(x, lw, cfg)
                assert rc == 0
            else:
                g = O.linear(x, lw["ffn_gate"], H, cfg.ffn, O.Q4_0)
                u = O.linear(x, lw["ffn_up"], H, cfg.ffn, O.Q4_0)
                g = (g / (np.float32(1) + np.exp(-g))).astype(np.float32)
                m = O.linear((g * u).astype(np.float32), lw["ffn_down"], cfg.ffn, H, O.Q4_0)
            h = (h + m).astype(np.float32)
        assert rel_l2(hidden, h) < 1e-6
    k_run, v_run = r.mha_cache()[0]
    assert np.array_equal(k_run[:3], kc[:3]) and np.array_equal(v_run[:3], vc[:3])


# ------------------------------------------- the DeepSeek2 step


def test_ds2_forward_composes_layers():
    """forward_pass.rs:703-909: the run's cache rows and expert ids equal what
    the per-layer restatements produce on the same residual stream."""
    cfg = small_cfg(k_norm=True)
    w = synth.ds2_weights(cfg, seed=8, norm_sigma=0.1)
    r = O.OracleDs2Run(cfg, w, 16)
    hidden = r.forward(5, 0)
    assert np.all(np.isfinite(hidden))
    # replay layer by layer with the unit restatements
    H = cfg.hidden
    emb = w["token_embd"].reshape(cfg.vocab_padded, H // 32, 34)[5]
    h = (emb[:, 2:].view(np.int8).astype(np.float32) * emb[:, :2].copy().view(np.float16).astype(np.float32))
    h = h.ravel().astype(np.float32)
    cache = np.zeros((cfg.n_layers, 16, cfg.kv_lora_rank + cfg.rope_dim), np.float32)
    ids_r, _ = r.expert_ids()
    for li, lw in enumerate(w["layers"]):
        x = O.rmsnorm(h, lw["attn_norm"], cfg.rms_eps)
        rc, a = O.mla_attention(x, lw, cfg, cache[li], 0)
        assert rc == 0
        h = (h + a).astype(np.float32)
        x = O.rmsnorm(h, lw["ffn_norm"], cfg.rms_eps)
        if cfg.is_moe(li):
            rc, m, ids, _ = O.moe_ffn(x, lw, cfg)
            assert rc == 0 and np.array_equal(ids, ids_r[li])
        else:
            g = O.linear(x, lw["ffn_gate"], H, cfg.ffn, O.Q4_0)
            u = O.linear(x, lw["ffn_up"], H, cfg.ffn, O.Q4_0)
            g = (g / (np.float32(1) + np.exp(-g))).astype(np.float32)
            m = O.linear((g * u).astype(np.float32), lw["ffn_down"], cfg.ffn, H, O.Q4_0)
        h = (h + m).astype(np.float32)
    assert rel_l2(hidden, h) < 1e-6
    assert rel_l2(r.cache()[:, :1], cache[:, :1]) < 1e-7


def test_ds2_generate_is_deterministic():
    cfg = small_cfg()
    w = synth.ds2_weights(cfg, seed=9)
    prompt = synth.ds2_prompt_ids(cfg, 5, seed=9)
    a = O.OracleDs2Run(cfg, w, 16).generate(prompt, 6)
    b = O.OracleDs2Run(cfg, w, 16).generate(prompt, 6)
    assert a[0] == 0 and np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])


# ---- the AVX-512 kernel order (inference_avx512.rs:2141-2825): the path the
# reference times, used for the config-3 CPU baseline

@pytest.mark.parametrize("variant", [dict(), dict(split_kv_b=True), dict(n_shared=0)])
def test_ds2_avx512_order_tracks_the_scalar_order(variant):
    """The AVX-512 order (16-lane matmul and dot accumulators, fused
    weighted adds, the polynomial SiLU) differs from the scalar crate order
    only in the last bits: same greedy tokens and expert ids, logits within
    1e-5."""
    kw = dict(n_layers=2, hidden=256, ffn=512, n_heads=2, n_experts=8, top_k=3, expert_ffn=128, n_shared=2,
              vocab=256)
    kw.update(variant)
    cfg = synth.ds2_small_config(**kw)
    w = synth.ds2_weights(cfg, seed=11, norm_sigma=0.1)
    prompt = synth.ds2_prompt_ids(cfg, 5, seed=11)
    a = O.OracleDs2Run(cfg, w, 16)
    b = O.OracleDs2Run(cfg, w, 16, order=O.ORDER_AVX512, threads=2)
    ra, rb = a.generate(prompt, 6, want_logits=True), b.generate(prompt, 6, want_logits=True)
    assert ra[0] == 0 and rb[0] == 0
    assert np.array_equal(ra[1], rb[1])
    assert np.array_equal(a.expert_ids()[0], b.expert_ids()[0])
    for s in range(6):
        assert rel_l2(rb[3][s], ra[3][s]) < 1e-5, s


def test_ds2_avx512_order_bits_do_not_depend_on_threads_or_simd():
    """Rows are independent, so the pool's split leaves every bit as it is,
    and the intrinsics reproduce the lane emulation exactly."""
    cfg = small_cfg()
    w = synth.ds2_weights(cfg, seed=12, norm_sigma=0.1)
    prompt = synth.ds2_prompt_ids(cfg, 4, seed=12)
    runs = [O.OracleDs2Run(cfg, w, 16, order=O.ORDER_AVX512, threads=t, simd=s) for t, s in ((1, 0), (1, 1), (3, 1))]
    outs = [r.generate(prompt, 5, want_logits=True) for r in runs]
    for o in outs[1:]:
        assert np.array_equal(o[1], outs[0][1])
        assert np.array_equal(o[3].view(np.uint32), outs[0][3].view(np.uint32))
    assert runs[2].threads == 3


def test_ds2_cache_rows_set_a_context_without_decoding_it():
    """A cache filled row by row from the decode equals one written by
    set_cache_rows from those rows: the next step's logits are identical."""
    cfg = small_cfg()
    w = synth.ds2_weights(cfg, seed=13, norm_sigma=0.1)
    prompt = synth.ds2_prompt_ids(cfg, 6, seed=13)
    a = O.OracleDs2Run(cfg, w, 16)
    for pos, t in enumerate(prompt):
        a.forward(int(t), pos)
    rows = a.cache()
    b = O.OracleDs2Run(cfg, w, 16)
    for layer in range(cfg.n_layers):
        b.set_cache_rows(layer, 0, rows[layer, :len(prompt)])
    a.forward(7, len(prompt))
    b.forward(7, len(prompt))
    assert np.array_equal(a.lm_head()[2].view(np.uint32), b.lm_head()[2].view(np.uint32))
    with pytest.raises(ValueError):
        b.set_cache_rows(cfg.n_layers, 0, rows[0, :1])
    with pytest.raises(ValueError):
        b.set_cache_rows(0, 15, rows[0, :2])
