"""GPU parity of the DeepSeek2 rows (MoE routing, grouped experts, MLA decode,
the DeepSeek2 step) with the CPU oracle, through the C ABI.

Bars: expert ids bit-identical to the reference order (the router repeats its
sequential unfused f32 dot); scores bit-identical in Softmax mode; weights to
expf rounding.  The MLA path absorbs kv_b into the query and the output (a
reordered sum), so hidden states, cache rows and logits are held to f32
rounding-level relative L2 (1e-4 here, 1e-2 is the north-star bar for
logits) and greedy tokens must be identical.
"""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


# ---------------------------------------------------------------- routing


@pytest.mark.parametrize("mode", [zb.ROUTE_SOFTMAX, zb.ROUTE_SIGMOID_NORMALIZE])
@pytest.mark.parametrize("dim,E,K,bias", [(2048, 64, 6, False), (512, 16, 4, True), (96, 24, 5, False),
                                          (4096, 160, 6, True)])
def test_route_matches_oracle(ctx, mode, dim, E, K, bias):
    seed = dim + E + K + mode
    h = synth.f32(seed, 1, dim, 0.0, 1.0)
    r = synth.f32(seed, 2, E * dim, 0.0, 1.0)
    b = synth.f32(seed, 3, E, 0.0, 1.0) if bias else None
    key = ctx.register(r, zb.F32, E, dim)
    for scale in (1.0, 2.5):
        ids, w, scores = ctx.moe_route_f32(h, key, E, K, mode, scale, router_bias=b)
        rc, rid, rw, rs = O.moe_route_f32(h, r, E, K, mode, scale, router_bias=b)
        assert rc == 0
        assert np.array_equal(ids, rid), (ids, rid)
        if mode == zb.ROUTE_SOFTMAX:
            assert np.array_equal(scores.view(np.uint32), rs.view(np.uint32))
        else:
            np.testing.assert_allclose(scores, rs, rtol=1e-6)
        np.testing.assert_allclose(w, rw, rtol=2e-6, atol=1e-7)


def test_route_reference_contracts(ctx):
    """deepseek2_moe_pipeline.rs:405-723 through the GPU entry point."""
    H, E, K = 256, 4, 2
    e = np.arange(E, dtype=np.float32)[:, None]
    i = np.arange(H)[None, :]
    skew = (np.float32(0.001) * e + np.float32(0.0001) * (i % 8).astype(np.float32)).astype(np.float32).ravel()
    ramp = (np.float32(0.1) + np.float32(0.01) * np.arange(H, dtype=np.float32)).astype(np.float32)
    ks = ctx.register(skew, zb.F32, E, H)
    ids, w, _ = ctx.moe_route_f32(ramp, ks, E, K)
    assert {2, 3} <= set(ids.tolist()) and abs(float(w.sum()) - 1) < 1e-5
    ids, w, _ = ctx.moe_route_f32(ramp, ks, E, K, zb.ROUTE_SIGMOID_NORMALIZE, 2.5)
    assert abs(float(w.sum()) - 2.5) < 1e-5
    nanr = np.zeros(E * H, np.float32)
    nanr[0] = np.nan
    kn = ctx.register(nanr, zb.F32, E, H)
    _, w, _ = ctx.moe_route_f32(np.ones(H, np.float32), kn, E, K)
    assert np.all(np.abs(w - 0.5) < 1e-6)
    alln = np.full(E * H, np.nan, np.float32)
    ka = ctx.register(alln, zb.F32, E, H)
    _, w, _ = ctx.moe_route_f32(np.ones(H, np.float32), ka, E, K, zb.ROUTE_SIGMOID_NORMALIZE, 2.5)
    assert np.all(np.abs(w - 1.25) < 1e-5)
    zero = np.zeros(E * H, np.float32)
    kz = ctx.register(zero, zb.F32, E, H)
    ids, w, _ = ctx.moe_route_f32(np.ones(H, np.float32), kz, E, K)
    assert ids.tolist() == [0, 1] and np.all(np.abs(w - 0.5) < 1e-6)
    bias = np.zeros(E, np.float32)
    bias[-1] = 10.0
    ids, w, _ = ctx.moe_route_f32(np.full(H, 0.5, np.float32), kz, E, K, zb.ROUTE_SIGMOID_NORMALIZE, 1.0,
                                  router_bias=bias)
    assert E - 1 in ids.tolist() and np.all(np.abs(w - 0.5) < 1e-6)
    for bad_k in (0, E + 1):
        with pytest.raises(zb.ZgpuError) as ei:
            ctx.moe_route_f32(ramp, ks, E, bad_k)
        assert ei.value.name == "INVALID_ARG"


# ---------------------------------------------------------------- MLA cache


def test_mla_cache_roundtrip(ctx):
    kv = zb.MlaKvCache(ctx, 8, 3, 512, 64)
    c = synth.f32(3, 1, 512, 0.0, 1.0)
    k = synth.f32(3, 2, 64, 0.0, 1.0)
    kv.store_compressed(2, 5, c, k)
    rows = kv.read(2, 6)
    assert np.array_equal(rows[5, :512], c) and np.array_equal(rows[5, 512:], k)
    assert not rows[:5].any()
    with pytest.raises(zb.ZgpuError) as ei:
        kv.store_compressed(3, 0, c, k)
    assert ei.value.name == "KV_LAYER_OUT_OF_RANGE"
    with pytest.raises(zb.ZgpuError) as ei:
        kv.store_compressed(0, 8, c, k)
    assert ei.value.name == "KV_TOKEN_OUT_OF_RANGE"
    with pytest.raises(zb.ZgpuError) as ei:
        kv.store_compressed(0, 0, c[:100], k)
    assert ei.value.name == "KV_INVALID_SLICE_LENGTH"
    with pytest.raises(zb.ZgpuError) as ei:
        kv.read(0, 9)
    assert ei.value.name == "KV_TOKEN_COUNT_EXCEEDS_MAX"
    kv.close()


# ---------------------------------------------------------------- the step

BASE = dict(n_layers=3, hidden=512, ffn=1024, n_heads=4, n_experts=8, top_k=3, expert_ffn=256, n_shared=2,
            vocab=1024)
VARIANTS = {
    "base": synth.ds2_small_config(**BASE),
    "split_knorm_sigmoid": synth.ds2_small_config(**{**BASE, "n_shared": 1}, split_kv_b=True, k_norm=True,
                                                  route_mode=1, router_bias=True, expert_weight_scale=2.5),
    "16heads_no_shared": synth.ds2_small_config(n_layers=2, hidden=1024, ffn=2048, n_heads=16, n_experts=16,
                                                top_k=6, expert_ffn=352, n_shared=0, vocab=2048),
}


def build(cfg, seed, **ctx_kw):
    ctx = zb.Context(**ctx_kw)
    w = synth.ds2_weights(cfg, seed=seed, norm_sigma=0.1)
    return ctx, w, zb.Ds2Model(ctx, cfg, w)


@pytest.mark.parametrize("name", list(VARIANTS))
def test_ds2_generate_matches_oracle(name):
    cfg = VARIANTS[name]
    ctx, w, m = build(cfg, seed=31)
    prompt = synth.ds2_prompt_ids(cfg, 7, seed=31)
    n_gen = 10
    kv = m.new_kv(48)
    toks, logits = m.generate_greedy(kv, prompt, n_gen, want_logits=True)
    r = O.OracleDs2Run(cfg, w, 48)
    rc, ref_t, margins, ref_l = r.generate(prompt, n_gen, want_logits=True)
    assert rc == 0
    assert np.array_equal(toks, ref_t), (toks, ref_t, margins)
    for s in range(n_gen):
        assert rel_l2(logits[s], ref_l[s]) < 1e-4, s
    used = len(prompt) + n_gen - 1
    ref_cache = r.cache()
    for layer in range(cfg.n_layers):
        assert rel_l2(kv.read(layer, used), ref_cache[layer, :used]) < 1e-4, layer
    # the last step's expert choices, layer by layer
    ids, wts = m.expert_ids()
    rid, rwt = r.expert_ids()
    for layer in range(cfg.n_dense, cfg.n_layers):
        assert np.array_equal(ids[layer], rid[layer]), (layer, ids[layer], rid[layer])
        np.testing.assert_allclose(wts[layer], rwt[layer], rtol=1e-3, atol=1e-5)
    perf = m.perf()
    assert perf["decode_launches"] > 0
    kv.close()
    m.close()
    ctx.close()


def test_ds2_forward_single_token_matches_oracle():
    cfg = VARIANTS["base"]
    ctx, w, m = build(cfg, seed=32)
    kv = m.new_kv(32)
    r = O.OracleDs2Run(cfg, w, 32)
    toks = synth.ds2_prompt_ids(cfg, 20, seed=32)
    agree = total = 0
    for pos, t in enumerate(toks):
        h = m.forward_single_token(kv, int(t), pos)
        ref = r.forward(int(t), pos)
        assert rel_l2(h, ref) < 1e-4, pos
        ids, _ = m.expert_ids()
        rid, _ = r.expert_ids()
        agree += int(np.array_equal(ids[cfg.n_dense:], rid[cfg.n_dense:]))
        total += 1
    assert agree == total
    tok, logits = m.lm_head_argmax()
    rc, rtok, rl = r.lm_head()
    assert rc == 0 and tok == rtok and rel_l2(logits, rl) < 1e-4
    # errors map to the reference's enums
    with pytest.raises(zb.ZgpuError) as ei:
        m.forward_single_token(kv, 1, 32)
    assert ei.value.name == "KV_TOKEN_OUT_OF_RANGE"
    m.close()
    ctx.close()


def test_ds2_graph_and_eager_agree():
    """The CUDA-graph step and the eagerly launched kernels are the same
    computation: bitwise equal tokens and logits."""
    cfg = VARIANTS["base"]
    prompt = synth.ds2_prompt_ids(cfg, 5, seed=33)
    out = []
    for graph in (True, False):
        ctx, w, m = build(cfg, seed=33, graph=graph)
        kv = m.new_kv(32)
        out.append(m.generate_greedy(kv, prompt, 6, want_logits=True))
        m.close()
        ctx.close()
    assert np.array_equal(out[0][0], out[1][0])
    assert np.array_equal(out[0][1].view(np.uint32), out[1][1].view(np.uint32))


def test_ds2_full_width_layers():
    """BASELINE config 3 widths (hidden 2048, 16 heads, kv_lora 512, q_lora
    1536, dense FFN 10944, 64 experts x 1408 top-6 + 2 shared) on two layers
    and a reduced vocab."""
    full = synth.DS2_V2_LITE
    cfg = synth.Ds2Config(**{**full.__dict__, "name": "ds2-full-width-2l", "n_layers": 2, "vocab_padded": 4096,
                             "vocab_real": 4096})
    ctx, w, m = build(cfg, seed=34)
    prompt = synth.ds2_prompt_ids(cfg, 4, seed=34)
    kv = m.new_kv(16)
    toks, logits = m.generate_greedy(kv, prompt, 4, want_logits=True)
    r = O.OracleDs2Run(cfg, w, 16)
    rc, rt, margins, rl = r.generate(prompt, 4, want_logits=True)
    assert rc == 0 and np.array_equal(toks, rt), (toks, rt, margins)
    for s in range(4):
        assert rel_l2(logits[s], rl[s]) < 1e-4
    ids, _ = m.expert_ids()
    rid, _ = r.expert_ids()
    assert np.array_equal(ids[1], rid[1])
    m.close()
    ctx.close()


# ------------------------------------------ layers with standard attention (AttnType::Mha)

MHA_VARIANTS = {
    # layer 0 as standard attention, as the builds that ship attn_q / attn_k / attn_v for it
    "mha_layer0": synth.ds2_small_config(**BASE, mha_layers=(0,)),
    # two MHA layers around an MLA layer, GQA 2, split k_b / v_b on the MLA layer
    "mha_gqa2_split": synth.ds2_small_config(**BASE, mha_layers=(0, 2), n_kv_heads=2, split_kv_b=True),
}


@pytest.mark.parametrize("name", list(MHA_VARIANTS))
def test_ds2_mha_layers_match_oracle(name):
    """mha_attention_single_token (mla.rs:449-618) inside the step: greedy
    tokens identical to the oracle's, logits and both caches within 1e-4."""
    cfg = MHA_VARIANTS[name]
    ctx, w, m = build(cfg, seed=34)
    prompt = synth.ds2_prompt_ids(cfg, 7, seed=34)
    n_gen = 8
    kv = m.new_kv(40)
    mkv = m.new_mha_kv(40)
    toks, logits = m.generate_greedy(kv, prompt, n_gen, want_logits=True)
    r = O.OracleDs2Run(cfg, w, 40)
    rc, ref_t, margins, ref_l = r.generate(prompt, n_gen, want_logits=True)
    assert rc == 0
    assert np.array_equal(toks, ref_t), (toks, ref_t, margins)
    for s in range(n_gen):
        assert rel_l2(logits[s], ref_l[s]) < 1e-4, s
    used = len(prompt) + n_gen - 1
    ref_cache = r.cache()
    for layer in range(cfg.n_layers):
        if not cfg.is_mha(layer):
            assert rel_l2(kv.read(layer, used), ref_cache[layer, :used]) < 1e-4, layer
    for slot, (rk, rv) in enumerate(r.mha_cache()):
        k, v = mkv.read(slot, used)
        assert rel_l2(k, rk[:used]) < 1e-4 and rel_l2(v, rv[:used]) < 1e-4, slot
    # the graph replays and the eager launches agree bit for bit
    ctx2 = zb.Context(graph=False)
    m2 = zb.Ds2Model(ctx2, cfg, w)
    kv2 = m2.new_kv(40)
    mkv2 = m2.new_mha_kv(40)
    t2, l2 = m2.generate_greedy(kv2, prompt, n_gen, want_logits=True)
    assert np.array_equal(t2, toks) and np.array_equal(l2.view(np.uint32), logits.view(np.uint32))
    for c in (kv2, mkv2):
        c.close()
    m2.close()
    ctx2.close()
    for c in (kv, mkv):
        c.close()
    m.close()
    ctx.close()


def test_ds2_mha_cache_errors():
    cfg = MHA_VARIANTS["mha_layer0"]
    ctx, w, m = build(cfg, seed=35)
    kv = m.new_kv(16)
    with pytest.raises(zb.ZgpuError) as ei:                 # forward_pass.rs:791-793: no MHA cache
        m.forward_single_token(kv, 1, 0)
    assert ei.value.name == "NUMERICAL_INSTABILITY"
    bad = zb.MhaKvCache(ctx, 16, 2, cfg.kv_heads, cfg.q_head, cfg.v_dim)   # two slots, one MHA layer
    with pytest.raises(zb.ZgpuError) as ei:
        m.set_mha_kv(bad)
    assert ei.value.name == "KV_LAYER_OUT_OF_RANGE"
    small = m.new_mha_kv(4)                                  # shorter than the MLA cache
    for pos in range(4):
        m.forward_single_token(kv, 1 + pos, pos)
    with pytest.raises(zb.ZgpuError) as ei:
        m.forward_single_token(kv, 7, 4)
    assert ei.value.name == "KV_TOKEN_OUT_OF_RANGE"
    # store / read round trip of the cache API
    k = np.arange(small.k_width, dtype=np.float32)
    v = -np.arange(small.v_width, dtype=np.float32)
    small.store(0, 3, k, v)
    rk, rv = small.read(0, 4)
    assert np.array_equal(rk[3], k) and np.array_equal(rv[3], v)
    for c in (kv, bad, small):
        c.close()
    m.close()
    ctx.close()
