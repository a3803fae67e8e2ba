"""End-to-end parity of the GPU decode path with the reference's CPU path (oracle).

The north-star bar: greedy token ids identical, logits within 1e-2 relative
L2.  The GPU path is held much tighter here (1e-4 on the small models) since
it reproduces the reference's RoPE/SiLU polynomials bit for bit and differs
only in reduction order.  Tests run through the C ABI (zgpu_generate_greedy,
zgpu_forward_single_token, zgpu_lm_head_argmax), on both execution paths: the
persistent step kernel (default) and the per-op kernels (persistent=False).
"""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def build(cfg, seed, norm_sigma=0.1, **ctx_kw):
    ctx = zb.Context(**ctx_kw)
    w = synth.qwen3_weights(cfg, seed=seed, norm_sigma=norm_sigma)
    return ctx, w, zb.Qwen3Model(ctx, cfg, w)


TINY = [
    synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512),
    synth.small_config(n_layers=3, hidden=512, ffn=1024, n_q=8, n_kv=2, vocab=1024),   # GQA 4
    synth.small_config(n_layers=2, hidden=1024, ffn=3072, n_q=8, n_kv=8, vocab=2048),  # MHA
    # BASELINE config 2 widths (Qwen3-8B: hidden 4096, FFN 12288, 32 q / 8 kv heads):
    # inputs wider than one round of float4s per consumer thread
    synth.small_config(n_layers=2, hidden=4096, ffn=12288, n_q=32, n_kv=8, vocab=1024),
]


PATHS = [True, False]


def assert_path(m, persistent, n_gen):
    """The last generate_greedy (no logits) ran on the requested path: the
    persistent kernel runs all decode steps as one launch."""
    launches = m.perf()["decode_launches"]
    if persistent:
        assert launches == 1, launches
    else:
        assert launches > n_gen, launches


@pytest.mark.parametrize("persistent", PATHS, ids=["persistent", "per_op"])
@pytest.mark.parametrize("cfg", TINY, ids=lambda c: c.name)
def test_generate_matches_oracle(cfg, persistent):
    ctx, w, m = build(cfg, seed=21, persistent=persistent)
    prompt = synth.prompt_ids(cfg, 7, seed=21)
    n_gen = 12
    kv = m.new_kv(64)
    toks, logits = m.generate_greedy(kv, prompt, n_gen, want_logits=True)
    # without logits the decode steps run as one launch: same tokens
    kv_b = m.new_kv(64)
    toks_b, _ = m.generate_greedy(kv_b, prompt, n_gen, want_logits=False)
    assert np.array_equal(toks_b, toks)
    assert_path(m, persistent, n_gen)
    kv_b.close()
    r = O.OracleRun(cfg, w, 64, order=O.ORDER_AVX512)
    rc, ref_t, margins, ref_l = r.generate(prompt, n_gen, want_logits=True)
    assert rc == 0
    assert np.array_equal(toks, ref_t), (toks, ref_t, margins)
    for s in range(n_gen):
        assert rel_l2(logits[s], ref_l[s]) < 1e-4, s
    # KV cache contents (kv_cache.rs layout) after the run
    used = len(prompt) + n_gen - 1
    ref_kv = r.kv().reshape(cfg.n_layers, 2, 64, cfg.kv_dim)
    for layer in range(cfg.n_layers):
        k, v = kv.read(layer, used)
        assert rel_l2(k, ref_kv[layer, 0, :used].ravel()) < 1e-5
        assert rel_l2(v, ref_kv[layer, 1, :used].ravel()) < 1e-5
    # the scalar crate order agrees too
    r0 = O.OracleRun(cfg, w, 64, order=O.ORDER_SCALAR)
    rc0, t0, _, l0 = r0.generate(prompt, n_gen, want_logits=True)
    assert rc0 == 0 and np.array_equal(toks, t0)
    assert max(rel_l2(logits[s], l0[s]) for s in range(n_gen)) < 1e-3
    m.close(); kv.close(); ctx.close()


@pytest.mark.parametrize("persistent", PATHS, ids=["persistent", "per_op"])
@pytest.mark.parametrize("cfg", TINY[:2], ids=lambda c: c.name)
def test_long_context_uses_split_attention(cfg, persistent):
    # > 256 cached tokens: the attention runs as several splits per kv-head
    # merged by the last CTA (flash-decoding partials).
    ctx, w, m = build(cfg, seed=25, persistent=persistent)
    prompt = synth.prompt_ids(cfg, 530, seed=25)
    kv = m.new_kv(600)
    toks, logits = m.generate_greedy(kv, prompt, 6, want_logits=True)
    r = O.OracleRun(cfg, w, 600, order=O.ORDER_AVX512)
    rc, ref_t, margins, ref_l = r.generate(prompt, 6, want_logits=True)
    assert rc == 0
    assert np.array_equal(toks, ref_t)
    assert max(rel_l2(logits[s], ref_l[s]) for s in range(6)) < 1e-4
    m.close(); kv.close(); ctx.close()


@pytest.mark.parametrize("persistent", PATHS, ids=["persistent", "per_op"])
def test_step_api_matches_generate(persistent):
    cfg = TINY[1]
    ctx, w, m = build(cfg, seed=22, persistent=persistent)
    prompt = synth.prompt_ids(cfg, 5, seed=22)
    kv = m.new_kv(32)
    toks, logits = m.generate_greedy(kv, prompt, 6, want_logits=True)
    kv2 = m.new_kv(32)
    r = O.OracleRun(cfg, w, 32, order=O.ORDER_AVX512)
    seq, out, pos = list(prompt), [], 0
    for t in prompt:
        h = m.forward_single_token(kv2, int(t), pos)
        hr = r.forward(int(t), pos)
        assert rel_l2(h, hr) < 1e-4
        pos += 1
    for s in range(6):
        tok, lg = m.lm_head_argmax()
        rc, rtok, rl = r.lm_head()
        assert rc == 0 and tok == rtok == toks[s]
        assert rel_l2(lg, rl) < 1e-4
        assert np.array_equal(lg, logits[s])     # same kernels, same order
        out.append(tok)
        if s < 5:
            m.forward_single_token(kv2, tok, pos)
            r.forward(tok, pos)
            pos += 1
    m.close(); kv.close(); kv2.close(); ctx.close()


def test_graph_replay_equals_eager_and_is_deterministic():
    cfg = TINY[0]
    w = synth.qwen3_weights(cfg, seed=23, norm_sigma=0.1)
    prompt = synth.prompt_ids(cfg, 6, seed=23)
    outs = []
    per_op = ({"persistent": False, "graph": True}, {"persistent": False, "graph": False},
              {"persistent": False, "graph": True, "pdl": False}, {"persistent": False, "graph": True})
    for kw in per_op + ({"persistent": True}, {"persistent": True}):
        ctx = zb.Context(**kw)
        m = zb.Qwen3Model(ctx, cfg, w)
        kv = m.new_kv(40)
        outs.append(m.generate_greedy(kv, prompt, 10, want_logits=True))
        m.close(); kv.close(); ctx.close()
    # per-op kernels: graph, eager, PDL or not -> identical bits
    for toks, logits in outs[1:4]:
        assert np.array_equal(toks, outs[0][0])
        assert np.array_equal(logits, outs[0][1])
    # persistent kernel: deterministic run to run; same tokens as the per-op
    # path, logits equal up to the RMSNorm summation order
    assert np.array_equal(outs[4][0], outs[5][0]) and np.array_equal(outs[4][1], outs[5][1])
    assert np.array_equal(outs[4][0], outs[0][0])
    assert max(rel_l2(outs[4][1][s], outs[0][1][s]) for s in range(10)) < 1e-5


def test_errors_follow_the_reference_enums():
    cfg = TINY[0]
    ctx, w, m = build(cfg, seed=24)
    kv = m.new_kv(8)
    prompt = synth.prompt_ids(cfg, 4, seed=24)
    with pytest.raises(zb.ZgpuError) as e:           # store_kv token >= max_tokens
        m.generate_greedy(kv, prompt, 6)
    assert e.value.status == 10
    with pytest.raises(zb.ZgpuError) as e:
        m.forward_single_token(kv, 1, 8)
    assert e.value.status == 10
    bad = zb.KvCache(ctx, 8, cfg.n_layers + 1, cfg.n_kv_heads, cfg.head_dim)
    with pytest.raises(zb.ZgpuError) as e:
        m.forward_single_token(bad, 1, 0)
    assert e.value.status == 11
    with pytest.raises(zb.ZgpuError):
        m.forward_single_token(kv, cfg.vocab_padded, 0)
    # LmHeadError::ArgmaxInPaddingRegion (lm_head.rs:161-163)
    m.forward_single_token(kv, 3, 0)
    tok, _ = m.lm_head_argmax()
    with pytest.raises(zb.ZgpuError) as e:
        m.lm_head_argmax(vocab_real=tok)
    assert e.value.status == 41
    # the context stays usable after the errors
    tok2, _ = m.lm_head_argmax()
    assert tok2 == tok
    bad.close(); kv.close(); m.close(); ctx.close()


# Weights of the full-size parity cases.  "baseline": BASELINE config 0's
# distributions (the bench's model); its greedy sequence repeats one id,
# because the uniform nibbles' mean of 7.5 gives every Q4_0 row a mean weight
# of -d/2 and that common mode, summed over 28 layers, decides the argmax.
# "varied": the same shapes with centred nibbles (synth.center_q4_0) and
# RMSNorm / QK-norm gains N(3, 0.3), whose 129 greedy tokens are all
# distinct on the oracle (smallest top-1/top-2 logit margin 3.6e-3 at logits
# of about 7), so the token check compares a sequence that really moves.
WEIGHTS = {"baseline": dict(), "varied": dict(centered=True, norm_mean=3.0, norm_sigma=0.3)}


@pytest.mark.slow
@pytest.mark.parametrize("variant", list(WEIGHTS))
@pytest.mark.parametrize("persistent", PATHS, ids=["persistent", "per_op"])
def test_config0_full_size_matches_oracle(persistent, variant):
    """Qwen3-1.7B shape, 16 prompt ids, 128 greedy decode steps."""
    cfg = synth.QWEN3_1_7B
    ctx = zb.Context(persistent=persistent)
    w = synth.qwen3_weights(cfg, seed=0, **WEIGHTS[variant])
    m = zb.Qwen3Model(ctx, cfg, w)
    prompt = synth.prompt_ids(cfg, 16, seed=0)
    n_gen = 129
    kv = m.new_kv(512)
    toks, logits = m.generate_greedy(kv, prompt, n_gen, want_logits=True)
    r = O.OracleRun(cfg, w, 512, order=O.ORDER_AVX512)
    rc, ref_t, margins, ref_l = r.generate(prompt, n_gen, want_logits=True)
    r.close()
    assert rc == 0
    distinct = len(set(ref_t.tolist()))
    print(f"{variant}: {distinct} distinct greedy ids of {n_gen}; top-1/top-2 margin min "
          f"{float(margins.min()):.3g} (step {int(margins.argmin())}), median {float(np.median(margins)):.3g}")
    if variant == "varied":
        assert distinct >= 100, distinct
    assert np.array_equal(toks, ref_t), f"first mismatch at step {np.argmax(toks != ref_t)}"
    worst = max(rel_l2(logits[s], ref_l[s]) for s in range(n_gen))
    assert worst < 1e-2, worst
    # what this path actually achieves: ~1e-5 on the baseline weights; the
    # varied model's gains of 3 amplify every layer's last-bit differences
    # (measured 3.5e-4 to 3.9e-4, with identical tokens)
    assert worst < (1e-4 if variant == "baseline" else 1e-3), worst
    # the decode steps as one launch give the same tokens
    kv_b = m.new_kv(512)
    toks_b, _ = m.generate_greedy(kv_b, prompt, n_gen, want_logits=False)
    assert np.array_equal(toks_b, toks)
    assert_path(m, persistent, n_gen)
    m.close(); kv.close(); kv_b.close(); ctx.close()
