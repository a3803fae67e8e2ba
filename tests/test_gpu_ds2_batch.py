"""Batched DeepSeek2 decode (BASELINE config 3's serving shape: up to 32
concurrent sequences, each on its own MLA cache at its own position) through
zgpu_ds2_decode_batch.

Bars:
- against the one-sequence path (zgpu_ds2_forward_single_token +
  zgpu_ds2_lm_head_argmax on a second set of caches): bit-identical greedy
  tokens, logits, per-layer expert ids and appended cache rows.  The batch
  widens every launch over the sequences and changes no arithmetic;
- against the CPU oracle (the reference's per-token order), free-running
  greedy: identical tokens and expert ids, logits within 1e-4 relative L2
  (the MLA path absorbs kv_b, a reordered sum; 1e-2 is the north-star bar).
"""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from ds2_batch_steps import prefill, prompts_for, run_batch, run_single
from zero_b200 import synth

pytestmark = pytest.mark.gpu

BASE = dict(n_layers=3, hidden=512, ffn=1024, n_heads=4, n_experts=8, top_k=3, expert_ffn=256, n_shared=2,
            vocab=1024)
VARIANTS = {
    "base": synth.ds2_small_config(**BASE),
    "split_knorm_sigmoid": synth.ds2_small_config(**{**BASE, "n_shared": 1}, split_kv_b=True, k_norm=True,
                                                  route_mode=1, router_bias=True, expert_weight_scale=2.5),
    "16heads_no_shared": synth.ds2_small_config(n_layers=2, hidden=1024, ffn=2048, n_heads=16, n_experts=16,
                                                top_k=6, expert_ffn=352, n_shared=0, vocab=2048),
}


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def build(cfg, seed, **ctx_kw):
    ctx = zb.Context(**ctx_kw)
    w = synth.ds2_weights(cfg, seed=seed, norm_sigma=0.1)
    return ctx, w, zb.Ds2Model(ctx, cfg, w)


def batch_vs_single(cfg, seed, n_seq, n_steps, max_tokens, max_len=9, **ctx_kw):
    ctx, w, m = build(cfg, seed, **ctx_kw)
    prompts = prompts_for(cfg, n_seq, seed, max_len=max_len)
    kb = [m.new_kv(max_tokens) for _ in range(n_seq)]
    ks = [m.new_kv(max_tokens) for _ in range(n_seq)]
    prefill(m, kb, prompts)
    prefill(m, ks, prompts)
    bt, bl, bi = run_batch(m, kb, prompts, n_steps)
    st, sl, si = run_single(m, ks, prompts, n_steps)
    assert np.array_equal(bt, st), (bt, st)
    assert np.array_equal(bl.view(np.uint32), sl.view(np.uint32))
    moe = slice(cfg.n_dense, cfg.n_layers)
    assert np.array_equal(bi[:, moe], si[:, moe])
    for b in range(n_seq):
        used = len(prompts[b]) + n_steps - 1
        for layer in range(cfg.n_layers):
            assert np.array_equal(kb[b].read(layer, used).view(np.uint32), ks[b].read(layer, used).view(np.uint32))
    for kv in kb + ks:
        kv.close()
    m.close()
    ctx.close()
    return prompts, bt, bl, bi, w


@pytest.mark.parametrize("name", list(VARIANTS))
def test_ds2_batch_equals_single_decodes(name):
    batch_vs_single(VARIANTS[name], seed=51, n_seq=5, n_steps=4, max_tokens=32)


def test_ds2_batch_graph_and_eager_agree():
    """The batch step replayed as a CUDA graph and launched eagerly."""
    cfg = VARIANTS["base"]
    _, t0, l0, _, _ = batch_vs_single(cfg, seed=52, n_seq=3, n_steps=3, max_tokens=24)
    _, t1, l1, _, _ = batch_vs_single(cfg, seed=52, n_seq=3, n_steps=3, max_tokens=24, graph=False)
    assert np.array_equal(t0, t1) and np.array_equal(l0.view(np.uint32), l1.view(np.uint32))


@pytest.mark.parametrize("name", ["base", "split_knorm_sigmoid"])
def test_ds2_batch_matches_oracle(name):
    """Free-running greedy per sequence on the CPU oracle."""
    cfg = VARIANTS[name]
    n_seq, n_steps, max_tokens = 4, 5, 32
    ctx, w, m = build(cfg, seed=53)
    prompts = prompts_for(cfg, n_seq, 53)
    kvs = [m.new_kv(max_tokens) for _ in range(n_seq)]
    prefill(m, kvs, prompts)
    bt, bl, bi = run_batch(m, kvs, prompts, n_steps)
    for b in range(n_seq):
        r = O.OracleDs2Run(cfg, w, max_tokens)
        p = prompts[b]
        for pos, t in enumerate(p[:-1]):
            r.forward(int(t), pos)
        cur, pos = int(p[-1]), len(p) - 1
        for s in range(n_steps):
            r.forward(cur, pos)
            rc, rtok, rl = r.lm_head()
            assert rc == 0
            rid, _ = r.expert_ids()
            assert bt[s, b] == rtok, (b, s, bt[:, b], rtok)
            assert rel_l2(bl[s, b], rl) < 1e-4, (b, s)
            for layer in range(cfg.n_dense, cfg.n_layers):
                assert np.array_equal(bi[s, layer, b], rid[layer]), (b, s, layer)
            cur, pos = rtok, pos + 1
        r.close()
    for kv in kvs:
        kv.close()
    m.close()
    ctx.close()


def test_ds2_batch_32_full_width():
    """BASELINE config 3 at its batch (32 sequences) and layer widths (hidden
    2048, 16 heads, kv_lora 512, q_lora 1536, 64 experts x 1408 top-6 + 2
    shared) on two layers and a reduced vocab, contexts 2..40 tokens: equal
    to 32 one-sequence decodes bit for bit, and two sequences held to the
    oracle."""
    full = synth.DS2_V2_LITE
    cfg = synth.Ds2Config(**{**full.__dict__, "name": "ds2-full-width-2l", "n_layers": 2, "vocab_padded": 4096,
                             "vocab_real": 4096})
    prompts, bt, bl, bi, w = batch_vs_single(cfg, seed=54, n_seq=32, n_steps=3, max_tokens=64, max_len=40)
    assert len({len(p) for p in prompts}) > 8
    for b in (0, 17):
        r = O.OracleDs2Run(cfg, w, 64)
        p = prompts[b]
        for pos, t in enumerate(p):
            r.forward(int(t), pos)
        rc, rtok, rl = r.lm_head()
        assert rc == 0 and bt[0, b] == rtok and rel_l2(bl[0, b], rl) < 1e-4
        rid, _ = r.expert_ids()
        assert np.array_equal(bi[0, 1, b], rid[1])
        r.close()


def test_ds2_batch_errors():
    cfg = VARIANTS["base"]
    ctx, w, m = build(cfg, seed=55)
    kvs = [m.new_kv(16) for _ in range(3)]
    other = m.new_kv(24)

    def err(kv_list, toks, pos):
        with pytest.raises(zb.ZgpuError) as ei:
            m.decode_batch(kv_list, toks, pos)
        return ei.value.name

    assert err(kvs[:2] + [kvs[0]], [1, 2, 3], [0, 0, 0]) == "INVALID_ARG"            # a cache twice
    assert err(kvs[:2] + [other], [1, 2, 3], [0, 0, 0]) == "INVALID_ARG"             # capacities differ
    assert err(kvs, [1, 2, 3], [0, 16, 0]) == "KV_TOKEN_OUT_OF_RANGE"
    assert err(kvs, [1, cfg.vocab_padded, 3], [0, 0, 0]) == "INVALID_ARG"
    many = [m.new_kv(4) for _ in range(33)]
    assert err(many, [1] * 33, [0] * 33) == "INVALID_ARG"
    for kv in many:
        kv.close()
    # still usable after the refusals
    t, _ = m.decode_batch(kvs, [1, 2, 3], [0, 0, 0])
    assert t.shape == (3,)
    for kv in kvs + [other]:
        kv.close()
    m.close()
    # MHA layers: one sequence at a time only
    mcfg = synth.ds2_small_config(**BASE, mha_layers=(0,))
    w2 = synth.ds2_weights(mcfg, seed=55, norm_sigma=0.1)
    m2 = zb.Ds2Model(ctx, mcfg, w2)
    mkv = m2.new_mha_kv(16)
    kv = m2.new_kv(16)
    with pytest.raises(zb.ZgpuError) as ei:
        m2.decode_batch([kv], [1], [0])
    assert ei.value.name == "INVALID_ARG"
    kv.close()
    m2.close()
    mkv.close()
    ctx.close()
