"""Batched greedy decode (zgpu_decode_batch): several sequences, each with its
own cache at its own position, one step at a time.

Per sequence, the step is forward_single_token + the LM head pick
(forward_pass.rs:515-631, lm_head.rs:98-166).  The batch runs every
projection and the LM head on the tensor cores with the single-token GEMV's
arithmetic (digit_mma.cu: int8 MMA over the three 8-bit digits of the
GEMV's activation integers, the GEMV's block and chunk order), so its f32
path is the reference's own, not a quantised one.  Bars:
- against the same sequences decoded one at a time on the per-op
  single-token path (zgpu_forward_single_token + zgpu_lm_head_argmax with
  ZGPU_FLAG_NO_PERSISTENT): the projections are that path's GEMVs bit for
  bit, the batched attention's exp (__expf) moves the last bits, so logits
  agree to 2e-5; bit-identical to the same sequences batched alone;
- against the oracle's f32 per-token path (the reference's AVX-512 order):
  logits within 1e-2 relative L2 at every step (the prompt goes through
  zgpu_prefill, whose Q8_0 activations leave the caches within 2e-2 of
  the oracle's, and the oracle's prompt runs with the same rounding), the KV
  cache within 2e-2, the same next token wherever the oracle's top-1/top-2
  margin is clear;
- free-running against the oracle's f32 path with no activation rounding
  anywhere at config-0 size and sixteen sequences at contexts past 2048
  tokens (run_f32_case).
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


def top2_gap(v):
    s = np.sort(v)
    return float(s[-1] - s[-2])


CASES = [
    # cfg, prompt lengths (one per sequence), decode steps
    (synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512), [5, 17, 33, 9], 6),
    (synth.small_config(n_layers=3, hidden=512, ffn=1024, n_q=8, n_kv=2, vocab=1024), [300, 12, 64], 5),
    # config-2 widths (hidden 4096, 32 / 8 heads, FFN 12288) on two layers, a short vocabulary
    (synth.small_config(n_layers=2, hidden=4096, ffn=12288, n_q=32, n_kv=8, vocab=1024), [40, 7], 4),
]


def run_case(cfg, lens, steps, seed=43):
    ctx = zb.Context()
    w = synth.qwen3_weights(cfg, seed=seed, norm_sigma=0.1)
    m = zb.Qwen3Model(ctx, cfg, w)
    max_tokens = max(lens) + steps + 8
    prompts = [synth.prompt_ids(cfg, n, seed=seed + i) for i, n in enumerate(lens)]
    kvs = [m.new_kv(max_tokens) for _ in lens]
    toks = np.array([m.prefill(kv, p, want_logits=False)[0] for kv, p in zip(kvs, prompts)], np.uint32)
    refs = []
    for p in prompts:
        r = O.OracleRun(cfg, w, max_tokens, order=O.ORDER_AVX512)
        r.set_q8act(1)
        for i, t in enumerate(p):
            r.forward(int(t), i)
        rc, rtok, _ = r.lm_head()
        assert rc == 0
        r.set_q8act(0)   # the decode steps: f32 activations, as the batch
        refs.append(r)
    worst, kv_worst = 0.0, 0.0
    for s in range(steps):
        pos = np.array([n + s for n in lens], np.uint32)
        nxt, logits = m.decode_batch(kvs, toks, pos)
        assert m.perf()["decode_ms"] > 0
        for i, r in enumerate(refs):
            r.forward(int(toks[i]), int(pos[i]))
            rc, rtok, rlog = r.lm_head()
            assert rc == 0
            err = rel_l2(logits[i], rlog)
            worst = max(worst, err)
            assert err < 1e-2, (s, i, err)
            if top2_gap(rlog) > 20 * err * float(np.abs(rlog).max()):
                assert nxt[i] == rtok, (s, i)
        toks = nxt
    for i, (r, kv) in enumerate(zip(refs, kvs)):
        n = lens[i] + steps
        ref_kv = r.kv().reshape(cfg.n_layers, 2, max_tokens, cfg.kv_dim)
        for layer in range(cfg.n_layers):
            k, v = kv.read(layer, n)
            kv_worst = max(kv_worst, rel_l2(k, ref_kv[layer, 0, :n].ravel()), rel_l2(v, ref_kv[layer, 1, :n].ravel()))
    assert kv_worst < 2e-2, kv_worst
    print(f"{cfg.name} lens={lens}: worst logits {worst:.2e}, kv {kv_worst:.2e}")
    for kv in kvs:
        kv.close()
    m.close()
    ctx.close()


@pytest.mark.parametrize("cfg,lens,steps", CASES, ids=[f"{c.name}-b{len(l)}" for c, l, _ in CASES])
def test_decode_batch_matches_per_token_path(cfg, lens, steps):
    run_case(cfg, lens, steps)


def test_decode_batch_config0_full_size():
    """BASELINE config 0 weights (28 layers, hidden 2048, vocab 151936), two sequences."""
    run_case(synth.QWEN3_1_7B, [16, 23], 3, seed=0)


def run_f32_case(cfg, lens, steps, seed, wkw):
    """Free-running batched greedy decode against the reference's own f32
    per-token path (ORDER_AVX512, no activation quantisation): each
    sequence's prompt goes through zgpu_prefill, then `steps` zgpu_decode_batch
    steps of all sequences; the oracle generates every sequence on its own
    (forward_single_token + lm_head_argmax, its prompt, then its own greedy
    tokens).  Per sequence and step: logits within the north-star 1e-2
    relative L2, and the same token.  A token may differ only where the
    oracle's top-1/top-2 margin is inside the logits error (the prompt's
    prefill quantises its matmul inputs to Q8_0); the sequences then part and
    that sequence's later steps are not compared.  At least 90% of the steps
    must be compared."""
    import os
    from concurrent.futures import ThreadPoolExecutor

    w = synth.qwen3_weights(cfg, seed=seed, **wkw)
    B = len(lens)
    max_tokens = max(lens) + steps + 8
    prompts = [synth.prompt_ids(cfg, n, seed=seed + i) for i, n in enumerate(lens)]
    ctx = zb.Context()
    m = zb.Qwen3Model(ctx, cfg, w)
    kvs = [m.new_kv(max_tokens) for _ in lens]
    first = [m.prefill(kv, p, want_logits=True) for kv, p in zip(kvs, prompts)]
    toks = np.array([t for t, _ in first], np.uint32)
    gpu_t = [[int(t)] for t in toks]
    gpu_l = [[l.copy()] for _, l in first]
    for s in range(steps):
        pos = np.array([n + s for n in lens], np.uint32)
        nxt, logits = m.decode_batch(kvs, toks, pos)
        for i in range(B):
            gpu_t[i].append(int(nxt[i]))
            gpu_l[i].append(logits[i].copy())
        toks = nxt
    for kv in kvs:
        kv.close()
    m.close()
    ctx.close()

    def ref(i):   # ctypes releases the GIL: the sequences run side by side
        r = O.OracleRun(cfg, w, max_tokens, order=O.ORDER_AVX512, threads=1)
        try:
            return r.generate(prompts[i], steps + 1, want_logits=True)
        finally:
            r.close()

    with ThreadPoolExecutor(min(B, os.cpu_count() or 1)) as ex:
        refs = list(ex.map(ref, range(B)))
    compared, worst, parted = 0, 0.0, []
    for i in range(B):
        rc, rt, margins, rl = refs[i]
        assert rc == 0
        for s in range(steps + 1):
            err = rel_l2(gpu_l[i][s], rl[s])
            worst = max(worst, err)
            assert err < 1e-2, (i, s, err)
            compared += 1
            if gpu_t[i][s] != int(rt[s]):
                assert not margins[s] > 20 * err * float(np.abs(rl[s]).max()), (i, s, float(margins[s]), err)
                parted.append((i, s))
                break
    distinct = len({t for seq in gpu_t for t in seq})
    print(f"{cfg.name} B={B} lens {min(lens)}..{max(lens)}: worst logits vs f32 path {worst:.2e}, "
          f"{compared} of {B * (steps + 1)} steps compared, parted at {parted}, {distinct} distinct ids")
    assert compared >= 0.9 * B * (steps + 1), (compared, parted)


# The weights are the tame ones (gains near 1).  The Q8_0 activation
# rounding of the batched path is a perturbation of ~0.5% per matmul; on the
# models whose greedy sequence moves (centred nibbles, gains of 2-3) the
# dynamics amplify it (the prefill's logits moved by 5.5e-2 on two layers and
# by 0.54 on 28), so those models are compared with the f32 path only on
# the f32 GPU step (test_gpu_model.py).
F32_CASES = [
    # two sequences at config-0 full size (28 layers, vocab 151936), BASELINE's distributions
    (synth.QWEN3_1_7B, [16, 23], 4, 0, dict()),
    # BASELINE config 2's batch of 16, each context past 2048 tokens, on a
    # two-layer model at config-0 widths
    (synth.small_config(n_layers=2, hidden=2048, ffn=6144, n_q=16, n_kv=8, vocab=4096),
     [2048 + 7 * i for i in range(16)], 4, 5, dict(norm_sigma=0.1)),
]


@pytest.mark.slow
@pytest.mark.parametrize("cfg,lens,steps,seed,wkw", F32_CASES,
                         ids=[f"{c.name}-b{len(l)}-ctx{max(l)}" for c, l, *_ in F32_CASES])
def test_decode_batch_matches_reference_f32_path(cfg, lens, steps, seed, wkw):
    run_f32_case(cfg, lens, steps, seed, wkw)


def test_batch_equals_sequences_alone():
    cfg = synth.small_config(n_layers=2, hidden=512, ffn=1024, n_q=8, n_kv=2, vocab=1024)
    ctx = zb.Context()
    w = synth.qwen3_weights(cfg, seed=5, norm_sigma=0.1)
    m = zb.Qwen3Model(ctx, cfg, w)
    lens = [3, 40, 300, 17, 1]
    prompts = [synth.prompt_ids(cfg, n, seed=70 + i) for i, n in enumerate(lens)]
    a = [m.new_kv(320) for _ in lens]
    b = [m.new_kv(320) for _ in lens]
    ta = np.array([m.prefill(kv, p, want_logits=False)[0] for kv, p in zip(a, prompts)], np.uint32)
    tb = np.array([m.prefill(kv, p, want_logits=False)[0] for kv, p in zip(b, prompts)], np.uint32)
    assert np.array_equal(ta, tb)
    for s in range(4):
        pos = np.array([n + s for n in lens], np.uint32)
        na, la = m.decode_batch(a, ta, pos)
        for i in range(len(lens)):
            nb, lb = m.decode_batch([b[i]], tb[i:i + 1], pos[i:i + 1])
            assert nb[0] == na[i]
            assert np.array_equal(lb[0].view(np.uint32), la[i].view(np.uint32)), (s, i)
            tb[i] = nb[0]
        ta = na
    for i, n in enumerate(lens):
        for layer in range(cfg.n_layers):
            ka, va = a[i].read(layer, n + 4)
            kb, vb = b[i].read(layer, n + 4)
            assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    for kv in a + b:
        kv.close()
    m.close()
    ctx.close()


@pytest.mark.parametrize("cfg", [synth.small_config(n_layers=2, hidden=512, ffn=1024, n_q=8, n_kv=2, vocab=1024),
                                 synth.small_config(n_layers=2, hidden=4096, ffn=12288, n_q=32, n_kv=8, vocab=2048)],
                         ids=["small", "config2-widths"])
def test_batch_equals_single_token_path(cfg):
    """Each sequence of a batch step against the per-op single-token step
    (forward_single_token + lm_head_argmax, ZGPU_FLAG_NO_PERSISTENT): the
    projections are the single-token GEMV's bit for bit; the batched
    attention reduces the q heads' scores together and takes exp by __expf,
    which moves the last bits, so logits agree to 2e-5 relative L2 and the
    tokens wherever the top-1/top-2 margin is clear."""
    ctx = zb.Context(persistent=False)
    w = synth.qwen3_weights(cfg, seed=6, norm_sigma=0.1)
    m = zb.Qwen3Model(ctx, cfg, w)
    lens = [3, 40, 17, 1, 9]
    prompts = [synth.prompt_ids(cfg, n, seed=80 + i) for i, n in enumerate(lens)]
    a = [m.new_kv(64) for _ in lens]
    b = [m.new_kv(64) for _ in lens]
    ta = np.zeros(len(lens), np.uint32)
    for i, p in enumerate(prompts):   # identical prompt caches through the single-token path
        for kvs in (a, b):
            for pos, t in enumerate(p[:-1]):
                m.forward_single_token(kvs[i], int(t), pos)
        ta[i] = p[-1]
    tb = ta.copy()
    for s in range(4):
        pos = np.array([n - 1 + s for n in lens], np.uint32)
        na, la = m.decode_batch(a, ta, pos)
        for i in range(len(lens)):
            m.forward_single_token(b[i], int(tb[i]), int(pos[i]))
            nb, lb = m.lm_head_argmax()
            err = rel_l2(la[i], lb)
            assert err < 2e-5, (s, i, err)
            if top2_gap(lb) > 20 * err * float(np.abs(lb).max()):
                assert nb == na[i], (s, i)
            tb[i] = na[i]   # both continue on the batch's token
        ta = na
    for i, n in enumerate(lens):
        for layer in range(cfg.n_layers):
            ka, va = a[i].read(layer, n + 3)
            kb, vb = b[i].read(layer, n + 3)
            assert rel_l2(ka, kb) < 2e-5 and rel_l2(va, vb) < 2e-5
    for kv in a + b:
        kv.close()
    m.close()
    ctx.close()


def test_generate_batch_runs_prefill_then_steps():
    cfg = synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512)
    ctx = zb.Context()
    w = synth.qwen3_weights(cfg, seed=9, norm_sigma=0.1)
    m = zb.Qwen3Model(ctx, cfg, w)
    prompts = np.stack([synth.prompt_ids(cfg, 12, seed=90 + i) for i in range(3)])
    kvs = [m.new_kv(40) for _ in range(3)]
    out, _ = m.generate_batch(kvs, prompts, 5)
    kv2 = [m.new_kv(40) for _ in range(3)]
    tok, _ = m.prefill_batch(kv2, prompts, want_logits=False)
    assert np.array_equal(out[:, 0], tok)
    for s in range(1, 5):
        tok, _ = m.decode_batch(kv2, tok, np.full(3, 12 + s - 1), want_logits=False)
        assert np.array_equal(out[:, s], tok)
    for kv in kvs + kv2:
        kv.close()
    m.close()
    ctx.close()


def test_decode_batch_errors():
    cfg = synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512)
    ctx = zb.Context()
    w = synth.qwen3_weights(cfg, seed=3)
    m = zb.Qwen3Model(ctx, cfg, w)
    a, b = m.new_kv(16), m.new_kv(16)
    with pytest.raises(zb.ZgpuError) as e:
        m.decode_batch([a, b], [1, 2], [3, 16])          # position at the capacity
    assert e.value.status == 10
    with pytest.raises(zb.ZgpuError) as e:
        m.decode_batch([a, a], [1, 2], [0, 1])           # one cache per sequence
    assert e.value.status == 1
    with pytest.raises(zb.ZgpuError) as e:
        m.decode_batch([a], [cfg.vocab_padded], [0])     # token beyond the vocabulary
    assert e.value.status == 1
    other = zb.KvCache(ctx, 16, cfg.n_layers, 1, cfg.head_dim)
    with pytest.raises(zb.ZgpuError):
        m.decode_batch([other], [1], [0])                # kv geometry
    toks, _ = m.decode_batch([a, b], [1, 2], [0, 0])     # a valid step still runs after the errors
    assert toks.shape == (2,)
    for kv in (a, b, other):
        kv.close()
    m.close()
    ctx.close()
