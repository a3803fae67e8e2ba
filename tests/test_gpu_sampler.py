"""Top-K + temperature sampling on the GPU (zgpu_sample_top_k,
zgpu_lm_head_sample) against the CPU oracle of sampler.rs:41-163: the
sampled token and the advanced xorshift64 state are bit-identical, over the
oracle's pinned cases (ties, -inf, NaN, short vocabularies, the vocab_real
cut), a full-size 151936-wide vector, and a model's own LM-head logits."""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

from test_sampler import CASES

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("i", range(len(CASES)))
def test_gpu_sampler_matches_oracle(ctx, i):
    logits, temp, st, vr = CASES[i]
    for _ in range(4):
        got = ctx.sample_top_k(logits, st, temp, vr)
        want = O.lm_head_sample(logits, st, temp, vr)
        assert got == want
        st = got[1]


def test_gpu_sampler_full_vocab(ctx):
    rng = np.random.default_rng(21)
    logits = (rng.standard_normal(151936) * 4).astype(np.float32)
    st = O.rng_seed(2024)
    for temp in (0.7, 1.0):
        for _ in range(5):
            got = ctx.sample_top_k(logits, st, temp)
            assert got == O.lm_head_sample(logits, st, temp)
            st = got[1]


def test_lm_head_sample_on_the_models_logits():
    cfg = synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512)
    w = synth.qwen3_weights(cfg, seed=9, norm_sigma=0.1)
    with zb.Context() as ctx:
        m = zb.Qwen3Model(ctx, cfg, w)
        kv = m.new_kv(16)
        for pos, t in enumerate(synth.prompt_ids(cfg, 4, seed=9)):
            m.forward_single_token(kv, int(t), pos)
        _, logits = m.lm_head_argmax(want_logits=True)
        st = O.rng_seed(77)
        for _ in range(3):
            got = m.lm_head_sample(st, 0.7)
            assert got == O.lm_head_sample(logits, st, 0.7, cfg.vocab_real)
            st = got[1]
        kv.close()
        m.close()
