"""CPU tests of the timed CPU baseline's machinery.

* The oracle library carries its own build of the seeded weight generator
  (zo_synth_*), so that the bench's reference arm never loads libzgpu; its
  bytes must equal libzgpu's (zgpu_synth_*) bit for bit.
* The AVX-512-order oracle runs on a persistent, pinned worker pool with the
  reference's fused dispatches (Q|K|V and gate|up as one row space,
  linear_fused_dispatch inference_avx512.rs:890-945; LM head + per-range
  argmax merged by lm_argmax_propose :1027-1044; attention heads split across
  cores, attn_heads_kernel :1459-1512).  Only row ownership changes with the
  thread count, so tokens, logits and the KV cache must be identical to the
  single-threaded run whatever the number of participants.
"""
import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from zero_b200 import synth

ROOT = Path(__file__).resolve().parents[1]


def _cpu_synth():
    name = "zero_b200_synth_cpu_test"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "zero_b200" / "synth.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    mod.use_generator(O.LIB, "zo_")
    return mod


def test_oracle_generator_equals_gpu_library_generator():
    cs = _cpu_synth()
    assert np.array_equal(cs.q4_0(3, 11, 64, 256, 0.02), synth.q4_0(3, 11, 64, 256, 0.02))
    assert np.array_equal(cs.q8_0(3, 12, 40, 128, 0.02 / 127), synth.q8_0(3, 12, 40, 128, 0.02 / 127))
    a, b = cs.f32(5, 2, 1000, 1.0, 0.1), synth.f32(5, 2, 1000, 1.0, 0.1)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(cs.tokens(9, 7, 500, 151936), synth.tokens(9, 7, 500, 151936))
    w = synth.q4_0(1, 1, 16, 96, 0.02)
    assert np.array_equal(cs.pack_x4(w, 16, 96, "q4_0"), synth.pack_x4(w, 16, 96, "q4_0"))


def test_oracle_generator_model_weights_equal():
    cfg = synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512)
    a = _cpu_synth().qwen3_weights(cfg, seed=7, x4=False, norm_sigma=0.1)
    b = synth.qwen3_weights(cfg, seed=7, x4=False, norm_sigma=0.1)
    for k in ("token_embd", "output", "output_norm"):
        assert np.array_equal(a[k].view(np.uint8), b[k].view(np.uint8)), k
    for la, lb in zip(a["layers"], b["layers"]):
        for k in la:
            assert np.array_equal(la[k].view(np.uint8), lb[k].view(np.uint8)), k


@pytest.mark.parametrize("threads", [2, 3, 5])
def test_pooled_avx512_run_is_thread_count_independent(threads):
    # 4 q heads over 2 kv heads: head splits of 1-2 per participant; 512-row
    # vocabulary: LM-head ranges of 25-64 groups
    cfg = synth.small_config(n_layers=2, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512)
    w = synth.qwen3_weights(cfg, seed=11, x4=False, norm_sigma=0.3)
    p = synth.prompt_ids(cfg, 5, seed=11)
    r1 = O.OracleRun(cfg, w, 24, order=O.ORDER_AVX512, threads=1)
    rn = O.OracleRun(cfg, w, 24, order=O.ORDER_AVX512, threads=threads)
    try:
        rc1, t1, m1, l1 = r1.generate(p, 8, want_logits=True)
        rcn, tn, mn, ln = rn.generate(p, 8, want_logits=True)
        assert rc1 == 0 and rcn == 0
        assert np.array_equal(t1, tn)
        assert np.array_equal(l1.view(np.uint32), ln.view(np.uint32))
        assert np.array_equal(r1.kv().view(np.uint32), rn.kv().view(np.uint32))
    finally:
        r1.close()
        rn.close()


def test_pooled_lm_head_ties_go_to_the_smallest_row():
    """Every LM-head row equal (one embedding row repeated, tied output):
    all logits tie, and the merged argmax must be row 0 as in the
    single-range scan, whichever participant owns it."""
    cfg = synth.small_config(n_layers=1, hidden=256, ffn=512, n_q=4, n_kv=2, vocab=512)
    w = synth.qwen3_weights(cfg, seed=2, x4=False)
    row = w["token_embd"][: 8 * 34].copy()
    w["token_embd"] = np.tile(row, cfg.vocab_padded)
    w["output"] = w["token_embd"]
    for threads in (1, 4, 7):
        r = O.OracleRun(cfg, w, 8, order=O.ORDER_AVX512, threads=threads)
        try:
            r.forward(3, 0)
            rc, tok, logits = r.lm_head()
            assert rc == 0 and tok == 0, (threads, rc, tok)
            assert np.all(logits == logits[0])
        finally:
            r.close()
