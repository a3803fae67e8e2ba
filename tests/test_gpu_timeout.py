"""A rank whose peer never arrives fails with a bounded device wait, on one GPU.

Rank 0 of a two-rank tensor-parallel Qwen3 model is connected with rank 1
absent (zgpu_qwen3_tp_connect_absent): rank 1's copies of the activation
vectors become local buffers that nothing reads, and the rows rank 1 owns
are never written.  The first stage that needs those rows (the O projection
after attention, which reads every rank's heads) polls tagged words that
nothing sets; its wait gives up after the kernel's limit (1 s on
%globaltimer), raises the launch's abort flag, every other wait of the launch
then fails at once, and the call returns ZGPU_ERR_DEVICE_TIMEOUT.  No fault,
trap or endless loop is involved.  Afterwards the same context decodes a
one-GPU model with the oracle's tokens, so the context stays usable.
"""
import time

import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu

DEVICE_TIMEOUT = 93   # ZGPU_ERR_DEVICE_TIMEOUT


def test_absent_peer_times_out_and_context_stays_usable(ctx):
    cfg = synth.small_config(n_layers=2, hidden=512, ffn=1024, n_q=8, n_kv=2, vocab=1024)
    w = synth.qwen3_weights(cfg, seed=3, norm_sigma=0.1)
    prompt = synth.prompt_ids(cfg, 4, seed=3)
    m = zb.Qwen3Model(ctx, cfg, w, rank=0, world=2)
    kv = m.new_kv(32)
    try:
        m.tp_connect_absent()
        t0 = time.perf_counter()
        with pytest.raises(zb.ZgpuError) as err:
            m.generate_greedy(kv, prompt, 3)
        dt = time.perf_counter() - t0
        assert err.value.status == DEVICE_TIMEOUT, err.value
        # at least one full wait limit, and the launches ran out soon after it
        assert 0.9 <= dt < 60.0, dt
        # the per-token entry points fail the same way
        with pytest.raises(zb.ZgpuError) as err:
            m.forward_single_token(kv, int(prompt[0]), 0)
        assert err.value.status == DEVICE_TIMEOUT, err.value
    finally:
        kv.close()
        m.close()
    # the context still runs a one-GPU decode, held to the CPU oracle
    m1 = zb.Qwen3Model(ctx, cfg, w)
    kv1 = m1.new_kv(32)
    try:
        toks, logits = m1.generate_greedy(kv1, prompt, 4, want_logits=True)
    finally:
        kv1.close()
        m1.close()
    r = O.OracleRun(cfg, w, 32, order=O.ORDER_AVX512)
    rc, ref_toks, _, ref_logits = r.generate(prompt, 4, want_logits=True)
    r.close()
    assert rc == 0
    assert np.array_equal(toks, ref_toks)
    assert np.linalg.norm(logits - ref_logits) / np.linalg.norm(ref_logits) < 1e-4
