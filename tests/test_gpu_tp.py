"""Tensor-parallel decode (BASELINE config 2's sharding) on 2-8 GPUs, one
process per GPU, against the one-GPU decode of the same model.

Bar: bit-identical.  Each rank reduces its output rows exactly as the
one-GPU step does (same K-chunk order, same RMSNorm), the all-gather is a
copy of tagged words, and the LM head's argmax merge keeps the smaller row on
ties, so the greedy tokens and the logits (the ranks' vocabulary slices
concatenated) equal the one-GPU run bit for bit.  The one-GPU run is itself
held to the reference's CPU path in test_gpu_model.py.  Skipped where fewer
GPUs are visible than the case needs.
"""
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu

CASES = [
    (dict(n_layers=2, hidden=512, ffn=1024, n_q=8, n_kv=2, vocab=1024), 2),
    # BASELINE config 0 widths (Qwen3-1.7B: hidden 2048, FFN 6144, 16 q / 8 kv heads), the
    # shapes bench.py --gpus N shards
    (dict(n_layers=2, hidden=2048, ffn=6144, n_q=16, n_kv=8, vocab=2048), 2),
    (dict(n_layers=2, hidden=2048, ffn=6144, n_q=16, n_kv=8, vocab=2048), 4),
    (dict(n_layers=2, hidden=2048, ffn=6144, n_q=16, n_kv=8, vocab=2048), 8),
    # BASELINE config 2 widths (Qwen3-8B: hidden 4096, FFN 12288, 32 q / 8 kv heads)
    (dict(n_layers=2, hidden=4096, ffn=12288, n_q=32, n_kv=8, vocab=2048), 2),
    (dict(n_layers=2, hidden=4096, ffn=12288, n_q=32, n_kv=8, vocab=2048), 4),
    (dict(n_layers=2, hidden=4096, ffn=12288, n_q=32, n_kv=8, vocab=2048), 8),
]
PROMPT_LEN, N_GEN, MAX_TOKENS = 7, 12, 64


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, cfg_kw, q):
    import torch.distributed as dist

    from zero_b200 import tp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = synth.small_config(**cfg_kw)
        ctx = zb.Context(device=rank)
        w = synth.qwen3_weights(cfg, seed=7, norm_sigma=0.1)
        m = zb.Qwen3Model(ctx, cfg, w, rank=rank, world=world)
        tp.connect(m)
        prompt = synth.prompt_ids(cfg, PROMPT_LEN, seed=7)
        kv = m.new_kv(MAX_TOKENS)
        toks, logits = m.generate_greedy(kv, prompt, N_GEN, want_logits=True)    # a launch per step
        kv2 = m.new_kv(MAX_TOKENS)
        toks2, _ = m.generate_greedy(kv2, prompt, N_GEN)                          # one launch
        launches = m.perf()["decode_launches"]
        # token by token through the per-token entry points, every rank in step
        kv3 = m.new_kv(MAX_TOKENS)
        for i, t in enumerate(prompt):
            m.forward_single_token(kv3, int(t), i)
        tok, lg = m.lm_head_argmax(want_logits=True)
        toks3, logits3 = [tok], [lg]
        for s in range(1, N_GEN):
            m.forward_single_token(kv3, tok, PROMPT_LEN + s - 1)
            tok, lg = m.lm_head_argmax(want_logits=True)
            toks3.append(tok)
            logits3.append(lg)
        assert np.array_equal(np.array(toks3, np.uint32), toks), (toks3, toks)
        assert np.array_equal(np.stack(logits3).view(np.uint32), logits.view(np.uint32))
        dist.barrier()
        kv.close()
        kv2.close()
        kv3.close()
        m.close()
        ctx.close()
        q.put((rank, toks, logits, toks2, launches, None))
    except Exception as e:   # reported to the test, which fails
        q.put((rank, None, None, None, 0, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg_kw,world", CASES, ids=[f"h{c['hidden']}-q{c['n_q']}-tp{w}" for c, w in CASES])
def test_tensor_parallel_decode_equals_one_gpu(cfg_kw, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, cfg_kw, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, toks, logits, toks2, launches, err = q.get(timeout=600)
            res[r] = (toks, logits, toks2, launches, err)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert res[r][4] is None, res[r][4]
    # the one-GPU decode of the same model
    cfg = synth.small_config(**cfg_kw)
    c1 = zb.Context(device=0)
    m1 = zb.Qwen3Model(c1, cfg, synth.qwen3_weights(cfg, seed=7, norm_sigma=0.1))
    kv = m1.new_kv(MAX_TOKENS)
    ref_toks, ref_logits = m1.generate_greedy(kv, synth.prompt_ids(cfg, PROMPT_LEN, seed=7), N_GEN,
                                              want_logits=True)
    kv.close()
    m1.close()
    c1.close()
    for r in range(world):
        toks, _, toks2, launches, _ = res[r]
        assert np.array_equal(toks, ref_toks), (r, toks, ref_toks)
        assert np.array_equal(toks2, ref_toks)
        assert launches == 1   # the decode steps ran as one persistent launch per GPU
    tp_logits = np.concatenate([res[r][1] for r in range(world)], axis=1)
    assert tp_logits.shape == ref_logits.shape
    assert np.array_equal(tp_logits.view(np.uint32), ref_logits.view(np.uint32))
