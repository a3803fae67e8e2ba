"""Expert-parallel DeepSeek2 decode (BASELINE config 3's sharding) on 2-8
GPUs, one process per GPU, against the one-GPU decode of the same model.

Bar: bit-identical.  The router runs on every rank with the same inputs, each
selected expert runs on the rank that owns it with the one-GPU GEMV, its
output crosses as a copy of tagged words, and every rank's combine adds the
slots in the reference's k order (moe.rs:486-590), so greedy tokens, logits
and the per-layer expert ids equal the one-GPU run bit for bit.  The one-GPU
run is itself held to the reference's CPU path in test_gpu_ds2.py.  Skipped
where fewer GPUs are visible than the case needs.
"""
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import zero_b200 as zb
from ds2_batch_steps import prefill, prompts_for, run_batch
from zero_b200 import synth

pytestmark = pytest.mark.gpu

VARIANTS = {
    "8experts_top3_2shared": dict(n_layers=3, hidden=512, ffn=1024, n_heads=4, n_experts=8, top_k=3,
                                  expert_ffn=256, n_shared=2, vocab=1024),
    "16experts_top6_no_shared": dict(n_layers=2, hidden=1024, ffn=2048, n_heads=16, n_experts=16, top_k=6,
                                     expert_ffn=352, n_shared=0, vocab=2048),
    # every token of every MoE layer routed to rank 0's experts (router bias
    # -1e4 on the others): rank 0's combine never waits for slot data, so
    # only the arrival words keep it from running two MoE layers ahead of
    # rank 1 and overwriting slots rank 1 has not read yet
    "8experts_top3_all_on_rank0": dict(n_layers=4, hidden=512, ffn=1024, n_heads=4, n_experts=8, top_k=3,
                                       expert_ffn=256, n_shared=1, vocab=1024, router_bias=True),
}
SKEWED = {"8experts_top3_all_on_rank0"}
CASES = [(name, 2) for name in VARIANTS] + [("16experts_top6_no_shared", 4)]
PROMPT_LEN, N_GEN, MAX_TOKENS = 7, 10, 48
BATCH_SEQ, BATCH_STEPS = 6, 4


def _weights(name, cfg):
    w = synth.ds2_weights(cfg, seed=41, norm_sigma=0.1)
    if name in SKEWED:
        for lw in w["layers"]:
            if "router_b" in lw:
                lw["router_b"][cfg.n_experts // 2:] = -1e4
    return w


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _batch(m, cfg):
    """Batched steps of BATCH_SEQ sequences with prompts of different lengths."""
    prompts = prompts_for(cfg, BATCH_SEQ, 42)
    kvs = [m.new_kv(MAX_TOKENS) for _ in prompts]
    prefill(m, kvs, prompts)
    toks, logits, ids = run_batch(m, kvs, prompts, BATCH_STEPS)
    for kv in kvs:
        kv.close()
    return toks, logits, ids


def _rank(rank, world, port, name, q, batch=False):
    import torch.distributed as dist

    from zero_b200 import tp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cfg = synth.ds2_small_config(**VARIANTS[name])
        ctx = zb.Context(device=rank)
        w = _weights(name, cfg)
        m = zb.Ds2Model(ctx, cfg, w, rank=rank, world=world)
        tp.connect(m)
        if batch:
            toks, logits, ids = _batch(m, cfg)
        else:
            prompt = synth.ds2_prompt_ids(cfg, PROMPT_LEN, seed=41)
            kv = m.new_kv(MAX_TOKENS)
            toks, logits = m.generate_greedy(kv, prompt, N_GEN, want_logits=True)
            ids, _ = m.expert_ids()
            kv.close()
        dist.barrier()
        m.close()
        ctx.close()
        q.put((rank, toks, logits, ids, None))
    except Exception as e:   # reported to the test, which fails
        q.put((rank, None, None, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _spawn(name, world, batch):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, name, q, batch)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            r, toks, logits, ids, err = q.get(timeout=600)
            res[r] = (toks, logits, ids, err)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert res[r][3] is None, res[r][3]
    return res


@pytest.mark.parametrize("name,world", CASES, ids=[f"{n}-ep{w}" for n, w in CASES])
def test_expert_parallel_decode_equals_one_gpu(name, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(name, world, False)
    cfg = synth.ds2_small_config(**VARIANTS[name])
    c1 = zb.Context(device=0)
    m1 = zb.Ds2Model(c1, cfg, _weights(name, cfg))
    kv = m1.new_kv(MAX_TOKENS)
    ref_toks, ref_logits = m1.generate_greedy(kv, synth.ds2_prompt_ids(cfg, PROMPT_LEN, seed=41), N_GEN,
                                              want_logits=True)
    ref_ids, _ = m1.expert_ids()
    kv.close()
    m1.close()
    c1.close()
    for r in range(world):
        toks, logits, ids, _ = res[r]
        assert np.array_equal(toks, ref_toks), (r, toks, ref_toks)
        assert np.array_equal(logits.view(np.uint32), ref_logits.view(np.uint32)), r
        assert np.array_equal(np.asarray(ids), np.asarray(ref_ids)), r
    if name in SKEWED:   # the routing really was all on rank 0
        moe = np.asarray(ref_ids)[cfg.n_dense:]
        assert moe.size and (moe < cfg.n_experts // world).all(), moe


BATCH_CASES = [("8experts_top3_2shared", 2), ("8experts_top3_all_on_rank0", 2), ("16experts_top6_no_shared", 4)]


@pytest.mark.parametrize("name,world", BATCH_CASES, ids=[f"{n}-ep{w}" for n, w in BATCH_CASES])
def test_expert_parallel_batch_equals_one_gpu(name, world):
    """zgpu_ds2_decode_batch with the experts sharded: every rank's tokens,
    logits and expert ids equal the one-GPU batch bit for bit (each rank runs
    its experts for every token that selected them; the outputs of all
    tokens cross in one publish per MoE layer)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _spawn(name, world, True)
    cfg = synth.ds2_small_config(**VARIANTS[name])
    c1 = zb.Context(device=0)
    m1 = zb.Ds2Model(c1, cfg, _weights(name, cfg))
    ref_toks, ref_logits, ref_ids = _batch(m1, cfg)
    m1.close()
    c1.close()
    for r in range(world):
        toks, logits, ids, _ = res[r]
        assert np.array_equal(toks, ref_toks), (r, toks, ref_toks)
        assert np.array_equal(logits.view(np.uint32), ref_logits.view(np.uint32)), r
        assert np.array_equal(ids[:, cfg.n_dense:], ref_ids[:, cfg.n_dense:]), r
