"""Steps shared by the batched DeepSeek2 decode tests (test_gpu_ds2_batch.py,
test_gpu_ep.py): per-sequence prompts of different lengths, a prefill of
each prompt through the one-token forward, then greedy steps either batched
(zgpu_ds2_decode_batch) or one sequence at a time
(zgpu_ds2_forward_single_token + zgpu_ds2_lm_head_argmax).
"""
import numpy as np

from zero_b200 import synth


def prompts_for(cfg, n_seq: int, seed: int, min_len: int = 2, max_len: int = 9):
    """n_seq prompts, lengths cycling through [min_len, max_len]."""
    span = max_len - min_len + 1
    return [synth.ds2_prompt_ids(cfg, min_len + (5 * b + seed) % span, seed=seed + 97 * b) for b in range(n_seq)]


def prefill(m, kvs, prompts):
    """Every prompt token but the last, one token at a time, into each cache."""
    for kv, p in zip(kvs, prompts):
        for pos, t in enumerate(p[:-1]):
            m.forward_single_token(kv, int(t), pos)


def run_batch(m, kvs, prompts, n_steps: int):
    """n_steps batched greedy steps from each prompt's last token: tokens
    [n_steps, n_seq], logits [n_steps, n_seq, vocab_padded], expert ids
    [n_steps, n_layers, n_seq, top_k]."""
    cur = np.array([p[-1] for p in prompts], np.uint32)
    pos = np.array([len(p) - 1 for p in prompts], np.uint32)
    toks, logits, ids = [], [], []
    for _ in range(n_steps):
        t, lg = m.decode_batch(kvs, cur, pos)
        toks.append(t.copy())
        logits.append(lg)
        ids.append(m.batch_expert_ids(len(kvs))[0])
        cur, pos = t, pos + 1
    return np.array(toks), np.array(logits), np.array(ids)


def run_single(m, kvs, prompts, n_steps: int):
    """The same steps one sequence at a time; same shapes as run_batch."""
    n = len(kvs)
    cur = [int(p[-1]) for p in prompts]
    pos = [len(p) - 1 for p in prompts]
    toks = np.zeros((n_steps, n), np.uint32)
    logits = np.zeros((n_steps, n, m.cfg.vocab_padded), np.float32)
    ids = np.zeros((n_steps, m.cfg.n_layers, n, m.cfg.top_k), np.uint32)
    for s in range(n_steps):
        for b in range(n):
            m.forward_single_token(kvs[b], cur[b], pos[b])
            ids[s, :, b] = m.expert_ids()[0]
            toks[s, b], logits[s, b] = m.lm_head_argmax()
        cur = [int(x) for x in toks[s]]
        pos = [p + 1 for p in pos]
    return toks, logits, ids
