"""A model decoded straight from a .smodel container the reference's packer
wrote (tests/golden/tiny_qwen3.smodel: Q8_0 embedding, Q8_0X4 LM head,
Q4_0X4 matmuls, F32 norms), through the C ABI, against the CPU oracle fed
the same bytes (the X4 group-blocks unpacked to plain rows): greedy tokens
identical and logits within 1e-4 relative L2, the bar of test_gpu_model.py.
The weights are the packer's own quantisation of a random F32 checkpoint,
not this project's synthetic generator."""
from pathlib import Path

import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth
from zero_b200.smodel import SmodelFile

pytestmark = pytest.mark.gpu

FIXTURE = Path(__file__).resolve().parent / "golden" / "tiny_qwen3.smodel"


def plain_weights(cfg, w):
    shapes = synth.layer_shapes(cfg)
    p = {"token_embd": np.array(w["token_embd"]), "output_norm": np.array(w["output_norm"]),
         "output": synth.unpack_x4(w["output_x4"], cfg.vocab_padded, cfg.hidden, cfg.output_quant), "layers": []}
    for lw in w["layers"]:
        d = {k: np.array(lw[k]) for k in synth.LAYER_NORMS}
        for name in synth.LAYER_MATS:
            rows, cols = shapes[name]
            d[name] = synth.unpack_x4(lw[name + "_x4"], rows, cols, "q4_0")
        p["layers"].append(d)
    return p


def test_decode_from_a_packed_container_matches_the_oracle():
    with SmodelFile(FIXTURE) as f, zb.Context() as ctx:
        assert ctx.register_smodel(f) == 16   # token_embd, 2 x 7 matmuls, output
        cfg = f.qwen3_config()
        w = f.qwen3_weights()
        m = zb.Qwen3Model(ctx, cfg, w)
        prompt = synth.prompt_ids(cfg, 6, seed=3)
        kv = m.new_kv(32)
        toks, logits = m.generate_greedy(kv, prompt, 8, want_logits=True)
        kv.close()
        m.close()
        r = O.OracleRun(cfg, plain_weights(cfg, w), 32, order=O.ORDER_AVX512)
        rc, ref_toks, _, ref_logits = r.generate(prompt, 8, want_logits=True)
        r.close()
    assert rc == 0
    assert np.array_equal(toks, ref_toks), (toks, ref_toks)
    rel = float(np.linalg.norm(logits - ref_logits) / np.linalg.norm(ref_logits))
    assert rel < 1e-4, rel
