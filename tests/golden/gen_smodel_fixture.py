"""Generate the .smodel container fixture with the reference's own packer.

    python tests/golden/gen_smodel_fixture.py <directory holding silicatepack.py>

Builds a tiny Qwen3-shaped Hugging Face checkpoint (config.json + one F32
SafeTensors file, seeded weights) in a temporary directory, packs it with
SilicatePack's `pack-hf` (quant auto: Q8_0 embedding and LM head, Q4_0
matmuls; --interleave 4: the .smodel-v2 X4 layout; 4 KB payload alignment so
the file stays small) and writes

  tiny_qwen3.smodel        the container as the packer wrote it
  tiny_qwen3_smodel.json   what the packer recorded about it: the header, the
                           model fields it put in the SIDX index, and per
                           tensor its name, dtype, shape, payload offset,
                           byte length, element count and SHA-256

next to this script.  tests/test_smodel.py reads the container through the C
ABI and checks it against the JSON; nothing at test time imports the packer.
"""
from __future__ import annotations

import json
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
H, F, L, NQ, NKV, HD, V = 256, 512, 2, 2, 1, 128, 256


def write_checkpoint(d: Path) -> None:
    cfg = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": H, "intermediate_size": F,
           "num_hidden_layers": L, "num_attention_heads": NQ, "num_key_value_heads": NKV, "head_dim": HD,
           "vocab_size": V, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "max_position_embeddings": 4096,
           "tie_word_embeddings": False, "eos_token_id": 1}
    (d / "config.json").write_text(json.dumps(cfg))
    rng = np.random.default_rng(7)
    shapes = {"model.embed_tokens.weight": (V, H), "lm_head.weight": (V, H), "model.norm.weight": (H,)}
    for layer in range(L):
        p = f"model.layers.{layer}."
        shapes.update({
            p + "self_attn.q_proj.weight": (NQ * HD, H), p + "self_attn.k_proj.weight": (NKV * HD, H),
            p + "self_attn.v_proj.weight": (NKV * HD, H), p + "self_attn.o_proj.weight": (H, NQ * HD),
            p + "self_attn.q_norm.weight": (HD,), p + "self_attn.k_norm.weight": (HD,),
            p + "input_layernorm.weight": (H,), p + "post_attention_layernorm.weight": (H,),
            p + "mlp.gate_proj.weight": (F, H), p + "mlp.up_proj.weight": (F, H), p + "mlp.down_proj.weight": (H, F),
        })
    header, blobs, off = {}, [], 0
    for name, shape in shapes.items():
        a = (1.0 + 0.1 * rng.standard_normal(shape)) if len(shape) == 1 else 0.05 * rng.standard_normal(shape)
        b = a.astype("<f4").tobytes()
        header[name] = {"dtype": "F32", "shape": list(shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header).encode()
    with open(d / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        f.write(b"".join(blobs))


def main(tools_dir: str) -> None:
    sys.path.insert(0, tools_dir)
    import silicatepack as sp

    with tempfile.TemporaryDirectory() as tmp:
        d = Path(tmp) / "hf"
        d.mkdir()
        write_checkpoint(d)
        out = Path(tmp) / "tiny_qwen3.smodel"
        rc = sp.main(["pack-hf", "--input-dir", str(d), "--output", str(out), "--quant", "auto",
                      "--interleave", "4", "--payload-alignment", "4096", "--force"])
        assert rc == 0, rc
        info = sp.inspect_path(out, json_output=True)
        cfg = json.loads((d / "config.json").read_text())
        fields = sp.native_model_config_fields(cfg)
        data = out.read_bytes()
    (HERE / "tiny_qwen3.smodel").write_bytes(data)
    expected = {
        "header": {k: info["header"][k] for k in ("version", "header_len", "manifest_offset", "manifest_len",
                                                  "payload_offset", "payload_len", "payload_kind", "flags",
                                                  "payload_sha256")},
        "config": {k: v for k, v in fields.items() if k != "architecture"},
        "tensors": [{k: t[k] for k in ("name", "dtype", "shape", "payload_offset", "byte_len", "elements", "sha256")}
                    for t in info["manifest"]["tensors"]],
        "dtype_ids": {k: sp.NATIVE_DTYPE_IDS[k] for k in ("F32", "Q4_0", "Q8_0", "Q4_0X4", "Q8_0X4")},
    }
    (HERE / "tiny_qwen3_smodel.json").write_text(json.dumps(expected, indent=1) + "\n")
    print(f"wrote {len(data)} bytes, {len(expected['tensors'])} tensors")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
