"""Generate the detokenizer fixture with the reference's own vocabulary tool.

    python tests/golden/gen_vocab_fixture.py <directory holding extract_vocab.py>

Writes, next to this script:

  tiny_tokenizer.json      a seeded synthetic byte-level BPE tokenizer.json:
                           about 5 000 model tokens of 1-6 characters of the
                           GPT-2 byte alphabet (some with a character outside
                           it) at ids spread over [0, 61 000), and added
                           tokens (one overriding a model id, two past the
                           model vocab)
  tiny_vocab_bytes.bin     what extract_vocab.py wrote for it: the token
  tiny_vocab_offsets.bin   byte strings and their u32 offsets

tests/test_detok.py checks zero_b200.detok's table builder and the C-ABI
detokenizer against these files; nothing at test time runs the tool.
"""
from __future__ import annotations

import json
import random
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent


def gpt2_alphabet() -> list[str]:
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return [chr(c) for c in cs]


def make_tokenizer() -> dict:
    rng = random.Random(20261202)
    alpha = gpt2_alphabet()
    # 5 000 ids spread over [0, 61 000) (the tool's own sample decodes reach
    # id 60 792); the ids in between are absent and decode to nothing
    ids = sorted(set(rng.sample(range(61000), 4990)) | {0, 25, 40, 271, 9707, 4337, 60792})
    vocab: dict[str, int] = {}
    for tid in ids:
        while True:
            s = "".join(rng.choice(alpha) for _ in range(rng.randint(1, 6)))
            if rng.random() < 0.005:
                s += "€"                            # outside the byte alphabet: dropped
            if s not in vocab:
                break
        vocab[s] = tid
    added = [
        {"id": 9707, "content": "<|override|>"},         # replaces a model token
        {"id": max(vocab.values()) + 3, "content": "<|im_start|>"},
        {"id": max(vocab.values()) + 5, "content": "<|endoftext|>"},
    ]
    return {"version": "1.0", "added_tokens": added, "model": {"type": "BPE", "vocab": vocab}}


def main(tools_dir: str) -> None:
    tok = make_tokenizer()
    path = HERE / "tiny_tokenizer.json"
    path.write_text(json.dumps(tok, ensure_ascii=False))
    with tempfile.TemporaryDirectory() as tmp:
        b, o = Path(tmp) / "b.bin", Path(tmp) / "o.bin"
        subprocess.run([sys.executable, str(Path(tools_dir) / "extract_vocab.py"), str(path), str(b), str(o)],
                       check=True, stderr=subprocess.DEVNULL)
        (HERE / "tiny_vocab_bytes.bin").write_bytes(b.read_bytes())
        (HERE / "tiny_vocab_offsets.bin").write_bytes(o.read_bytes())
    print(f"{len(tok['model']['vocab'])} model tokens, {(HERE / 'tiny_vocab_bytes.bin').stat().st_size} bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    main(sys.argv[1])
