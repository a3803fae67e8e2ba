"""Token ids -> text bytes for streaming output (the kernel's detokenizer,
kernel/src/detokenizer.rs), over the C-ABI zgpu_detok_* tables.

vocab_tables() builds the two tables from a Hugging Face tokenizer.json the
way the reference's tools/extract_vocab.py does: every id up to the largest
model or added-token id gets an entry; model tokens are byte-level BPE
strings mapped back to bytes through the GPT-2 byte alphabet (characters
outside it are dropped), added tokens are taken as UTF-8 text and replace a
model token of the same id, absent ids are empty.
"""
from __future__ import annotations

import ctypes as C
import json
from pathlib import Path

import numpy as np

from ._lib import LIB


def byte_decoder() -> dict[str, int]:
    """The GPT-2 byte-level alphabet, inverted: character -> byte.  Bytes
    '!'..'~', '¡'..'¬' and '®'..'ÿ' stand for themselves; the other 68 take
    the characters from U+0100 upwards in byte order."""
    keep = [*range(0x21, 0x7F), *range(0xA1, 0xAD), *range(0xAE, 0x100)]
    dec = {chr(b): b for b in keep}
    extra = 0
    for b in range(256):
        if b not in dec.values():
            dec[chr(0x100 + extra)] = b
            extra += 1
    return dec


def vocab_tables(tokenizer) -> tuple[bytes, np.ndarray]:
    """(byte table, u32 offsets [vocab + 1]) of a tokenizer.json (path or parsed dict)."""
    if not isinstance(tokenizer, dict):
        tokenizer = json.loads(Path(tokenizer).read_text(encoding="utf-8"))
    vocab = tokenizer.get("model", {}).get("vocab", {})
    if not vocab:
        raise ValueError("tokenizer.json has no model vocab")
    added = {t["id"]: t["content"] for t in tokenizer.get("added_tokens", [])}
    size = max(max(vocab.values()), max(added, default=0)) + 1
    text = {i: s for s, i in vocab.items()}
    text.update(added)
    dec = byte_decoder()
    table = bytearray()
    offsets = np.zeros(size + 1, np.uint32)
    for i in range(size):
        s = text.get(i, "")
        if s and i in added:
            table += s.encode("utf-8")
        elif s:
            table += bytes(dec[c] for c in s if c in dec)
        offsets[i + 1] = len(table)
    return bytes(table), offsets


class Detokenizer:
    """zgpu_detok: the tables copied once, then bytes per token id."""

    def __init__(self, table: bytes, offsets: np.ndarray):
        offsets = np.ascontiguousarray(offsets, np.uint32)
        if offsets.size < 2:
            raise ValueError("offsets need vocab_size + 1 >= 2 entries")
        buf = (C.c_uint8 * max(len(table), 1)).from_buffer_copy(bytes(table) or b"\0")
        h = C.c_void_p()
        st = LIB.zgpu_detok_create(buf, len(table), offsets.ctypes.data, offsets.size - 1, C.byref(h))
        if st:
            raise ValueError(f"zgpu_detok_create failed: {st}")
        self.h = h

    @classmethod
    def from_tokenizer_json(cls, tokenizer) -> "Detokenizer":
        return cls(*vocab_tables(tokenizer))

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_detok_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def __len__(self) -> int:
        return LIB.zgpu_detok_vocab_size(self.h)

    def token(self, token_id: int) -> bytes:
        p = C.POINTER(C.c_uint8)()
        n = C.c_uint64()
        if LIB.zgpu_detok_token(self.h, token_id, C.byref(p), C.byref(n)):
            raise ValueError("zgpu_detok_token failed")
        return C.string_at(p, n.value) if n.value else b""

    def decode(self, ids) -> bytes:
        ids = np.ascontiguousarray(ids, np.uint32)
        need = C.c_uint64()
        LIB.zgpu_detok_decode(self.h, ids.ctypes.data, ids.size, None, 0, C.byref(need))
        out = (C.c_uint8 * max(need.value, 1))()
        st = LIB.zgpu_detok_decode(self.h, ids.ctypes.data, ids.size, out, need.value, C.byref(need))
        if st:
            raise ValueError(f"zgpu_detok_decode failed: {st}")
        return bytes(out)[:need.value]
