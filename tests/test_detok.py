"""The detokenizer (zgpu_detok_*, zero_b200/csrc/detok.cpp; zero_b200.detok)
on CPU, against tables written by the reference's own tools/extract_vocab.py
(tests/golden/gen_vocab_fixture.py ran it on tests/golden/tiny_tokenizer.json).

  * vocab_tables() rebuilds the reference tool's byte and offset tables bit
    for bit (model tokens through the GPT-2 byte alphabet, added tokens as
    UTF-8 overriding a model id, absent ids empty, characters outside the
    alphabet dropped);
  * the C-ABI lookup returns each id's slice of those tables, the batch
    decode their concatenation, and follows decode_token's empty-slice rules
    (detokenizer.rs:110-205) for ids past the vocabulary and for offsets that
    run backwards or past the byte table.
"""
from pathlib import Path

import numpy as np
import pytest

from zero_b200 import detok

GOLDEN = Path(__file__).resolve().parent / "golden"
REF_BYTES = (GOLDEN / "tiny_vocab_bytes.bin").read_bytes()
REF_OFFSETS = np.fromfile(GOLDEN / "tiny_vocab_offsets.bin", "<u4")


def test_tables_equal_the_reference_tool():
    table, offsets = detok.vocab_tables(GOLDEN / "tiny_tokenizer.json")
    assert table == REF_BYTES
    assert np.array_equal(offsets, REF_OFFSETS)


def test_byte_alphabet_is_a_bijection():
    dec = detok.byte_decoder()
    assert len(dec) == 256 and sorted(dec.values()) == list(range(256))
    assert all(dec[chr(b)] == b for b in range(0x21, 0x7F))       # printable ASCII stands for itself
    assert dec["Ġ"] == 0x20 and dec["Ċ"] == 0x0A                  # the familiar space and newline


def test_lookup_and_decode_follow_the_tables():
    d = detok.Detokenizer(REF_BYTES, REF_OFFSETS)
    assert len(d) == REF_OFFSETS.size - 1
    rng = np.random.default_rng(1)
    ids = rng.integers(0, len(d), 3000)
    for i in ids[:500]:
        assert d.token(int(i)) == REF_BYTES[REF_OFFSETS[i]:REF_OFFSETS[i + 1]]
    assert d.decode(ids) == b"".join(REF_BYTES[REF_OFFSETS[i]:REF_OFFSETS[i + 1]] for i in ids)
    assert d.token(9707) == b"<|override|>"                      # added token over a model id
    assert d.token(len(d)) == b"" and d.token(2**32 - 1) == b""  # past the vocabulary
    assert d.decode([]) == b""


def test_inconsistent_offsets_decode_to_nothing():
    table = b"abcdef"
    offsets = np.array([0, 2, 1, 4, 99], np.uint32)   # id 1 runs backwards, id 3 past the table
    d = detok.Detokenizer(table, offsets)
    assert [d.token(i) for i in range(4)] == [b"ab", b"", b"bcd", b""]
    assert d.decode([0, 1, 2, 3, 0]) == b"abbcdab"


def test_small_output_buffer_and_empty_vocab_are_refused():
    from zero_b200._lib import LIB
    import ctypes as C

    d = detok.Detokenizer(b"xyz", np.array([0, 3], np.uint32))
    ids = np.array([0, 0], np.uint32)
    out = (C.c_uint8 * 4)()
    need = C.c_uint64()
    assert LIB.zgpu_detok_decode(d.h, ids.ctypes.data, 2, out, 4, C.byref(need)) == 1
    assert need.value == 6
    with pytest.raises(ValueError):
        detok.Detokenizer(b"", np.array([0], np.uint32))        # vocab_size 0
