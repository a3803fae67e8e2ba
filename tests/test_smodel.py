"""The .smodel container reader (zgpu_smodel_*, zero_b200/csrc/smodel.cpp) on
CPU, against a container written by the reference's own packer
(tests/golden/gen_smodel_fixture.py runs SilicatePack's pack-hf and records
what the packer wrote).

  * every header field, SIDX model field and tensor record (name, dtype id,
    shape, payload offset, byte length, elements) equals the packer's record,
    and the SHA-256 of each tensor's mapped bytes equals the packer's;
  * malformed containers are refused with the reference loader's error
    classes (model_loader.rs:256-661): MagicMismatch, UnsupportedFormat,
    InvalidContainer;
  * the X4 group-block unpacking used to feed the CPU oracle inverts the packer.
"""
import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from zero_b200 import synth
from zero_b200.smodel import SmodelError, SmodelFile

GOLDEN = Path(__file__).resolve().parent / "golden"
FIXTURE = GOLDEN / "tiny_qwen3.smodel"
EXPECTED = json.loads((GOLDEN / "tiny_qwen3_smodel.json").read_text())
MAGIC, UNSUPPORTED, INVALID, IO = 50, 51, 52, 53


def test_reader_matches_the_packers_record():
    with SmodelFile(FIXTURE) as f:
        h = EXPECTED["header"]
        for k in ("version", "manifest_offset", "manifest_len", "payload_offset", "payload_len", "payload_kind",
                  "flags"):
            assert f.info[k] == h[k], k
        for k, v in EXPECTED["config"].items():
            if isinstance(v, float):
                assert f.info[k] == np.float32(v), k
            else:
                assert f.info[k] == v, k
        ids = EXPECTED["dtype_ids"]
        assert len(f.tensors) == len(EXPECTED["tensors"])
        for t, e in zip(f.tensors, EXPECTED["tensors"]):
            assert t.name == e["name"]
            assert t.dtype == ids[e["dtype"]], t.name
            assert list(t.shape) == e["shape"], t.name
            assert (t.payload_offset, t.byte_len, t.elements) == (e["payload_offset"], e["byte_len"], e["elements"])
            assert hashlib.sha256(f.raw(t).tobytes()).hexdigest() == e["sha256"], t.name
        assert f.manifest()["tensor_count"] == len(f.tensors)
    data = FIXTURE.read_bytes()
    po, pl = EXPECTED["header"]["payload_offset"], EXPECTED["header"]["payload_len"]
    assert hashlib.sha256(data[po:po + pl]).hexdigest() == EXPECTED["header"]["payload_sha256"]


def test_qwen3_view_of_the_container():
    with SmodelFile(FIXTURE) as f:
        cfg = f.qwen3_config()
        assert (cfg.n_layers, cfg.hidden, cfg.ffn, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim) == (2, 256, 512, 2, 1, 128)
        assert (cfg.vocab_padded, cfg.embd_quant, cfg.output_quant) == (256, "q8_0", "q8_0")
        w = f.qwen3_weights()
        assert w["token_embd"].size == 256 * 8 * 34
        assert w["output_x4"].size == 256 * 8 * 34
        assert sorted(w["layers"][1]) == sorted([m + "_x4" for m in synth.LAYER_MATS] + list(synth.LAYER_NORMS))
        assert w["layers"][0]["q_norm"].dtype == np.float32 and w["layers"][0]["q_norm"].size == 128


@pytest.mark.parametrize("quant,rows,cols", [("q4_0", 64, 256), ("q8_0", 8, 128)])
def test_unpack_x4_inverts_the_packer(quant, rows, cols):
    plain = synth.q4_0(3, 1, rows, cols, 0.02) if quant == "q4_0" else synth.q8_0(3, 1, rows, cols, 0.01)
    assert np.array_equal(synth.unpack_x4(synth.pack_x4(plain, rows, cols, quant), rows, cols, quant), plain)


def _u32(b: bytearray, off: int, v: int):
    struct.pack_into("<I", b, off, v)


def _u64(b: bytearray, off: int, v: int):
    struct.pack_into("<Q", b, off, v)


PO = EXPECTED["header"]["payload_offset"]
ENTRY0 = PO + 128


def _names_offset(b: bytes) -> int:
    return struct.unpack_from("<I", b, PO + 20)[0]


MUTATIONS = {
    "magic": (lambda b: _u32(b, 0, 0x46554747), MAGIC),
    "version_3": (lambda b: _u32(b, 4, 3), UNSUPPORTED),
    "header_len": (lambda b: _u32(b, 8, 64), UNSUPPORTED),
    "gguf_compat_payload": (lambda b: _u32(b, 44, 1), UNSUPPORTED),
    "unknown_payload_kind": (lambda b: _u32(b, 44, 7), UNSUPPORTED),
    "empty_manifest": (lambda b: _u64(b, 20, 0), INVALID),
    "payload_past_eof": (lambda b: _u64(b, 36, EXPECTED["header"]["payload_len"] + 4096), INVALID),
    "flagged_2mib_alignment": (lambda b: _u32(b, 48, 1), INVALID),
    "sidx_magic": (lambda b: _u32(b, PO, 0x0), UNSUPPORTED),
    "sidx_version": (lambda b: _u32(b, PO + 4, 2), UNSUPPORTED),
    "tensor_count_cap": (lambda b: _u32(b, PO + 12, 10001), INVALID),
    "entry_size": (lambda b: _u32(b, PO + 16, 96), UNSUPPORTED),
    "rank_9": (lambda b: _u32(b, ENTRY0 + 12, 9), INVALID),
    "unknown_dtype": (lambda b: _u32(b, ENTRY0 + 8, 99), UNSUPPORTED),
    "tensor_past_payload": (lambda b: _u64(b, ENTRY0 + 88, 1 << 40), INVALID),
    "x4_rows_not_multiple_of_4": (lambda b: _u64(b, ENTRY0 + 2 * 104 + 16, 255), INVALID),
    "name_not_utf8": (lambda b: b.__setitem__(PO + _names_offset(b), 0xFF), INVALID),
}


@pytest.mark.parametrize("name", list(MUTATIONS))
def test_malformed_containers_are_refused(tmp_path, name):
    mutate, status = MUTATIONS[name]
    b = bytearray(FIXTURE.read_bytes())
    mutate(b)
    p = tmp_path / "bad.smodel"
    p.write_bytes(bytes(b))
    with pytest.raises(SmodelError) as ei:
        SmodelFile(p)
    assert ei.value.status == status, (name, ei.value)


def test_truncated_and_missing_files(tmp_path):
    p = tmp_path / "short.smodel"
    p.write_bytes(FIXTURE.read_bytes()[:100])
    with pytest.raises(SmodelError) as ei:
        SmodelFile(p)
    assert ei.value.status == INVALID
    with pytest.raises(SmodelError) as ei:
        SmodelFile(tmp_path / "absent.smodel")
    assert ei.value.status == IO
