"""Generate the packer golden fixtures from the reference's own tools/silicatepack.py.

Run where the reference tree is available (--reference PATH, the directory
holding tools/silicatepack.py's checkout).  Writes tests/golden/packer_golden.npz, which the CPU tests
use to pin the oracle's block encoders, fp16 conversion and X4 permutation
(and, through the oracle, the GPU quantiser).  The fixture is committed; the
tests never read the reference tree.

    python tests/golden/gen_packer_golden.py --reference <reference checkout>
"""
from __future__ import annotations

import argparse
import hashlib
import io
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "packer_golden.npz"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (holds tools/silicatepack.py)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "tools"))
    import silicatepack as sp  # the reference's packer, imported read-only

    rng = np.random.default_rng(20261201)

    # fp16 conversion of doubles (float_to_fp16_bytes), including edges.
    edges = [0.0, -0.0, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 6.1035156e-05,
             6.0e-08, 5.9604645e-08, 2.98e-08, 2.9802322387695312e-08, 1e-10, 0.333333333,
             1.0009765625, 1.00048828125, 1.00146484375, float("nan"), float("inf")]
    vals = np.concatenate([np.array(edges), rng.standard_normal(200) * 10.0 ** rng.integers(-8, 5, 200)])
    fp16 = np.array([struct.unpack("<H", sp.float_to_fp16_bytes(float(v)))[0] for v in vals], np.uint16)

    # Block encoders on f32-representable inputs (what the packer sees from
    # an F32 checkpoint): random blocks plus edge blocks.
    def blocks(n):
        out = []
        for i in range(n):
            scale = 10.0 ** rng.uniform(-4, 2)
            out.append((rng.standard_normal(32) * scale).astype(np.float32))
        z = np.zeros(32, np.float32)
        out.append(z.copy())                                   # all zero
        e = z.copy(); e[0] = -8.0; e[1] = 4.0; e[2] = 1.0; out.append(e)   # test_silicatepack.py:283
        e = z.copy(); e[0] = 8.0; e[1] = -4.0; out.append(e)               # :297
        e = z.copy(); e[5] = 3.0e-7; out.append(e)             # tiny single value (fp16 subnormal d)
        e = np.linspace(-1, 1, 32).astype(np.float32); out.append(e)
        e = np.full(32, 0.5, np.float32); e[0] = 127.0; out.append(e)     # exact ties for q8
        e = (np.arange(32, dtype=np.float32) - 16.0) * 0.25; out.append(e)
        e = np.full(32, 1.0e6, np.float32); out.append(e)      # d above fp16 max (q8 clamp)
        return np.stack(out)

    xb = blocks(96)
    q4 = np.stack([np.frombuffer(sp.quantize_q4_0_block(tuple(float(v) for v in b)), np.uint8) for b in xb])
    q8 = np.stack([np.frombuffer(sp.quantize_q8_0_block(tuple(float(v) for v in b)), np.uint8) for b in xb])

    # X4 permutation through the packer's writer (as its own unit test does).
    rows, cols = 12, 96
    src_vals = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    data = src_vals.tobytes()
    outs = {}
    with tempfile.TemporaryDirectory() as tmp:
        p = Path(tmp) / "w.bin"
        p.write_bytes(data)
        src = sp.TensorSource(name="blk.0.attn_q.weight", dtype="F32", shape=(rows, cols), file=p,
                              data_begin=0, data_end=len(data), file_data_offset=0)
        for t in ("q4_0", "q4_0x4", "q8_0", "q8_0x4"):
            buf = io.BytesIO()
            sp.write_transformed_tensor(src=src, dst=buf, payload_hash=hashlib.sha256(), transform=t)
            outs[t] = np.frombuffer(buf.getvalue(), np.uint8)

    np.savez_compressed(
        OUT, fp16_in=vals, fp16_out=fp16, blocks_in=xb, q4_0=q4, q8_0=q8,
        x4_src=src_vals, x4_rows=np.int64(rows), x4_cols=np.int64(cols),
        plain_q4_0=outs["q4_0"], x4_q4_0=outs["q4_0x4"], plain_q8_0=outs["q8_0"], x4_q8_0=outs["q8_0x4"])
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
