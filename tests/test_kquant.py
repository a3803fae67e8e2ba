"""GGUF K-quant restatement in the CPU oracle (Q4_K / Q6_K), pinned three ways:

  * the known-answer blocks of the reference's own tests
    (zero-gguf-parser/src/dequant.rs:664-830 for Q4_K, :1093-1295 for Q6_K),
    held exactly (every expected value is representable);
  * an independent vectorised numpy restatement of dequant_q4k_block and
    dequant_q6k_block (dequant.rs:98-138, :328-360), bit-exact on random
    blocks (numpy rounds every float32 product and difference on its own, as
    the reference's scalar Rust does);
  * linear_q4k / linear_q6k (zero-llm-inference/src/ops.rs:179-292): the
    oracle equals a sequential float32 sum over the dequantised row
    bit-for-bit, and sits within in_dim * 2^-24 * sum|x w| of float64.
"""
import numpy as np
import pytest

import oracle as O
from zero_b200 import synth


def q4k_block(d: int, dmin: int, scales=None, qs=None) -> bytes:
    """dequant.rs:664 build_q4k_block: d, dmin as fp16 bit patterns."""
    b = bytearray(144)
    b[0:2] = d.to_bytes(2, "little")
    b[2:4] = dmin.to_bytes(2, "little")
    b[4:16] = bytes(scales or [0] * 12)
    b[16:144] = bytes(qs or [0] * 128)
    return bytes(b)


def q6k_block(ql=None, qh=None, scales=None, d: int = 0) -> bytes:
    """dequant.rs:1099 build_q6k_block."""
    b = bytearray(210)
    b[0:128] = bytes(ql or [0] * 128)
    b[128:192] = bytes(qh or [0] * 64)
    b[192:208] = bytes((s & 0xFF) for s in (scales or [0] * 16))
    b[208:210] = d.to_bytes(2, "little")
    return bytes(b)


# ------------------------------------------------- reference known answers
def test_q4k_known_answers():
    deq = lambda blk: O.dequant_kquant_block(blk, "q4_k")
    assert np.all(deq(q4k_block(0, 0)) == 0.0)                         # zero d, zero dmin
    sc = [1, 1, 1, 1, 1, 1, 1, 1, 0x11, 0x11, 0x11, 0x11]
    assert np.all(deq(q4k_block(0x3C00, 0x3800, sc)) == -0.5)          # zero quants, min 1
    sc = [1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1]
    assert np.all(deq(q4k_block(0x3C00, 0, sc, [0xFF] * 128)) == 15.0)  # max quants
    sc = [3, 5, 0, 0, 2, 4, 0, 0, 0, 0, 0, 0]
    out = deq(q4k_block(0x4000, 0x3C00, sc, [0x73] + [0] * 127))
    assert out[0] == 16.0 and out[32] == 66.0                          # 2*3*3-1*2, 2*5*7-1*4
    sc = [0, 0, 0, 0, 10, 10, 10, 10, 0xA0, 0xA0, 0xA0, 0xA0]
    assert np.all(deq(q4k_block(0, 0x4000, sc)) == -20.0)              # min dominates
    assert np.all(deq(q4k_block(0x3C00, 0, None, [0xFF] * 128)) == 0.0)  # zero scales
    b0 = q4k_block(0x3C00, 0, [2] + [0] * 11, [0x05] + [0] * 127)
    b1 = q4k_block(0x3800, 0, [4] + [0] * 11, [0x03] + [0] * 127)
    assert deq(b0)[0] == 10.0 and deq(b1)[0] == 6.0                    # row of distinct blocks


def test_q6k_known_answers():
    deq = lambda blk: O.dequant_kquant_block(blk, "q6_k")
    assert np.all(deq(q6k_block()) == 0.0)
    out = deq(q6k_block(scales=[2] + [0] * 15, d=0x3C00))
    assert np.all(out[:16] == -64.0) and np.all(out[16:32] == 0.0)     # quant -32, scale 2
    assert np.all(deq(q6k_block([0xFF] * 128, [0xFF] * 64, [1] * 16, 0x3C00)) == 31.0)
    out = deq(q6k_block([0x05] + [0] * 127, [0x01] + [0] * 63, [3] + [0] * 15, 0x4000))
    assert out[0] == -66.0                                             # 2*3*((1<<4|5)-32)
    assert deq(q6k_block(scales=[-4] + [0] * 15, d=0x3C00))[0] == 128.0  # negative scale


# ------------------------------------------- independent numpy restatement
def np_q4k(blocks: np.ndarray) -> np.ndarray:
    n = blocks.shape[0]
    d = blocks[:, 0:2].copy().view("<f2").astype(np.float32)
    dmin = blocks[:, 2:4].copy().view("<f2").astype(np.float32)
    s = blocks[:, 4:16].astype(np.uint32)
    sc = np.empty((n, 8), np.uint32)
    mn = np.empty((n, 8), np.uint32)
    sc[:, :4], mn[:, :4] = s[:, 0:4] & 63, s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    qs = blocks[:, 16:].reshape(n, 4, 1, 32)
    q = np.concatenate([qs & 15, qs >> 4], axis=2).astype(np.float32)    # [g][half][l]
    dd = d[:, :, None] * sc.reshape(n, 4, 2).astype(np.float32)
    mm = dmin[:, :, None] * mn.reshape(n, 4, 2).astype(np.float32)
    return (dd[..., None] * q - mm[..., None]).reshape(n, 256)


def np_q6k(blocks: np.ndarray) -> np.ndarray:
    n = blocks.shape[0]
    ql = blocks[:, 0:128].reshape(n, 2, 64)
    qh = blocks[:, 128:192].reshape(n, 2, 32)
    sc = blocks[:, 192:208].view(np.int8).reshape(n, 2, 4, 2)
    d = blocks[:, 208:210].copy().view("<f2").astype(np.float32)[:, 0]
    a, b = ql[:, :, :32], ql[:, :, 32:]
    q = np.stack([(a & 15) | ((qh & 3) << 4), (b & 15) | (((qh >> 2) & 3) << 4),
                  (a >> 4) | (((qh >> 4) & 3) << 4), (b >> 4) | (((qh >> 6) & 3) << 4)], axis=2)
    q = q.astype(np.int32) - 32                                          # [half][k][l]
    s = sc[:, :, :, np.arange(32) // 16].astype(np.float32)
    return ((d[:, None, None, None] * s) * q.astype(np.float32)).reshape(n, 256)


@pytest.mark.parametrize("quant", ["q4_k", "q6_k"])
def test_oracle_dequant_matches_numpy_restatement(quant):
    bb = 144 if quant == "q4_k" else 210
    blocks = synth.kquant(5, 64, 256, quant).reshape(64, bb)
    if quant == "q4_k":   # also subnormal and large fp16 scales
        blocks[0, 0:4] = np.array([1e-7, 3.0], "<f2").view(np.uint8)
        blocks[1, 0:4] = np.array([-2.5, 6e-6], "<f2").view(np.uint8)
    else:
        blocks[0, 208:210] = np.array([5e-7], "<f2").view(np.uint8)
        blocks[1, 208:210] = np.array([-1.5], "<f2").view(np.uint8)
    ref = np_q4k(blocks) if quant == "q4_k" else np_q6k(blocks)
    got = np.stack([O.dequant_kquant_block(b.tobytes(), quant) for b in blocks])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("quant", ["q4_k", "q6_k"])
def test_oracle_linear_is_the_sequential_sum(quant):
    rows, cols = 3, 512
    w = synth.kquant(9, rows, cols, quant)
    x = np.random.default_rng(2).standard_normal(cols).astype(np.float32)
    deq = np_q4k if quant == "q4_k" else np_q6k
    wd = deq(w.reshape(rows * cols // 256, -1)).reshape(rows, cols)
    y = O.linear_kquant(x, w, cols, rows, quant)
    for r in range(rows):
        acc = np.float32(0.0)
        for k in range(cols):
            acc = np.float32(acc + np.float32(x[k] * wd[r, k]))
        assert y[r].view(np.uint32) == acc.view(np.uint32)


@pytest.mark.parametrize("quant", ["q4_k", "q6_k"])
@pytest.mark.parametrize("rows,cols", [(17, 256), (64, 4096)])
def test_oracle_linear_within_float_bound(quant, rows, cols):
    w = synth.kquant(rows + cols, rows, cols, quant)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    deq = np_q4k if quant == "q4_k" else np_q6k
    wd = deq(w.reshape(rows * cols // 256, -1)).reshape(rows, cols).astype(np.float64)
    y = O.linear_kquant(x, w, cols, rows, quant).astype(np.float64)
    mag = np.abs(wd) @ np.abs(x.astype(np.float64))
    assert np.all(np.abs(y - wd @ x.astype(np.float64)) <= cols * 2.0 ** -24 * mag)
