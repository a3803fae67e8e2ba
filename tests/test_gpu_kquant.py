"""GPU K-quant GEMV (zgpu_linear_dispatch with Q4_K / Q6_K, kquant.cu) against
the CPU oracle's linear_q4k / linear_q6k restatement (ops.rs:179-292).

  * a one-hot input returns one column of the dequantised matrix exactly, so
    every weight the kernel rebuilds equals the oracle's dequantisation
    bit-for-bit (each lane position of both super-block layouts is hit);
  * on random matrices each row is within 2e-6 * sum_j |x_j w_j| of a float64
    evaluation of the same weights (the kernel sums in a fixed warp order,
    the reference sequentially), and so is the oracle;
  * geometry and quant mismatches are refused.
"""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu

QUANTS = {"q4_k": (zb.Q4_K, 144), "q6_k": (zb.Q6_K, 210)}


def dequant(w: np.ndarray, rows: int, cols: int, quant: str) -> np.ndarray:
    bb = QUANTS[quant][1]
    blocks = w.reshape(rows * cols // 256, bb)
    return np.stack([O.dequant_kquant_block(b.tobytes(), quant) for b in blocks]).reshape(rows, cols)


@pytest.mark.parametrize("quant", list(QUANTS))
def test_one_hot_columns_are_the_dequantised_weights(ctx, quant):
    qt, _ = QUANTS[quant]
    rows, cols = 24, 512
    w = synth.kquant(3, rows, cols, quant)
    key = ctx.register(w, qt, rows, cols)
    wd = dequant(w, rows, cols, quant)
    for k in range(cols):
        x = np.zeros(cols, np.float32)
        x[k] = 1.0
        y = ctx.linear_dispatch(x, key, cols, rows, qt)
        assert np.array_equal(y, wd[:, k]), (quant, k)


@pytest.mark.parametrize("quant", list(QUANTS))
@pytest.mark.parametrize("rows,cols", [(8, 256), (1001, 2048), (4096, 4096), (1024, 12288), (151, 256 * 9)])
def test_random_gemv_matches_oracle(ctx, quant, rows, cols):
    qt, _ = QUANTS[quant]
    w = synth.kquant(rows * 7 + cols, rows, cols, quant)
    key = ctx.register(w, qt, rows, cols)
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    y = ctx.linear_dispatch(x, key, cols, rows, qt)
    ref = O.linear_kquant(x, w, cols, rows, quant)
    wd = dequant(w, rows, cols, quant).astype(np.float64)
    y64 = wd @ x.astype(np.float64)
    mag = np.abs(wd) @ np.abs(x.astype(np.float64))
    for got in (y, ref):
        worst = np.max(np.abs(got.astype(np.float64) - y64) / np.maximum(mag, 1e-30))
        assert worst <= 2e-6, worst
    assert np.array_equal(y, ctx.linear_dispatch(x, key, cols, rows, qt))   # deterministic


def test_kquant_geometry_and_quant_errors(ctx):
    with pytest.raises(zb.ZgpuError) as e:
        ctx.register(np.zeros(144, np.uint8), zb.Q4_K, 1, 128)           # cols not a multiple of 256
    assert e.value.status == 1
    with pytest.raises(zb.ZgpuError) as e:
        ctx.register(np.zeros(209, np.uint8), zb.Q6_K, 1, 256)           # wrong byte length
    assert e.value.status == 1
    w = synth.kquant(1, 8, 256, "q4_k")
    key = ctx.register(w, zb.Q4_K, 8, 256)
    x = np.zeros(256, np.float32)
    with pytest.raises(zb.ZgpuError) as e:
        ctx.linear_dispatch(x, key, 256, 8, zb.Q6_K)                     # registered as Q4_K
    assert e.value.status == 1
    assert np.array_equal(ctx.linear_dispatch(x, key, 256, 8, zb.Q4_K), np.zeros(8, np.float32))
