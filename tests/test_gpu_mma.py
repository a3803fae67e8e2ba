"""Batched Q4_0 x Q8_0 matmul on the tcgen05 int8 path (mma_gemm.cu).

Bar: bit-identical to the CPU restatement of the single-row Q4_0 x Q8_0
product (per block sumi exact, then acc += (sumi * d_w) * d_x in block order)
for every token row, because each block is one integer MMA whose int32 result
is scaled and added in the same order.  Activations are quantised on the GPU
with the packer's Q8_0 rule, pinned bit-exact against the oracle quantiser.
"""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 32, 1),        # one tile, one block
    (256, 1024, 7),      # ragged token count
    (512, 2048, 64),     # exactly one token tile
    (384, 6144, 100),    # down-projection width, two token tiles
    (128, 2048, 130),    # three token tiles
]


@pytest.mark.parametrize("rows,cols,T", SHAPES)
def test_q4q8_batch_bit_exact(ctx, rows, cols, T):
    seed = rows + cols + T
    w = synth.q4_0(seed, 1, rows, cols, 0.02)
    key = ctx.register(w, zb.Q4_0, rows, cols)
    x = synth.f32(seed, 2, T * cols, 0.0, 1.0).reshape(T, cols)
    y = ctx.linear_q8act_batch(x, key, cols, rows)
    assert y.shape == (T, rows)
    for t in range(T):
        xq = O.quantize_row_q8_0(x[t])
        ref = O.linear_q4_0_q8act(xq, w, cols, rows)
        assert np.array_equal(y[t].view(np.uint32), ref.view(np.uint32)), t


def test_q4q8_batch_x4_registration_and_gemv_agree(ctx):
    """The .smodel-v2 X4 registration gives the same device layout; the
    single-row dp4a GEMV (another summation order) agrees to f32 rounding."""
    rows, cols, T = 1024, 2048, 16
    w = synth.q4_0(5, 3, rows, cols, 0.02)
    w4 = synth.pack_x4(w, rows, cols, "q4_0")
    key = ctx.register(w4, zb.Q4_0X4, rows, cols)
    x = synth.f32(5, 4, T * cols, 0.0, 1.0).reshape(T, cols)
    y = ctx.linear_q8act_batch(x, key, cols, rows)
    for t in (0, 7, 15):
        xq = ctx.quantize_q8_0(x[t])
        assert np.array_equal(xq, O.quantize_row_q8_0(x[t]))
        g = ctx.linear_q8act(xq, key, cols, rows)
        np.testing.assert_allclose(y[t], g, rtol=1e-5, atol=1e-5 * float(np.abs(g).max()))
        ref = O.linear_q4_0_q8act(xq, w, cols, rows)
        assert np.array_equal(y[t].view(np.uint32), ref.view(np.uint32))


def test_q4q8_batch_rejects_bad_shapes(ctx):
    rows, cols = 96, 64      # rows not a multiple of 128
    w = synth.q4_0(6, 5, rows, cols, 0.02)
    key = ctx.register(w, zb.Q4_0, rows, cols)
    with pytest.raises(zb.ZgpuError) as ei:
        ctx.linear_q8act_batch(np.zeros((2, cols), np.float32), key, cols, rows)
    assert ei.value.name == "INVALID_ARG"
