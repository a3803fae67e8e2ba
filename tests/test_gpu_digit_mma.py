"""The batched tensor-core matvec (zgpu_linear_dispatch_batch: tcgen05 int8
MMA over the activation digits) against the single-vector GEMV
(zgpu_linear_dispatch), which the op tests hold to the reference.

Bar: bit-identical for every vector, at every vector count (1..32), for Q4_0
and Q8_0 weights, full and partial 128-row tiles, full and short last
32-block chunks, and activation blocks that are zero, negligible, huge or
of mixed magnitude.
"""
import numpy as np
import pytest

import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu

# (out, in): config-1 / ds2 shapes, a partial last row tile (2112 = 16.5 tiles),
# short last chunks (48 and 44 blocks), tiny matrices
SHAPES = [(4096, 2048), (2112, 2048), (3072, 1536), (2048, 1408), (128, 6144), (8, 32), (100, 64)]


def inputs(n_vec, in_dim, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n_vec, in_dim)).astype(np.float32)
    if n_vec > 1:
        x[1] = 0.0                                   # an all-zero vector
    if n_vec > 2:
        x[2, :32] *= 1e-33                           # a negligible block (maximum below 2^-100)
        x[2, 32:64] = 0.0                            # a zero block
        x[2, 64:96] *= 1e30 if in_dim > 64 else 1.0  # a huge block
    if n_vec > 3:
        x[3] *= np.exp2(rng.integers(-20, 20, in_dim)).astype(np.float32)   # mixed magnitudes
    if n_vec > 5:
        # blocks just above the negligible limit (2^-100): block scales near
        # 2^-120, so scale products fall into the f32 subnormal range
        x[4] *= np.float32(2.0 ** -97)
        x[5] *= np.float32(2.0 ** -99)
    return x


@pytest.mark.parametrize("quant", [zb.Q4_0, zb.Q8_0])
@pytest.mark.parametrize("out_dim,in_dim", SHAPES)
def test_batch_equals_single_gemv(ctx, quant, out_dim, in_dim):
    if quant == zb.Q4_0:
        w = synth.q4_0(21, out_dim + in_dim, out_dim, in_dim, 0.02)
    else:
        w = synth.q8_0(22, out_dim + in_dim, out_dim, in_dim, 0.02 / 127)
    key = ctx.register(w, quant, out_dim, in_dim)
    x = inputs(32, in_dim, out_dim + in_dim)
    single = np.stack([ctx.linear_dispatch(x[v], key, in_dim, out_dim, quant) for v in range(32)])
    for n_vec in (1, 3, 16, 17, 32):
        y = ctx.linear_dispatch_batch(x[:n_vec], key, in_dim, out_dim, quant)
        same = y.view(np.uint32) == single[:n_vec].view(np.uint32)
        assert same.all(), (n_vec, np.argwhere(~same)[:5], y[~same][:5], single[:n_vec][~same][:5])


def test_batch_many_vector_groups(ctx):
    """100 and 256 vectors (7 and 16 vector groups of one launch)."""
    out_dim, in_dim = 1024, 4096
    w = synth.q4_0(25, 3, out_dim, in_dim, 0.02)
    key = ctx.register(w, zb.Q4_0, out_dim, in_dim)
    x = inputs(256, in_dim, 9)
    for n_vec in (100, 256):
        y = ctx.linear_dispatch_batch(x[:n_vec], key, in_dim, out_dim, zb.Q4_0)
        for v in (0, 5, 16, 47, n_vec - 1):
            assert np.array_equal(y[v].view(np.uint32),
                                  ctx.linear_dispatch(x[v], key, in_dim, out_dim, zb.Q4_0).view(np.uint32)), (n_vec, v)


def test_batch_lm_head_shape(ctx):
    """The ds2 LM head shape (Q8_0, 102400 x 2048) with 32 vectors."""
    out_dim, in_dim = 102400, 2048
    w = synth.q8_0(23, 7, out_dim, in_dim, 0.02 / 127)
    key = ctx.register(w, zb.Q8_0, out_dim, in_dim)
    x = inputs(32, in_dim, 5)
    y = ctx.linear_dispatch_batch(x, key, in_dim, out_dim, zb.Q8_0)
    for v in (0, 1, 2, 3, 17, 31):
        assert np.array_equal(y[v].view(np.uint32), ctx.linear_dispatch(x[v], key, in_dim, out_dim, zb.Q8_0).view(np.uint32))


def test_batch_rejects_bad_args(ctx):
    w = synth.q4_0(24, 1, 64, 64, 0.02)
    key = ctx.register(w, zb.Q4_0, 64, 64)
    with pytest.raises(zb.ZgpuError) as ei:
        ctx.linear_dispatch_batch(np.zeros((257, 64), np.float32), key, 64, 64, zb.Q4_0)
    assert ei.value.name == "INVALID_ARG"
    with pytest.raises(zb.ZgpuError) as ei:
        ctx.linear_dispatch_batch(np.zeros((2, 64), np.float32), key, 64, 64, zb.Q4_K)
    assert ei.value.name == "UNSUPPORTED_QUANT"
