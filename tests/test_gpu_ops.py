"""GPU parity of the op-level entry points against the CPU oracle (through the C ABI).

Tolerances: the GEMV reduces in a different (fixed) order than the
reference, so each output row is held to |y - y64| <= 2e-6 * sum_j |x_j w_j|
against an fp64 evaluation of the same dequantised weights — a few f32
roundings of the row's magnitude — and the oracle's AVX-512-order result is
checked against the same bound.  Ops restated from the reference's own
polynomials (RoPE LUT, SiLU*up) and the Q8_0 quantiser are bit-exact.
"""
import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200 import synth

pytestmark = pytest.mark.gpu

REL_BOUND = 2e-6


def dequant_rows(plain: np.ndarray, rows: int, cols: int, quant: int) -> np.ndarray:
    bb = 18 if quant == zb.Q4_0 else 34
    blk = plain.reshape(rows * cols // 32, bb)
    d = blk[:, :2].copy().view(np.float16).astype(np.float64)
    if quant == zb.Q4_0:
        lo = (blk[:, 2:] & 0xF).astype(np.float64) - 8
        hi = (blk[:, 2:] >> 4).astype(np.float64) - 8
        vals = np.concatenate([lo, hi], axis=1)
    else:
        vals = blk[:, 2:].view(np.int8).astype(np.float64)
    return (vals * d).reshape(rows, cols)


def check_rows(y: np.ndarray, x: np.ndarray, wd: np.ndarray, bound=REL_BOUND):
    x64 = x.astype(np.float64)
    y64 = wd @ x64
    mag = np.abs(wd) @ np.abs(x64)
    err = np.abs(y.astype(np.float64) - y64)
    worst = np.max(err / np.maximum(mag, 1e-30))
    assert worst <= bound, f"worst row error {worst:.3e} x magnitude"
    return worst


# BASELINE config 1's four shapes (out x in) first, the LM-head one in Q4_0 as config 1 states it
SHAPES = [(4096, 2048), (12288, 2048), (2048, 6144), (151936, 2048), (2048, 2048), (64, 2048), (8, 32),
          (4, 64), (400, 1024), (1028, 4096), (4, 8192)]


@pytest.mark.parametrize("out_dim,in_dim", SHAPES)
def test_q4_0x4_gemv_matches_oracle(ctx, out_dim, in_dim):
    w = synth.q4_0(11, out_dim + in_dim, out_dim, in_dim, 0.02)
    wx = synth.pack_x4(w, out_dim, in_dim, "q4_0")
    key = ctx.register(wx, zb.Q4_0X4, out_dim, in_dim)
    assert ctx.group_of(key) == 4
    x = np.random.default_rng(out_dim).standard_normal(in_dim).astype(np.float32)
    y = ctx.linear_dispatch(x, key, in_dim, out_dim, zb.Q4_0)
    wd = dequant_rows(w, out_dim, in_dim, zb.Q4_0)
    check_rows(y, x, wd)
    ref = O.linear_x4_avx512(x, wx, in_dim, out_dim, O.Q4_0)
    check_rows(ref, x, wd)
    # deterministic: a second call is bitwise identical
    assert np.array_equal(y, ctx.linear_dispatch(x, key, in_dim, out_dim, zb.Q4_0))


@pytest.mark.parametrize("out_dim,in_dim", [(151936, 2048), (4096, 2048), (8, 64), (64, 6144)])
def test_q8_0x4_gemv_matches_oracle(ctx, out_dim, in_dim):
    w = synth.q8_0(12, out_dim, out_dim, in_dim, 0.02 / 127)
    wx = synth.pack_x4(w, out_dim, in_dim, "q8_0")
    key = ctx.register(wx, zb.Q8_0X4, out_dim, in_dim)
    x = np.random.default_rng(1).standard_normal(in_dim).astype(np.float32)
    y = ctx.linear_dispatch(x, key, in_dim, out_dim, zb.Q8_0)
    wd = dequant_rows(w, out_dim, in_dim, zb.Q8_0)
    check_rows(y, x, wd)
    ref = O.linear_x4_avx512(x, wx, in_dim, out_dim, O.Q8_0)
    check_rows(ref, x, wd)


@pytest.mark.parametrize("out_dim", [1, 2, 3, 5, 6, 7, 33])
def test_plain_layout_ragged_rows(ctx, out_dim):
    # plain Q4_0 registration with rows not a multiple of the group (padded on device)
    in_dim = 96
    w = synth.q4_0(13, out_dim, out_dim, in_dim, 0.02)
    key = ctx.register(w, zb.Q4_0, out_dim, in_dim)
    assert ctx.group_of(key) == 1
    x = np.random.default_rng(2).standard_normal(in_dim).astype(np.float32)
    y = ctx.linear_dispatch(x, key, in_dim, out_dim, zb.Q4_0)
    check_rows(y, x, dequant_rows(w, out_dim, in_dim, zb.Q4_0))
    ref = O.linear(x, w, in_dim, out_dim, O.Q4_0)
    assert np.allclose(y, ref, rtol=0, atol=1e-5 * np.max(np.abs(ref)))


def test_reference_linear_kats_on_gpu(ctx):
    # ops.rs:967-1131 hand-math values through the GPU path (exact).
    unit_q4 = np.frombuffer(bytes([0x00, 0x3C] + [0x99] * 16), np.uint8).copy()
    unit_q8 = np.frombuffer(bytes([0x00, 0x3C] + [1] * 32), np.uint8).copy()
    x = np.arange(1, 33, dtype=np.float32)
    assert ctx.linear_dispatch(x, ctx.register(unit_q4, zb.Q4_0, 1, 32), 32, 1, zb.Q4_0)[0] == 528.0
    assert ctx.linear_dispatch(x, ctx.register(unit_q8, zb.Q8_0, 1, 32), 32, 1, zb.Q8_0)[0] == 528.0
    two = np.concatenate([unit_q4, np.frombuffer(bytes([0x00, 0x3C] + [0] * 16), np.uint8)]).copy()
    out = ctx.linear_dispatch(np.ones(32, np.float32), ctx.register(two, zb.Q4_0, 2, 32), 32, 2, zb.Q4_0)
    assert out[0] == 32.0 and out[1] == -256.0
    neg = np.frombuffer(bytes([0x00, 0x3C] + [0xFF] * 32), np.uint8).copy()
    assert ctx.linear_dispatch(np.full(32, 0.5, np.float32), ctx.register(neg, zb.Q8_0, 1, 32),
                               32, 1, zb.Q8_0)[0] == -16.0


def test_linear_dispatch_errors(ctx):
    w = synth.q4_0(14, 0, 8, 64, 0.02)
    key = ctx.register(w, zb.Q4_0, 8, 64)
    x = np.zeros(64, np.float32)
    with pytest.raises(zb.ZgpuError) as e:
        ctx.linear_dispatch(x, key, 64, 8, zb.F16)          # ops.rs:513-521 unsupported quant
    assert e.value.status == 2
    with pytest.raises(zb.ZgpuError) as e:
        ctx.linear_dispatch(x, w.ctypes.data + 16, 64, 8, zb.Q4_0)   # interior pointer: not registered
    assert e.value.status == 3
    with pytest.raises(zb.ZgpuError) as e:
        ctx.linear_dispatch(x, key, 64, 4, zb.Q4_0)         # shape mismatch
    assert e.value.status == 1
    assert ctx.group_of(w.ctypes.data + 16) == 1             # weight_layout.rs:163 interior miss


def test_register_rejects_bad_geometry(ctx):
    with pytest.raises(zb.ZgpuError):
        ctx.register(np.zeros(6 * 2 * 18, np.uint8), zb.Q4_0X4, 6, 64)   # partial group
    with pytest.raises(zb.ZgpuError):
        ctx.register(np.zeros(10, np.uint8), zb.Q4_0, 1, 64)             # wrong length


def test_rmsnorm_matches_oracle(ctx):
    rng = np.random.default_rng(3)
    for n in (2, 4, 128, 2048, 4096):
        x = rng.standard_normal(n).astype(np.float32)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        y = ctx.rmsnorm(x, w, 1e-6)
        ref = O.rmsnorm(x, w, 1e-6)
        assert np.max(np.abs(y - ref) / np.maximum(np.abs(ref), 1e-6)) < 1e-5
    out = ctx.rmsnorm(np.array([3, 4], np.float32), np.ones(2, np.float32), 1e-6)   # ops.rs:559
    assert abs(out[0] - 0.8485281) < 1e-4 and abs(out[1] - 1.1313708) < 1e-4
    assert np.all(ctx.rmsnorm(np.zeros(8, np.float32), np.ones(8, np.float32), 1e-6) == 0.0)


@pytest.mark.parametrize("pos", [0, 1, 17, 143, 511, 4095])
def test_rope_bit_exact_with_reference_lut(ctx, pos):
    rng = np.random.default_rng(pos)
    heads = rng.standard_normal(24 * 128).astype(np.float32)
    y = ctx.rope(heads, 24, 128, pos, 1e6)
    inv = O.rope_ctx(1e6, 64)
    c, s = O.rope_lut_avx512(pos, inv)
    ref = np.concatenate([O.rope_apply_avx512(heads[h * 128:(h + 1) * 128], c, s) for h in range(24)])
    assert np.array_equal(y, ref)


def test_rope_reference_vector(ctx):
    ramp = (0.01 * (np.arange(128) + 1)).astype(np.float32)
    ref_pos1 = [-0.5415531171, -0.4622832390, -0.3812512551, -0.3051765074, -0.2368033646,
                -0.1767538593, -0.1246151535, -0.0795384381, -0.0405505749, -0.0067053730,
                0.0228510916, 0.0488593503, 0.0719468978, 0.0926380198, 0.1113669505,
                0.1284913603]   # ops.rs:692-709 (gguf-py dump)
    assert np.allclose(ctx.rope(ramp, 1, 128, 1, 1e6)[:16], ref_pos1, atol=1e-4)


def test_silu_mul_bit_exact(ctx):
    rng = np.random.default_rng(5)
    g = (rng.standard_normal(6144) * 4).astype(np.float32)
    g[:6] = [0.0, -0.0, 88.0, -88.0, 100.0, -100.0]
    u = rng.standard_normal(6144).astype(np.float32)
    assert np.array_equal(ctx.silu_mul(g, u), O.silu_mul_avx512(g, u))


def test_q8_0_quantiser_bit_exact_with_packer(ctx, golden):
    x = golden["blocks_in"].reshape(-1)
    assert np.array_equal(ctx.quantize_q8_0(x), golden["q8_0"].reshape(-1))
    rng = np.random.default_rng(6)
    x = rng.standard_normal(6144).astype(np.float32)
    assert np.array_equal(ctx.quantize_q8_0(x), O.quantize_row_q8_0(x))


@pytest.mark.parametrize("out_dim,in_dim", [(4096, 2048), (2048, 6144), (12288, 2048), (151936, 2048), (64, 96)])
def test_q8_activation_gemv_matches_oracle(ctx, out_dim, in_dim):
    w = synth.q4_0(15, out_dim, out_dim, in_dim, 0.02)
    key = ctx.register(w, zb.Q4_0, out_dim, in_dim)
    x = np.random.default_rng(7).standard_normal(in_dim).astype(np.float32)
    xq = ctx.quantize_q8_0(x)
    y = ctx.linear_q8act(xq, key, in_dim, out_dim)
    ref = O.linear_q4_0_q8act(xq, w, in_dim, out_dim)
    # integer block sums are exact; only the f32 block combination order differs
    mag = np.abs(dequant_rows(w, out_dim, in_dim, zb.Q4_0)) @ np.abs(x.astype(np.float64))
    assert np.max(np.abs(y - ref) / mag) < 2e-6


def test_kv_cache_store_read_layout(ctx):
    # kv_cache.rs:620-728: strides and layer isolation
    kv = zb.KvCache(ctx, max_tokens=8, n_layers=3, n_kv_heads=2, head_dim=128)
    stride = 2 * 128
    for layer in range(3):
        for t in range(8):
            k = np.full(stride, layer * 100 + t, np.float32)
            kv.store_kv(layer, t, k, -k)
    for layer in range(3):
        k, v = kv.read(layer, 8)
        assert np.array_equal(k.reshape(8, stride)[:, 0], layer * 100 + np.arange(8, dtype=np.float32))
        assert np.array_equal(v, -k)
    with pytest.raises(zb.ZgpuError) as e:
        kv.store_kv(3, 0, np.zeros(stride, np.float32), np.zeros(stride, np.float32))
    assert e.value.status == 11
    with pytest.raises(zb.ZgpuError) as e:
        kv.store_kv(0, 8, np.zeros(stride, np.float32), np.zeros(stride, np.float32))
    assert e.value.status == 10
    with pytest.raises(zb.ZgpuError) as e:
        kv.store_kv(0, 0, np.zeros(3, np.float32), np.zeros(3, np.float32))
    assert e.value.status == 12
    with pytest.raises(zb.ZgpuError) as e:
        kv.read(0, 9)
    assert e.value.status == 13
    kv.close()
