"""The arithmetic identities the exact batched matvec (digit_mma.cu) rests on,
checked on the host in numpy (CPU only).

1. Digits.  The GEMV splits each activation integer N (|N| < 2^23) into
   d0, d1 (unsigned bytes) and d2 (the signed top byte) and forms
   s_d = sum_j w_j d_dj; the tensor-core path stores d0 - 128, d1 - 128 (so
   every operand byte is signed) and restores s_d = sum_j w_j (d_dj - 128) +
   128 sum_j w_j.  Both give the same integers, and the same
   t = fma(s2, 65536, float(s0 + 256 s1)).
2. Conversion.  For |S| < 2^22 the float with bits (0x4B400000 + S), minus
   1.5 * 2^23, is S exactly; fma(float(S1), 256, float(S0)) rounds once, to
   float(S0 + 256 S1).
3. Order.  A warp's xor-butterfly over 32 lanes (pairs 16 apart first, then 8,
   4, 2, 1) equals a left-to-right binary-counter fold of the lanes taken in
   bit-reversed order, in float32, for any values.
"""
import numpy as np

MAGIC_BITS = 0x4B400000
M = np.float32(12582912.0)


def block_ints(x):
    """N_j = rint(x_j * 2^(22-e)) for one 32-element block (am in [2^e, 2^(e+1))), capped at 2^23 - 1."""
    am = np.max(np.abs(x))
    if am < np.float32(2.0 ** -100):
        return np.zeros(32, np.int64)
    e = int((np.float32(am).view(np.uint32) >> 23)) - 127
    up = np.float32(2.0 ** (22 - e))
    n = np.rint((x * up).astype(np.float32)).astype(np.int64)
    return np.minimum(n, 0x7FFFFF)


def f32_fma(a, b, c):
    """a * b + c rounded once to float32 (exact in float64 for these magnitudes)."""
    return np.float32(np.float64(a) * np.float64(b) + np.float64(c))


def magic(s):
    bits = np.array([MAGIC_BITS + int(s)], np.int64).astype(np.uint32)
    return np.float32(bits.view(np.float32)[0] - M)


def test_digits_and_t_agree():
    rng = np.random.default_rng(1)
    for trial in range(400):
        scale = np.float32(2.0 ** rng.integers(-30, 30))
        x = (rng.standard_normal(32) * scale).astype(np.float32)
        n = block_ints(x)
        d0, d1, d2 = n & 255, (n >> 8) & 255, n >> 16
        assert np.array_equal(d0 + 256 * d1 + 65536 * d2, n)
        assert d2.min() >= -128 and d2.max() <= 127
        w = rng.integers(-8, 8, 32) if trial % 2 else rng.integers(-127, 128, 32)
        s0, s1, s2 = int(w @ d0), int(w @ d1), int(w @ d2)
        rs = int(w.sum())
        S0 = int(w @ (d0 - 128)) + 128 * rs
        S1 = int(w @ (d1 - 128)) + 128 * rs
        assert (S0, S1) == (s0, s1)
        assert max(abs(S0), abs(S1), abs(s2)) < 2 ** 22
        X = s0 + 256 * s1
        assert abs(X) < 2 ** 31
        t_gemv = f32_fma(np.float32(s2), np.float32(65536.0), np.float32(X))
        f0, f1, f2 = magic(S0), magic(S1), magic(s2)
        assert (f0, f1, f2) == (np.float32(S0), np.float32(S1), np.float32(s2))
        t_mma = f32_fma(f2, np.float32(65536.0), f32_fma(f1, np.float32(256.0), f0))
        assert t_mma.view(np.uint32) == t_gemv.view(np.uint32), (trial, s0, s1, s2)


def butterfly(v):
    """The GEMV's warp reduce: pairs 16 apart first, then 8, 4, 2, 1."""
    v = v.astype(np.float32).copy()
    off = 16
    while off:
        v = np.array([np.float32(v[l] + v[l ^ off]) for l in range(32)], np.float32)
        off >>= 1
    return v[0]


def bitrev_fold(v):
    """Leaves in bit-reversed lane order, folded by a binary counter (left + right)."""
    order = [int(f"{i:05b}"[::-1], 2) for i in range(32)]
    stack = []
    for i, lane in enumerate(order):
        x = np.float32(v[lane])
        k = 0
        while (i >> k) & 1:
            x = np.float32(stack.pop() + x)
            k += 1
        stack.append(x)
    assert len(stack) == 1
    return stack[0]


def test_bit_reversed_fold_is_the_butterfly():
    rng = np.random.default_rng(2)
    for trial in range(300):
        v = (rng.standard_normal(32) * np.exp2(rng.integers(-40, 40, 32))).astype(np.float32)
        if trial % 5 == 0:
            v[rng.integers(0, 32, 8)] = 0.0          # idle lanes of a short chunk
        a, b = butterfly(v), bitrev_fold(v)
        assert a.view(np.uint32) == b.view(np.uint32), trial
