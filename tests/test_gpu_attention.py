"""GPU parity of the single-layer decode attention entry points (through the C ABI).

zgpu_gqa_attention_decode restates steps 2-5 of
gqa_attention_single_token_dispatch (crates/zero-llm-inference/src/
attention.rs:344-425); the oracle is zo_gqa_attention_decode in the AVX-512
order (inference_avx512.rs:1612-1800).  RoPE is bit-exact with the oracle's
LUT; the QK-norm sum of squares, the score dot products and the softmax
exponentials reduce in a different order, so outputs are held to a relative
L2 error of 1e-5 and the newly stored k row to 1e-6.  The stored v row and the
single-token case (softmax weight exactly 1) are bit-exact.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import zero_b200 as zb
from zero_b200._lib import LIB

pytestmark = pytest.mark.gpu

HD = 128
EPS = 1e-6
THETA = 1e6
REL_L2 = 1e-5


def make_case(seed: int, n_q: int, n_kv: int, max_tokens: int):
    rng = np.random.default_rng(seed)
    kvd = n_kv * HD
    return dict(
        k_prev=rng.standard_normal((max_tokens, kvd)).astype(np.float32),
        v_prev=rng.standard_normal((max_tokens, kvd)).astype(np.float32),
        qkv=rng.standard_normal((n_q + 2 * n_kv) * HD).astype(np.float32),
        q_norm=(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32),
        k_norm=(1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32),
    )


def rel_l2(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def oracle_step(case, kb, vb, pos, n_q, n_kv):
    inv = O.rope_ctx(THETA, HD // 2)
    rc, out = O.gqa_attention_decode(case["qkv"], case["q_norm"], case["k_norm"], inv, kb, vb, pos, n_q,
                                     n_kv, HD, EPS, order=1)
    assert rc == 0
    return out


@pytest.mark.parametrize("n_q,n_kv", [(16, 8), (8, 8), (32, 8), (4, 1)])
@pytest.mark.parametrize("pos", [0, 1, 143, 255, 256, 257, 600, 1023])
def test_attention_matches_oracle_prefilled_cache(ctx, n_q, n_kv, pos):
    """Cache rows 0..pos-1 written by store_kv, then one decode step at pos:
    one split up to 256 tokens, flash-decoding partials merged in split order
    beyond (1024 tokens = 4 splits)."""
    max_tokens, layers, layer = 1024, 2, 1
    case = make_case(1000 + pos + n_q, n_q, n_kv, max_tokens)
    kv = zb.KvCache(ctx, max_tokens, layers, n_kv, HD)
    try:
        for t in range(pos):
            kv.store_kv(layer, t, case["k_prev"][t], case["v_prev"][t])
        out = kv.gqa_attention_decode(layer, pos, n_q, case["qkv"], case["q_norm"], case["k_norm"], THETA, EPS)
        kb, vb = case["k_prev"].copy(), case["v_prev"].copy()
        ref = oracle_step(case, kb.reshape(-1), vb.reshape(-1), pos, n_q, n_kv)
        if pos == 0:
            # one token: softmax weight exactly 1, so out = v of the head's kv head
            v = case["qkv"][(n_q + n_kv) * HD:].reshape(n_kv, HD)
            assert np.array_equal(out.reshape(n_q, HD), np.repeat(v, n_q // n_kv, axis=0))
        assert rel_l2(out, ref) <= REL_L2
        k, v = kv.read(layer, pos + 1)
        assert np.array_equal(v.reshape(pos + 1, -1)[pos], vb[pos])
        assert rel_l2(k.reshape(pos + 1, -1)[pos], kb[pos]) <= 1e-6
        if pos:
            assert np.array_equal(k.reshape(pos + 1, -1)[:pos], case["k_prev"][:pos])
        k0, _ = kv.read(0, max_tokens)
        assert not k0.any(), "other layers untouched"
    finally:
        kv.close()


def test_attention_lockstep_decode_crosses_split_boundary(ctx):
    """Consecutive decode steps, each appending its own k/v, in lockstep with
    the oracle's cache, across the 256-token split boundary."""
    n_q, n_kv, max_tokens = 16, 8, 320
    kv = zb.KvCache(ctx, max_tokens, 1, n_kv, HD)
    kb = np.zeros(max_tokens * n_kv * HD, np.float32)
    vb = np.zeros_like(kb)
    inv = O.rope_ctx(THETA, HD // 2)
    worst = 0.0
    try:
        for pos in range(max_tokens):
            case = make_case(pos, n_q, n_kv, 1)
            out = kv.gqa_attention_decode(0, pos, n_q, case["qkv"], case["q_norm"], case["k_norm"], THETA, EPS)
            rc, ref = O.gqa_attention_decode(case["qkv"], case["q_norm"], case["k_norm"], inv, kb, vb, pos,
                                             n_q, n_kv, HD, EPS, order=1)
            assert rc == 0
            worst = max(worst, rel_l2(out, ref))
        assert worst <= REL_L2, worst
        k, v = kv.read(0, max_tokens)
        assert np.array_equal(v, vb)
        assert rel_l2(k, kb) <= 1e-6
    finally:
        kv.close()


def test_attention_errors(ctx):
    n_q, n_kv = 16, 8
    case = make_case(5, n_q, n_kv, 1)
    kv = zb.KvCache(ctx, 16, 2, n_kv, HD)
    args = (case["qkv"], case["q_norm"], case["k_norm"], THETA, EPS)
    try:
        with pytest.raises(zb.ZgpuError) as e:       # KvCacheError::TokenOutOfRange (kv_cache.rs:148)
            kv.gqa_attention_decode(0, 16, n_q, *args)
        assert e.value.status == 10
        with pytest.raises(zb.ZgpuError) as e:       # KvCacheError::LayerOutOfRange
            kv.gqa_attention_decode(2, 0, n_q, *args)
        assert e.value.status == 11
        for bad_nq in (0, 12, 40):                    # not 1..4 x n_kv
            with pytest.raises(zb.ZgpuError) as e:
                kv.gqa_attention_decode(0, 0, bad_nq, *args)
            assert e.value.status == 1
        # attention.rs:57-66: a non-finite max score is NumericalInstability
        bad = case["qkv"].copy()
        bad[:n_q * HD] = np.nan
        with pytest.raises(zb.ZgpuError) as e:
            kv.gqa_attention_decode(0, 3, n_q, bad, case["q_norm"], case["k_norm"], THETA, EPS)
        assert e.value.status == 20
        # the error is reported once; the next call is clean
        out = kv.gqa_attention_decode(0, 3, n_q, *args)
        assert np.isfinite(out).all()
    finally:
        kv.close()
    kv64 = zb.KvCache(ctx, 16, 1, n_kv, 64)
    try:
        with pytest.raises(zb.ZgpuError) as e:
            kv64.gqa_attention_decode(0, 0, n_q, np.zeros((n_q + 2 * n_kv) * 64, np.float32),
                                      np.ones(64, np.float32), np.ones(64, np.float32), THETA, EPS)
        assert e.value.status == 1
    finally:
        kv64.close()


def test_attention_device_entry_matches_host_entry(ctx):
    """zgpu_gqa_attention_decode_device on caller-owned device buffers gives
    the same bits as the host-buffer entry point."""
    torch = pytest.importorskip("torch")
    n_q, n_kv, max_tokens, pos = 16, 8, 700, 611
    case = make_case(77, n_q, n_kv, max_tokens)
    kv = zb.KvCache(ctx, max_tokens, 1, n_kv, HD)
    try:
        for t in range(pos):
            kv.store_kv(0, t, case["k_prev"][t], case["v_prev"][t])
        host = kv.gqa_attention_decode(0, pos, n_q, case["qkv"], case["q_norm"], case["k_norm"], THETA, EPS)
        dev = torch.device("cuda", 0)
        d_qkv = torch.from_numpy(case["qkv"]).to(dev)
        d_qn = torch.from_numpy(case["q_norm"]).to(dev)
        d_kn = torch.from_numpy(case["k_norm"]).to(dev)
        d_inv = torch.from_numpy(O.rope_ctx(THETA, HD // 2)).to(dev)
        d_out = torch.full((n_q * HD,), float("nan"), device=dev)
        torch.cuda.synchronize(dev)
        stream = torch.cuda.Stream(dev)
        for _ in range(2):
            st = LIB.zgpu_gqa_attention_decode_device(ctx.h, kv.h, 0, pos, n_q, d_qkv.data_ptr(), d_qn.data_ptr(),
                                                      d_kn.data_ptr(), d_inv.data_ptr(), C.c_float(EPS),
                                                      d_out.data_ptr(), C.c_void_p(stream.cuda_stream))
            ctx._check(st)
            stream.synchronize()
            assert np.array_equal(d_out.cpu().numpy(), host)
    finally:
        kv.close()
