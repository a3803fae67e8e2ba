"""The allocation-free attention entry point against the allocating one.

zgpu_gqa_attention_decode_noalloc exists for callers that may not allocate
device memory once they are running: hosts that reserve every byte up front
and hand out fixed buffers, per-token loops in which an allocation could
synchronise the device, and plugins whose memory belongs to another
allocator.  Instead of context-owned scratch it uses a fixed array in the
library's device image, shared by every call on the device.

The test runs two decode steps in a row through both entry points, each on
its own copy of the same KV cache.  Both run the same kernel with the same
launch shape and a fixed reduction order, so the outputs and the appended
cache rows must be equal bit for bit.  The context is 1024 tokens (four
splits), so the second call finds the partials and counters that the first
call left in the shared array.  This file sorts last so that a stop at the
first failure has already run every other test.
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


def _call(fn, ctx, kv, pos, n_q, bufs, stream):
    d_qkv, d_qn, d_kn, d_inv, d_out = bufs
    return fn(ctx.h, kv.h, 0, pos, n_q, d_qkv.data_ptr(), d_qn.data_ptr(), d_kn.data_ptr(), d_inv.data_ptr(),
              C.c_float(EPS), d_out.data_ptr(), C.c_void_p(stream.cuda_stream))


def test_noalloc_attention_matches_allocating_entry_point(ctx):
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda", 0)
    n_q, n_kv, max_tokens, first_pos = 16, 8, 1024, 600
    rng = np.random.default_rng(2024)
    kvd = n_kv * HD
    k_prev = rng.standard_normal((first_pos, kvd)).astype(np.float32)
    v_prev = rng.standard_normal((first_pos, kvd)).astype(np.float32)
    kv_ref = zb.KvCache(ctx, max_tokens, 1, n_kv, HD)
    kv_new = zb.KvCache(ctx, max_tokens, 1, n_kv, HD)
    try:
        for t in range(first_pos):
            kv_ref.store_kv(0, t, k_prev[t], v_prev[t])
            kv_new.store_kv(0, t, k_prev[t], v_prev[t])
        d_qn = torch.from_numpy((1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32)).to(dev)
        d_kn = torch.from_numpy((1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32)).to(dev)
        d_inv = torch.from_numpy(O.rope_ctx(THETA, HD // 2)).to(dev)
        stream = torch.cuda.Stream(dev)
        for pos in (first_pos, first_pos + 1):
            d_qkv = torch.from_numpy(rng.standard_normal((n_q + 2 * n_kv) * HD).astype(np.float32)).to(dev)
            d_ref = torch.full((n_q * HD,), float("nan"), device=dev)
            d_new = torch.full((n_q * HD,), float("nan"), device=dev)
            torch.cuda.synchronize(dev)
            ctx._check(_call(LIB.zgpu_gqa_attention_decode_device, ctx, kv_ref, pos, n_q,
                             (d_qkv, d_qn, d_kn, d_inv, d_ref), stream))
            ctx._check(_call(LIB.zgpu_gqa_attention_decode_noalloc, ctx, kv_new, pos, n_q,
                             (d_qkv, d_qn, d_kn, d_inv, d_new), stream))
            stream.synchronize()
            ctx.synchronize()
            ref, new = d_ref.cpu().numpy(), d_new.cpu().numpy()
            assert np.isfinite(ref).all()
            assert np.array_equal(new.view(np.uint32), ref.view(np.uint32)), f"call at pos {pos}"
            k_ref, v_ref = kv_ref.read(0, pos + 1)
            k_new, v_new = kv_new.read(0, pos + 1)
            assert np.array_equal(k_new.view(np.uint32), k_ref.view(np.uint32))
            assert np.array_equal(v_new.view(np.uint32), v_ref.view(np.uint32))
    finally:
        kv_ref.close()
        kv_new.close()


def test_noalloc_attention_rejects_oversized_cache(ctx):
    """32 q heads over a 16384-token cache need 266240 partial floats, more
    than the fixed array holds: the call fails before launching anything."""
    torch = pytest.importorskip("torch")
    dev = torch.device("cuda", 0)
    n_q, n_kv = 32, 8
    kv = zb.KvCache(ctx, 16384, 1, n_kv, HD)
    try:
        bufs = (torch.zeros((n_q + 2 * n_kv) * HD, device=dev), torch.ones(HD, device=dev),
                torch.ones(HD, device=dev), torch.ones(HD // 2, device=dev), torch.zeros(n_q * HD, device=dev))
        torch.cuda.synchronize(dev)
        st = _call(LIB.zgpu_gqa_attention_decode_noalloc, ctx, kv, 0, n_q, bufs, torch.cuda.Stream(dev))
        assert st == 1
        assert b"static scratch" in LIB.zgpu_last_error(ctx.h)
    finally:
        kv.close()
