"""CPU parity oracle for the zero-llm-inference decode hot path (ctypes wrapper).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm may import this module, and only
as the checker or the timed CPU baseline.  The product package ``zero_b200``
never imports it.  The C sources (``zoracle.c``) restate the reference's
scalar crate order and its AVX-512 kernel order; see ``zoracle.h``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

Q4_0, Q8_0 = 2, 8
ORDER_SCALAR, ORDER_AVX512 = 0, 1

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_u32p = C.POINTER(C.c_uint32)


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, no GPU)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _load() -> C.CDLL:
    srcs = [HERE / "zoracle.c", HERE / "zoracle_ds2.c", HERE / "zoracle.h", HERE / "Makefile",
            HERE.parent / "zero_b200" / "csrc" / "synth.cpp"]
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < max(p.stat().st_mtime for p in srcs):
        build()
    lib = C.CDLL(str(LIB_PATH))
    sz = C.c_size_t
    sig = {
        "zo_fp16_to_f32": (C.c_float, [C.c_uint16]),
        "zo_f64_to_fp16": (C.c_uint16, [C.c_double]),
        "zo_dequant_q4_0_block": (None, [_u8p, _f32p]),
        "zo_dequant_q8_0_block": (None, [_u8p, _f32p]),
        "zo_quantize_q4_0_block": (None, [_f32p, _u8p]),
        "zo_quantize_q8_0_block": (None, [_f32p, _u8p]),
        "zo_quantize_row_q8_0": (None, [_f32p, _u8p, sz]),
        "zo_rng_next_u32": (C.c_uint32, [C.POINTER(C.c_uint64)]),
        "zo_dequant_q4_k_block": (None, [_u8p, _f32p]),
        "zo_dequant_q6_k_block": (None, [_u8p, _f32p]),
        "zo_linear_q4_k": (None, [_f32p, _u8p, _f32p, sz, sz]),
        "zo_linear_q6_k": (None, [_f32p, _u8p, _f32p, sz, sz]),
        "zo_exp_approx": (C.c_float, [C.c_float]),
        "zo_lm_head_sample": (C.c_uint32, [_f32p, C.c_uint32, C.POINTER(C.c_uint64), C.c_float, C.c_uint32]),
        "zo_linear_q4_0_q8act": (None, [_u8p, _u8p, _f32p, sz, sz]),
        "zo_linear_q8_0_q8act": (None, [_u8p, _u8p, _f32p, sz, sz]),
        "zo_interleave_x4": (C.c_int, [_u8p, _u8p, sz, sz, C.c_int]),
        "zo_rmsnorm": (None, [_f32p, _f32p, _f32p, sz, C.c_float]),
        "zo_rope_ctx": (None, [C.c_float, sz, _f32p]),
        "zo_rope": (None, [_f32p, _f32p, sz, sz]),
        "zo_linear_q4_0": (None, [_f32p, _u8p, _f32p, sz, sz]),
        "zo_linear_q8_0": (None, [_f32p, _u8p, _f32p, sz, sz]),
        "zo_linear_dispatch": (C.c_int, [_f32p, _u8p, _f32p, sz, sz, C.c_int]),
        "zo_softmax": (C.c_int, [_f32p, sz]),
        "zo_gqa_attention_decode": (C.c_int, [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                              C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                              C.c_float, C.c_int, _f32p, _f32p]),
        "zo_linear_q4_0x4_avx512": (None, [_f32p, _u8p, _f32p, sz, sz, C.c_int, C.c_int]),
        "zo_linear_q8_0x4_avx512": (None, [_f32p, _u8p, _f32p, sz, sz, C.c_int, C.c_int]),
        "zo_linear_q4_0_avx512": (None, [_f32p, _u8p, _f32p, sz, sz, C.c_int, C.c_int]),
        "zo_linear_q8_0_avx512": (None, [_f32p, _u8p, _f32p, sz, sz, C.c_int, C.c_int]),
        "zo_dot_product_avx512": (C.c_float, [_f32p, _f32p, sz]),
        "zo_weighted_add_avx512": (None, [C.c_float, _f32p, _f32p, sz]),
        "zo_argmax_avx512": (sz, [_f32p, sz, _f32p]),
        "zo_exp_avx512": (None, [_f32p, _f32p, sz]),
        "zo_silu_mul_avx512": (None, [_f32p, _f32p, _f32p, sz]),
        "zo_rope_sincos_lut_avx512": (None, [sz, _f32p, _f32p, _f32p, sz]),
        "zo_rope_apply_avx512": (None, [_f32p, _f32p, _f32p, sz]),
        "zo_have_avx512": (C.c_int, []),
        "zo_run_create": (C.c_void_p, [C.c_void_p, C.c_uint32, C.c_int, C.c_int, C.c_int]),
        "zo_synth_q4_0": (None, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_void_p]),
        "zo_synth_q8_0": (None, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_void_p]),
        "zo_synth_f32": (None, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.c_void_p]),
        "zo_synth_tokens": (None, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32, C.c_void_p]),
        "zo_pack_x4": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint32]),
        "zo_run_destroy": (None, [C.c_void_p]),
        "zo_run_forward": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, _f32p]),
        "zo_run_lm_head": (C.c_int, [C.c_void_p, _u32p, _f32p]),
        "zo_run_kv": (_f32p, [C.c_void_p]),
        "zo_run_set_q8act": (None, [C.c_void_p, C.c_int]),
        "zo_run_generate": (C.c_int, [C.c_void_p, _u32p, C.c_uint32, C.c_uint32, _u32p, _f32p, _f32p]),
        "zo_moe_route_f32": (C.c_int, [_f32p, sz, _f32p, _f32p, sz, sz, _f32p, _u32p, _f32p, C.c_int, C.c_float]),
        "zo_expert_swiglu": (C.c_int, [_f32p, _u8p, _u8p, _u8p, sz, sz, C.c_int, _f32p, _f32p]),
        "zo_moe_ffn": (C.c_int, [_f32p, _f32p, _f32p, _u8p, _u8p, _u8p, _u8p, _u8p, _u8p, sz, sz, sz, sz,
                                 sz, C.c_int, C.c_int, C.c_float, _f32p, _u32p, _f32p, _f32p]),
        "zo_mla_work_floats": (sz, [C.c_void_p, C.c_uint32]),
        "zo_mla_attention": (C.c_int, [_f32p, C.c_void_p, C.c_void_p, _f32p, C.c_uint32, C.c_uint32, _f32p,
                                       _f32p]),
        "zo_ds2_run_create": (C.c_void_p, [C.c_void_p, C.c_uint32]),
        "zo_ds2_run_create_order": (C.c_void_p, [C.c_void_p, C.c_uint32, C.c_int, C.c_int, C.c_int]),
        "zo_ds2_run_threads": (C.c_int, [C.c_void_p]),
        "zo_ds2_run_set_cache_rows": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, _f32p]),
        "zo_linear_plain_pool": (C.c_int, [C.c_void_p, _f32p, _u8p, _f32p, sz, sz, C.c_int, C.c_int]),
        "zo_ds2_run_destroy": (None, [C.c_void_p]),
        "zo_ds2_run_forward": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, _f32p]),
        "zo_ds2_run_lm_head": (C.c_int, [C.c_void_p, _u32p, _f32p]),
        "zo_ds2_run_generate": (C.c_int, [C.c_void_p, _u32p, C.c_uint32, C.c_uint32, _u32p, _f32p, _f32p]),
        "zo_ds2_run_cache": (_f32p, [C.c_void_p]),
        "zo_ds2_run_mha_cache": (_f32p, [C.c_void_p]),
        "zo_mha_work_floats": (sz, [C.c_void_p, C.c_uint32, C.c_uint32]),
        "zo_mha_attention": (C.c_int, [_f32p, _u8p, _u8p, _u8p, _u8p, C.c_void_p, C.c_uint32, _f32p, _f32p,
                                       C.c_uint32, C.c_uint32, _f32p, _f32p]),
        "zo_ds2_run_expert_ids": (_u32p, [C.c_void_p]),
        "zo_ds2_run_expert_weights": (_f32p, [C.c_void_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _b(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(_u8p)


def _u(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_u32p)


# ---------------------------------------------------------------- codecs
def fp16_to_f32(bits: int) -> float:
    return LIB.zo_fp16_to_f32(bits)


def f64_to_fp16(v: float) -> int:
    return LIB.zo_f64_to_fp16(v)


def quantize_q4_0_block(v) -> bytes:
    x = np.ascontiguousarray(np.asarray(v, dtype=np.float32))
    out = np.zeros(18, np.uint8)
    LIB.zo_quantize_q4_0_block(_f(x), _b(out))
    return out.tobytes()


def quantize_q8_0_block(v) -> bytes:
    x = np.ascontiguousarray(np.asarray(v, dtype=np.float32))
    out = np.zeros(34, np.uint8)
    LIB.zo_quantize_q8_0_block(_f(x), _b(out))
    return out.tobytes()


def quantize_row_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32 * 34, np.uint8)
    LIB.zo_quantize_row_q8_0(_f(x), _b(out), x.size)
    return out


RNG_ZERO_SEED = 0x853C49E6748FEA9B   # Rng::new(0) (rng.rs:27-33)


def rng_seed(seed: int) -> int:
    return seed if seed != 0 else RNG_ZERO_SEED


def lm_head_sample(logits: np.ndarray, rng_state: int, temperature: float, vocab_real: int = 151643):
    """sampler.rs:41-120: returns (token, the advanced rng state)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    st = C.c_uint64(rng_state)
    tok = LIB.zo_lm_head_sample(_f(x), x.size, C.byref(st), C.c_float(temperature), vocab_real)
    return int(tok), int(st.value)


def dequant_kquant_block(blk, quant: str) -> np.ndarray:
    """One Q4_K (144 bytes) or Q6_K (210 bytes) super-block -> 256 floats."""
    b = np.ascontiguousarray(np.frombuffer(bytes(blk), np.uint8))
    out = np.zeros(256, np.float32)
    (LIB.zo_dequant_q4_k_block if quant == "q4_k" else LIB.zo_dequant_q6_k_block)(_b(b), _f(out))
    return out


def linear_kquant(x: np.ndarray, w: np.ndarray, in_dim: int, out_dim: int, quant: str) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(out_dim, np.float32)
    (LIB.zo_linear_q4_k if quant == "q4_k" else LIB.zo_linear_q6_k)(_f(x), _b(np.ascontiguousarray(w, np.uint8)),
                                                                    _f(out), in_dim, out_dim)
    return out


def exp_approx(x: float) -> float:
    return float(LIB.zo_exp_approx(C.c_float(x)))


def linear_q8_0_q8act(xq: np.ndarray, w: np.ndarray, in_dim: int, out_dim: int) -> np.ndarray:
    out = np.zeros(out_dim, np.float32)
    LIB.zo_linear_q8_0_q8act(_b(np.ascontiguousarray(xq, np.uint8)), _b(np.ascontiguousarray(w, np.uint8)),
                             _f(out), in_dim, out_dim)
    return out


def linear_q4_0_q8act(xq: np.ndarray, w: np.ndarray, in_dim: int, out_dim: int) -> np.ndarray:
    out = np.zeros(out_dim, np.float32)
    LIB.zo_linear_q4_0_q8act(_b(np.ascontiguousarray(xq, np.uint8)), _b(np.ascontiguousarray(w, np.uint8)),
                             _f(out), in_dim, out_dim)
    return out


def dequant_q4_0_block(blk: bytes) -> np.ndarray:
    b = np.frombuffer(blk, np.uint8).copy()
    out = np.zeros(32, np.float32)
    LIB.zo_dequant_q4_0_block(_b(b), _f(out))
    return out


def dequant_q8_0_block(blk: bytes) -> np.ndarray:
    b = np.frombuffer(blk, np.uint8).copy()
    out = np.zeros(32, np.float32)
    LIB.zo_dequant_q8_0_block(_b(b), _f(out))
    return out


def interleave_x4(plain: np.ndarray, rows: int, cols: int, quant: int) -> np.ndarray:
    plain = np.ascontiguousarray(plain, dtype=np.uint8)
    out = np.zeros_like(plain)
    rc = LIB.zo_interleave_x4(_b(plain), _b(out), rows, cols, quant)
    if rc:
        raise ValueError(f"interleave_x4 rejected rows={rows} cols={cols}")
    return out


# ------------------------------------------------------------ scalar ops
def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    LIB.zo_rmsnorm(_f(x), _f(w), _f(out), x.size, eps)
    return out


def rope_ctx(base: float, half: int) -> np.ndarray:
    out = np.zeros(half, np.float32)
    LIB.zo_rope_ctx(base, half, _f(out))
    return out


def rope(qk: np.ndarray, inv: np.ndarray, pos: int) -> np.ndarray:
    qk = np.ascontiguousarray(qk, np.float32).copy()
    inv = np.ascontiguousarray(inv, np.float32)
    LIB.zo_rope(_f(qk), _f(inv), inv.size, pos)
    return qk


def linear(x: np.ndarray, w: np.ndarray, in_dim: int, out_dim: int, quant: int) -> np.ndarray:
    """Scalar linear_dispatch (ops.rs:486) on plain blocks."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(out_dim, np.float32)
    rc = LIB.zo_linear_dispatch(_f(x), _b(np.ascontiguousarray(w, np.uint8)), _f(out), in_dim, out_dim, quant)
    if rc:
        raise ValueError(f"linear_dispatch: unsupported quant {quant}")
    return out


def linear_x4_avx512(x, w_x4, in_dim, out_dim, quant, threads=0, simd=1) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(out_dim, np.float32)
    fn = LIB.zo_linear_q4_0x4_avx512 if quant == Q4_0 else LIB.zo_linear_q8_0x4_avx512
    fn(_f(x), _b(np.ascontiguousarray(w_x4, np.uint8)), _f(out), in_dim, out_dim, threads, simd)
    return out


def linear_plain_avx512(x, w, in_dim, out_dim, quant, threads=0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(out_dim, np.float32)
    fn = LIB.zo_linear_q4_0_avx512 if quant == Q4_0 else LIB.zo_linear_q8_0_avx512
    fn(_f(x), _b(np.ascontiguousarray(w, np.uint8)), _f(out), in_dim, out_dim, threads, 0)
    return out


def softmax(s: np.ndarray):
    s = np.ascontiguousarray(s, np.float32).copy()
    rc = LIB.zo_softmax(_f(s), s.size)
    return rc, s


def gqa_attention_decode(qkv: np.ndarray, q_norm: np.ndarray, k_norm: np.ndarray, inv: np.ndarray,
                         k_block: np.ndarray, v_block: np.ndarray, pos: int, n_q: int, n_kv: int,
                         hd: int, eps: float, order: int = 1):
    """One layer of decode attention (attention.rs:344-425 / inference_avx512.rs:1612-1800).

    k_block / v_block are the layer's cache blocks [max_tokens * n_kv * hd],
    updated in place at `pos`.  Returns (rc, out[n_q * hd])."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    qd, kvd = n_q * hd, n_kv * hd
    q, k, v = qkv[:qd].copy(), qkv[qd:qd + kvd].copy(), qkv[qd + kvd:qd + 2 * kvd].copy()
    assert k_block.dtype == np.float32 and k_block.flags.c_contiguous
    assert v_block.dtype == np.float32 and v_block.flags.c_contiguous
    max_tokens = k_block.size // kvd
    work = np.zeros((n_q + n_kv + 1) * hd + max_tokens, np.float32)
    out = np.zeros(qd, np.float32)
    rc = LIB.zo_gqa_attention_decode(_f(q), _f(k), _f(v), _f(np.ascontiguousarray(q_norm, np.float32)),
                                     _f(np.ascontiguousarray(k_norm, np.float32)),
                                     _f(np.ascontiguousarray(inv, np.float32)), _f(k_block), _f(v_block),
                                     pos, max_tokens, n_q, n_kv, hd, eps, order, _f(work), _f(out))
    return rc, out


def exp_avx512(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    LIB.zo_exp_avx512(_f(x), _f(y), x.size)
    return y


def silu_mul_avx512(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.zeros_like(g)
    LIB.zo_silu_mul_avx512(_f(g), _f(u), _f(out), g.size)
    return out


def rope_lut_avx512(pos: int, inv: np.ndarray):
    inv = np.ascontiguousarray(inv, np.float32)
    c = np.zeros_like(inv)
    s = np.zeros_like(inv)
    LIB.zo_rope_sincos_lut_avx512(pos, _f(inv), _f(c), _f(s), inv.size)
    return c, s


def rope_apply_avx512(qk: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    qk = np.ascontiguousarray(qk, np.float32).copy()
    LIB.zo_rope_apply_avx512(_f(qk), _f(np.ascontiguousarray(c, np.float32)),
                             _f(np.ascontiguousarray(s, np.float32)), c.size)
    return qk


def argmax_avx512(v: np.ndarray):
    v = np.ascontiguousarray(v, np.float32)
    mx = C.c_float(0)
    idx = LIB.zo_argmax_avx512(_f(v), v.size, C.byref(mx))
    return idx, mx.value


def have_avx512() -> bool:
    return bool(LIB.zo_have_avx512())


# ------------------------------------------------------------ model runs
class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "attn_norm", "attn_q", "attn_k", "attn_v", "attn_o", "q_norm", "k_norm",
        "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")]


class _Model(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32), ("hidden", C.c_uint32), ("ffn", C.c_uint32),
        ("n_q_heads", C.c_uint32), ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
        ("vocab_padded", C.c_uint32), ("vocab_real", C.c_uint32),
        ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("token_embd_quant", C.c_int), ("token_embd", C.c_void_p),
        ("output_quant", C.c_int), ("output", C.c_void_p), ("output_norm", C.c_void_p),
        ("layers", C.POINTER(_Layer)),
    ]


class OracleRun:
    """A Qwen3-shaped decode run on the CPU oracle.

    ``weights`` is the dict produced by ``zero_b200.synth.qwen3_weights``
    (plain-layout blocks).  order: ORDER_SCALAR (crate, forward_pass.rs:515)
    or ORDER_AVX512 (inference_avx512.rs:1826).
    """

    def __init__(self, cfg, weights, max_tokens: int, order: int = ORDER_AVX512,
                 threads: int = 0, simd: int = 1):
        self._keep = weights
        L = cfg.n_layers
        self._layers = (_Layer * L)()
        for i in range(L):
            lw = weights["layers"][i]
            for name in _Layer._fields_:
                setattr(self._layers[i], name[0], lw[name[0]].ctypes.data)
        self._m = _Model(
            cfg.n_layers, cfg.hidden, cfg.ffn, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim,
            cfg.vocab_padded, cfg.vocab_real, cfg.rms_eps, cfg.rope_theta,
            Q8_0 if cfg.embd_quant == "q8_0" else Q4_0, weights["token_embd"].ctypes.data,
            Q8_0 if cfg.output_quant == "q8_0" else Q4_0, weights["output"].ctypes.data,
            weights["output_norm"].ctypes.data, self._layers)
        self.cfg = cfg
        self.max_tokens = max_tokens
        self._r = LIB.zo_run_create(C.byref(self._m), max_tokens, order, threads, simd)
        if not self._r:
            raise MemoryError("oracle run allocation failed")

    def close(self):
        if self._r:
            LIB.zo_run_destroy(self._r)
            self._r = None

    def __del__(self):
        self.close()

    def set_q8act(self, on=True):
        """Q4_0 matmuls on Q8_0-quantised inputs (the prefill path's
        arithmetic); on=2 quantises the Q8_0 LM head's input too (the batched
        decode path)."""
        LIB.zo_run_set_q8act(self._r, 2 if on == 2 else (1 if on else 0))

    def forward(self, token: int, pos: int) -> np.ndarray:
        h = np.zeros(self.cfg.hidden, np.float32)
        rc = LIB.zo_run_forward(self._r, token, pos, _f(h))
        if rc:
            raise RuntimeError(f"oracle forward failed: {rc}")
        return h

    def lm_head(self):
        logits = np.zeros(self.cfg.vocab_padded, np.float32)
        tok = C.c_uint32(0)
        rc = LIB.zo_run_lm_head(self._r, C.byref(tok), _f(logits))
        return rc, tok.value, logits

    def kv(self) -> np.ndarray:
        c = self.cfg
        n = 2 * c.n_layers * self.max_tokens * c.n_kv_heads * c.head_dim
        return np.ctypeslib.as_array(LIB.zo_run_kv(self._r), shape=(n,)).copy()

    def generate(self, prompt, n_gen: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.zeros(n_gen, np.uint32)
        margins = np.zeros(n_gen, np.float32)
        logits = np.zeros((n_gen, self.cfg.vocab_padded), np.float32) if want_logits else None
        rc = LIB.zo_run_generate(self._r, _u(p), p.size, n_gen, _u(toks), _f(margins),
                                 _f(logits) if want_logits else None)
        return rc, toks, margins, logits


# ------------------------------------------------------------ DeepSeek2
ROUTE_SOFTMAX, ROUTE_SIGMOID_NORMALIZE = 0, 1


def _fopt(a):
    return None if a is None else _f(np.ascontiguousarray(a, np.float32))


def moe_route_f32(hidden, router_w, n_experts: int, top_k: int, mode: int = ROUTE_SOFTMAX,
                  expert_weight_scale: float = 1.0, router_bias=None):
    """moe_route_f32 (moe.rs:132-317).  Returns (rc, ids, weights, scores)."""
    x = np.ascontiguousarray(hidden, np.float32)
    w = np.ascontiguousarray(router_w, np.float32)
    b = None if router_bias is None else np.ascontiguousarray(router_bias, np.float32)
    scores = np.zeros(max(n_experts, 1), np.float32)
    ids = np.zeros(max(top_k, 1), np.uint32)
    wts = np.zeros(max(top_k, 1), np.float32)
    rc = LIB.zo_moe_route_f32(_f(x), x.size, _f(w), None if b is None else _f(b), n_experts, top_k,
                              _f(scores), _u(ids), _f(wts), mode, expert_weight_scale)
    return rc, ids[:top_k], wts[:top_k], scores[:n_experts]


def expert_swiglu(x, gate, up, down, dim: int, inter: int, quant: int = Q4_0) -> np.ndarray:
    """expert_swiglu (moe.rs:345-397) on plain blocks."""
    x = np.ascontiguousarray(x, np.float32)
    work = np.zeros(3 * inter, np.float32)
    out = np.zeros(dim, np.float32)
    rc = LIB.zo_expert_swiglu(_f(x), _b(gate), _b(up), _b(down), dim, inter, quant, _f(work), _f(out))
    if rc:
        raise ValueError(f"expert_swiglu failed: {rc}")
    return out


def moe_ffn(x, lw: dict, cfg, quant: int = Q4_0):
    """moe_ffn (moe.rs:486-590) over one synth.ds2_weights() layer dict.
    Returns (rc, out, ids, weights)."""
    x = np.ascontiguousarray(x, np.float32)
    H, EF, E, K, NS = cfg.hidden, cfg.expert_ffn, cfg.n_experts, cfg.top_k, cfg.n_shared
    work = np.zeros(E + 3 * EF + H, np.float32)
    ids = np.zeros(K, np.uint32)
    wts = np.zeros(K, np.float32)
    out = np.zeros(H, np.float32)
    empty = np.zeros(1, np.uint8)
    rc = LIB.zo_moe_ffn(_f(x), _f(lw["router_w"]), _fopt(lw.get("router_b")), _b(lw["gate_exps"]),
                        _b(lw["up_exps"]), _b(lw["down_exps"]), _b(lw.get("gate_shexp", empty)),
                        _b(lw.get("up_shexp", empty)), _b(lw.get("down_shexp", empty)), NS, E, K, H, EF,
                        quant, cfg.route_mode, cfg.expert_weight_scale, _f(work), _u(ids), _f(wts), _f(out))
    return rc, out, ids, wts


class _MlaDims(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("n_heads", C.c_uint32), ("kv_lora_rank", C.c_uint32),
                ("q_lora_rank", C.c_uint32), ("nope_dim", C.c_uint32), ("rope_dim", C.c_uint32),
                ("v_dim", C.c_uint32), ("quant", C.c_int), ("eps", C.c_float), ("rope_base", C.c_float)]


class _MlaWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("kv_a_mqa", "kv_a_norm", "kv_b", "k_b", "v_b", "q_a", "q_a_norm",
                                          "q_b", "output", "k_norm")]


class _Ds2Layer(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p), ("mla", _MlaWeights), ("moe", C.c_int),
                ("ffn_gate", C.c_void_p), ("ffn_up", C.c_void_p), ("ffn_down", C.c_void_p),
                ("router_w", C.c_void_p), ("router_b", C.c_void_p), ("gate_exps", C.c_void_p),
                ("up_exps", C.c_void_p), ("down_exps", C.c_void_p), ("gate_shexp", C.c_void_p),
                ("up_shexp", C.c_void_p), ("down_shexp", C.c_void_p), ("mha", C.c_int),
                ("q_mha", C.c_void_p), ("k_mha", C.c_void_p), ("v_mha", C.c_void_p)]


class _Ds2(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("ffn", C.c_uint32), ("n_experts", C.c_uint32),
                ("top_k", C.c_uint32), ("expert_ffn", C.c_uint32), ("n_shared", C.c_uint32),
                ("vocab_padded", C.c_uint32), ("vocab_real", C.c_uint32), ("mla", _MlaDims),
                ("route_mode", C.c_int), ("expert_weight_scale", C.c_float), ("token_embd_quant", C.c_int),
                ("token_embd", C.c_void_p), ("output_quant", C.c_int), ("output", C.c_void_p),
                ("output_norm", C.c_void_p), ("layers", C.POINTER(_Ds2Layer)), ("n_kv_heads", C.c_uint32)]


def _addr(d: dict, name: str):
    a = d.get(name)
    return None if a is None else a.ctypes.data


def _mla_dims(cfg) -> _MlaDims:
    return _MlaDims(cfg.hidden, cfg.n_heads, cfg.kv_lora_rank, cfg.q_lora_rank, cfg.nope_dim, cfg.rope_dim,
                    cfg.v_dim, Q4_0, cfg.rms_eps, cfg.rope_theta)


def _mla_weights(lw: dict) -> _MlaWeights:
    return _MlaWeights(*[_addr(lw, n) for n in ("kv_a_mqa", "kv_a_norm", "kv_b", "k_b", "v_b", "q_a",
                                                 "q_a_norm", "q_b", "attn_output", "k_norm")])


def mla_attention(x, lw: dict, cfg, cache_layer: np.ndarray, pos: int):
    """mla_attention_single_token (mla.rs:122-414) for one layer; cache_layer
    ([max_tokens, kv_lora + rope] f32) is updated in place.  Returns (rc, out)."""
    x = np.ascontiguousarray(x, np.float32)
    assert cache_layer.dtype == np.float32 and cache_layer.flags.c_contiguous
    max_tokens = cache_layer.shape[0]
    dims = _mla_dims(cfg)
    w = _mla_weights(lw)
    work = np.zeros(LIB.zo_mla_work_floats(C.byref(dims), max_tokens), np.float32)
    out = np.zeros(cfg.hidden, np.float32)
    rc = LIB.zo_mla_attention(_f(x), C.byref(w), C.byref(dims), _f(cache_layer), pos, max_tokens, _f(work),
                              _f(out))
    return rc, out


def mha_attention(x, lw: dict, cfg, k_cache: np.ndarray, v_cache: np.ndarray, pos: int):
    """mha_attention_single_token (mla.rs:449-618) for one MHA layer; the K / V
    blocks ([max_tokens, n_kv * q_head], [max_tokens, n_kv * v_dim] f32) are
    updated in place.  Returns (rc, out)."""
    x = np.ascontiguousarray(x, np.float32)
    for c in (k_cache, v_cache):
        assert c.dtype == np.float32 and c.flags.c_contiguous
    max_tokens = k_cache.shape[0]
    dims = _mla_dims(cfg)
    work = np.zeros(LIB.zo_mha_work_floats(C.byref(dims), cfg.kv_heads, max_tokens), np.float32)
    out = np.zeros(cfg.hidden, np.float32)
    rc = LIB.zo_mha_attention(_f(x), *(_b(lw[n]) for n in ("q_mha", "k_mha", "v_mha", "attn_output")),
                              C.byref(dims), cfg.kv_heads, _f(k_cache), _f(v_cache), pos, max_tokens, _f(work),
                              _f(out))
    return rc, out


class OracleDs2Run:
    """A DeepSeek2-shaped decode run on the CPU oracle, over synth.ds2_weights()
    tensors.  order: ORDER_SCALAR (the crate's scalar path,
    forward_pass.rs:703-909; the parity oracle) or ORDER_AVX512 (its AVX-512
    kernel path, inference_avx512.rs:2141-2825, the one the reference times),
    the latter over a persistent pool of `threads` participants (<= 0: one per
    physical core); simd 0 runs the lane emulation (same bits)."""

    def __init__(self, cfg, weights, max_tokens: int, order: int = ORDER_SCALAR, threads: int = 1,
                 simd: int = 1):
        self._keep = weights
        self.cfg = cfg
        self.max_tokens = max_tokens
        L = cfg.n_layers
        self._layers = (_Ds2Layer * L)()
        for i in range(L):
            lw = weights["layers"][i]
            ly = self._layers[i]
            ly.attn_norm = _addr(lw, "attn_norm")
            ly.ffn_norm = _addr(lw, "ffn_norm")
            ly.mla = _mla_weights(lw)
            ly.moe = 1 if cfg.is_moe(i) else 0
            if cfg.is_mha(i):
                ly.mha = 1
                ly.q_mha, ly.k_mha, ly.v_mha = (_addr(lw, n) for n in ("q_mha", "k_mha", "v_mha"))
            for n in ("ffn_gate", "ffn_up", "ffn_down", "router_w", "router_b", "gate_exps", "up_exps",
                      "down_exps", "gate_shexp", "up_shexp", "down_shexp"):
                setattr(ly, n, _addr(lw, n))
        self._m = _Ds2(cfg.n_layers, cfg.ffn, cfg.n_experts, cfg.top_k, cfg.expert_ffn, cfg.n_shared,
                       cfg.vocab_padded, cfg.vocab_real, _mla_dims(cfg), cfg.route_mode, cfg.expert_weight_scale,
                       Q8_0 if cfg.embd_quant == "q8_0" else Q4_0, weights["token_embd"].ctypes.data,
                       Q8_0 if cfg.output_quant == "q8_0" else Q4_0, weights["output"].ctypes.data,
                       weights["output_norm"].ctypes.data, self._layers, cfg.kv_heads)
        self._r = LIB.zo_ds2_run_create_order(C.byref(self._m), max_tokens, order, threads, simd)
        if not self._r:
            raise MemoryError("oracle ds2 run allocation failed")
        self.order = order

    @property
    def threads(self) -> int:
        return LIB.zo_ds2_run_threads(self._r)

    def set_cache_rows(self, layer: int, t0: int, rows: np.ndarray):
        """Cached latent rows [t0, t0 + len(rows)) of one layer := rows [n, kv_lora + rope]."""
        rows = np.ascontiguousarray(rows, np.float32)
        rc = LIB.zo_ds2_run_set_cache_rows(self._r, layer, t0, rows.shape[0], _f(rows))
        if rc:
            raise ValueError(f"oracle ds2 cache rows refused: {rc}")

    def close(self):
        if self._r:
            LIB.zo_ds2_run_destroy(self._r)
            self._r = None

    def __del__(self):
        self.close()

    def forward(self, token: int, pos: int) -> np.ndarray:
        h = np.zeros(self.cfg.hidden, np.float32)
        rc = LIB.zo_ds2_run_forward(self._r, token, pos, _f(h))
        if rc:
            raise RuntimeError(f"oracle ds2 forward failed: {rc}")
        return h

    def lm_head(self):
        logits = np.zeros(self.cfg.vocab_padded, np.float32)
        tok = C.c_uint32(0)
        rc = LIB.zo_ds2_run_lm_head(self._r, C.byref(tok), _f(logits))
        return rc, tok.value, logits

    def mha_cache(self):
        """[(K [max_tokens, n_kv * q_head], V [max_tokens, n_kv * v_dim])] per MHA layer, in layer order."""
        c = self.cfg
        kb, vb = self.max_tokens * c.kv_heads * c.q_head, self.max_tokens * c.kv_heads * c.v_dim
        n = len(c.mha_layers)
        a = np.ctypeslib.as_array(LIB.zo_ds2_run_mha_cache(self._r), shape=(max(n, 1) * (kb + vb),)).copy()
        return [(a[i * (kb + vb):i * (kb + vb) + kb].reshape(self.max_tokens, -1),
                 a[i * (kb + vb) + kb:(i + 1) * (kb + vb)].reshape(self.max_tokens, -1)) for i in range(n)]

    def cache(self) -> np.ndarray:
        c = self.cfg
        n = c.n_layers * self.max_tokens * (c.kv_lora_rank + c.rope_dim)
        return np.ctypeslib.as_array(LIB.zo_ds2_run_cache(self._r), shape=(n,)).copy().reshape(
            c.n_layers, self.max_tokens, c.kv_lora_rank + c.rope_dim)

    def expert_ids(self):
        c = self.cfg
        n = c.n_layers * c.top_k
        ids = np.ctypeslib.as_array(LIB.zo_ds2_run_expert_ids(self._r), shape=(n,)).copy()
        wts = np.ctypeslib.as_array(LIB.zo_ds2_run_expert_weights(self._r), shape=(n,)).copy()
        return ids.reshape(c.n_layers, c.top_k), wts.reshape(c.n_layers, c.top_k)

    def generate(self, prompt, n_gen: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.zeros(n_gen, np.uint32)
        margins = np.zeros(n_gen, np.float32)
        logits = np.zeros((n_gen, self.cfg.vocab_padded), np.float32) if want_logits else None
        rc = LIB.zo_ds2_run_generate(self._r, _u(p), p.size, n_gen, _u(toks), _f(margins),
                                     _f(logits) if want_logits else None)
        return rc, toks, margins, logits
