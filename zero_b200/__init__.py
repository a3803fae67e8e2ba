"""zero_b200 — B200 (sm_100a) drop-in for the zero-llm-inference decode hot path.

Python mirror of the crate API the C ABI (include/zgpu.h) exports, used by
the tests and the benchmark.  The names follow the reference crate
(crates/zero-llm-inference): ``linear_dispatch`` (ops.rs:486), ``rmsnorm``
(ops.rs:29), ``KvCache`` (kv_cache.rs:32), ``forward_single_token``
(forward_pass.rs:515), ``lm_head_argmax_dynamic`` (lm_head.rs:98), and the
greedy loop of kernel/src/inference.rs:1836.  Errors surface as ZgpuError
carrying the status code that mirrors the Rust error enum.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import LIB, ZgpuDs2Desc, ZgpuDs2Layer, ZgpuOpts, ZgpuPerf, ZgpuQwen3Desc, ZgpuQwen3Layer
from . import synth
from .synth import DS2_V2_LITE, QWEN3_1_7B, Ds2Config, Qwen3Config

ABI_VERSION = 1
F32, F16, Q4_0, Q8_0, Q4_0X4, Q8_0X4 = 0, 1, 2, 8, 100, 101
Q4_K, Q6_K = 12, 14     # GGUF K-quants (plain rows of 256-element super-blocks)
IPC_HANDLE_BYTES = 64   # ZGPU_IPC_HANDLE_BYTES
FLAG_NO_GRAPH, FLAG_NO_PDL, FLAG_NO_PERSISTENT = 0x1, 0x2, 0x4
ROUTE_SOFTMAX, ROUTE_SIGMOID_NORMALIZE = 0, 1

STATUS = {
    0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED_QUANT", 3: "UNREGISTERED_WEIGHT",
    10: "KV_TOKEN_OUT_OF_RANGE", 11: "KV_LAYER_OUT_OF_RANGE", 12: "KV_INVALID_SLICE_LENGTH",
    13: "KV_TOKEN_COUNT_EXCEEDS_MAX", 20: "NUMERICAL_INSTABILITY", 30: "EMBED_UNSUPPORTED_QUANT",
    31: "EMBED_DIM_MISALIGNMENT", 40: "LM_NON_FINITE_LOGITS", 41: "LM_ARGMAX_IN_PADDING",
    90: "NO_DEVICE", 91: "CUDA", 92: "OUT_OF_MEMORY", 93: "DEVICE_TIMEOUT",
}


class ZgpuError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.name = STATUS.get(status, str(status))


def _ptr(a: np.ndarray) -> int:
    if not a.flags.c_contiguous:
        raise ValueError("array must be C-contiguous")
    return a.ctypes.data


class Context:
    """A device context (zgpu_init).  Keeps every registered host array alive."""

    def __init__(self, device: int = 0, graph: bool = True, pdl: bool = True, persistent: bool = True):
        flags = ((0 if graph else FLAG_NO_GRAPH) | (0 if pdl else FLAG_NO_PDL)
                 | (0 if persistent else FLAG_NO_PERSISTENT))
        opts = ZgpuOpts(ABI_VERSION, device, flags)
        h = C.c_void_p()
        st = LIB.zgpu_init(C.byref(opts), C.byref(h))
        if st:
            raise ZgpuError(st, LIB.zgpu_status_string(st).decode())
        self.h = h
        self._keep: dict[int, np.ndarray] = {}

    def _check(self, st: int):
        if st:
            raise ZgpuError(st, (LIB.zgpu_last_error(self.h) or b"").decode())

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def device_info(self) -> tuple[int, int, int]:
        sm, ma, mi = C.c_int32(), C.c_int32(), C.c_int32()
        self._check(LIB.zgpu_device_info(self.h, C.byref(sm), C.byref(ma), C.byref(mi)))
        return sm.value, ma.value, mi.value

    def synchronize(self):
        self._check(LIB.zgpu_synchronize(self.h))

    # -------------------------------------------------- weight registry
    def register(self, arr: np.ndarray, dtype: int, rows: int, cols: int) -> int:
        """weight_layout::register + upload; returns the key (host address)."""
        self._check(LIB.zgpu_register_weights(self.h, _ptr(arr), arr.nbytes, dtype, rows, cols))
        self._keep[_ptr(arr)] = arr
        return _ptr(arr)

    def sample_top_k(self, logits: np.ndarray, rng_state: int, temperature: float, vocab_real: int = 151643):
        """lm_head_sample (sampler.rs:41-163) on the GPU: (token, advanced rng state)."""
        x = np.ascontiguousarray(logits, np.float32)
        st, tok = C.c_uint64(rng_state), C.c_uint32()
        self._check(LIB.zgpu_sample_top_k(self.h, _ptr(x), x.size, vocab_real, C.c_float(temperature),
                                          C.byref(st), C.byref(tok)))
        return tok.value, st.value

    def register_smodel(self, smodel) -> int:
        """zgpu_smodel_register: every rank-2 matmul tensor of an open
        SmodelFile, keyed by its mapped address; returns how many."""
        n = C.c_uint32()
        self._check(LIB.zgpu_smodel_register(self.h, smodel.h, C.byref(n)))
        return n.value

    def group_of(self, arr_or_key) -> int:
        key = arr_or_key if isinstance(arr_or_key, int) else _ptr(arr_or_key)
        return int(LIB.zgpu_group_of(self.h, key))

    def clear_weights(self):
        self._check(LIB.zgpu_clear_weights(self.h))
        self._keep.clear()

    # -------------------------------------------------------- matmul ops
    def linear_dispatch(self, x: np.ndarray, w, in_dim: int, out_dim: int, quant: int) -> np.ndarray:
        """linear_dispatch (ops.rs:486) with the registered weight `w` (array or key)."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(out_dim, np.float32)
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_dispatch(self.h, _ptr(x), key, _ptr(out), in_dim, out_dim, quant))
        return out

    def linear_dispatch_device(self, d_x: int, w, d_out: int, in_dim: int, out_dim: int, quant: int,
                               stream: int = 0):
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_dispatch_device(self.h, d_x, key, d_out, in_dim, out_dim, quant,
                                                    stream or None))

    def quantize_q8_0(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.size // 32 * 34, np.uint8)
        self._check(LIB.zgpu_quantize_q8_0(self.h, _ptr(x), _ptr(out), x.size))
        return out

    def linear_q8act(self, xq: np.ndarray, w, in_dim: int, out_dim: int) -> np.ndarray:
        out = np.empty(out_dim, np.float32)
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_q8act(self.h, _ptr(np.ascontiguousarray(xq, np.uint8)), key,
                                          _ptr(out), in_dim, out_dim))
        return out

    def linear_q8act_device(self, d_xq: int, w, d_out: int, in_dim: int, out_dim: int, stream: int = 0):
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_q8act_device(self.h, d_xq, key, d_out, in_dim, out_dim, stream or None))

    def linear_dispatch_batch(self, x: np.ndarray, w, in_dim: int, out_dim: int, quant: int) -> np.ndarray:
        """linear_dispatch of each row of x [n_vec, in_dim] (n_vec <= 32) on the
        tensor cores; row v equals linear_dispatch(x[v]) bit for bit."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, in_dim)
        out = np.empty((x.shape[0], out_dim), np.float32)
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_dispatch_batch(self.h, _ptr(x), key, _ptr(out), x.shape[0], in_dim, out_dim,
                                                   quant))
        return out

    def linear_q8act_batch(self, x: np.ndarray, w, in_dim: int, out_dim: int) -> np.ndarray:
        """T rows of activations (x [T, in_dim] f32) quantised to Q8_0 and
        multiplied by Q4_0 weights on the tcgen05 int8 path; returns [T, out_dim]."""
        x = np.ascontiguousarray(x, np.float32).reshape(-1, in_dim)
        out = np.empty((x.shape[0], out_dim), np.float32)
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_q8act_batch(self.h, _ptr(x), key, _ptr(out), x.shape[0], in_dim, out_dim))
        return out

    def linear_q8act_batch_device(self, d_x: int, w, d_out: int, T: int, in_dim: int, out_dim: int,
                                  stream: int = 0):
        key = w if isinstance(w, int) else _ptr(w)
        self._check(LIB.zgpu_linear_q8act_batch_device(self.h, d_x, key, d_out, T, in_dim, out_dim,
                                                       stream or None))

    # ---------------------------------------------------------- small ops
    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        self._check(LIB.zgpu_rmsnorm(self.h, _ptr(x), _ptr(w), _ptr(out), x.size, eps))
        return out

    def rope(self, qk: np.ndarray, n_heads: int, head_dim: int, pos: int, base: float) -> np.ndarray:
        qk = np.ascontiguousarray(qk, np.float32).copy()
        self._check(LIB.zgpu_rope(self.h, _ptr(qk), n_heads, head_dim, pos, base))
        return qk

    def silu_mul(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        out = np.empty_like(g)
        self._check(LIB.zgpu_silu_mul(self.h, _ptr(g), _ptr(u), _ptr(out), g.size))
        return out


    # ------------------------------------------------------- MoE routing
    def moe_route_f32(self, hidden: np.ndarray, router, n_experts: int, top_k: int,
                      mode: int = ROUTE_SOFTMAX, expert_weight_scale: float = 1.0,
                      router_bias: np.ndarray | None = None):
        """moe_route_f32 (moe.rs:132-317) with a registered f32 router.
        Returns (indices u32[top_k], weights f32[top_k], scores f32[n_experts])."""
        x = np.ascontiguousarray(hidden, np.float32)
        key = router if isinstance(router, int) else _ptr(router)
        b = None if router_bias is None else np.ascontiguousarray(router_bias, np.float32)
        idx = np.empty(top_k, np.uint32)
        wts = np.empty(top_k, np.float32)
        scores = np.empty(max(n_experts, 1), np.float32)
        self._check(LIB.zgpu_moe_route_f32(self.h, _ptr(x), key, None if b is None else _ptr(b), x.size,
                                           n_experts, top_k, mode, expert_weight_scale, _ptr(scores),
                                           _ptr(idx), _ptr(wts)))
        return idx, wts, scores[:n_experts]


class KvCache:
    """KvCache::new (kv_cache.rs:100) in device memory, same logical layout."""

    def __init__(self, ctx: Context, max_tokens: int, n_layers: int, n_kv_heads: int, head_dim: int):
        self.ctx = ctx
        self.max_tokens, self.n_layers, self.n_kv_heads, self.head_dim = max_tokens, n_layers, n_kv_heads, head_dim
        h = C.c_void_p()
        ctx._check(LIB.zgpu_kv_create(ctx.h, max_tokens, n_layers, n_kv_heads, head_dim, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_kv_destroy(self.h)
            self.h = None

    def store_kv(self, layer: int, token: int, k: np.ndarray, v: np.ndarray):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self.ctx._check(LIB.zgpu_kv_store(self.h, layer, token, _ptr(k), _ptr(v), k.size))

    def read(self, layer: int, token_count: int):
        n = token_count * self.n_kv_heads * self.head_dim
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        self.ctx._check(LIB.zgpu_kv_read(self.h, layer, token_count, _ptr(k), _ptr(v)))
        return k, v

    def causal_attention(self, layer: int, pos0: int, n_q_heads: int, q: np.ndarray) -> np.ndarray:
        """The prefill's causal attention (zgpu_causal_attention): rotated
        queries q [T, n_q_heads * head_dim] at positions pos0.. over the cached
        keys of `layer`; returns [T, n_q_heads * head_dim]."""
        q = np.ascontiguousarray(q, np.float32)
        T = q.shape[0]
        out = np.empty((T, n_q_heads * self.head_dim), np.float32)
        self.ctx._check(LIB.zgpu_causal_attention(self.ctx.h, self.h, layer, pos0, T, n_q_heads, _ptr(q), _ptr(out)))
        return out

    def gqa_attention_decode(self, layer: int, pos: int, n_q_heads: int, qkv: np.ndarray,
                             q_norm: np.ndarray, k_norm: np.ndarray, freq_base: float,
                             eps: float) -> np.ndarray:
        """Steps 2-5 of gqa_attention_single_token_dispatch (attention.rs:344-425)
        for one layer: QK-norm, RoPE, store k/v at `pos`, softmax attention over
        tokens 0..pos.  Returns the attention output [n_q_heads * head_dim]."""
        qkv = np.ascontiguousarray(qkv, np.float32)
        qn = np.ascontiguousarray(q_norm, np.float32)
        kn = np.ascontiguousarray(k_norm, np.float32)
        out = np.empty(n_q_heads * self.head_dim, np.float32)
        self.ctx._check(LIB.zgpu_gqa_attention_decode(self.ctx.h, self.h, layer, pos, n_q_heads, _ptr(qkv),
                                                      _ptr(qn), _ptr(kn), freq_base, eps, _ptr(out)))
        return out


class Qwen3Model:
    """A Qwen3-shaped model on the device, built from synth.qwen3_weights() tensors.

    Matmul tensors are registered in the .smodel-v2 X4 layout (dtype 100/101)
    when `<name>_x4` copies exist, else as plain Q4_0 blocks.
    """

    def __init__(self, ctx: Context, cfg: Qwen3Config, weights: dict, rank: int = 0, world: int = 1):
        """rank / world > 1: one tensor-parallel rank (zgpu_qwen3_create_tp);
        call tp_export() on every rank, exchange the handles, then
        tp_connect(handles) before decoding."""
        self.ctx, self.cfg, self.w = ctx, cfg, weights
        self.rank, self.world = rank, world
        H = cfg.hidden
        eq = Q8_0 if cfg.embd_quant == "q8_0" else Q4_0
        oq = Q8_0 if cfg.output_quant == "q8_0" else Q4_0
        emb_key = ctx.register(weights["token_embd"], eq, cfg.vocab_padded, H)
        if "output_x4" in weights:
            out_key = ctx.register(weights["output_x4"], Q8_0X4 if oq == Q8_0 else Q4_0X4, cfg.vocab_padded, H)
        elif weights["output"] is weights["token_embd"]:
            out_key = emb_key
        else:
            out_key = ctx.register(weights["output"], oq, cfg.vocab_padded, H)
        shapes = synth.layer_shapes(cfg)
        self._layers = (ZgpuQwen3Layer * cfg.n_layers)()
        for i, lw in enumerate(weights["layers"]):
            L = self._layers[i]
            for name in synth.LAYER_MATS:
                rows, cols = shapes[name]
                if name + "_x4" in lw:
                    key = ctx.register(lw[name + "_x4"], Q4_0X4, rows, cols)
                else:
                    key = ctx.register(lw[name], Q4_0, rows, cols)
                setattr(L, name, key)
            for name in synth.LAYER_NORMS:
                setattr(L, name, _ptr(lw[name]))
        desc = ZgpuQwen3Desc(
            cfg.n_layers, H, cfg.ffn, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim,
            cfg.vocab_padded, cfg.vocab_real, cfg.rms_eps, cfg.rope_theta, eq, emb_key, oq, out_key,
            _ptr(weights["output_norm"]), self._layers)
        h = C.c_void_p()
        if world == 1:
            ctx._check(LIB.zgpu_qwen3_create(ctx.h, C.byref(desc), C.byref(h)))
        else:
            ctx._check(LIB.zgpu_qwen3_create_tp(ctx.h, C.byref(desc), rank, world, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_qwen3_destroy(self.h)
            self.h = None

    def tp_export(self) -> bytes:
        """This rank's CUDA IPC handle of its activation vectors (zgpu_qwen3_tp_export)."""
        buf = (C.c_uint8 * IPC_HANDLE_BYTES)()
        self.ctx._check(LIB.zgpu_qwen3_tp_export(self.h, buf))
        return bytes(buf)

    def tp_connect(self, handles) -> None:
        """Map every rank's activation vectors (handles in rank order)."""
        if len(handles) != self.world or any(len(x) != IPC_HANDLE_BYTES for x in handles):
            raise ZgpuError(3, "tp_connect: one handle per rank")
        blob = (C.c_uint8 * (IPC_HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        self.ctx._check(LIB.zgpu_qwen3_tp_connect(self.h, blob))

    def tp_connect_absent(self):
        """Connect this rank with every other rank absent (zgpu_qwen3_tp_connect_absent):
        a test of the device-side timeout when a peer never arrives."""
        self.ctx._check(LIB.zgpu_qwen3_tp_connect_absent(self.h))

    @property
    def vocab_rows(self) -> int:
        """LM-head rows (logits) of this rank."""
        return self.cfg.vocab_padded // self.world

    def new_kv(self, max_tokens: int) -> KvCache:
        c = self.cfg
        return KvCache(self.ctx, max_tokens, c.n_layers, c.n_kv_heads // self.world, c.head_dim)

    def forward_single_token(self, kv: KvCache, token: int, pos: int) -> np.ndarray:
        hidden = np.empty(self.cfg.hidden, np.float32)
        self.ctx._check(LIB.zgpu_forward_single_token(self.h, kv.h, token, pos, _ptr(hidden)))
        return hidden

    def lm_head_argmax(self, vocab_real: int | None = None, want_logits: bool = True):
        """(token, logits); a tensor-parallel rank's logits are its own vocabulary rows."""
        tok = C.c_uint32()
        logits = np.empty(self.vocab_rows, np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_lm_head_argmax(
            self.h, self.cfg.vocab_real if vocab_real is None else vocab_real, C.byref(tok),
            _ptr(logits) if want_logits else None))
        return tok.value, logits

    def generate_greedy(self, kv: KvCache, prompt, n_gen: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.empty(n_gen, np.uint32)
        logits = np.empty((n_gen, self.vocab_rows), np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_generate_greedy(self.h, kv.h, _ptr(p), p.size, n_gen, _ptr(toks),
                                                 _ptr(logits) if want_logits else None))
        return toks, logits

    def lm_head_sample(self, rng_state: int, temperature: float, vocab_real: int | None = None):
        """lm_head_sample on the logits of the last LM-head call: (token, advanced rng state)."""
        st, tok = C.c_uint64(rng_state), C.c_uint32()
        self.ctx._check(LIB.zgpu_lm_head_sample(self.h, self.cfg.vocab_real if vocab_real is None else vocab_real,
                                                C.c_float(temperature), C.byref(st), C.byref(tok)))
        return tok.value, st.value

    def prefill(self, kv: KvCache, tokens, want_logits: bool = True):
        """Token-parallel prompt prefill on the tensor cores (zgpu_prefill):
        fills cache positions [0, n) and returns (next token, logits)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        tok = C.c_uint32()
        logits = np.empty(self.cfg.vocab_padded, np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_prefill(self.h, kv.h, _ptr(t), t.size, C.byref(tok),
                                         _ptr(logits) if want_logits else None))
        return tok.value, logits

    def prefill_batch(self, kvs, prompts, want_logits: bool = True):
        """zgpu_prefill_batch: prompts [n_seq, n] (equal lengths), one cache per
        sequence; returns (next tokens [n_seq], logits [n_seq, vocab] or None)."""
        t = np.ascontiguousarray(prompts, np.uint32)
        n_seq, n = t.shape
        handles = (C.c_void_p * n_seq)(*[kv.h.value if isinstance(kv.h, C.c_void_p) else kv.h for kv in kvs])
        toks = np.empty(n_seq, np.uint32)
        logits = np.empty((n_seq, self.cfg.vocab_padded), np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_prefill_batch(self.h, handles, n_seq, _ptr(t), n, _ptr(toks),
                                               _ptr(logits) if want_logits else None))
        return toks, logits

    def decode_batch(self, kvs, tokens, positions, want_logits: bool = True):
        """zgpu_decode_batch: one greedy step for len(kvs) sequences, sequence
        i feeding tokens[i] at positions[i] of its own cache; returns (next
        tokens [n_seq], logits [n_seq, vocab] or None)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        pos = np.ascontiguousarray(positions, np.uint32)
        n_seq = len(kvs)
        if t.size != n_seq or pos.size != n_seq:
            raise ValueError("one token and one position per sequence")
        handles = (C.c_void_p * n_seq)(*[kv.h.value if isinstance(kv.h, C.c_void_p) else kv.h for kv in kvs])
        toks = np.empty(n_seq, np.uint32)
        logits = np.empty((n_seq, self.cfg.vocab_padded), np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_decode_batch(self.h, handles, n_seq, _ptr(t), _ptr(pos), _ptr(toks),
                                              _ptr(logits) if want_logits else None))
        return toks, logits

    def generate_batch(self, kvs, prompts, n_gen: int, want_logits: bool = False):
        """Greedy generation for several sequences: the prompts [n_seq, n]
        through zgpu_prefill_batch, then n_gen - 1 zgpu_decode_batch steps.
        Returns (tokens [n_seq, n_gen], logits [n_gen, n_seq, vocab] or None)."""
        p = np.ascontiguousarray(prompts, np.uint32)
        n_seq, n = p.shape
        out = np.empty((n_seq, n_gen), np.uint32)
        lg = [] if want_logits else None
        tok, logits = self.prefill_batch(kvs, p, want_logits)
        out[:, 0] = tok
        if want_logits:
            lg.append(logits)
        for s in range(1, n_gen):
            tok, logits = self.decode_batch(kvs, tok, np.full(n_seq, n + s - 1), want_logits)
            out[:, s] = tok
            if want_logits:
                lg.append(logits)
        return out, (np.stack(lg) if want_logits else None)

    def perf(self) -> dict:
        p = ZgpuPerf()
        self.ctx._check(LIB.zgpu_perf_snapshot(self.h, C.byref(p)))
        return {"steps": p.steps, "kernel_launches": p.kernel_launches, "decode_ms": p.decode_ms,
                "prefill_ms": p.prefill_ms, "decode_launches": p.decode_launches,
                "prefill_gemm_ms": p.prefill_gemm_ms, "prefill_attn_ms": p.prefill_attn_ms,
                "batch_gemm_ms": p.batch_gemm_ms, "batch_attn_ms": p.batch_attn_ms}


class MlaKvCache:
    """MlaKvCache::new (kv_cache.rs:257-305) in device memory: per layer
    max_tokens rows of [kv_lora_rank | rope_dim] f32."""

    def __init__(self, ctx: Context, max_tokens: int, n_layers: int, kv_lora_rank: int, rope_dim: int):
        self.ctx = ctx
        self.max_tokens, self.n_layers, self.kv_lora_rank, self.rope_dim = max_tokens, n_layers, kv_lora_rank, rope_dim
        h = C.c_void_p()
        ctx._check(LIB.zgpu_mla_kv_create(ctx.h, max_tokens, n_layers, kv_lora_rank, rope_dim, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_mla_kv_destroy(self.h)
            self.h = None

    def store_compressed(self, layer: int, token: int, c_kv: np.ndarray, k_rope: np.ndarray):
        c = np.ascontiguousarray(c_kv, np.float32)
        k = np.ascontiguousarray(k_rope, np.float32)
        if c.size != self.kv_lora_rank or k.size != self.rope_dim:
            raise ZgpuError(12, "store_compressed: slice length differs from the cache geometry")
        self.ctx._check(LIB.zgpu_mla_kv_store(self.h, layer, token, _ptr(c), _ptr(k)))

    def read(self, layer: int, token_count: int) -> np.ndarray:
        out = np.empty((token_count, self.kv_lora_rank + self.rope_dim), np.float32)
        self.ctx._check(LIB.zgpu_mla_kv_read(self.h, layer, token_count, _ptr(out)))
        return out

    def copy_from(self, src: "MlaKvCache", token_count: int) -> None:
        """Rows [0, token_count) of every layer of src, copied on the device (zgpu_mla_kv_copy)."""
        self.ctx._check(LIB.zgpu_mla_kv_copy(self.h, src.h, token_count))


class MhaKvCache:
    """MhaKvCache (kv_cache.rs:433-560) in device memory: per MHA layer a K
    block [max_tokens, n_kv * head_dim_qk] and a V block [max_tokens, n_kv * head_dim_v]."""

    def __init__(self, ctx: Context, max_tokens: int, n_mha_layers: int, n_kv_heads: int, head_dim_qk: int,
                 head_dim_v: int):
        self.ctx = ctx
        self.max_tokens, self.n_layers = max_tokens, n_mha_layers
        self.k_width, self.v_width = n_kv_heads * head_dim_qk, n_kv_heads * head_dim_v
        h = C.c_void_p()
        ctx._check(LIB.zgpu_mha_kv_create(ctx.h, max_tokens, n_mha_layers, n_kv_heads, head_dim_qk, head_dim_v,
                                          C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_mha_kv_destroy(self.h)
            self.h = None

    def store(self, layer: int, token: int, k: np.ndarray, v: np.ndarray):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self.ctx._check(LIB.zgpu_mha_kv_store(self.h, layer, token, _ptr(k), _ptr(v)))

    def read(self, layer: int, token_count: int):
        k = np.empty((token_count, self.k_width), np.float32)
        v = np.empty((token_count, self.v_width), np.float32)
        self.ctx._check(LIB.zgpu_mha_kv_read(self.h, layer, token_count, _ptr(k), _ptr(v)))
        return k, v


class Ds2Model:
    """A DeepSeek2-shaped (MLA + MoE) model on the device, built from
    synth.ds2_weights() tensors (plain Q4_0 blocks; routers registered f32)."""

    def __init__(self, ctx: Context, cfg: Ds2Config, weights: dict, rank: int = 0, world: int = 1):
        """rank / world > 1: one expert-parallel rank (zgpu_ds2_create_ep);
        call tp_export() on every rank, exchange the handles, then
        tp_connect(handles) (zero_b200.tp.connect does both) before use."""
        self.rank, self.world = rank, world
        self.ctx, self.cfg, self.w = ctx, cfg, weights
        H = cfg.hidden
        eq = Q8_0 if cfg.embd_quant == "q8_0" else Q4_0
        oq = Q8_0 if cfg.output_quant == "q8_0" else Q4_0
        emb_key = ctx.register(weights["token_embd"], eq, cfg.vocab_padded, H)
        out_key = ctx.register(weights["output"], oq, cfg.vocab_padded, H)
        self._layers = (ZgpuDs2Layer * cfg.n_layers)()
        for i, lw in enumerate(weights["layers"]):
            L = self._layers[i]
            for name, (rows, cols) in synth.ds2_layer_shapes(cfg, i).items():
                setattr(L, name, ctx.register(lw[name], Q4_0, rows, cols))
            for name in ("attn_norm", "ffn_norm", "kv_a_norm", "q_a_norm", "k_norm", "router_b"):
                if name in lw:
                    setattr(L, name, _ptr(lw[name]))
            if cfg.is_moe(i):
                L.moe = 1
                L.router_w = ctx.register(lw["router_w"], F32, cfg.n_experts, H)
            if cfg.is_mha(i):
                L.attn_type = 1   # ZGPU_ATTN_MHA
        desc = ZgpuDs2Desc(
            cfg.n_layers, H, cfg.ffn, cfg.n_heads, cfg.kv_lora_rank, cfg.q_lora_rank, cfg.nope_dim,
            cfg.rope_dim, cfg.v_dim, cfg.n_experts, cfg.top_k, cfg.expert_ffn, cfg.n_shared,
            cfg.vocab_padded, cfg.vocab_real, cfg.rms_eps, cfg.rope_theta, cfg.route_mode,
            cfg.expert_weight_scale, Q4_0, eq, emb_key, oq, out_key, _ptr(weights["output_norm"]),
            self._layers, cfg.n_kv_heads)
        h = C.c_void_p()
        if world == 1:
            ctx._check(LIB.zgpu_ds2_create(ctx.h, C.byref(desc), C.byref(h)))
        else:
            ctx._check(LIB.zgpu_ds2_create_ep(ctx.h, C.byref(desc), rank, world, C.byref(h)))
        self.h = h

    def tp_export(self) -> bytes:
        """This rank's CUDA IPC handle of its expert exchange buffer (zgpu_ds2_ep_export)."""
        buf = (C.c_uint8 * IPC_HANDLE_BYTES)()
        self.ctx._check(LIB.zgpu_ds2_ep_export(self.h, buf))
        return bytes(buf)

    def tp_connect(self, handles) -> None:
        """Map every rank's exchange buffer (handles in rank order)."""
        if len(handles) != self.world or any(len(x) != IPC_HANDLE_BYTES for x in handles):
            raise ZgpuError(3, "tp_connect: one handle per rank")
        blob = (C.c_uint8 * (IPC_HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        self.ctx._check(LIB.zgpu_ds2_ep_connect(self.h, blob))

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_ds2_destroy(self.h)
            self.h = None

    def new_kv(self, max_tokens: int) -> MlaKvCache:
        c = self.cfg
        return MlaKvCache(self.ctx, max_tokens, c.n_layers, c.kv_lora_rank, c.rope_dim)

    def new_mha_kv(self, max_tokens: int, bind: bool = True) -> MhaKvCache:
        """A cache for the model's MHA layers (zgpu_mha_kv_create), bound to the
        model (zgpu_ds2_set_mha_kv) unless bind is False."""
        c = self.cfg
        kv = MhaKvCache(self.ctx, max_tokens, len(c.mha_layers), c.kv_heads, c.q_head, c.v_dim)
        if bind:
            self.set_mha_kv(kv)
        return kv

    def set_mha_kv(self, kv) -> None:
        self.ctx._check(LIB.zgpu_ds2_set_mha_kv(self.h, kv.h if kv is not None else None))

    def forward_single_token(self, kv: MlaKvCache, token: int, pos: int) -> np.ndarray:
        hidden = np.empty(self.cfg.hidden, np.float32)
        self.ctx._check(LIB.zgpu_ds2_forward_single_token(self.h, kv.h, token, pos, _ptr(hidden)))
        return hidden

    def lm_head_argmax(self, vocab_real: int | None = None, want_logits: bool = True):
        tok = C.c_uint32()
        logits = np.empty(self.cfg.vocab_padded, np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_ds2_lm_head_argmax(
            self.h, self.cfg.vocab_real if vocab_real is None else vocab_real, C.byref(tok),
            _ptr(logits) if want_logits else None))
        return tok.value, logits

    def expert_ids(self):
        """[n_layers][top_k] expert ids and weights of the last forward (zeros for dense layers)."""
        k = self.cfg.top_k
        ids = np.empty((self.cfg.n_layers, k), np.uint32)
        wts = np.empty((self.cfg.n_layers, k), np.float32)
        self.ctx._check(LIB.zgpu_ds2_expert_ids(self.h, _ptr(ids), _ptr(wts)))
        return ids, wts

    def generate_greedy(self, kv: MlaKvCache, prompt, n_gen: int, want_logits: bool = False):
        p = np.ascontiguousarray(prompt, np.uint32)
        toks = np.empty(n_gen, np.uint32)
        logits = np.empty((n_gen, self.cfg.vocab_padded), np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_ds2_generate_greedy(self.h, kv.h, _ptr(p), p.size, n_gen, _ptr(toks),
                                                     _ptr(logits) if want_logits else None))
        return toks, logits

    def decode_batch(self, kvs, tokens, positions, want_logits: bool = True):
        """zgpu_ds2_decode_batch: one greedy step for len(kvs) sequences,
        sequence i feeding tokens[i] at positions[i] of its own cache; returns
        (next tokens [n_seq], logits [n_seq, vocab_padded] or None)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        pos = np.ascontiguousarray(positions, np.uint32)
        n_seq = len(kvs)
        if t.size != n_seq or pos.size != n_seq:
            raise ValueError("one token and one position per sequence")
        handles = (C.c_void_p * n_seq)(*[kv.h.value if isinstance(kv.h, C.c_void_p) else kv.h for kv in kvs])
        toks = np.empty(n_seq, np.uint32)
        logits = np.empty((n_seq, self.cfg.vocab_padded), np.float32) if want_logits else None
        self.ctx._check(LIB.zgpu_ds2_decode_batch(self.h, handles, n_seq, _ptr(t), _ptr(pos), _ptr(toks),
                                                  _ptr(logits) if want_logits else None))
        return toks, logits

    def batch_expert_ids(self, n_seq: int):
        """[n_layers][n_seq][top_k] expert ids and weights of the last decode_batch."""
        k = self.cfg.top_k
        ids = np.empty((self.cfg.n_layers, n_seq, k), np.uint32)
        wts = np.empty((self.cfg.n_layers, n_seq, k), np.float32)
        self.ctx._check(LIB.zgpu_ds2_batch_expert_ids(self.h, n_seq, _ptr(ids), _ptr(wts)))
        return ids, wts

    def perf(self) -> dict:
        p = ZgpuPerf()
        self.ctx._check(LIB.zgpu_ds2_perf_snapshot(self.h, C.byref(p)))
        return {"steps": p.steps, "kernel_launches": p.kernel_launches, "decode_ms": p.decode_ms,
                "prefill_ms": p.prefill_ms, "decode_launches": p.decode_launches,
                "prefill_gemm_ms": p.prefill_gemm_ms, "prefill_attn_ms": p.prefill_attn_ms}


__all__ = ["Context", "KvCache", "Qwen3Model", "Qwen3Config", "QWEN3_1_7B", "ZgpuError", "synth",
           "MlaKvCache", "MhaKvCache", "Ds2Model", "Ds2Config", "DS2_V2_LITE", "ROUTE_SOFTMAX", "ROUTE_SIGMOID_NORMALIZE",
           "F32", "Q4_0", "Q8_0", "Q4_0X4", "Q8_0X4", "Q4_K", "Q6_K"]
