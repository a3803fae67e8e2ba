"""ctypes binding of libzgpu.so (the in-tree sm_100a library).

The library must exist: there is no CPU fallback for the decode path.  Build
it with ``python zero_b200/build.py``.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libzgpu.so"

if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing: build the CUDA extension with `python zero_b200/build.py` "
        "(zero_b200 has no CPU fallback)"
    )

LIB = C.CDLL(str(LIB_PATH))

_vp, _u32, _u64, _i32, _f = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32, C.c_float


class ZgpuOpts(C.Structure):
    _fields_ = [("abi_version", _u32), ("device", _i32), ("flags", _u32)]


class ZgpuQwen3Layer(C.Structure):
    _fields_ = [(n, _vp) for n in (
        "attn_norm", "attn_q", "attn_k", "attn_v", "attn_o", "q_norm", "k_norm", "ffn_norm",
        "ffn_gate", "ffn_up", "ffn_down")]


class ZgpuQwen3Desc(C.Structure):
    _fields_ = [
        ("n_layers", _u32), ("hidden", _u32), ("ffn", _u32), ("n_q_heads", _u32),
        ("n_kv_heads", _u32), ("head_dim", _u32), ("vocab_padded", _u32), ("vocab_real", _u32),
        ("rms_eps", _f), ("rope_theta", _f), ("token_embd_quant", _u32), ("token_embd", _vp),
        ("output_quant", _u32), ("output", _vp), ("output_norm", _vp),
        ("layers", C.POINTER(ZgpuQwen3Layer)),
    ]


class ZgpuDs2Layer(C.Structure):
    _fields_ = [
        ("attn_norm", _vp), ("ffn_norm", _vp), ("kv_a_mqa", _vp), ("kv_a_norm", _vp), ("kv_b", _vp),
        ("k_b", _vp), ("v_b", _vp), ("q_a", _vp), ("q_a_norm", _vp), ("q_b", _vp), ("attn_output", _vp),
        ("k_norm", _vp), ("moe", _u32), ("ffn_gate", _vp), ("ffn_up", _vp), ("ffn_down", _vp),
        ("router_w", _vp), ("router_b", _vp), ("gate_exps", _vp), ("up_exps", _vp), ("down_exps", _vp),
        ("gate_shexp", _vp), ("up_shexp", _vp), ("down_shexp", _vp),
        ("attn_type", _u32), ("q_mha", _vp), ("k_mha", _vp), ("v_mha", _vp),
    ]


class ZgpuDs2Desc(C.Structure):
    _fields_ = [
        ("n_layers", _u32), ("hidden", _u32), ("ffn", _u32), ("n_heads", _u32),
        ("kv_lora_rank", _u32), ("q_lora_rank", _u32), ("nope_dim", _u32), ("rope_dim", _u32),
        ("v_dim", _u32), ("n_experts", _u32), ("top_k", _u32), ("expert_ffn", _u32), ("n_shared", _u32),
        ("vocab_padded", _u32), ("vocab_real", _u32), ("rms_eps", _f), ("rope_theta", _f),
        ("route_mode", _u32), ("expert_weight_scale", _f), ("attn_quant", _u32),
        ("token_embd_quant", _u32), ("token_embd", _vp), ("output_quant", _u32), ("output", _vp),
        ("output_norm", _vp), ("layers", C.POINTER(ZgpuDs2Layer)), ("n_kv_heads", _u32),
    ]


class ZgpuPerf(C.Structure):
    _fields_ = [("steps", _u64), ("kernel_launches", _u64), ("decode_ms", C.c_double),
                ("prefill_ms", C.c_double), ("decode_launches", _u64),
                ("prefill_gemm_ms", C.c_double), ("prefill_attn_ms", C.c_double),
                ("batch_gemm_ms", C.c_double), ("batch_attn_ms", C.c_double)]


class ZgpuSmodelInfo(C.Structure):
    _fields_ = [("version", _u32), ("payload_kind", _u32), ("flags", _u32), ("tensor_count", _u32),
                ("manifest_offset", _u64), ("manifest_len", _u64), ("payload_offset", _u64), ("payload_len", _u64),
                ("data_base", _u64),
                ("architecture_id", _u32), ("block_count", _u32), ("context_length", _u32),
                ("embedding_length", _u32), ("feed_forward_length", _u32),
                ("head_count", _u32), ("head_count_kv", _u32), ("key_length", _u32), ("value_length", _u32),
                ("rope_freq_base", _f), ("layer_norm_rms_epsilon", _f),
                ("vocab_size", _u32), ("eos_token_id", _u32), ("expert_count", _u32), ("expert_used_count", _u32),
                ("expert_shared_count", _u32), ("expert_feed_forward_length", _u32), ("kv_lora_rank", _u32),
                ("q_lora_rank", _u32), ("qk_nope_head_dim", _u32), ("qk_rope_head_dim", _u32),
                ("v_head_dim", _u32), ("expert_weights_scale", _f)]


class ZgpuSmodelTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", _u32), ("rank", _u32), ("shape", _u64 * 8),
                ("payload_offset", _u64), ("byte_len", _u64), ("elements", _u64), ("data", _vp)]


_SIGS = {
    "zgpu_init": (_i32, [C.POINTER(ZgpuOpts), C.POINTER(_vp)]),
    "zgpu_destroy": (None, [_vp]),
    "zgpu_last_error": (C.c_char_p, [_vp]),
    "zgpu_status_string": (C.c_char_p, [_i32]),
    "zgpu_device_info": (_i32, [_vp, C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_i32)]),
    "zgpu_synchronize": (_i32, [_vp]),
    "zgpu_register_weights": (_i32, [_vp, _vp, C.c_size_t, _u32, _u64, _u64]),
    "zgpu_group_of": (_u32, [_vp, _vp]),
    "zgpu_clear_weights": (_i32, [_vp]),
    "zgpu_linear_dispatch": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64, _u32]),
    "zgpu_linear_dispatch_device": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64, _u32, _vp]),
    "zgpu_quantize_q8_0": (_i32, [_vp, _vp, _vp, _u64]),
    "zgpu_linear_q8act": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64]),
    "zgpu_linear_q8act_device": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64, _vp]),
    "zgpu_linear_dispatch_batch": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64, _u64, _u32]),
    "zgpu_linear_q8act_batch": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64, _u64]),
    "zgpu_linear_q8act_batch_device": (_i32, [_vp, _vp, _vp, _vp, _u64, _u64, _u64, _vp]),
    "zgpu_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _u64, _f]),
    "zgpu_rope": (_i32, [_vp, _vp, _u32, _u32, _u32, _f]),
    "zgpu_silu_mul": (_i32, [_vp, _vp, _vp, _vp, _u64]),
    "zgpu_kv_create": (_i32, [_vp, _u32, _u32, _u32, _u32, C.POINTER(_vp)]),
    "zgpu_kv_destroy": (None, [_vp]),
    "zgpu_kv_store": (_i32, [_vp, _u32, _u32, _vp, _vp, _u64]),
    "zgpu_kv_read": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "zgpu_causal_attention": (_i32, [_vp, _vp, _u32, _u32, _u32, _u32, _vp, _vp]),
    "zgpu_gqa_attention_decode": (_i32, [_vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _f, _f, _vp]),
    "zgpu_gqa_attention_decode_device": (_i32, [_vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _f, _vp,
                                                _vp]),
    "zgpu_gqa_attention_decode_noalloc": (_i32, [_vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _f, _vp,
                                                 _vp]),
    "zgpu_qwen3_create_tp": (_i32, [_vp, C.POINTER(ZgpuQwen3Desc), _u32, _u32, C.POINTER(_vp)]),
    "zgpu_qwen3_tp_export": (_i32, [_vp, _vp]),
    "zgpu_qwen3_tp_connect": (_i32, [_vp, _vp]),
    "zgpu_qwen3_tp_connect_absent": (_i32, [_vp]),
    "zgpu_sample_top_k": (_i32, [_vp, _vp, _u32, _u32, _f, C.POINTER(_u64), C.POINTER(_u32)]),
    "zgpu_lm_head_sample": (_i32, [_vp, _u32, _f, C.POINTER(_u64), C.POINTER(_u32)]),
    "zgpu_smodel_open": (_i32, [C.c_char_p, C.POINTER(_vp)]),
    "zgpu_smodel_close": (None, [_vp]),
    "zgpu_smodel_error": (C.c_char_p, []),
    "zgpu_smodel_info_get": (_i32, [_vp, C.POINTER(ZgpuSmodelInfo)]),
    "zgpu_smodel_manifest": (_i32, [_vp, C.POINTER(C.c_void_p), C.POINTER(_u64)]),
    "zgpu_smodel_tensor_at": (_i32, [_vp, _u32, C.POINTER(ZgpuSmodelTensor)]),
    "zgpu_smodel_find": (_i32, [_vp, C.c_char_p, C.POINTER(ZgpuSmodelTensor)]),
    "zgpu_smodel_register": (_i32, [_vp, _vp, C.POINTER(_u32)]),
    "zgpu_qwen3_create": (_i32, [_vp, C.POINTER(ZgpuQwen3Desc), C.POINTER(_vp)]),
    "zgpu_qwen3_destroy": (None, [_vp]),
    "zgpu_forward_single_token": (_i32, [_vp, _vp, _u32, _u32, _vp]),
    "zgpu_lm_head_argmax": (_i32, [_vp, _u32, _vp, _vp]),
    "zgpu_generate_greedy": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp, _vp]),
    "zgpu_perf_snapshot": (_i32, [_vp, C.POINTER(ZgpuPerf)]),
    "zgpu_prefill_batch": (_i32, [_vp, _vp, _u32, _vp, _u32, _vp, _vp]),
    "zgpu_decode_batch": (_i32, [_vp, _vp, _u32, _vp, _vp, _vp, _vp]),
    "zgpu_prefill": (_i32, [_vp, _vp, _vp, _u32, _vp, _vp]),
    "zgpu_moe_route_f32": (_i32, [_vp, _vp, _vp, _vp, _u64, _u32, _u32, _u32, _f, _vp, _vp, _vp]),
    "zgpu_mla_kv_create": (_i32, [_vp, _u32, _u32, _u32, _u32, C.POINTER(_vp)]),
    "zgpu_mha_kv_create": (_i32, [_vp, _u32, _u32, _u32, _u32, _u32, C.POINTER(_vp)]),
    "zgpu_mha_kv_destroy": (None, [_vp]),
    "zgpu_detok_create": (_i32, [_vp, _u64, _vp, _u32, C.POINTER(_vp)]),
    "zgpu_detok_destroy": (None, [_vp]),
    "zgpu_detok_vocab_size": (_u32, [_vp]),
    "zgpu_detok_token": (_i32, [_vp, _u32, _vp, C.POINTER(_u64)]),
    "zgpu_detok_decode": (_i32, [_vp, _vp, _u64, _vp, _u64, C.POINTER(_u64)]),
    "zgpu_mha_kv_store": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "zgpu_mha_kv_read": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "zgpu_ds2_set_mha_kv": (_i32, [_vp, _vp]),
    "zgpu_mla_kv_destroy": (None, [_vp]),
    "zgpu_mla_kv_store": (_i32, [_vp, _u32, _u32, _vp, _vp]),
    "zgpu_mla_kv_read": (_i32, [_vp, _u32, _u32, _vp]),
    "zgpu_mla_kv_copy": (_i32, [_vp, _vp, _u32]),
    "zgpu_ds2_create_ep": (_i32, [_vp, C.POINTER(ZgpuDs2Desc), _u32, _u32, C.POINTER(_vp)]),
    "zgpu_ds2_ep_export": (_i32, [_vp, _vp]),
    "zgpu_ds2_ep_connect": (_i32, [_vp, _vp]),
    "zgpu_ds2_create": (_i32, [_vp, C.POINTER(ZgpuDs2Desc), C.POINTER(_vp)]),
    "zgpu_ds2_destroy": (None, [_vp]),
    "zgpu_ds2_forward_single_token": (_i32, [_vp, _vp, _u32, _u32, _vp]),
    "zgpu_ds2_lm_head_argmax": (_i32, [_vp, _u32, _vp, _vp]),
    "zgpu_ds2_expert_ids": (_i32, [_vp, _vp, _vp]),
    "zgpu_ds2_generate_greedy": (_i32, [_vp, _vp, _vp, _u32, _u32, _vp, _vp]),
    "zgpu_ds2_decode_batch": (_i32, [_vp, _vp, _u32, _vp, _vp, _vp, _vp]),
    "zgpu_ds2_batch_expert_ids": (_i32, [_vp, _u32, _vp, _vp]),
    "zgpu_ds2_perf_snapshot": (_i32, [_vp, C.POINTER(ZgpuPerf)]),
    "zgpu_synth_q4_0": (None, [_u64, _u64, _u64, _u64, _f, _vp]),
    "zgpu_synth_q8_0": (None, [_u64, _u64, _u64, _u64, _f, _vp]),
    "zgpu_synth_f32": (None, [_u64, _u64, _u64, _f, _f, _vp]),
    "zgpu_synth_tokens": (None, [_u64, _u64, _u64, _u32, _vp]),
    "zgpu_pack_x4": (_i32, [_vp, _vp, _u64, _u64, _u32]),
}

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(LIB, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)
