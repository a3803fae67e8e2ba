"""SilicatePack `.smodel` containers (zgpu_smodel_* in the C ABI).

    with SmodelFile("model.smodel") as f:
        cfg = f.qwen3_config()
        model = Qwen3Model(ctx, cfg, f.qwen3_weights())

The file is mapped read-only and validated as the reference's loader does
(kernel/src/model_loader.rs:256-661).  Tensors are numpy views of the
mapping, so registering them keys the device copies by their mapped
addresses, as weight_layout::register does.  Keep the file open while models
are built from it.
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass

import numpy as np

from ._lib import LIB, ZgpuSmodelInfo, ZgpuSmodelTensor

DTYPE_NAMES = {0: "F32", 1: "F16", 2: "Q4_0", 8: "Q8_0", 100: "Q4_0X4", 101: "Q8_0X4"}
NONE_U32 = 0xFFFFFFFF


class SmodelError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{status}: {message}")
        self.status = status


@dataclass
class SmodelTensor:
    name: str
    dtype: int
    shape: tuple
    payload_offset: int
    byte_len: int
    elements: int
    data: int   # mapped address

    @property
    def dtype_name(self) -> str:
        return DTYPE_NAMES.get(self.dtype, str(self.dtype))


class SmodelFile:
    def __init__(self, path):
        h = C.c_void_p()
        st = LIB.zgpu_smodel_open(str(path).encode(), C.byref(h))
        if st:
            raise SmodelError(st, (LIB.zgpu_smodel_error() or b"").decode())
        self.h = h
        info = ZgpuSmodelInfo()
        LIB.zgpu_smodel_info_get(self.h, C.byref(info))
        self.info = {k: getattr(info, k) for k, _ in ZgpuSmodelInfo._fields_}
        self.tensors: list[SmodelTensor] = []
        for i in range(info.tensor_count):
            t = ZgpuSmodelTensor()
            LIB.zgpu_smodel_tensor_at(self.h, i, C.byref(t))
            self.tensors.append(SmodelTensor(t.name.decode(), t.dtype, tuple(t.shape[: t.rank]), t.payload_offset,
                                             t.byte_len, t.elements, t.data or 0))
        self._by_name = {t.name: t for t in self.tensors}

    def close(self):
        if getattr(self, "h", None):
            LIB.zgpu_smodel_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def manifest(self) -> dict:
        p, n = C.c_void_p(), C.c_uint64()
        LIB.zgpu_smodel_manifest(self.h, C.byref(p), C.byref(n))
        return json.loads(C.string_at(p, n.value).decode())

    def raw(self, name_or_tensor) -> np.ndarray:
        """The tensor's bytes: a read-only uint8 view of the mapping."""
        t = name_or_tensor if isinstance(name_or_tensor, SmodelTensor) else self._by_name[name_or_tensor]
        buf = (C.c_uint8 * t.byte_len).from_address(t.data)
        a = np.frombuffer(buf, np.uint8)
        a.flags.writeable = False
        return a

    def f32(self, name: str) -> np.ndarray:
        t = self._by_name[name]
        if t.dtype != 0:
            raise SmodelError(2, f"{name} is {t.dtype_name}, not F32")
        return self.raw(t).view(np.float32)

    def has(self, name: str) -> bool:
        return name in self._by_name

    def tensor(self, name: str) -> SmodelTensor:
        return self._by_name[name]

    # ------------------------------------------------------------ Qwen3
    def qwen3_config(self):
        from .synth import Qwen3Config

        i = self.info
        emb = self._by_name["token_embd.weight"]
        out = self._by_name.get("output.weight", emb)
        q = lambda t: "q8_0" if t.dtype in (8, 101) else "q4_0"   # noqa: E731
        vocab_real = i["vocab_size"] if i["vocab_size"] != NONE_U32 else emb.shape[0]
        return Qwen3Config("smodel-qwen3", i["block_count"], i["embedding_length"], i["feed_forward_length"],
                           i["head_count"], i["head_count_kv"], i["key_length"], emb.shape[0], vocab_real,
                           rms_eps=i["layer_norm_rms_epsilon"], rope_theta=i["rope_freq_base"],
                           embd_quant=q(emb), output_quant=q(out))

    def qwen3_weights(self) -> dict:
        """The weights dict Qwen3Model takes, as views of the mapping (the
        runtime names of silicatepack.py native_tensor_name)."""
        names = {"attn_q": "attn_q", "attn_k": "attn_k", "attn_v": "attn_v", "attn_o": "attn_output",
                 "ffn_gate": "ffn_gate", "ffn_up": "ffn_up", "ffn_down": "ffn_down"}
        norms = {"attn_norm": "attn_norm", "q_norm": "attn_q_norm", "k_norm": "attn_k_norm", "ffn_norm": "ffn_norm"}
        w = {"token_embd": self.raw("token_embd.weight"), "output_norm": self.f32("output_norm.weight")}
        if self.has("output.weight"):
            t = self._by_name["output.weight"]
            w["output_x4" if t.dtype in (100, 101) else "output"] = self.raw(t)
            if t.dtype in (100, 101):
                w["output"] = None
        else:
            w["output"] = w["token_embd"]
        w["layers"] = []
        for layer in range(self.info["block_count"]):
            lw = {}
            for key, n in names.items():
                t = self._by_name[f"blk.{layer}.{n}.weight"]
                lw[key + "_x4" if t.dtype in (100, 101) else key] = self.raw(t)
            for key, n in norms.items():
                lw[key] = self.f32(f"blk.{layer}.{n}.weight")
            w["layers"].append(lw)
        return w
