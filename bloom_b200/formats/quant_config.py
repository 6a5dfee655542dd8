"""Quantisation metadata of a model: weight method, bit width, group size and
KV-cache dtype, read from an HF `config.json` (`quantization_config`) or from
a GGUF file type, plus the conversion of packed AWQ / GPTQ / bitsandbytes
checkpoint tensors into the bf16 weights the tcgen05 GEMM consumes.

Behaviour follows the reference's `QuantMethod`, `KvCacheDtype` and
`QuantizationConfig` (crates/engine/src/core/quantization.rs:46-390): the same
method labels and HF `quant_method` aliases, the same default bit widths, the
same GGUF file-type table (most specific name first), and the `torch_dtype`
fallback for the KV dtype.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from enum import Enum
from typing import Dict, Optional

SUB_BYTE = {"gguf", "awq", "gptq", "nvfp4", "nf4", "fp4", "hqq", "aqlm", "exl2", "quanto", "torchao"}


class QuantMethod(str, Enum):
    NONE = "none"
    GGUF = "gguf"
    AWQ = "awq"
    GPTQ = "gptq"
    FP8 = "fp8"
    NVFP4 = "nvfp4"
    INT8 = "int8"
    NF4 = "nf4"
    FP4 = "fp4"
    HQQ = "hqq"
    EETQ = "eetq"
    AQLM = "aqlm"
    EXL2 = "exl2"
    QUANTO = "quanto"
    TORCHAO = "torchao"

    @property
    def label(self) -> str:
        return self.value

    def is_sub_byte(self) -> bool:
        return self.value in SUB_BYTE

    @classmethod
    def from_hf_quant_config(cls, qc: dict) -> Optional["QuantMethod"]:
        m = qc.get("quant_method") if isinstance(qc, dict) else None
        if not isinstance(m, str):
            return None
        m = m.lower()
        aliases = {"awq": cls.AWQ, "awq_marlin": cls.AWQ, "gptq": cls.GPTQ, "marlin": cls.GPTQ,
                   "gptq_marlin": cls.GPTQ, "fp8": cls.FP8, "fbgemm_fp8": cls.FP8, "fp8_marlin": cls.FP8,
                   "hqq": cls.HQQ, "eetq": cls.EETQ, "aqlm": cls.AQLM, "exl2": cls.EXL2, "quanto": cls.QUANTO,
                   "torchao": cls.TORCHAO}
        if m in aliases:
            return aliases[m]
        if m in ("bitsandbytes", "bnb"):
            four = bool(qc.get("load_in_4bit", False)) or "bnb_4bit_compute_dtype" in qc
            if not four:
                return cls.INT8
            return cls.NF4 if str(qc.get("bnb_4bit_quant_type", "fp4")).lower() == "nf4" else cls.FP4
        return None

    @classmethod
    def from_gguf_type(cls, name: str) -> "QuantMethod":
        low = name.lower()
        hit = any(t in low for t in ("q4", "q5", "q8", "q2", "q3", "q6", "iq2", "iq3", "iq4"))
        return cls.GGUF if hit else cls.NONE


class KvCacheDtype(str, Enum):
    F16 = "f16"
    BF16 = "bf16"
    F32 = "f32"
    INT8 = "int8"
    FP8 = "fp8"

    def element_size(self) -> int:
        return {"f32": 4, "f16": 2, "bf16": 2, "int8": 1, "fp8": 1}[self.value]

    def needs_dequant(self) -> bool:
        return self in (KvCacheDtype.INT8, KvCacheDtype.FP8)


_DEFAULT_BITS = {QuantMethod.AWQ: 4, QuantMethod.GPTQ: 4, QuantMethod.FP8: 8, QuantMethod.INT8: 8,
                 QuantMethod.EETQ: 8, QuantMethod.NVFP4: 4, QuantMethod.NF4: 4, QuantMethod.FP4: 4,
                 QuantMethod.AQLM: 2, QuantMethod.HQQ: 4, QuantMethod.EXL2: 4, QuantMethod.QUANTO: 4,
                 QuantMethod.TORCHAO: 4}

# GGUF file types, most specific first: (substring, bits); the source label is "gguf_" + substring
_GGUF_TYPES = (("iq2_xxs", 2), ("iq2_xs", 2), ("iq3_xxs", 3), ("iq3_s", 3), ("iq4_xs", 4), ("iq4_nl", 4),
               ("q2_k", 2), ("q3_k_s", 3), ("q3_k_m", 3), ("q3_k_l", 3), ("q4_k_s", 4), ("q4_k_m", 4),
               ("q4_0", 4), ("q4_1", 4), ("q5_k_s", 5), ("q5_k_m", 5), ("q5_0", 5), ("q5_1", 5), ("q6_k", 6),
               ("q8_0", 8))


@dataclass
class QuantizationConfig:
    weight_method: QuantMethod = QuantMethod.NONE
    weight_bits: int = 16
    group_size: int = 0
    kv_cache_dtype: KvCacheDtype = KvCacheDtype.F16
    activation_quant: bool = False
    source_format: str = ""
    raw: Optional[dict] = None  # the checkpoint's quantization_config (sym, desc_act, version, ...)

    def is_quantized(self) -> bool:
        return self.weight_method != QuantMethod.NONE

    def has_kv_cache_quant(self) -> bool:
        return self.kv_cache_dtype.needs_dequant()

    def memory_ratio(self) -> float:
        return self.weight_bits / 16.0

    @classmethod
    def from_model_config(cls, config: dict) -> "QuantizationConfig":
        qc = config.get("quantization_config") if isinstance(config, dict) else None
        if isinstance(qc, dict):
            m = QuantMethod.from_hf_quant_config(qc)
            if m is not None:
                kv = {"int8": KvCacheDtype.INT8, "fp8": KvCacheDtype.FP8, "bf16": KvCacheDtype.BF16,
                      "f32": KvCacheDtype.F32}.get(qc.get("kv_cache_dtype"), KvCacheDtype.F16)
                return cls(weight_method=m, weight_bits=int(qc.get("bits", _DEFAULT_BITS.get(m, 16))),
                           group_size=int(qc.get("group_size", 128)), kv_cache_dtype=kv,
                           activation_quant=bool(qc.get("activation_quant", False)), source_format=m.label, raw=qc)
        td = config.get("torch_dtype") if isinstance(config, dict) else None
        if isinstance(td, str):
            return cls(kv_cache_dtype={"bfloat16": KvCacheDtype.BF16, "float32": KvCacheDtype.F32}.get(
                td, KvCacheDtype.F16))
        return cls()

    @classmethod
    def from_gguf_metadata(cls, general_type: Optional[str]) -> "QuantizationConfig":
        if general_type is None:
            return cls()
        low = general_type.lower()
        for key, bits in _GGUF_TYPES:
            if key in low:
                return cls(weight_method=QuantMethod.GGUF, weight_bits=bits, source_format="gguf_" + key)
        if "q2" in low or "q3" in low:
            return cls(weight_method=QuantMethod.GGUF, weight_bits=3, source_format="gguf_q3")
        return cls()

    @classmethod
    def from_model_dir(cls, model_dir: str) -> "QuantizationConfig":
        p = os.path.join(model_dir, "config.json")
        if not os.path.exists(p):
            return cls()
        with open(p) as f:
            return cls.from_model_config(json.load(f))


# ---------------------------------------------------------------- checkpoint conversion


def dequantize_checkpoint(sd: Dict[str, object], qc: QuantizationConfig, device=None) -> Dict[str, object]:
    """Replace packed linear layers by dense bf16 `<p>.weight` [N, K]:

    * AWQ / GPTQ 4-bit: `<p>.qweight`, `<p>.qzeros`, `<p>.scales` (GPTQ also
      `<p>.g_idx`; without it groups are consecutive runs of `group_size`).
    * bitsandbytes NF4 / FP4: `<p>.weight` holds the uint8 codes and
      `<p>.weight.absmax` one fp32 scale per block (the block size follows from
      the two element counts); an optional `<p>.weight.shape` gives the shape.

    Runs the CUDA dequantisers when `device` is a GPU, the fp32 torch
    restatements otherwise."""
    import torch

    from ..ops import reference as R

    if qc.weight_method not in (QuantMethod.AWQ, QuantMethod.GPTQ, QuantMethod.NF4, QuantMethod.FP4):
        return sd
    use_gpu = device is not None and torch.device(device).type == "cuda"
    out = dict(sd)
    if qc.weight_method in (QuantMethod.AWQ, QuantMethod.GPTQ):
        if qc.weight_bits != 4:
            raise ValueError(f"{qc.weight_method.label}: only 4-bit checkpoints are supported")
        for k in [k for k in sd if k.endswith(".qweight")]:
            p = k[: -len(".qweight")]
            qw, qz, sc = sd[k], sd[p + ".qzeros"], sd[p + ".scales"]
            if qc.weight_method == QuantMethod.GPTQ:
                K = qw.shape[0] * 8
                gi = sd.get(p + ".g_idx")
                if gi is None:
                    gi = torch.arange(K, dtype=torch.int32) // max(1, qc.group_size)
                if use_gpu:
                    from .. import ops

                    w = ops.dequant_gptq(qw.to(device), qz.to(device), sc.to(device), gi.to(device))
                else:
                    w = R.dequant_gptq(qw, qz, sc, gi).to(torch.bfloat16)
            else:
                if use_gpu:
                    from .. import ops

                    w = ops.dequant_awq(qw.to(device), qz.to(device), sc.to(device), qc.group_size)
                else:
                    w = R.dequant_awq(qw, qz, sc, qc.group_size).to(torch.bfloat16)
            for suffix in (".qweight", ".qzeros", ".scales", ".g_idx"):
                out.pop(p + suffix, None)
            out[p + ".weight"] = w
    else:
        nf4 = qc.weight_method == QuantMethod.NF4
        for k in [k for k in sd if k.endswith(".weight.absmax")]:
            p = k[: -len(".absmax")]
            codes = sd[p]
            absmax = sd[k].float()
            shape = sd.get(p + ".shape")
            block = max(1, (codes.numel() * 2) // absmax.numel())
            if use_gpu:
                from .. import ops

                w = ops.dequant_bnb4(codes.to(device), absmax.to(device), block, nf4=nf4)
            else:
                w = R.dequant_bnb4(codes, absmax, block, nf4=nf4).to(torch.bfloat16)
            if shape is not None:
                w = w.view(*[int(s) for s in shape.tolist()])
            out.pop(k, None)
            out.pop(p + ".shape", None)
            out[p] = w
    return out
