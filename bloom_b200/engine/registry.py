"""Engine registry and router.

Each engine declares a capability matrix; the router picks the first engine
that supports a model Natively, else the first Fallback, else reports
Unsupported (reference: crates/engine/src/core/engine.rs:16-27 maturity,
:44-70 EngineCapability, :139-228 default_engine_supports, :305-405
EngineRouter::select_engine; skeleton engines are never auto-routed).

Engines here:
  b200    the GPU engine (this repository's sm_100a kernels, TP/EP over NVLink)
  cpu     host engine for small GGUF Q8_0/Q4_0 and fp32 models (C++ block kernels)
  echo    deterministic test engine (echoes the prompt), like the reference's
          EchoTextModel / "mock" engine used by the C ABI demo
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import List, Optional

NATIVE, FALLBACK, UNSUPPORTED = "Native", "Fallback", "Unsupported"


@dataclass
class EngineCapability:
    name: str
    maturity: str  # Production | Beta | Experimental | Skeleton
    devices: List[str]
    families: List[str]
    formats: List[str]
    native_dtypes: List[str]
    fallback_dtypes: List[str] = field(default_factory=list)
    modalities: List[str] = field(default_factory=lambda: ["Text"])
    parallel_strategies: List[str] = field(default_factory=lambda: ["None"])
    max_tp: int = 1


class EngineRegistry:
    def __init__(self):
        self.engines: List[EngineCapability] = []

    def register(self, cap: EngineCapability) -> None:
        self.engines.append(cap)

    def get(self, name: str) -> Optional[EngineCapability]:
        for e in self.engines:
            if e.name == name:
                return e
        return None

    def support(self, cap: EngineCapability, family: str, fmt: str, dtype: str, device: str,
                modality: str = "Text") -> str:
        if cap.maturity == "Skeleton":
            return UNSUPPORTED
        if device not in cap.devices or modality not in cap.modalities:
            return UNSUPPORTED
        if family not in cap.families or fmt not in cap.formats:
            return UNSUPPORTED
        if dtype in cap.native_dtypes:
            return NATIVE
        if dtype in cap.fallback_dtypes:
            return FALLBACK
        return UNSUPPORTED

    def route(self, family: str, fmt: str, dtype: str, device: str, modality: str = "Text",
              preferred: Optional[str] = None):
        """(engine name, support level) or (None, Unsupported)."""
        if preferred:
            cap = self.get(preferred)
            if cap is None:
                return None, UNSUPPORTED
            return cap.name, self.support(cap, family, fmt, dtype, device, modality)
        fallback = None
        for cap in self.engines:
            lvl = self.support(cap, family, fmt, dtype, device, modality)
            if lvl == NATIVE:
                return cap.name, NATIVE
            if lvl == FALLBACK and fallback is None:
                fallback = cap.name
        return (fallback, FALLBACK) if fallback else (None, UNSUPPORTED)

    def describe(self) -> list:
        return [asdict(e) for e in self.engines]


def default_registry() -> EngineRegistry:
    r = EngineRegistry()
    r.register(EngineCapability(
        name="b200", maturity="Beta", devices=["gpu"], families=["Llama", "Qwen", "Bert", "Gemma"],
        formats=["Safetensors", "Gguf", "Preset"], native_dtypes=["BF16", "F16", "Q8", "Q4"], fallback_dtypes=["F32"],
        modalities=["Text", "Embedding"], parallel_strategies=["None", "TensorParallel", "ExpertParallel",
                                                               "DataParallel"], max_tp=8))
    r.register(EngineCapability(
        name="cpu", maturity="Beta", devices=["cpu"], families=["Llama", "Qwen"], formats=["Gguf", "Safetensors"],
        native_dtypes=["Q8", "Q4", "F32"], fallback_dtypes=["BF16", "F16"]))
    r.register(EngineCapability(
        name="echo", maturity="Experimental", devices=["cpu", "gpu"], families=["Echo"], formats=["Preset"],
        native_dtypes=["F32"]))
    r.register(EngineCapability(
        name="qwen3-vl", maturity="Experimental", devices=["gpu"], families=["QwenVL"], formats=["Preset", "Safetensors"],
        native_dtypes=["BF16"], modalities=["Text", "Vision"]))
    r.register(EngineCapability(
        name="wan", maturity="Experimental", devices=["gpu"], families=["Wan"], formats=["Preset", "Safetensors"],
        native_dtypes=["BF16"], modalities=["Text", "Video"]))
    r.register(EngineCapability(
        name="longcat", maturity="Experimental", devices=["gpu"], families=["LongCat"],
        formats=["Preset", "Safetensors"], native_dtypes=["BF16"], modalities=["Text", "Vision"]))
    # external runtimes (explicit --backend only: their availability depends on binaries outside this build)
    r.register(EngineCapability(
        name="llamacpp", maturity="Beta", devices=["cpu", "gpu"], families=["*"], formats=["Gguf"],
        native_dtypes=["F32", "F16", "BF16", "Q8", "Q4"]))
    r.register(EngineCapability(
        name="script", maturity="Experimental", devices=["cpu", "gpu"], families=["*"], formats=["Script"],
        native_dtypes=["F32"], modalities=["Text", "Audio", "Vision"]))
    return r
