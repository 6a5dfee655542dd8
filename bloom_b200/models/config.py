"""Model architecture descriptions.

`ModelConfig` covers the decoder families the reference serves (Llama incl.
Mistral/DeepSeek-style GGUF, Qwen2 with QKV bias, Qwen3 with per-head q/k
RMSNorm; crates/engine/src/executor/candle.rs:28-70) plus Qwen3-MoE, and the
BERT encoder for embeddings.  `from_hf_config` reads a Hugging Face
config.json; `PRESETS` names the benchmark shapes.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import List, Optional


@dataclass
class ModelConfig:
    arch: str = "llama"  # llama | qwen2 | qwen3 | qwen3_moe | mistral | bert | gemma4
    vocab_size: int = 32000
    hidden_size: int = 4096
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = None
    max_position_embeddings: int = 8192
    tie_word_embeddings: bool = False
    qkv_bias: bool = False
    qk_norm: bool = False
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    # Gemma4 (executor/gemma4.rs Config :175-336): every `sliding_window_pattern`-th
    # layer is global (head_dim_global, num_kv_heads_global, rope_theta,
    # partial rotary, optional k = v), the others slide over `sliding_window`
    # keys with head_dim / num_kv_heads / rope_local_theta
    head_dim_global: int = 0
    num_kv_heads_global: int = 0
    sliding_window: int = 0
    sliding_window_pattern: int = 6
    rope_local_theta: float = 10000.0
    partial_rotary_factor: float = 1.0
    attn_logit_softcapping: float = 0.0
    final_logit_softcapping: float = 0.0
    attention_k_eq_v: bool = False
    hidden_activation: str = "silu"
    # BERT
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12
    bos_token_id: Optional[int] = None
    eos_token_ids: List[int] = field(default_factory=list)
    name: str = ""

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def is_sliding(self, layer: int) -> bool:
        """Gemma4: layer `layer` attends over a sliding window (the reference's
        (i + 1) % pattern > 0 rule, executor/gemma4.rs:1000)."""
        return self.arch == "gemma4" and (layer + 1) % self.sliding_window_pattern > 0

    def layer_attn(self, layer: int):
        """(head_dim, num_kv_heads) of one layer's attention."""
        if self.arch == "gemma4" and not self.is_sliding(layer):
            return self.head_dim_global, self.num_kv_heads_global
        return self.head_dim, self.num_kv_heads

    def num_params(self) -> int:
        H, L, V = self.hidden_size, self.num_layers, self.vocab_size
        if self.arch == "gemma4":
            n = V * H + H
            for i in range(L):
                d, kvh = self.layer_attn(i)
                nv = 0 if (self.attention_k_eq_v and not self.is_sliding(i)) else 1
                n += H * self.num_heads * d * 2 + H * kvh * d * (1 + nv) + 2 * d + 3 * H * self.intermediate_size
                n += 4 * H + 1
            return n
        attn = H * (self.q_size + 2 * self.kv_size) + self.q_size * H
        if self.is_moe:
            mlp = self.num_experts * 3 * H * self.moe_intermediate_size + H * self.num_experts
        else:
            mlp = 3 * H * self.intermediate_size
        emb = V * H * (1 if self.tie_word_embeddings else 2)
        return L * (attn + mlp + 2 * H) + emb + H

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        # KV/token = 2 * L * kv_heads * head_dim * bytes (reference core/manifest.rs:252)
        if self.arch == "gemma4":  # every layer's slot is sized for the widest layer
            return 2 * self.num_layers * max(d * k for d, k in map(self.layer_attn, range(self.num_layers))) \
                * dtype_bytes
        return 2 * self.num_layers * self.num_kv_heads * self.head_dim * dtype_bytes

    def to_json(self) -> str:
        return json.dumps(dataclasses.asdict(self))

    @staticmethod
    def from_dict(d: dict) -> "ModelConfig":
        names = {f.name for f in dataclasses.fields(ModelConfig)}
        return ModelConfig(**{k: v for k, v in d.items() if k in names})


def _gemma4_from_hf(cfg: dict) -> ModelConfig:
    """Gemma4 text config (top level or `text_config`), with the reference's
    defaults (executor/gemma4.rs:201-336)."""
    t = cfg.get("text_config") or cfg
    rp = t.get("rope_parameters") or {}
    full, slide = rp.get("full_attention") or {}, rp.get("sliding_attention") or {}
    eos = cfg.get("eos_token_id", t.get("eos_token_id"))
    eos_ids = eos if isinstance(eos, list) else ([eos] if eos is not None else [1, 106])
    hd = t["head_dim"]
    return ModelConfig(
        arch="gemma4", vocab_size=t["vocab_size"], hidden_size=t["hidden_size"], num_layers=t["num_hidden_layers"],
        num_heads=t["num_attention_heads"], num_kv_heads=t["num_key_value_heads"], head_dim=hd,
        intermediate_size=t["intermediate_size"], rms_norm_eps=t.get("rms_norm_eps", 1e-6),
        rope_theta=full.get("rope_theta", 1_000_000.0), max_position_embeddings=t.get("max_position_embeddings", 131072),
        tie_word_embeddings=True, qkv_bias=bool(t.get("attention_bias", False)), qk_norm=True,
        head_dim_global=t.get("global_head_dim") or 512, num_kv_heads_global=t.get("num_global_key_value_heads") or 1,
        sliding_window=t.get("sliding_window") or 1024, sliding_window_pattern=6,
        rope_local_theta=slide.get("rope_theta", 10000.0),
        partial_rotary_factor=full.get("partial_rotary_factor", 1.0),
        attn_logit_softcapping=t.get("attn_logit_softcapping") or 0.0,
        final_logit_softcapping=t.get("final_logit_softcapping") or 0.0,
        attention_k_eq_v=bool(t.get("attention_k_eq_v", False)),
        hidden_activation=t.get("hidden_activation", "gelu_pytorch_tanh"),
        bos_token_id=cfg.get("bos_token_id", t.get("bos_token_id")), eos_token_ids=eos_ids,
        name=cfg.get("_name_or_path", ""))


def from_hf_config(cfg: dict) -> ModelConfig:
    """Map a Hugging Face config.json onto ModelConfig."""
    mt = (cfg.get("model_type") or "llama").lower()
    if mt in ("gemma4", "gemma4_text", "gemma4_unified"):
        return _gemma4_from_hf(cfg)
    arch = {"llama": "llama", "mistral": "llama", "qwen2": "qwen2", "qwen3": "qwen3", "qwen3_moe": "qwen3_moe",
            "bert": "bert"}.get(mt, "llama")
    H = cfg.get("hidden_size", 4096)
    nh = cfg.get("num_attention_heads", 32)
    eos = cfg.get("eos_token_id")
    eos_ids = eos if isinstance(eos, list) else ([eos] if eos is not None else [])
    if arch == "bert":
        return ModelConfig(
            arch="bert", vocab_size=cfg.get("vocab_size", 30522), hidden_size=H,
            num_layers=cfg.get("num_hidden_layers", 12), num_heads=nh, num_kv_heads=nh, head_dim=H // nh,
            intermediate_size=cfg.get("intermediate_size", 4 * H),
            max_position_embeddings=cfg.get("max_position_embeddings", 512),
            type_vocab_size=cfg.get("type_vocab_size", 2), layer_norm_eps=cfg.get("layer_norm_eps", 1e-12),
            name=cfg.get("_name_or_path", ""))
    return ModelConfig(
        arch=arch,
        vocab_size=cfg.get("vocab_size", 32000),
        hidden_size=H,
        num_layers=cfg.get("num_hidden_layers", 32),
        num_heads=nh,
        num_kv_heads=cfg.get("num_key_value_heads", nh),
        head_dim=cfg.get("head_dim") or H // nh,
        intermediate_size=cfg.get("intermediate_size", 4 * H),
        rms_norm_eps=cfg.get("rms_norm_eps", 1e-6),
        rope_theta=cfg.get("rope_theta", 10000.0),
        rope_scaling=cfg.get("rope_scaling"),
        max_position_embeddings=cfg.get("max_position_embeddings", 4096),
        tie_word_embeddings=bool(cfg.get("tie_word_embeddings", False)),
        qkv_bias=(arch == "qwen2") or bool(cfg.get("attention_bias", False)),
        qk_norm=arch in ("qwen3", "qwen3_moe"),
        num_experts=cfg.get("num_experts", 0) if arch == "qwen3_moe" else 0,
        num_experts_per_tok=cfg.get("num_experts_per_tok", 0),
        moe_intermediate_size=cfg.get("moe_intermediate_size", 0),
        norm_topk_prob=bool(cfg.get("norm_topk_prob", True)),
        bos_token_id=cfg.get("bos_token_id"),
        eos_token_ids=eos_ids,
        name=cfg.get("_name_or_path", ""),
    )


def to_hf_config(c: ModelConfig) -> dict:
    if c.arch == "bert":
        return {"model_type": "bert", "architectures": ["BertModel"], "vocab_size": c.vocab_size,
                "hidden_size": c.hidden_size, "num_hidden_layers": c.num_layers, "num_attention_heads": c.num_heads,
                "intermediate_size": c.intermediate_size, "max_position_embeddings": c.max_position_embeddings,
                "type_vocab_size": c.type_vocab_size, "layer_norm_eps": c.layer_norm_eps, "hidden_act": "gelu"}
    mt = {"llama": "llama", "qwen2": "qwen2", "qwen3": "qwen3", "qwen3_moe": "qwen3_moe"}.get(c.arch, "llama")
    d = {"model_type": mt, "vocab_size": c.vocab_size, "hidden_size": c.hidden_size,
         "num_hidden_layers": c.num_layers, "num_attention_heads": c.num_heads,
         "num_key_value_heads": c.num_kv_heads, "head_dim": c.head_dim, "intermediate_size": c.intermediate_size,
         "rms_norm_eps": c.rms_norm_eps, "rope_theta": c.rope_theta, "rope_scaling": c.rope_scaling,
         "max_position_embeddings": c.max_position_embeddings, "tie_word_embeddings": c.tie_word_embeddings,
         "torch_dtype": "bfloat16", "hidden_act": "silu"}
    if c.eos_token_ids:
        d["eos_token_id"] = c.eos_token_ids if len(c.eos_token_ids) > 1 else c.eos_token_ids[0]
    if c.bos_token_id is not None:
        d["bos_token_id"] = c.bos_token_id
    if c.is_moe:
        d.update(num_experts=c.num_experts, num_experts_per_tok=c.num_experts_per_tok,
                 moe_intermediate_size=c.moe_intermediate_size, norm_topk_prob=c.norm_topk_prob)
    return d


PRESETS = {
    # Llama-3-8B shape (headline serving benchmark)
    "llama3-8b": ModelConfig(arch="llama", vocab_size=128256, hidden_size=4096, num_layers=32, num_heads=32,
                             num_kv_heads=8, head_dim=128, intermediate_size=14336, rms_norm_eps=1e-5,
                             rope_theta=500000.0, max_position_embeddings=8192, eos_token_ids=[128001, 128009],
                             bos_token_id=128000, name="llama3-8b"),
    "llama3-70b": ModelConfig(arch="llama", vocab_size=128256, hidden_size=8192, num_layers=80, num_heads=64,
                              num_kv_heads=8, head_dim=128, intermediate_size=28672, rms_norm_eps=1e-5,
                              rope_theta=500000.0, max_position_embeddings=8192, eos_token_ids=[128001, 128009],
                              bos_token_id=128000, name="llama3-70b"),
    # 1B-shape draft for speculative decoding
    "llama3-1b-draft": ModelConfig(arch="llama", vocab_size=128256, hidden_size=2048, num_layers=16, num_heads=32,
                                   num_kv_heads=8, head_dim=64, intermediate_size=8192, rms_norm_eps=1e-5,
                                   rope_theta=500000.0, max_position_embeddings=8192, tie_word_embeddings=True,
                                   eos_token_ids=[128001, 128009], bos_token_id=128000, name="llama3-1b-draft"),
    "qwen3-moe-30b-a3b": ModelConfig(arch="qwen3_moe", vocab_size=151936, hidden_size=2048, num_layers=48,
                                     num_heads=32, num_kv_heads=4, head_dim=128, intermediate_size=6144,
                                     rms_norm_eps=1e-6, rope_theta=1000000.0, max_position_embeddings=32768,
                                     qk_norm=True, num_experts=128, num_experts_per_tok=8, moe_intermediate_size=768,
                                     eos_token_ids=[151645, 151643], name="qwen3-moe-30b-a3b"),
    # SmolLM2-135M shape (CPU GGUF Q8_0 config)
    "smollm2-135m": ModelConfig(arch="llama", vocab_size=49152, hidden_size=576, num_layers=30, num_heads=9,
                                num_kv_heads=3, head_dim=64, intermediate_size=1536, rms_norm_eps=1e-5,
                                rope_theta=10000.0, max_position_embeddings=2048, tie_word_embeddings=True,
                                eos_token_ids=[2], bos_token_id=1, name="smollm2-135m"),
    "minilm-l6": ModelConfig(arch="bert", vocab_size=30522, hidden_size=384, num_layers=6, num_heads=12,
                             num_kv_heads=12, head_dim=32, intermediate_size=1536, max_position_embeddings=512,
                             type_vocab_size=2, layer_norm_eps=1e-12, name="minilm-l6"),
    # tiny shapes for tests
    "tiny-llama": ModelConfig(arch="llama", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=128, intermediate_size=512, rms_norm_eps=1e-5,
                              rope_theta=10000.0, max_position_embeddings=1024, eos_token_ids=[2], bos_token_id=1,
                              name="tiny-llama"),
    "tiny-qwen3": ModelConfig(arch="qwen3", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=128, intermediate_size=512, rms_norm_eps=1e-6,
                              rope_theta=1000000.0, max_position_embeddings=1024, qk_norm=True, eos_token_ids=[2],
                              name="tiny-qwen3"),
    "tiny-qwen2": ModelConfig(arch="qwen2", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=128, intermediate_size=512, rms_norm_eps=1e-6,
                              rope_theta=1000000.0, max_position_embeddings=1024, qkv_bias=True, eos_token_ids=[2],
                              name="tiny-qwen2"),
    # tiny shape that shards over 8 ranks (8 q heads, 2 KV heads replicated at TP 4/8)
    "tiny-tp": ModelConfig(arch="llama", vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8,
                           num_kv_heads=2, head_dim=128, intermediate_size=1024, rms_norm_eps=1e-5,
                           rope_theta=10000.0, max_position_embeddings=1024, eos_token_ids=[2], name="tiny-tp"),
    "tiny-moe-tp": ModelConfig(arch="qwen3_moe", vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8,
                               num_kv_heads=4, head_dim=128, intermediate_size=1024, rms_norm_eps=1e-6,
                               rope_theta=1000000.0, max_position_embeddings=1024, qk_norm=True, num_experts=16,
                               num_experts_per_tok=4, moe_intermediate_size=128, eos_token_ids=[2],
                               name="tiny-moe-tp"),
    # head_dim 64 (the 1B draft and SmolLM2 layouts)
    "tiny-hd64": ModelConfig(arch="llama", vocab_size=512, hidden_size=256, num_layers=2, num_heads=8,
                             num_kv_heads=2, head_dim=64, intermediate_size=512, rms_norm_eps=1e-5,
                             rope_theta=10000.0, max_position_embeddings=1024, tie_word_embeddings=True,
                             eos_token_ids=[2], name="tiny-hd64"),
    # Gemma4 layout at test size: 5 sliding layers (head_dim 256, window 24) + 1 global
    # (head_dim 512, one KV head, k = v, quarter rotary), both soft-caps on
    "tiny-gemma4": ModelConfig(arch="gemma4", vocab_size=512, hidden_size=256, num_layers=6, num_heads=4,
                               num_kv_heads=2, head_dim=256, intermediate_size=512, rms_norm_eps=1e-6,
                               rope_theta=1_000_000.0, max_position_embeddings=1024, tie_word_embeddings=True,
                               qk_norm=True, head_dim_global=512, num_kv_heads_global=1, sliding_window=24,
                               sliding_window_pattern=6, rope_local_theta=10000.0, partial_rotary_factor=0.25,
                               attn_logit_softcapping=50.0, final_logit_softcapping=30.0, attention_k_eq_v=True,
                               hidden_activation="gelu_pytorch_tanh", eos_token_ids=[1, 106], name="tiny-gemma4"),
    "tiny-moe": ModelConfig(arch="qwen3_moe", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                            num_kv_heads=2, head_dim=128, intermediate_size=512, rms_norm_eps=1e-6,
                            rope_theta=1000000.0, max_position_embeddings=1024, qk_norm=True, num_experts=8,
                            num_experts_per_tok=2, moe_intermediate_size=128, eos_token_ids=[2], name="tiny-moe"),
}


def preset(name: str) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return dataclasses.replace(PRESETS[name])
