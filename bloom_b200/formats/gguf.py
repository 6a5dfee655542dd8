"""GGUF model files: reading (native parser + memory-mapped tensors), writing,
config and tokenizer synthesis.

Reading uses the C++ parser in bloom_b200._runtime (header, metadata, tensor
table); tensor bytes are numpy memmaps into the file.  Writing is used by the
model generators and tests.  Config synthesis maps the `{arch}.*` keys the
same way the reference does (crates/engine/src/executor/candle.rs:682-841);
tokenizer synthesis turns `tokenizer.ggml.*` into a Hugging Face
tokenizer.json (candle.rs:843-1077: BPE with byte-level pre-tokenisation for
gpt2-style vocabularies, special tokens from token_type 3/4).

llama.cpp stores the Q and K projections of "llama" architectures with the
head dimension permuted for its interleaved RoPE; they are un-permuted on
load so the HF rotate_half kernels apply (and permuted again when written).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from .._ext import runtime as _rt

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_BF16 = 0, 1, 2, 8, 30
GGML_TYPES = {"F32": GGML_F32, "F16": GGML_F16, "Q4_0": GGML_Q4_0, "Q8_0": GGML_Q8_0, "BF16": GGML_BF16}
BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q4_0: (32, 18), GGML_Q8_0: (32, 34), GGML_BF16: (1, 2)}

# GGUF value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)


@dataclass
class GGUFTensor:
    name: str
    shape: Tuple[int, ...]  # row-major (numpy/torch) order
    ggml_type: int
    type_name: str
    offset: int
    n_bytes: int


class GGUFFile:
    def __init__(self, path: str):
        self.path = path
        info = _rt().read_gguf(path)
        self.version = info["version"]
        self.metadata: Dict[str, Any] = dict(info["metadata"])
        self.alignment = info["alignment"]
        self.data_offset = info["data_offset"]
        self.tensors: Dict[str, GGUFTensor] = {}
        for t in info["tensors"]:
            self.tensors[t["name"]] = GGUFTensor(t["name"], tuple(int(x) for x in t["shape"]), int(t["type"]),
                                                 t["type_name"], int(t["offset"]), int(t["n_bytes"]))
        self._mm = None

    @property
    def arch(self) -> str:
        return str(self.metadata.get("general.architecture", "llama"))

    def raw(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        start = self.data_offset + t.offset
        return self._mm[start:start + t.n_bytes]

    def tensor(self, name: str, unpermute_rope: bool = True):
        """Dequantised torch.float32 tensor in row-major shape."""
        import torch

        t = self.tensors[name]
        raw = self.raw(name)
        n = int(np.prod(t.shape)) if t.shape else 1
        if t.ggml_type == GGML_F32:
            out = torch.from_numpy(np.frombuffer(raw, dtype=np.float32, count=n).copy())
        elif t.ggml_type == GGML_F16:
            out = torch.from_numpy(np.frombuffer(raw, dtype=np.float16, count=n).astype(np.float32))
        elif t.ggml_type == GGML_BF16:
            u = np.frombuffer(raw, dtype=np.uint16, count=n).astype(np.uint32) << 16
            out = torch.from_numpy(u.view(np.float32).copy())
        elif t.ggml_type == GGML_Q8_0:
            out = _rt().dequant_q8_0(torch.from_numpy(np.ascontiguousarray(raw)), n)
        elif t.ggml_type == GGML_Q4_0:
            out = _rt().dequant_q4_0(torch.from_numpy(np.ascontiguousarray(raw)), n)
        else:
            raise NotImplementedError(f"ggml type {t.type_name} for {name}")
        out = out.view(*t.shape)
        if unpermute_rope and self.arch in ("llama",) and _is_qk(name):
            heads = self._heads_for(name)
            out = unpermute_qk(out, heads)
        return out

    def _heads_for(self, name: str) -> int:
        a = self.arch
        if name.endswith("attn_q.weight"):
            return int(self.metadata[f"{a}.attention.head_count"])
        return int(self.metadata.get(f"{a}.attention.head_count_kv", self.metadata[f"{a}.attention.head_count"]))

    def primary_dtype(self) -> str:
        """Most common tensor type by bytes (the mixed-dtype rule of the reference's
        GGUF summary: the dtype that holds the most weight bytes wins)."""
        acc: Dict[str, int] = {}
        for t in self.tensors.values():
            acc[t.type_name] = acc.get(t.type_name, 0) + t.n_bytes
        return max(acc.items(), key=lambda kv: kv[1])[0] if acc else "F32"


def _is_qk(name: str) -> bool:
    return name.endswith("attn_q.weight") or name.endswith("attn_k.weight")


def permute_qk(w, heads: int):
    """HF rotate_half layout -> llama.cpp interleaved layout (rows of each head)."""
    out_f, in_f = w.shape
    hd = out_f // heads
    return w.reshape(heads, 2, hd // 2, in_f).transpose(1, 2).reshape(out_f, in_f)


def unpermute_qk(w, heads: int):
    out_f, in_f = w.shape
    hd = out_f // heads
    return w.reshape(heads, hd // 2, 2, in_f).transpose(1, 2).reshape(out_f, in_f)


# ---------------------------------------------------------------- config synthesis
def config_from_gguf(g: GGUFFile):
    """ModelConfig from {arch}.* metadata (head_dim = embedding_length / head_count)."""
    from ..models.config import ModelConfig

    m, a = g.metadata, g.arch
    H = int(m[f"{a}.embedding_length"])
    nh = int(m[f"{a}.attention.head_count"])
    nkv = int(m.get(f"{a}.attention.head_count_kv", nh))
    hd = int(m.get(f"{a}.attention.key_length", H // nh))
    vocab = int(m.get(f"{a}.vocab_size", len(m.get("tokenizer.ggml.tokens", [])) or 32000))
    eos = m.get("tokenizer.ggml.eos_token_id")
    arch = {"llama": "llama", "mistral": "llama", "deepseek": "llama", "qwen2": "qwen2", "qwen3": "qwen3",
            "qwen3moe": "qwen3_moe"}.get(a, "llama")
    cfg = ModelConfig(
        arch=arch, vocab_size=vocab, hidden_size=H, num_layers=int(m[f"{a}.block_count"]), num_heads=nh,
        num_kv_heads=nkv, head_dim=hd, intermediate_size=int(m.get(f"{a}.feed_forward_length", 4 * H)),
        rms_norm_eps=float(m.get(f"{a}.attention.layer_norm_rms_epsilon", 1e-5)),
        rope_theta=float(m.get(f"{a}.rope.freq_base", 10000.0)),
        max_position_embeddings=int(m.get(f"{a}.context_length", 2048)),
        tie_word_embeddings="output.weight" not in g.tensors,
        qkv_bias="blk.0.attn_q.bias" in g.tensors, qk_norm="blk.0.attn_q_norm.weight" in g.tensors,
        bos_token_id=m.get("tokenizer.ggml.bos_token_id"), eos_token_ids=[int(eos)] if eos is not None else [],
        name=str(m.get("general.name", os.path.basename(g.path))))
    return cfg


GGUF_TO_HF = {
    "token_embd.weight": "model.embed_tokens.weight",
    "output_norm.weight": "model.norm.weight",
    "output.weight": "lm_head.weight",
}
BLK_TO_HF = {
    "attn_norm.weight": "input_layernorm.weight", "ffn_norm.weight": "post_attention_layernorm.weight",
    "attn_q.weight": "self_attn.q_proj.weight", "attn_k.weight": "self_attn.k_proj.weight",
    "attn_v.weight": "self_attn.v_proj.weight", "attn_output.weight": "self_attn.o_proj.weight",
    "attn_q.bias": "self_attn.q_proj.bias", "attn_k.bias": "self_attn.k_proj.bias",
    "attn_v.bias": "self_attn.v_proj.bias", "attn_q_norm.weight": "self_attn.q_norm.weight",
    "attn_k_norm.weight": "self_attn.k_norm.weight", "ffn_gate.weight": "mlp.gate_proj.weight",
    "ffn_up.weight": "mlp.up_proj.weight", "ffn_down.weight": "mlp.down_proj.weight",
}
HF_TO_BLK = {v: k for k, v in BLK_TO_HF.items()}


def gguf_name_to_hf(name: str) -> Optional[str]:
    if name in GGUF_TO_HF:
        return GGUF_TO_HF[name]
    if name.startswith("blk."):
        _, idx, rest = name.split(".", 2)
        if rest in BLK_TO_HF:
            return f"model.layers.{idx}.{BLK_TO_HF[rest]}"
    return None


def hf_name_to_gguf(name: str) -> Optional[str]:
    for k, v in GGUF_TO_HF.items():
        if v == name:
            return k
    if name.startswith("model.layers."):
        parts = name.split(".", 3)
        idx, rest = parts[2], parts[3]
        if rest in HF_TO_BLK:
            return f"blk.{idx}.{HF_TO_BLK[rest]}"
    return None


def load_hf_weights(g: GGUFFile, dtype=None) -> Dict[str, Any]:
    """All tensors of a GGUF decoder under Hugging Face names (dequantised)."""
    import torch

    dtype = dtype or torch.bfloat16
    out = {}
    for name in g.tensors:
        hf = gguf_name_to_hf(name)
        if hf is None:
            continue
        out[hf] = g.tensor(name).to(dtype)
    return out


# ---------------------------------------------------------------- tokenizer synthesis
def tokenizer_json_from_gguf(g: GGUFFile) -> Optional[dict]:
    """A Hugging Face tokenizer.json built from tokenizer.ggml.* (BPE vocabularies)."""
    m = g.metadata
    toks = m.get("tokenizer.ggml.tokens")
    if not toks:
        return None
    model_kind = str(m.get("tokenizer.ggml.model", "gpt2"))
    types = m.get("tokenizer.ggml.token_type") or [1] * len(toks)
    vocab = {t: i for i, t in enumerate(toks)}
    added = [{"id": i, "content": t, "single_word": False, "lstrip": False, "rstrip": False, "normalized": False,
              "special": True} for i, t in enumerate(toks) if i < len(types) and types[i] in (3, 4)]
    if model_kind == "gpt2":
        merges = m.get("tokenizer.ggml.merges") or []
        return {
            "version": "1.0", "truncation": None, "padding": None, "added_tokens": added,
            "normalizer": None,
            "pre_tokenizer": {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": True},
            "post_processor": None,
            "decoder": {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": True},
            "model": {"type": "BPE", "dropout": None, "unk_token": None, "continuing_subword_prefix": None,
                      "end_of_word_suffix": None, "fuse_unk": False, "byte_fallback": False,
                      "vocab": vocab, "merges": merges},
        }
    # fallback: whole-word vocabulary split on whitespace (the reference's last resort)
    return {
        "version": "1.0", "truncation": None, "padding": None, "added_tokens": added,
        "normalizer": None, "pre_tokenizer": {"type": "WhitespaceSplit"}, "post_processor": None,
        "decoder": None, "model": {"type": "WordLevel", "vocab": vocab, "unk_token": toks[0]},
    }


# ---------------------------------------------------------------- writer
def _w_str(f, s: str):
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f, v):
    if isinstance(v, bool):
        f.write(struct.pack("<I", _BOOL))
        f.write(struct.pack("<B", int(v)))
    elif isinstance(v, int):
        if 0 <= v < 2 ** 32:
            f.write(struct.pack("<II", _U32, v))
        else:
            f.write(struct.pack("<Iq", _I64, v))
    elif isinstance(v, float):
        f.write(struct.pack("<If", _F32, v))
    elif isinstance(v, str):
        f.write(struct.pack("<I", _STR))
        _w_str(f, v)
    elif isinstance(v, (list, tuple)):
        f.write(struct.pack("<I", _ARR))
        if len(v) == 0 or isinstance(v[0], str):
            f.write(struct.pack("<IQ", _STR, len(v)))
            for s in v:
                _w_str(f, s)
        elif isinstance(v[0], float):
            f.write(struct.pack("<IQ", _F32, len(v)))
            f.write(np.asarray(v, dtype=np.float32).tobytes())
        else:
            f.write(struct.pack("<IQ", _I32, len(v)))
            f.write(np.asarray(v, dtype=np.int32).tobytes())
    else:
        raise TypeError(f"gguf: unsupported metadata value {type(v)}")


def encode_tensor(x, ggml_type: int) -> bytes:
    import torch

    xf = x.detach().to(torch.float32).contiguous().cpu()
    if ggml_type == GGML_F32:
        return xf.numpy().tobytes()
    if ggml_type == GGML_F16:
        return xf.numpy().astype(np.float16).tobytes()
    if ggml_type == GGML_BF16:
        return (xf.view(torch.int32) >> 16).to(torch.int16).numpy().tobytes()
    if ggml_type == GGML_Q8_0:
        return _rt().quantize_q8_0(xf).numpy().tobytes()
    if ggml_type == GGML_Q4_0:
        return _rt().quantize_q4_0(xf).numpy().tobytes()
    raise NotImplementedError(ggml_type)


def write_gguf(path: str, metadata: Dict[str, Any], tensors: List[Tuple[str, Any, int]], alignment: int = 32):
    """tensors: (name, torch tensor in row-major shape, ggml type)."""
    infos = []
    blobs = []
    off = 0
    for name, x, t in tensors:
        blob = encode_tensor(x, t)
        infos.append((name, tuple(x.shape), t, off))
        blobs.append(blob)
        off += len(blob)
        off = (off + alignment - 1) // alignment * alignment
    meta = dict(metadata)
    meta.setdefault("general.alignment", alignment)
    with open(path, "wb") as f:
        f.write(b"GGUF")
        f.write(struct.pack("<IQQ", 3, len(infos), len(meta)))
        for k, v in meta.items():
            _w_str(f, k)
            _w_value(f, v)
        for name, shape, t, o in infos:
            _w_str(f, name)
            f.write(struct.pack("<I", len(shape)))
            for d in reversed(shape):
                f.write(struct.pack("<Q", d))
            f.write(struct.pack("<IQ", t, o))
        pos = f.tell()
        pad = (pos + alignment - 1) // alignment * alignment - pos
        f.write(b"\0" * pad)
        base = f.tell()
        for (name, shape, t, o), blob in zip(infos, blobs):
            cur = f.tell() - base
            if cur < o:
                f.write(b"\0" * (o - cur))
            f.write(blob)


def write_decoder_gguf(path: str, cfg, weights: Dict[str, Any], ggml_type: int = GGML_Q8_0,
                       tokenizer: Optional[dict] = None):
    """Write a decoder (HF-named weights) as a llama.cpp-compatible GGUF.

    2-D projection matrices use `ggml_type`; norms stay F32.  Q/K of the
    "llama" architecture are permuted to llama.cpp's RoPE layout."""
    arch = {"llama": "llama", "qwen2": "qwen2", "qwen3": "qwen3"}.get(cfg.arch, "llama")
    meta: Dict[str, Any] = {
        "general.architecture": arch, "general.name": cfg.name or "bloom-b200-model",
        f"{arch}.block_count": cfg.num_layers, f"{arch}.context_length": cfg.max_position_embeddings,
        f"{arch}.embedding_length": cfg.hidden_size, f"{arch}.feed_forward_length": cfg.intermediate_size,
        f"{arch}.attention.head_count": cfg.num_heads, f"{arch}.attention.head_count_kv": cfg.num_kv_heads,
        f"{arch}.attention.layer_norm_rms_epsilon": float(cfg.rms_norm_eps),
        f"{arch}.rope.freq_base": float(cfg.rope_theta), f"{arch}.vocab_size": cfg.vocab_size,
    }
    if cfg.head_dim != cfg.hidden_size // cfg.num_heads:
        meta[f"{arch}.attention.key_length"] = cfg.head_dim
        meta[f"{arch}.attention.value_length"] = cfg.head_dim
    if tokenizer is not None:
        meta.update(tokenizer)
    else:
        meta["tokenizer.ggml.model"] = "gpt2"
        meta["tokenizer.ggml.tokens"] = [f"<t{i}>" for i in range(cfg.vocab_size)]
        meta["tokenizer.ggml.token_type"] = [1] * cfg.vocab_size
        meta["tokenizer.ggml.merges"] = []
    if cfg.bos_token_id is not None:
        meta["tokenizer.ggml.bos_token_id"] = int(cfg.bos_token_id)
    if cfg.eos_token_ids:
        meta["tokenizer.ggml.eos_token_id"] = int(cfg.eos_token_ids[0])
    tens = []
    for hf_name, x in weights.items():
        g = hf_name_to_gguf(hf_name)
        if g is None:
            continue
        if arch == "llama" and _is_qk(g):
            heads = cfg.num_heads if g.endswith("attn_q.weight") else cfg.num_kv_heads
            x = permute_qk(x, heads)
        t = ggml_type if (x.dim() == 2 and x.shape[-1] % 32 == 0) else GGML_F32
        tens.append((g, x, t))
    write_gguf(path, meta, tens)
