"""Host (CPU) execution path for small GGUF decoders.

Linear layers run on GGUF blocks directly through the C++ kernels of
bloom_b200._runtime (Q8_0 x Q8_0 int8 dot products with the activation row
quantised on the fly, AVX2); everything else (RMSNorm, RoPE, attention,
SwiGLU) runs in fp32 PyTorch on the CPU with a contiguous per-request KV
cache.  This is the path for CPU-only hosts and for the SmolLM2-135M-shape
Q8_0 configuration; it mirrors the reference's Candle CPU quantized Llama
(crates/engine/src/executor/candle.rs:1533-1568).
"""
from __future__ import annotations

import math
from typing import Dict, Iterator, List, Optional

import torch

from .._ext import runtime as _rt
from ..formats.gguf import GGML_Q8_0, GGUFFile, config_from_gguf, gguf_name_to_hf
from ..models.config import ModelConfig
from ..ops import reference as R
from ..ops import rope_cos_sin


class QLinear:
    """A GGUF Q8_0 weight [N, K] used as y = x @ W^T."""

    def __init__(self, raw: torch.Tensor, n: int, k: int):
        self.raw, self.n, self.k = raw, n, k

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return _rt().q8_0_matmul(x, self.raw, self.n, self.k)


class FLinear:
    def __init__(self, w: torch.Tensor):
        self.w = w.float().contiguous()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return x.float() @ self.w.t()


def _fuse(parts: List[object]) -> Optional[object]:
    """Rows of several Q8_0 / fp32 linears with the same K as one linear."""
    if all(isinstance(p, QLinear) for p in parts) and len({p.k for p in parts}) == 1:
        return QLinear(torch.cat([p.raw.view(p.n, -1) for p in parts], 0).reshape(-1).contiguous(),
                       sum(p.n for p in parts), parts[0].k)
    if all(isinstance(p, FLinear) for p in parts) and len({p.w.shape[1] for p in parts}) == 1:
        return FLinear(torch.cat([p.w for p in parts], 0))
    return None


class CpuDecoder:
    def __init__(self, cfg: ModelConfig, linears: Dict[str, object], dense: Dict[str, torch.Tensor]):
        import os

        # the native thread pool parallelises the matmuls; the PyTorch glue
        # between them is tiny, and torch's own intra-op threads would only
        # compete with the pool's workers for the cores
        torch.set_num_threads(int(os.environ.get("BLOOM_TORCH_THREADS", "1")))
        self.cfg = cfg
        self.L = linears
        self.D = dense
        # one matmul for q|k|v and one for gate|up per layer: the decode step is
        # a chain of small matmuls, so fewer and larger ones run faster
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            qkv = _fuse([linears[p + f"self_attn.{x}_proj.weight"] for x in "qkv"])
            if qkv is not None:
                linears[p + "self_attn.qkv"] = qkv
            gu = _fuse([linears[p + "mlp.gate_proj.weight"], linears[p + "mlp.up_proj.weight"]])
            if gu is not None:
                linears[p + "mlp.gate_up"] = gu
        self.cos_sin = rope_cos_sin(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta,
                                    scaling=cfg.rope_scaling)

    @staticmethod
    def from_gguf(path: str) -> "CpuDecoder":
        from ..formats.gguf import _is_qk, unpermute_qk

        g = GGUFFile(path)
        cfg = config_from_gguf(g)
        lin, dense = {}, {}
        for name, t in g.tensors.items():
            hf = gguf_name_to_hf(name)
            if hf is None:
                continue
            if t.ggml_type == GGML_Q8_0 and len(t.shape) == 2 and "embed_tokens" not in hf:
                if g.arch == "llama" and _is_qk(name):
                    # un-permute RoPE rows on the dequantised matrix, then re-block
                    w = g.tensor(name)
                    lin[hf] = QLinear(_rt().quantize_q8_0(w), t.shape[0], t.shape[1])
                else:
                    raw = torch.from_numpy(g.raw(name).copy())
                    lin[hf] = QLinear(raw, t.shape[0], t.shape[1])
            else:
                dense[hf] = g.tensor(name).float()
        if "lm_head.weight" not in lin and "lm_head.weight" not in dense:
            emb = dense["model.embed_tokens.weight"]
            lin["lm_head.weight"] = QLinear(_rt().quantize_q8_0(emb), emb.shape[0], emb.shape[1])
        for k in list(dense):
            if k.endswith("proj.weight") and dense[k].dim() == 2:
                lin[k] = FLinear(dense.pop(k))
        return CpuDecoder(cfg, lin, dense)

    @staticmethod
    def from_weights(cfg: ModelConfig, w: Dict[str, torch.Tensor], quantize: bool = True) -> "CpuDecoder":
        lin, dense = {}, {}
        for k, v in w.items():
            if v.dim() == 2 and k != "model.embed_tokens.weight":
                lin[k] = QLinear(_rt().quantize_q8_0(v.float()), v.shape[0], v.shape[1]) if quantize else FLinear(v)
            else:
                dense[k] = v.float()
        if "lm_head.weight" not in lin:
            e = dense["model.embed_tokens.weight"]
            lin["lm_head.weight"] = QLinear(_rt().quantize_q8_0(e), e.shape[0], e.shape[1]) if quantize else FLinear(e)
        return CpuDecoder(cfg, lin, dense)

    def new_cache(self, max_len: int):
        c = self.cfg
        return {"k": torch.zeros(c.num_layers, max_len, c.num_kv_heads, c.head_dim),
                "v": torch.zeros(c.num_layers, max_len, c.num_kv_heads, c.head_dim), "len": 0}

    @torch.no_grad()
    def forward(self, tokens: List[int], cache) -> torch.Tensor:
        """Logits of the last position after appending `tokens` to the cache."""
        c = self.cfg
        L, D = self.L, self.D
        T = len(tokens)
        start = cache["len"]
        pos = torch.arange(start, start + T)
        x = D["model.embed_tokens.weight"][torch.tensor(tokens)]
        for i in range(c.num_layers):
            p = f"model.layers.{i}."
            h = R.rmsnorm(x, D[p + "input_layernorm.weight"], c.rms_norm_eps)
            if p + "self_attn.qkv" in L:
                q, k, v = L[p + "self_attn.qkv"](h).split([c.q_size, c.kv_size, c.kv_size], dim=-1)
            else:
                q = L[p + "self_attn.q_proj.weight"](h)
                k = L[p + "self_attn.k_proj.weight"](h)
                v = L[p + "self_attn.v_proj.weight"](h)
            if c.qkv_bias:
                q = q + D[p + "self_attn.q_proj.bias"]
                k = k + D[p + "self_attn.k_proj.bias"]
                v = v + D[p + "self_attn.v_proj.bias"]
            q = q.view(T, c.num_heads, c.head_dim)
            k = k.view(T, c.num_kv_heads, c.head_dim)
            v = v.view(T, c.num_kv_heads, c.head_dim)
            if c.qk_norm:
                q = R.rmsnorm(q, D[p + "self_attn.q_norm.weight"], c.rms_norm_eps)
                k = R.rmsnorm(k, D[p + "self_attn.k_norm.weight"], c.rms_norm_eps)
            q = R.rope(q, pos, self.cos_sin)
            k = R.rope(k, pos, self.cos_sin)
            cache["k"][i, start:start + T] = k
            cache["v"][i, start:start + T] = v
            kk = cache["k"][i, :start + T]
            vv = cache["v"][i, :start + T]
            a = R.attention(q, kk, vv, causal=True, q_offset=start).reshape(T, c.q_size)
            x = x + L[p + "self_attn.o_proj.weight"](a)
            h = R.rmsnorm(x, D[p + "post_attention_layernorm.weight"], c.rms_norm_eps)
            if p + "mlp.gate_up" in L:
                g, u = L[p + "mlp.gate_up"](h).split([c.intermediate_size, c.intermediate_size], dim=-1)
            else:
                g = L[p + "mlp.gate_proj.weight"](h)
                u = L[p + "mlp.up_proj.weight"](h)
            x = x + L[p + "mlp.down_proj.weight"](R.swiglu(g, u))
        cache["len"] = start + T
        h = R.rmsnorm(x[-1:], D["model.norm.weight"], c.rms_norm_eps)
        return L["lm_head.weight"](h)[0]

    def generate(self, prompt: List[int], max_tokens: int, temperature: float = 0.0, top_p: float = 1.0,
                 seed: Optional[int] = None, eos: Optional[List[int]] = None, ignore_eos: bool = False) -> Iterator[int]:
        cache = self.new_cache(min(self.cfg.max_position_embeddings, len(prompt) + max_tokens + 1))
        gen = torch.Generator().manual_seed(seed if seed is not None else 42)
        logits = self.forward(prompt, cache)
        for _ in range(max_tokens):
            tok = sample_host(logits, temperature, top_p, gen)
            yield tok
            if not ignore_eos and eos and tok in eos:
                return
            if cache["len"] >= cache["k"].shape[1]:
                return
            logits = self.forward([tok], cache)


def sample_host(logits: torch.Tensor, temperature: float, top_p: float, gen: torch.Generator) -> int:
    if temperature <= 0:
        return int(torch.argmax(logits))
    p = torch.softmax(logits.float() / temperature, -1)
    if 0 < top_p < 1:
        sp, si = torch.sort(p, descending=True)
        keep = torch.cumsum(sp, 0) - sp < top_p
        sp = sp * keep
        idx = torch.multinomial(sp / sp.sum(), 1, generator=gen)
        return int(si[idx])
    return int(torch.multinomial(p, 1, generator=gen))
