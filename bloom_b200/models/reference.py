"""Plain PyTorch fp32 forward of the decoder family (the oracle for GPU tests).

Takes full, unsharded Hugging Face-named weights and computes logits for one
token sequence with no KV cache.  Semantics: HF Llama/Qwen2/Qwen3 modelling
(RMSNorm, rotate_half RoPE, GQA, SwiGLU, optional QKV bias, optional q/k norm).
"""
from __future__ import annotations

from typing import Dict

import torch

from ..ops import reference as R
from ..ops import rope_cos_sin
from .config import ModelConfig


def forward_logits(cfg: ModelConfig, w: Dict[str, torch.Tensor], tokens) -> torch.Tensor:
    dev = w["model.embed_tokens.weight"].device
    ids = torch.as_tensor(tokens, device=dev).long()
    T = ids.numel()
    hd = cfg.head_dim
    x = w["model.embed_tokens.weight"][ids].float()
    cs = rope_cos_sin(max(cfg.max_position_embeddings, T), hd, cfg.rope_theta, dev, cfg.rope_scaling)
    pos = torch.arange(T, device=dev)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        h = R.rmsnorm(x, w[p + "input_layernorm.weight"], cfg.rms_norm_eps)
        q = h @ w[p + "self_attn.q_proj.weight"].float().t()
        k = h @ w[p + "self_attn.k_proj.weight"].float().t()
        v = h @ w[p + "self_attn.v_proj.weight"].float().t()
        if cfg.qkv_bias:
            q = q + w[p + "self_attn.q_proj.bias"].float()
            k = k + w[p + "self_attn.k_proj.bias"].float()
            v = v + w[p + "self_attn.v_proj.bias"].float()
        q = q.view(T, cfg.num_heads, hd)
        k = k.view(T, cfg.num_kv_heads, hd)
        v = v.view(T, cfg.num_kv_heads, hd)
        if cfg.qk_norm:
            q = R.rmsnorm(q, w[p + "self_attn.q_norm.weight"], cfg.rms_norm_eps)
            k = R.rmsnorm(k, w[p + "self_attn.k_norm.weight"], cfg.rms_norm_eps)
        q = R.rope(q, pos, cs)
        k = R.rope(k, pos, cs)
        a = R.attention(q, k, v, causal=True).reshape(T, cfg.q_size)
        x = x + a @ w[p + "self_attn.o_proj.weight"].float().t()
        h = R.rmsnorm(x, w[p + "post_attention_layernorm.weight"], cfg.rms_norm_eps)
        if cfg.is_moe:
            x = x + moe_mlp(cfg, w, p, h)
        else:
            g = h @ w[p + "mlp.gate_proj.weight"].float().t()
            u = h @ w[p + "mlp.up_proj.weight"].float().t()
            x = x + R.swiglu(g, u) @ w[p + "mlp.down_proj.weight"].float().t()
    x = R.rmsnorm(x, w["model.norm.weight"], cfg.rms_norm_eps)
    lm = w.get("lm_head.weight", w["model.embed_tokens.weight"])
    return x @ lm.float().t()


def moe_mlp(cfg: ModelConfig, w, p, h):
    """Dense reference of a top-k softmax-routed SwiGLU expert layer."""
    logits = h @ w[p + "mlp.gate.weight"].float().t()
    probs = torch.softmax(logits, -1)
    topv, topi = probs.topk(cfg.num_experts_per_tok, dim=-1)
    if cfg.norm_topk_prob:
        topv = topv / topv.sum(-1, keepdim=True)
    out = torch.zeros_like(h)
    G, U, D = (w[p + "mlp.experts.gate_proj"].float(), w[p + "mlp.experts.up_proj"].float(),
               w[p + "mlp.experts.down_proj"].float())
    for t in range(h.shape[0]):
        for j in range(cfg.num_experts_per_tok):
            e = int(topi[t, j])
            y = R.swiglu(h[t] @ G[e].t(), h[t] @ U[e].t()) @ D[e].t()
            out[t] += topv[t, j] * y
    return out


def random_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02, device="cpu") -> Dict[str, torch.Tensor]:
    """Full HF-named random weights (bf16) for tests and fixtures."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    H, hd = cfg.hidden_size, cfg.head_dim

    def rn(*s):
        return (torch.randn(*s, generator=g) * std).to(torch.bfloat16).to(device)

    def ones(n):
        return torch.ones(n, dtype=torch.bfloat16, device=device)

    w = {"model.embed_tokens.weight": rn(cfg.vocab_size, H), "model.norm.weight": ones(H)}
    if not cfg.tie_word_embeddings:
        w["lm_head.weight"] = rn(cfg.vocab_size, H)
    for i in range(cfg.num_layers):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = ones(H)
        w[p + "post_attention_layernorm.weight"] = ones(H)
        w[p + "self_attn.q_proj.weight"] = rn(cfg.q_size, H)
        w[p + "self_attn.k_proj.weight"] = rn(cfg.kv_size, H)
        w[p + "self_attn.v_proj.weight"] = rn(cfg.kv_size, H)
        w[p + "self_attn.o_proj.weight"] = rn(H, cfg.q_size)
        if cfg.qkv_bias:
            w[p + "self_attn.q_proj.bias"] = rn(cfg.q_size)
            w[p + "self_attn.k_proj.bias"] = rn(cfg.kv_size)
            w[p + "self_attn.v_proj.bias"] = rn(cfg.kv_size)
        if cfg.qk_norm:
            w[p + "self_attn.q_norm.weight"] = ones(hd)
            w[p + "self_attn.k_norm.weight"] = ones(hd)
        if cfg.is_moe:
            E, Im = cfg.num_experts, cfg.moe_intermediate_size
            w[p + "mlp.gate.weight"] = rn(E, H)
            w[p + "mlp.experts.gate_proj"] = rn(E, Im, H)
            w[p + "mlp.experts.up_proj"] = rn(E, Im, H)
            w[p + "mlp.experts.down_proj"] = rn(E, H, Im)
        else:
            w[p + "mlp.gate_proj.weight"] = rn(cfg.intermediate_size, H)
            w[p + "mlp.up_proj.weight"] = rn(cfg.intermediate_size, H)
            w[p + "mlp.down_proj.weight"] = rn(H, cfg.intermediate_size)
    return w
