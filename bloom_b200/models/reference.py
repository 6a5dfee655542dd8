"""Plain PyTorch fp32 forward of the decoder family (the oracle for GPU tests).

Takes full, unsharded Hugging Face-named weights and computes logits for one
token sequence with no KV cache.  Semantics: HF Llama/Qwen2/Qwen3 modelling
(RMSNorm, rotate_half RoPE, GQA, SwiGLU, optional QKV bias, optional q/k norm).
"""
from __future__ import annotations

import math
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


# ---------------------------------------------------------------- Gemma4
GEMMA4_PREFIX = "model.language_model."


def gemma4_random_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02,
                          device="cpu") -> Dict[str, torch.Tensor]:
    """HF-named random Gemma4 text weights (bf16).  Norm weights and layer
    scalars are drawn around 1 so the test exercises them."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    H, I, nh = cfg.hidden_size, cfg.intermediate_size, cfg.num_heads
    P = GEMMA4_PREFIX

    def rn(*s):
        return (torch.randn(*s, generator=g) * std).to(torch.bfloat16).to(device)

    def near1(*s):
        return (1.0 + 0.2 * torch.randn(*s, generator=g)).to(torch.bfloat16).to(device)

    w = {P + "embed_tokens.weight": rn(cfg.vocab_size, H), P + "norm.weight": near1(H)}
    for i in range(cfg.num_layers):
        p = f"{P}layers.{i}."
        d, kvh = cfg.layer_attn(i)
        w[p + "self_attn.q_proj.weight"] = rn(nh * d, H)
        w[p + "self_attn.k_proj.weight"] = rn(kvh * d, H)
        if not (cfg.attention_k_eq_v and not cfg.is_sliding(i)):
            w[p + "self_attn.v_proj.weight"] = rn(kvh * d, H)
        w[p + "self_attn.o_proj.weight"] = rn(H, nh * d)
        # q / k norm weights near 1/2 each: with attention scale 1, q.k of unit-RMS heads would have a
        # standard deviation of sqrt(head_dim) (16 to 23 here) and an almost one-hot softmax whose
        # near-ties flip under bf16 rounding; at 1/4 of that the oracle comparison stays well posed
        w[p + "self_attn.q_norm.weight"] = (near1(d).float() * 0.5).to(torch.bfloat16)
        w[p + "self_attn.k_norm.weight"] = (near1(d).float() * 0.5).to(torch.bfloat16)
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            w[p + n + ".weight"] = near1(H)
        w[p + "mlp.gate_proj.weight"] = rn(I, H)
        w[p + "mlp.up_proj.weight"] = rn(I, H)
        w[p + "mlp.down_proj.weight"] = rn(H, I)
        w[p + "layer_scalar"] = (0.75 + 0.5 * torch.rand(1, generator=g)).to(torch.bfloat16).to(device)
    return w


def _gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def gemma4_forward_logits(cfg: ModelConfig, w: Dict[str, torch.Tensor], tokens, trace=None) -> torch.Tensor:
    """fp32 Gemma4 text forward over one sequence (executor/gemma4.rs semantics:
    scaled embedding, q/k/v norms, partial RoPE on global layers, attention
    scale 1, soft-capped scores, sliding-window masks of `sliding_window` keys,
    sandwich norms, layer scalar, tied lm_head, soft-capped logits)."""
    P = GEMMA4_PREFIX
    emb = w[P + "embed_tokens.weight"]
    dev = emb.device
    ids = torch.as_tensor(tokens, device=dev).long()
    T = ids.numel()
    H, eps, nh = cfg.hidden_size, cfg.rms_norm_eps, cfg.num_heads
    x = emb[ids].float() * math.sqrt(H)
    x = x.to(torch.bfloat16).float()  # the embedding runs in bf16 in the model
    pos = torch.arange(T, device=dev)
    qi, kj = pos[:, None], pos[None, :]

    def rms(t, wt=None):
        y = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps)
        return y * wt.float() if wt is not None else y

    def rope(t, rot, denom, theta):
        half = rot // 2
        inv = 1.0 / (theta ** (torch.arange(0, half, device=dev, dtype=torch.float64) * 2 / denom))
        ang = (pos.double()[:, None] * inv[None, :]).float()
        c, s = ang.cos()[:, None, :], ang.sin()[:, None, :]
        x1, x2, rest = t[..., :half], t[..., half:rot], t[..., rot:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s, rest], dim=-1)

    for i in range(cfg.num_layers):
        p = f"{P}layers.{i}."
        sliding = cfg.is_sliding(i)
        d, kvh = cfg.layer_attn(i)
        rot = d if sliding else int(d * cfg.partial_rotary_factor)
        theta = cfg.rope_local_theta if sliding else cfg.rope_theta
        h = rms(x, w[p + "input_layernorm.weight"])
        q = (h @ w[p + "self_attn.q_proj.weight"].float().t()).view(T, nh, d)
        k = (h @ w[p + "self_attn.k_proj.weight"].float().t()).view(T, kvh, d)
        vw = w.get(p + "self_attn.v_proj.weight")
        v = (h @ vw.float().t()).view(T, kvh, d) if vw is not None else k
        q = rope(rms(q, w[p + "self_attn.q_norm.weight"]), rot, d, theta)
        k2 = rope(rms(k, w[p + "self_attn.k_norm.weight"]), rot, d, theta)
        v = rms(v)
        G = nh // kvh
        kk = k2.repeat_interleave(G, dim=1)
        vv = v.repeat_interleave(G, dim=1)
        sc = torch.einsum("qhd,khd->hqk", q, kk)  # attention scale 1
        if cfg.attn_logit_softcapping:
            sc = cfg.attn_logit_softcapping * torch.tanh(sc / cfg.attn_logit_softcapping)
        vis = kj <= qi
        if sliding:
            vis = vis & (kj > qi - cfg.sliding_window)
        sc = sc.masked_fill(~vis[None], float("-inf"))
        a = torch.einsum("hqk,khd->qhd", sc.softmax(-1), vv).reshape(T, nh * d)
        a = a @ w[p + "self_attn.o_proj.weight"].float().t()
        x = x + rms(a, w[p + "post_attention_layernorm.weight"])
        if trace is not None:
            trace.append(x.clone())
        h = rms(x, w[p + "pre_feedforward_layernorm.weight"])
        gt = h @ w[p + "mlp.gate_proj.weight"].float().t()
        up = h @ w[p + "mlp.up_proj.weight"].float().t()
        m = (_gelu_tanh(gt) * up) @ w[p + "mlp.down_proj.weight"].float().t()
        x = (x + rms(m, w[p + "post_feedforward_layernorm.weight"])) * w[p + "layer_scalar"].float()
        if trace is not None:
            trace.append(x.clone())
    logits = rms(x, w[P + "norm.weight"]) @ emb.float().t()
    if cfg.final_logit_softcapping:
        logits = cfg.final_logit_softcapping * torch.tanh(logits / cfg.final_logit_softcapping)
    return logits
