"""umT5 text encoder (Wan 2.1's prompt encoder) on the B200 kernels.

Shape (executor/wan/t5_encoder.rs T5Config::umt5_xxl :31-41): d_model 4096,
24 layers, 64 heads of 64, d_ff 10240, vocabulary 256,384, prompts padded to
512 tokens.  Each layer: x += o(Attn(RMSNorm(x))) with T5's relative
position bias (one learned [32 buckets, heads] table per layer in umT5, no
1/sqrt(d) scale, padding keys masked), x += wo(gelu_tanh(wi_0 h) * wi_1 h)
with h = RMSNorm(x); a final RMSNorm; padded positions are zeroed (the DiT
reads a zero-padded 512-token context).

The reference's encoder (t5_encoder.rs:155-343) stands in LayerNorm, a ReLU
FFN and scaled attention without the position bias; this module follows the
published T5 v1.1 / umT5 definition so checkpoint weights load as trained.

GPU path: embedding gather, fused residual-add + RMSNorm (`add_rmsnorm`),
tcgen05 GEMMs (q|k|v in one, the gated FFN with the GeGLU epilogue), and
`t5_rel_attention` for the biased attention.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from .. import ops


@dataclass
class T5Config:
    max_length: int = 512
    d_model: int = 4096
    vocab_size: int = 256384
    num_layers: int = 24
    num_heads: int = 64
    d_ff: int = 10240
    num_buckets: int = 32
    max_distance: int = 128
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads


def t5_preset(name: str = "umt5-xxl") -> T5Config:
    if name == "umt5-xxl":
        return T5Config()
    if name == "tiny":
        return T5Config(max_length=24, d_model=256, vocab_size=512, num_layers=2, num_heads=4, d_ff=512)
    raise KeyError(f"unknown T5 preset {name!r}")


def relative_buckets(rel: torch.Tensor, num_buckets: int = 32, max_distance: int = 128) -> torch.Tensor:
    """T5's bidirectional relative position buckets (Raffel et al. 2020):
    half the buckets per direction, exact for |rel| < num_buckets / 4, then
    logarithmic up to max_distance."""
    nb = num_buckets // 2
    ret = (rel > 0).long() * nb
    n = rel.abs()
    max_exact = nb // 2
    large = max_exact + (torch.log(n.float().clamp(min=1) / max_exact) / math.log(max_distance / max_exact)
                         * (nb - max_exact)).long()
    large = large.clamp(max=nb - 1)
    return ret + torch.where(n < max_exact, n, large)


def bias_table(cfg: T5Config, emb: torch.Tensor, L: int) -> torch.Tensor:
    """[2L - 1, heads] f32: row (j - i) + L - 1 = emb[bucket(j - i)] (j key, i query)."""
    rel = torch.arange(-(L - 1), L, device=emb.device)
    return emb.float()[relative_buckets(rel, cfg.num_buckets, cfg.max_distance)].contiguous()


def t5_random_weights(cfg: T5Config, seed: int = 0, device="cpu") -> Dict[str, torch.Tensor]:
    g = torch.Generator(device="cpu").manual_seed(seed)
    D, F = cfg.d_model, cfg.d_ff

    def rn(*s, scale):
        return (torch.randn(*s, generator=g) * scale).to(torch.bfloat16).to(device)

    def near1(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16).to(device)

    w = {"encoder.embed_tokens.weight": rn(cfg.vocab_size, D, scale=1.0), "encoder.final_layer_norm.weight": near1(D)}
    for i in range(cfg.num_layers):
        p = f"encoder.block.{i}.layer."
        for n in "qkv":
            w[p + f"0.SelfAttention.{n}.weight"] = rn(D, D, scale=D ** -0.5)
        w[p + "0.SelfAttention.o.weight"] = rn(D, D, scale=D ** -0.5)
        w[p + "0.SelfAttention.relative_attention_bias.weight"] = rn(cfg.num_buckets, cfg.num_heads, scale=0.5)
        w[p + "0.layer_norm.weight"] = near1(D)
        w[p + "1.DenseReluDense.wi_0.weight"] = rn(F, D, scale=D ** -0.5)
        w[p + "1.DenseReluDense.wi_1.weight"] = rn(F, D, scale=D ** -0.5)
        w[p + "1.DenseReluDense.wo.weight"] = rn(D, F, scale=F ** -0.5)
        w[p + "1.layer_norm.weight"] = near1(D)
    return w


def t5_encode_reference(cfg: T5Config, w: Dict[str, torch.Tensor], ids: torch.Tensor,
                        lens: Sequence[int]) -> torch.Tensor:
    """fp32 oracle: ids [B, L] (padded), lens -> [B, L, d_model] (padding zeroed)."""
    f = {k: v.float() for k, v in w.items()}
    B, L = ids.shape
    nh, hd, eps = cfg.num_heads, cfg.head_dim, cfg.eps
    x = f["encoder.embed_tokens.weight"][ids.long()]

    def rms(v, wt):
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * wt

    key_ok = torch.arange(L, device=ids.device)[None, :] < torch.tensor(list(lens), device=ids.device)[:, None]
    for i in range(cfg.num_layers):
        p = f"encoder.block.{i}.layer."
        h = rms(x, f[p + "0.layer_norm.weight"])
        q, k, v = (h @ f[p + f"0.SelfAttention.{n}.weight"].t() for n in "qkv")
        q, k, v = (t.view(B, L, nh, hd) for t in (q, k, v))
        bias = bias_table(cfg, f[p + "0.SelfAttention.relative_attention_bias.weight"], L)  # [2L-1, nh]
        idx = torch.arange(L, device=ids.device)
        b = bias[(idx[None, :] - idx[:, None]) + L - 1]  # [Lq, Lk, nh]
        s = torch.einsum("bqhd,bkhd->bhqk", q, k) + b.permute(2, 0, 1)[None]
        s = s.masked_fill(~key_ok[:, None, None, :], float("-inf"))
        a = torch.einsum("bhqk,bkhd->bqhd", s.softmax(-1), v).reshape(B, L, -1)
        x = x + a @ f[p + "0.SelfAttention.o.weight"].t()
        h = rms(x, f[p + "1.layer_norm.weight"])
        g0 = h @ f[p + "1.DenseReluDense.wi_0.weight"].t()
        g1 = h @ f[p + "1.DenseReluDense.wi_1.weight"].t()
        gelu = 0.5 * g0 * (1.0 + torch.tanh(0.7978845608028654 * (g0 + 0.044715 * g0 ** 3)))
        x = x + (gelu * g1) @ f[p + "1.DenseReluDense.wo.weight"].t()
    x = rms(x, f["encoder.final_layer_norm.weight"])
    return x * key_ok[..., None]


class UMT5Encoder:
    """umT5 encoder on one GPU: `encode(ids, lens)` -> bf16 [B, L, d_model]."""

    def __init__(self, cfg: T5Config, device=None):
        if cfg.head_dim != 64:
            raise ValueError("the relative-bias attention kernel needs head_dim 64")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.cfg = cfg
        self.device = dev
        self.layers: List[Dict[str, torch.Tensor]] = []

    def load(self, full: Dict[str, torch.Tensor]) -> None:
        dev, bf = self.device, torch.bfloat16
        g = lambda n: full[n].to(dev, bf).contiguous()  # noqa: E731
        emb = full.get("encoder.embed_tokens.weight", full.get("shared.weight"))
        self.embed = emb.to(dev, bf).contiguous()
        self.final_norm = g("encoder.final_layer_norm.weight")
        self.layers = []
        for i in range(self.cfg.num_layers):
            p = f"encoder.block.{i}.layer."
            self.layers.append({
                "qkv": torch.cat([g(p + f"0.SelfAttention.{n}.weight") for n in "qkv"], 0).contiguous(),
                "o": g(p + "0.SelfAttention.o.weight"),
                "rel": full[p + "0.SelfAttention.relative_attention_bias.weight"].to(dev).float(),
                "ln0": g(p + "0.layer_norm.weight"),
                "wi": ops.interleave_gate_up(g(p + "1.DenseReluDense.wi_0.weight"),
                                             g(p + "1.DenseReluDense.wi_1.weight")),
                "wo": g(p + "1.DenseReluDense.wo.weight"),
                "ln1": g(p + "1.layer_norm.weight"),
            })
        self._bias: Dict[int, List[torch.Tensor]] = {}

    def random_init(self, seed: int = 0) -> None:
        self.load(t5_random_weights(self.cfg, seed, self.device))

    def encode(self, ids: torch.Tensor, lens: Sequence[int]) -> torch.Tensor:
        cfg, dev = self.cfg, self.device
        B, L = ids.shape
        if L not in self._bias:
            self._bias[L] = [bias_table(cfg, lay["rel"], L) for lay in self.layers]
        flat = ids.to(dev, torch.int32).reshape(-1).contiguous()
        x = ops.embedding(flat, self.embed)  # residual (bf16)
        lens_t = torch.tensor(list(lens), dtype=torch.int32, device=dev)
        h = ops.rmsnorm(x, self.layers[0]["ln0"], cfg.eps)
        C = _C()
        for i, lay in enumerate(self.layers):
            qkv = ops.gemm(h, lay["qkv"])
            a = torch.empty(B * L, cfg.d_model, dtype=torch.bfloat16, device=dev)
            C.t5_rel_attention(qkv, B, cfg.num_heads, lens_t, self._bias[L][i], a)
            ops._count()
            h = ops.add_rmsnorm(ops.gemm(a, lay["o"]), x, lay["ln1"], cfg.eps)  # x += attn; h = norm(x)
            m = ops.gemm(h, lay["wi"], epi=ops.EPI_GEGLU)
            nxt = self.layers[i + 1]["ln0"] if i + 1 < len(self.layers) else self.final_norm
            h = ops.add_rmsnorm(ops.gemm(m, lay["wo"]), x, nxt, cfg.eps)
        out = h.view(B, L, cfg.d_model)
        for b, n in enumerate(lens):  # zero-padded context, as the DiT reads it
            if n < L:
                out[b, n:].zero_()
        return out


def _C():
    from .._ext import cuda

    return cuda()
