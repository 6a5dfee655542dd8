"""Plain PyTorch fp32 restatements of every kernel in bloom_b200._C.

These are the numerics oracles for the GPU tests and the math used by the
CPU execution path.  They operate on any device and upcast to fp32.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def gemm(x, w, bias=None):
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y


def swiglu(gate, up):
    g = gate.float()
    return g * torch.sigmoid(g) * up.float()


def rmsnorm(x, w, eps):
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def layernorm(x, w, b, eps):
    return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), eps)


def rope(x, positions, cos_sin):
    """x [..., T, H, D]; HF rotate_half with the [cos | sin] table."""
    D = x.shape[-1]
    half = D // 2
    cs = cos_sin[positions.long()].float()  # [T, D]
    cos, sin = cs[:, :half], cs[:, half:]
    cos = torch.cat([cos, cos], -1)[:, None, :]
    sin = torch.cat([sin, sin], -1)[:, None, :]
    xf = x.float()
    rot = torch.cat([-xf[..., half:], xf[..., :half]], -1)
    return xf * cos + rot * sin


def attention(q, k, v, causal: bool = True, q_offset: int = 0, scale: Optional[float] = None):
    """q [Tq, Hq, D], k/v [Tk, Hkv, D]; GQA by head repetition; query i sits at kv position q_offset + i."""
    Tq, Hq, D = q.shape
    Tk, Hkv, _ = k.shape
    G = Hq // Hkv
    kk = k.float().repeat_interleave(G, dim=1)
    vv = v.float().repeat_interleave(G, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * (scale if scale is not None else 1.0 / math.sqrt(D))
    if causal:
        qi = torch.arange(Tq, device=q.device)[:, None] + q_offset
        ki = torch.arange(Tk, device=q.device)[None, :]
        s = s.masked_fill((ki > qi)[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hqk,khd->qhd", p, vv)


def gather_paged(kv_cache, layer, block_table_row, length):
    """(k, v) [length, Hkv, D] of one sequence from the paged cache [L, NB, 2, Hkv, 16, D]."""
    nb = (length + 15) // 16
    blocks = block_table_row[:nb].long()
    kv = kv_cache[layer, blocks]  # [nb, 2, Hkv, 16, D]
    k = kv[:, 0].permute(0, 2, 1, 3).reshape(nb * 16, kv.shape[2], kv.shape[4])[:length]
    v = kv[:, 1].permute(0, 2, 1, 3).reshape(nb * 16, kv.shape[2], kv.shape[4])[:length]
    return k, v
