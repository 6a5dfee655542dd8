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


def q8_perm16(i: int) -> int:
    """Byte position of element i of an int8 page row (MMA fragment order:
    within each group of 16, elements 2t, 2t+1, 2t+8, 2t+9 are bytes 4t..4t+3)."""
    return (i & ~15) | (((i & 7) >> 1) << 2) | (((i >> 3) & 1) << 1) | (i & 1)


def dequant_q8_cache(kv_u8, num_kv_heads: int, head_dim: int = 128):
    """fp32 [L, NB, 2, Hkv, 16, D] of an int8 cache [L, NB, block bytes]: K
    pages [Hkv][16][D] in natural order, dim-major V pages [Hkv][D][16] with
    each 16-token row in fragment order (`q8_perm16`), then fp32 scales
    [2][Hkv][16] per block (the layout rope_kv_write writes for int8)."""
    L, NB, BB = kv_u8.shape
    P = num_kv_heads * 16 * head_dim
    dev = kv_u8.device
    tp = torch.tensor([q8_perm16(t) for t in range(16)], device=dev)
    k = kv_u8[:, :, :P].contiguous().view(torch.int8).view(L, NB, num_kv_heads, 16, head_dim).float()
    v = kv_u8[:, :, P:2 * P].contiguous().view(torch.int8).view(L, NB, num_kv_heads, head_dim, 16)[..., tp]
    v = v.transpose(-1, -2).float()
    sc = kv_u8[:, :, 2 * P:].contiguous().view(torch.float32).view(L, NB, 2, num_kv_heads, 16)
    return torch.stack([k * sc[:, :, 0, :, :, None], v * sc[:, :, 1, :, :, None]], 2)


def quantize_q8_rows(x):
    """Symmetric int8 of the last dimension: (int8 values, fp32 scale = absmax / 127)."""
    am = x.float().abs().amax(-1, keepdim=True)
    inv = torch.where(am > 0, 127.0 / am, torch.zeros_like(am))
    q = torch.round(x.float() * inv).clamp(-127, 127)
    return q, (am / 127.0).squeeze(-1)


# ---------------------------------------------------------------- quantised formats (fp32 restatements)

NF4_CODEBOOK = (-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453, -0.28444138169288635,
                -0.18477343022823334, -0.09105003625154495, 0.0, 0.07958029955625534, 0.16093020141124725,
                0.24611230194568634, 0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                0.7229568362236023, 1.0)
FP4_CODEBOOK = (0.0, 0.0625, 8.0, 12.0, 4.0, 6.0, 2.0, 3.0, -0.0, -0.0625, -8.0, -12.0, -4.0, -6.0, -2.0, -3.0)


def _nibbles(words: torch.Tensor) -> torch.Tensor:
    """int32 words [...] -> their 8 nibbles [..., 8], nibble i = bits 4i..4i+3."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    return torch.stack([(w >> (4 * i)) & 0xF for i in range(8)], dim=-1)


def dequant_int4_flat(qweight, scales, qzeros, n: int, g_idx=None) -> torch.Tensor:
    """Flat AWQ (g_idx None, groups of 128) / GPTQ (g = g_idx[id]) int4 -> fp32 [n]."""
    q = _nibbles(qweight.flatten()).flatten()
    out = torch.zeros(n, dtype=torch.float32)
    ids = torch.arange(n)
    ok = ids < q.numel()
    if g_idx is None:
        g = ids // 128
    else:
        ok &= ids < g_idx.numel()
        g = torch.zeros(n, dtype=torch.int64)
        m = ids < g_idx.numel()
        g[m] = g_idx.flatten()[ids[m]].to(torch.int64) & 0xFFFFFFFF
    sc = scales.flatten().float()
    ok &= g < sc.numel()
    zw = _nibbles(qzeros.flatten()).flatten()
    z = torch.zeros(n)
    zm = ok & (g < zw.numel())
    z[zm] = zw[g[zm]].float()
    out[ok] = (q[ids[ok]].float() - z[ok]) * sc[g[ok]]
    return out


def dequant_gptq(qweight, qzeros, scales, g_idx) -> torch.Tensor:
    """HF GPTQ tensors (qweight [K/8, N], qzeros [G, N/8], scales [G, N], g_idx [K]) -> W [N, K] fp32."""
    Kw, N = qweight.shape
    q = _nibbles(qweight).permute(0, 2, 1).reshape(Kw * 8, N)  # [K, N]
    z = _nibbles(qzeros).reshape(qzeros.shape[0], N) + 1       # [G, N]
    g = g_idx.to(torch.int64)
    w = (q.float() - z[g].float()) * scales.float()[g]
    return w.t().contiguous()


AWQ_ORDER = (0, 4, 1, 5, 2, 6, 3, 7)  # column j of 8 sits in nibble AWQ_ORDER[j]


def dequant_awq(qweight, qzeros, scales, group: int) -> torch.Tensor:
    """AWQ GEMM-format tensors (qweight [K, N/8], qzeros [K/group, N/8], scales [K/group, N]) -> W [N, K] fp32."""
    K, Nw = qweight.shape
    order = torch.tensor(AWQ_ORDER)
    q = _nibbles(qweight)[..., order].reshape(K, Nw * 8)
    z = _nibbles(qzeros)[..., order].reshape(qzeros.shape[0], Nw * 8)
    g = torch.arange(K) // group
    w = (q.float() - z[g].float()) * scales.float()[g]
    return w.t().contiguous()


def dequant_bnb4(packed, scale, block: int, nf4: bool = True) -> torch.Tensor:
    """bitsandbytes 4-bit codes (high nibble first) -> fp32 [2 * bytes], one scale per `block` outputs."""
    b = packed.flatten().to(torch.int64)
    codes = torch.stack([b >> 4, b & 15], dim=-1).flatten()
    book = torch.tensor(NF4_CODEBOOK if nf4 else FP4_CODEBOOK, dtype=torch.float32)
    s = scale.flatten().float()
    return book[codes] * s[torch.arange(codes.numel()) // block]


def mrope(x, cos, sin, sections=(24, 20, 20)):
    """Rotate-half M-RoPE of x [B, H, S, D] with cos / sin [3, B, S, D] (fp32)."""
    D = x.shape[-1]
    half = D // 2
    comp = torch.cat([torch.full((n,), i, dtype=torch.long) for i, n in enumerate(sections)])
    comp = torch.cat([comp, comp])  # [D]: position plane of every channel
    idx = torch.arange(D)
    c = cos.float()[comp, :, :, idx].permute(1, 2, 0)[:, None]  # [B, 1, S, D]
    s = sin.float()[comp, :, :, idx].permute(1, 2, 0)[:, None]
    x = x.float()
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * c + rot * s


def kv_quantize_int8(x):
    """Symmetric per-row int8: scale = max|x| / 127 (1 for a zero row), q = clamp(round(x / scale))."""
    x = x.float()
    mx = x.abs().amax(dim=-1)
    scale = torch.where(mx > 0, mx / 127.0, torch.ones_like(mx))
    inv = 1.0 / scale
    v = x * inv[:, None]
    q = torch.clamp(torch.sign(v) * torch.floor(v.abs() + 0.5), -128, 127).to(torch.int8)
    return q, scale


def kv_dequantize_int8(q, scale):
    return q.float() * scale.float()[:, None]
