"""LongCat image edit: a Flux-style MMDiT over [text; image] tokens and a KL
VAE, on the B200 kernels.

Transformer (executor/longcat_native.rs forward_complete_transformer
:1080-1123): x_embedder over 2x2-packed latents, context_embedder over the
prompt embeddings, timestep embedding -> SiLU -> one AdaLN linear per block,
then
  * joint blocks (:966-1024): AdaLayerNormZero on each stream, joint
    attention over the concatenated text and image tokens (per-head q/k
    RMSNorm, 3-axis interleaved RoPE), gated residuals, GELU-tanh FFNs per
    stream;
  * single blocks (:1026-1057): one AdaLN, parallel attention and MLP whose
    concatenation is projected back, gated residual;
  * AdaLayerNormContinuous (scale then shift) and proj_out on the image tokens.
VAE (AutoEncoderKL): encoder (conv_in, down blocks with stride-2
convolutions padded (0, 1, 0, 1), mid block with one-head attention,
GroupNorm -> SiLU -> conv_out to mean / log-variance) and decoder (conv_in,
mid block, up blocks with nearest x2 + conv, GroupNorm -> SiLU -> conv_out);
latents are (mean - shift) * scale.
Draft edit (run_draft_image_edit :257-307): encode the image, one
transformer pass at t = 0.5, the un-packed output rescaled to at most the
latent's RMS, latent + 0.12 * delta, decode.

B200 mapping: the residual stream of both streams is one fp32 buffer
[text; image] (the joint blocks work on its two row ranges, the single
blocks on all of it, so no concatenation is ever copied); all AdaLN
linears of a step are one GEMM; `wan_residual_norm` applies each gate,
adds the residual and writes the next modulated LayerNorm in one pass;
`wan_qkv_norm_rope` places the text and image rows of q and the paged K / V
in joint order with per-head RMSNorm and RoPE fused; the joint attention is
the paged tcgen05 prefill kernel with causal masking off; the single
block's projection of [attn | mlp] is two GEMMs, the second adding the first
in its epilogue.  RoPE positions of image tokens use the packed grid
(row = idx // width); the reference derives them from sqrt(tokens), which
is the same for square images.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from .wan_vae import VaeConfig, WanVAE


@dataclass
class LongCatConfig:
    dim: int = 3072
    num_heads: int = 24
    head_dim: int = 128
    num_layers: int = 19
    num_single_layers: int = 38
    in_channels: int = 64
    joint_attention_dim: int = 3584
    axes_dims_rope: Tuple[int, int, int] = (16, 56, 56)
    ff_mult: int = 4
    eps: float = 1e-6
    name: str = ""


LONGCAT_PRESETS = {
    "longcat-image-edit": LongCatConfig(name="longcat-image-edit"),
    "tiny-longcat": LongCatConfig(dim=256, num_heads=2, num_layers=2, num_single_layers=2, joint_attention_dim=128,
                                  name="tiny-longcat"),
}


def longcat_preset(name: str) -> LongCatConfig:
    if name not in LONGCAT_PRESETS:
        raise KeyError(f"unknown LongCat preset {name!r}; known: {sorted(LONGCAT_PRESETS)}")
    return dataclasses.replace(LONGCAT_PRESETS[name])


def rope_table(cfg: LongCatConfig, positions: int = 1024) -> torch.Tensor:
    """[positions, head_dim / 2, 2] (cos, sin): pair i of axis a at position n
    turns by n * 10000^(-2 i / axes[a]) (longcat_native.rs:2040-2087)."""
    inv = torch.cat([1.0 / 10000.0 ** (torch.arange(a // 2, dtype=torch.float64) * 2 / a) for a in cfg.axes_dims_rope])
    ang = torch.arange(positions, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([ang.cos(), ang.sin()], -1).float().contiguous()


def token_positions(text_tokens: int, grid_h: int, grid_w: int) -> torch.Tensor:
    """int32 [text + image, 3]: text (0, 0, i), image (0, row, column)."""
    t = torch.stack([torch.zeros(text_tokens, dtype=torch.int32), torch.zeros(text_tokens, dtype=torch.int32),
                     torch.arange(text_tokens, dtype=torch.int32)], 1)
    idx = torch.arange(grid_h * grid_w, dtype=torch.int32)
    im = torch.stack([torch.zeros_like(idx), idx // grid_w, idx % grid_w], 1)
    return torch.cat([t, im], 0).contiguous()


def timestep_embedding(t: float, dim: int = 256) -> torch.Tensor:
    """[1, dim] = [cos | sin](t * 1000 * 10000^(-i / half)) (longcat_native.rs:2025-2038)."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    a = t * 1000.0 * freqs
    return torch.cat([a.cos(), a.sin()])[None, :]


def pack_latents(lat: torch.Tensor) -> torch.Tensor:
    """[C, H, W] -> [(H/2) (W/2), C * 4] (longcat_native.rs:1204-1213)."""
    C, H, W = lat.shape
    return lat.reshape(C, H // 2, 2, W // 2, 2).permute(1, 3, 0, 2, 4).reshape((H // 2) * (W // 2), C * 4)


def unpack_latents(p: torch.Tensor, C: int, H: int, W: int) -> torch.Tensor:
    return p.reshape(H // 2, W // 2, C, 2, 2).permute(2, 0, 3, 1, 4).reshape(C, H, W)


def longcat_random_weights(cfg: LongCatConfig, seed: int = 0, device="cpu") -> Dict[str, torch.Tensor]:
    """Random weights drawn on `device` (a CUDA device draws them there: the full-size model
    has ~12 B parameters)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    D, hd, Fd = cfg.dim, cfg.head_dim, cfg.ff_mult * cfg.dim

    def lin(name, o, i, scale=None):
        s = scale if scale is not None else i ** -0.5
        w[name + ".weight"] = (torch.randn(o, i, generator=g, device=dev) * s).to(torch.bfloat16)
        w[name + ".bias"] = (torch.randn(o, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    def nrm(name, n):
        w[name + ".weight"] = (1.0 + 0.1 * torch.randn(n, generator=g, device=dev)).float()

    w: Dict[str, torch.Tensor] = {}
    lin("x_embedder", D, cfg.in_channels)
    lin("context_embedder", D, cfg.joint_attention_dim)
    lin("time_embed.timestep_embedder.linear_1", D, 256)
    lin("time_embed.timestep_embedder.linear_2", D, D)
    for i in range(cfg.num_layers):
        p = f"transformer_blocks.{i}."
        lin(p + "norm1.linear", 6 * D, D, 0.02)
        lin(p + "norm1_context.linear", 6 * D, D, 0.02)
        for n in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0", "to_add_out"):
            lin(p + "attn." + n, D, D)
        for n in ("norm_q", "norm_k", "norm_added_q", "norm_added_k"):
            nrm(p + "attn." + n, hd)
        for f in ("ff", "ff_context"):
            lin(p + f + ".net.0.proj", Fd, D)
            lin(p + f + ".net.2", D, Fd)
    for i in range(cfg.num_single_layers):
        p = f"single_transformer_blocks.{i}."
        lin(p + "norm.linear", 3 * D, D, 0.02)
        lin(p + "proj_mlp", Fd, D)
        for n in ("to_q", "to_k", "to_v"):
            lin(p + "attn." + n, D, D)
        nrm(p + "attn.norm_q", hd)
        nrm(p + "attn.norm_k", hd)
        lin(p + "proj_out", D, D + Fd)
    lin("norm_out.linear", 2 * D, D, 0.02)
    lin("proj_out", cfg.in_channels, D)
    return w


# ---------------------------------------------------------------- fp32 oracle
def _gelu(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def longcat_transformer_reference(cfg: LongCatConfig, w: Dict[str, torch.Tensor], packed: torch.Tensor,
                                  ctx: torch.Tensor, t: float, grid: Tuple[int, int]) -> torch.Tensor:
    """fp32 transformer: packed [Li, C*4], ctx [Lt, J] -> [Li, C*4]."""
    f = {k: v.float() for k, v in w.items()}
    dev = packed.device
    D, nh, hd, eps = cfg.dim, cfg.num_heads, cfg.head_dim, cfg.eps
    Lt, Li = ctx.shape[0], packed.shape[0]
    lin = lambda v, n: v @ f[n + ".weight"].t() + f[n + ".bias"]  # noqa: E731
    ln = lambda v: F.layer_norm(v, (D,), eps=eps)  # noqa: E731
    x = lin(packed.float(), "x_embedder")
    enc = lin(ctx.float(), "context_embedder")
    emb = lin(F.silu(lin(timestep_embedding(t).float().to(dev), "time_embed.timestep_embedder.linear_1")),
              "time_embed.timestep_embedder.linear_2")
    se = F.silu(emb)
    tab = rope_table(cfg).to(dev)
    pos = token_positions(Lt, *grid).to(dev).long()
    a0, a1, _ = (a // 2 for a in cfg.axes_dims_rope)
    pidx = torch.arange(hd // 2, device=dev)
    axis = torch.where(pidx < a0, 0, torch.where(pidx < a0 + a1, 1, 2))
    cs = tab[pos[:, axis], pidx[None, :]]  # [T, hd/2, 2]

    def rope(v):  # [T, nh, hd] interleaved pairs
        v2 = v.view(v.shape[0], nh, hd // 2, 2)
        c, s = cs[:, None, :, 0], cs[:, None, :, 1]
        return torch.stack([v2[..., 0] * c - v2[..., 1] * s, v2[..., 0] * s + v2[..., 1] * c], -1).view(v.shape)

    def rms(v, wt):
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * wt

    def heads(v, n):
        return v.view(v.shape[0], nh, hd) if n is None else rms(v.view(v.shape[0], nh, hd), f[n + ".weight"])

    def attend(q, k, v):
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd)
        return torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(q.shape[0], D)

    for i in range(cfg.num_layers):
        p = f"transformer_blocks.{i}."
        mi = lin(se, p + "norm1.linear")[0].view(6, D)
        mt = lin(se, p + "norm1_context.linear")[0].view(6, D)
        yi = ln(x) * (1 + mi[1]) + mi[0]
        yt = ln(enc) * (1 + mt[1]) + mt[0]
        q = torch.cat([heads(lin(yt, p + "attn.add_q_proj"), p + "attn.norm_added_q"),
                       heads(lin(yi, p + "attn.to_q"), p + "attn.norm_q")])
        k = torch.cat([heads(lin(yt, p + "attn.add_k_proj"), p + "attn.norm_added_k"),
                       heads(lin(yi, p + "attn.to_k"), p + "attn.norm_k")])
        v = torch.cat([heads(lin(yt, p + "attn.add_v_proj"), None), heads(lin(yi, p + "attn.to_v"), None)])
        a = attend(rope(q), rope(k), v)
        x = x + lin(a[Lt:], p + "attn.to_out.0") * mi[2]
        enc = enc + lin(a[:Lt], p + "attn.to_add_out") * mt[2]
        x = x + lin(_gelu(lin(ln(x) * (1 + mi[4]) + mi[3], p + "ff.net.0.proj")), p + "ff.net.2") * mi[5]
        enc = enc + lin(_gelu(lin(ln(enc) * (1 + mt[4]) + mt[3], p + "ff_context.net.0.proj")),
                        p + "ff_context.net.2") * mt[5]
    c = torch.cat([enc, x])
    for i in range(cfg.num_single_layers):
        p = f"single_transformer_blocks.{i}."
        m = lin(se, p + "norm.linear")[0].view(3, D)
        y = ln(c) * (1 + m[1]) + m[0]
        mlp = _gelu(lin(y, p + "proj_mlp"))
        a = attend(rope(heads(lin(y, p + "attn.to_q"), p + "attn.norm_q")),
                   rope(heads(lin(y, p + "attn.to_k"), p + "attn.norm_k")), heads(lin(y, p + "attn.to_v"), None))
        c = c + lin(torch.cat([a, mlp], 1), p + "proj_out") * m[2]
    mo = lin(se, "norm_out.linear")[0].view(2, D)
    y = ln(c[Lt:]) * (1 + mo[0]) + mo[1]
    return lin(y, "proj_out")


# ---------------------------------------------------------------- B200 transformer
class LongCatTransformer:
    def __init__(self, cfg: LongCatConfig, device=None):
        if cfg.head_dim != 128 or sum(cfg.axes_dims_rope) != cfg.head_dim:
            raise ValueError("LongCat needs head_dim 128 with RoPE axes summing to it")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.cfg, self.device = cfg, dev

    def load(self, full: Dict[str, torch.Tensor]) -> None:
        cfg, dev, D = self.cfg, self.device, self.cfg.dim
        bf = lambda n: full[n].to(dev, torch.bfloat16).contiguous()  # noqa: E731
        f32 = lambda n: full[n].to(dev, torch.float32).contiguous()  # noqa: E731
        cat = lambda ns: torch.cat([bf(n) for n in ns], 0).contiguous()  # noqa: E731
        self.w = {n: bf(n + s) for n in ("x_embedder", "context_embedder", "time_embed.timestep_embedder.linear_1",
                                         "time_embed.timestep_embedder.linear_2", "proj_out")
                  for s in (".weight",)}
        self.b = {n: bf(n + ".bias") for n in ("x_embedder", "context_embedder", "time_embed.timestep_embedder.linear_1",
                                               "time_embed.timestep_embedder.linear_2", "proj_out")}
        # every AdaLN linear of a step in one GEMM: [joint img 6D | joint txt 6D]* [single 3D]* [out 2D]
        names, self.mod_off = [], []
        off = 0
        for i in range(cfg.num_layers):
            p = f"transformer_blocks.{i}."
            names += [p + "norm1.linear", p + "norm1_context.linear"]
            self.mod_off.append((off, off + 6 * D))
            off += 12 * D
        self.single_off = []
        for i in range(cfg.num_single_layers):
            names.append(f"single_transformer_blocks.{i}.norm.linear")
            self.single_off.append(off)
            off += 3 * D
        names.append("norm_out.linear")
        self.out_off = off
        self.mod_w = cat([n + ".weight" for n in names])
        self.mod_b = cat([n + ".bias" for n in names])
        self.joint, self.single = [], []
        for i in range(cfg.num_layers):
            p = f"transformer_blocks.{i}.attn."
            q = f"transformer_blocks.{i}."
            self.joint.append({
                "qkv_i": cat([p + n + ".weight" for n in ("to_q", "to_k", "to_v")]),
                "qkv_i_b": cat([p + n + ".bias" for n in ("to_q", "to_k", "to_v")]),
                "qkv_t": cat([p + n + ".weight" for n in ("add_q_proj", "add_k_proj", "add_v_proj")]),
                "qkv_t_b": cat([p + n + ".bias" for n in ("add_q_proj", "add_k_proj", "add_v_proj")]),
                "out_i": bf(p + "to_out.0.weight"), "out_i_b": bf(p + "to_out.0.bias"),
                "out_t": bf(p + "to_add_out.weight"), "out_t_b": bf(p + "to_add_out.bias"),
                "nq": f32(p + "norm_q.weight"), "nk": f32(p + "norm_k.weight"),
                "naq": f32(p + "norm_added_q.weight"), "nak": f32(p + "norm_added_k.weight"),
                "ff0_i": bf(q + "ff.net.0.proj.weight"), "ff0_i_b": bf(q + "ff.net.0.proj.bias"),
                "ff2_i": bf(q + "ff.net.2.weight"), "ff2_i_b": bf(q + "ff.net.2.bias"),
                "ff0_t": bf(q + "ff_context.net.0.proj.weight"), "ff0_t_b": bf(q + "ff_context.net.0.proj.bias"),
                "ff2_t": bf(q + "ff_context.net.2.weight"), "ff2_t_b": bf(q + "ff_context.net.2.bias"),
            })
        for i in range(cfg.num_single_layers):
            p = f"single_transformer_blocks.{i}."
            po = bf(p + "proj_out.weight")
            self.single.append({
                "qkv": cat([p + "attn." + n + ".weight" for n in ("to_q", "to_k", "to_v")]),
                "qkv_b": cat([p + "attn." + n + ".bias" for n in ("to_q", "to_k", "to_v")]),
                "nq": f32(p + "attn.norm_q.weight"), "nk": f32(p + "attn.norm_k.weight"),
                "mlp": bf(p + "proj_mlp.weight"), "mlp_b": bf(p + "proj_mlp.bias"),
                "po_a": po[:, :D].contiguous(), "po_m": po[:, D:].contiguous(), "po_b": bf(p + "proj_out.bias"),
            })
        self.zeros6 = torch.zeros(6, D, dtype=torch.float32, device=dev)
        self.rope = rope_table(cfg).to(dev)

    def random_init(self, seed: int = 0) -> None:
        self.load(longcat_random_weights(self.cfg, seed, self.device))

    def forward(self, packed: torch.Tensor, ctx: torch.Tensor, t: float, grid: Tuple[int, int]) -> torch.Tensor:
        """packed [Li, C*4], ctx [Lt, J] (bf16 or f32) -> bf16 [Li, C*4]."""
        cfg, dev, C = self.cfg, self.device, _C()
        D, nh, hd, eps = cfg.dim, cfg.num_heads, cfg.head_dim, cfg.eps
        Lt, Li = ctx.shape[0], packed.shape[0]
        T = Lt + Li
        Z = self.zeros6
        c = torch.empty(T, D, dtype=torch.float32, device=dev)  # residual stream [text; image]
        c[:Lt] = ops.gemm(ctx.to(dev, torch.bfloat16).contiguous(), self.w["context_embedder"],
                          bias=self.b["context_embedder"]).float()
        c[Lt:] = ops.gemm(packed.to(dev, torch.bfloat16).contiguous(), self.w["x_embedder"],
                          bias=self.b["x_embedder"]).float()
        te = timestep_embedding(t).to(torch.bfloat16).to(dev)
        h = ops.gemm(te, self.w["time_embed.timestep_embedder.linear_1"], bias=self.b["time_embed.timestep_embedder.linear_1"])
        C.silu_bf16(h, h)
        emb = ops.gemm(h, self.w["time_embed.timestep_embedder.linear_2"], bias=self.b["time_embed.timestep_embedder.linear_2"])
        C.silu_bf16(emb, emb)
        mods = ops.gemm(emb, self.mod_w, bias=self.mod_b, epi=ops.EPI_F32)  # [1, all AdaLN rows]
        M = lambda o, n: mods[:, o:o + n * D]  # noqa: E731
        pos3 = token_positions(Lt, *grid).to(dev)
        a0, a1 = cfg.axes_dims_rope[0] // 2, cfg.axes_dims_rope[1] // 2
        bpb = (T + 15) // 16
        bt = torch.arange(bpb, dtype=torch.int32, device=dev)[None, :].contiguous()
        lens = torch.tensor([T], dtype=torch.int32, device=dev)
        cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
        ts, tst = [x.to(dev) for x in ops.prefill_tiles([0, T], [T])]
        y = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        ct, ci = c[:Lt], c[Lt:]
        yt, yi = y[:Lt], y[Lt:]

        def norm(x, yv, delta, gmod, gi, nmod, ish, isc):
            """x += gate * delta (gate = gmod row gi); yv = LN(x) * (1 + scale) + shift."""
            C.wan_residual_norm(x, delta, Z if delta is not None and gi >= 0 else None,
                                gmod if delta is not None and gi >= 0 else None, gi if delta is not None else -1, 0, D,
                                2, None, None, Z, nmod, ish, isc, 0, D, x.shape[0], eps, yv)

        def attention(q, kv):
            out = torch.empty_like(q)
            ops.paged_prefill_attention(q, kv, 0, bt, lens, cu, ts, tst, out, scale=1.0 / math.sqrt(hd), causal=False)
            return out.view(T, D)

        if cfg.num_layers:
            o_i, o_t = self.mod_off[0]
            norm(ci, yi, None, None, -1, M(o_i, 6), 0, 1)
            norm(ct, yt, None, None, -1, M(o_t, 6), 0, 1)
        else:
            norm(c, y, None, None, -1, M(self.single_off[0], 3), 0, 1)
        nlaunch = 8
        for i, blk in enumerate(self.joint):
            o_i, o_t = self.mod_off[i]
            mi, mt = M(o_i, 6), M(o_t, 6)
            qkv_i = ops.gemm(yi, blk["qkv_i"], bias=blk["qkv_i_b"])
            qkv_t = ops.gemm(yt, blk["qkv_t"], bias=blk["qkv_t_b"])
            q = torch.empty(T, nh, hd, dtype=torch.bfloat16, device=dev)
            kv = torch.zeros(1, bpb, 2, nh, 16, hd, dtype=torch.bfloat16, device=dev)
            C.wan_qkv_norm_rope(qkv_t, 0, D, 2 * D, nh, hd, blk["naq"], blk["nak"], eps, self.rope, a0, a1, 1, 1, 1, Lt,
                                q, kv, bpb, True, pos3, T, 0)
            C.wan_qkv_norm_rope(qkv_i, 0, D, 2 * D, nh, hd, blk["nq"], blk["nk"], eps, self.rope, a0, a1, 1, 1, 1, Li,
                                q, kv, bpb, True, pos3, T, Lt)
            a = attention(q, kv)
            oi = ops.gemm(a[Lt:], blk["out_i"], bias=blk["out_i_b"])
            ot = ops.gemm(a[:Lt], blk["out_t"], bias=blk["out_t_b"])
            norm(ci, yi, oi, mi, 2, mi, 3, 4)
            norm(ct, yt, ot, mt, 2, mt, 3, 4)
            fi = ops.gemm(ops.gemm(yi, blk["ff0_i"], bias=blk["ff0_i_b"], epi=ops.EPI_GELU_TANH), blk["ff2_i"],
                          bias=blk["ff2_i_b"])
            ft = ops.gemm(ops.gemm(yt, blk["ff0_t"], bias=blk["ff0_t_b"], epi=ops.EPI_GELU_TANH), blk["ff2_t"],
                          bias=blk["ff2_t_b"])
            if i + 1 < cfg.num_layers:
                n_i, n_t = self.mod_off[i + 1]
                norm(ci, yi, fi, mi, 5, M(n_i, 6), 0, 1)
                norm(ct, yt, ft, mt, 5, M(n_t, 6), 0, 1)
            elif cfg.num_single_layers:
                ms = M(self.single_off[0], 3)
                norm(ci, yi, fi, mi, 5, ms, 0, 1)
                norm(ct, yt, ft, mt, 5, ms, 0, 1)
            else:
                mo = M(self.out_off, 2)
                norm(ci, yi, fi, mi, 5, mo, 1, 0)
                norm(ct, yt, ft, mt, 5, mo, 1, 0)
            nlaunch += 10
        for j, blk in enumerate(self.single):
            ms = M(self.single_off[j], 3)
            mlp = ops.gemm(y, blk["mlp"], bias=blk["mlp_b"], epi=ops.EPI_GELU_TANH)
            qkv = ops.gemm(y, blk["qkv"], bias=blk["qkv_b"])
            q = torch.empty(T, nh, hd, dtype=torch.bfloat16, device=dev)
            kv = torch.zeros(1, bpb, 2, nh, 16, hd, dtype=torch.bfloat16, device=dev)
            C.wan_qkv_norm_rope(qkv, 0, D, 2 * D, nh, hd, blk["nq"], blk["nk"], eps, self.rope, a0, a1, 1, 1, 1, T, q,
                                kv, bpb, True, pos3, T, 0)
            a = attention(q, kv)
            o = ops.gemm(mlp, blk["po_m"], bias=blk["po_b"], resid=ops.gemm(a, blk["po_a"]), epi=ops.EPI_RESIDUAL)
            if j + 1 < cfg.num_single_layers:
                norm(c, y, o, ms, 2, M(self.single_off[j + 1], 3), 0, 1)
            else:
                norm(c, y, o, ms, 2, M(self.out_off, 2), 1, 0)  # AdaLayerNormContinuous: scale first, then shift
            nlaunch += 3
        ops._count(nlaunch)
        return ops.gemm(yi, self.w["proj_out"], bias=self.b["proj_out"])


# ---------------------------------------------------------------- KL VAE
@dataclass
class KLVaeConfig:
    block_out_channels: List[int] = field(default_factory=lambda: [128, 256, 512, 512])
    latent_channels: int = 16
    layers_per_block: int = 2
    scaling_factor: float = 0.3611
    shift_factor: float = 0.1159
    groups: int = 32
    eps: float = 1e-6


def klvae_preset(name: str = "flux") -> KLVaeConfig:
    if name == "flux":
        return KLVaeConfig()
    if name == "tiny":  # mid attention at 256 channels (a wide-attention head dim)
        return KLVaeConfig(block_out_channels=[128, 256], layers_per_block=1)
    raise KeyError(f"unknown KL VAE preset {name!r}")


def klvae_random_weights(cfg: KLVaeConfig, seed: int = 0, device="cpu") -> Dict[str, torch.Tensor]:
    g = torch.Generator(device="cpu").manual_seed(seed)
    w: Dict[str, torch.Tensor] = {}

    def conv(n, co, ci, k=3):
        w[n + ".weight"] = (torch.randn(co, ci, k, k, generator=g) / math.sqrt(ci * k * k)).to(device)
        w[n + ".bias"] = (0.02 * torch.randn(co, generator=g)).to(device)

    def gn(n, c):
        w[n + ".weight"] = (1.0 + 0.1 * torch.randn(c, generator=g)).to(device)
        w[n + ".bias"] = (0.05 * torch.randn(c, generator=g)).to(device)

    def res(p, ci, co):
        gn(p + "norm1", ci)
        conv(p + "conv1", co, ci)
        gn(p + "norm2", co)
        conv(p + "conv2", co, co)
        if ci != co:
            conv(p + "conv_shortcut", co, ci, 1)

    def attn(p, c):
        gn(p + "group_norm", c)
        for n in ("to_q", "to_k", "to_v", "to_out.0"):
            w[p + n + ".weight"] = (torch.randn(c, c, generator=g) / math.sqrt(c)).to(device)
            w[p + n + ".bias"] = (0.02 * torch.randn(c, generator=g)).to(device)

    ch = cfg.block_out_channels
    conv("encoder.conv_in", ch[0], 3)
    cin = ch[0]
    for i, co in enumerate(ch):
        for j in range(cfg.layers_per_block):
            res(f"encoder.down_blocks.{i}.resnets.{j}.", cin, co)
            cin = co
        if i + 1 < len(ch):
            conv(f"encoder.down_blocks.{i}.downsamplers.0.conv", co, co)
    for side in ("encoder", "decoder"):
        res(f"{side}.mid_block.resnets.0.", ch[-1], ch[-1])
        attn(f"{side}.mid_block.attentions.0.", ch[-1])
        res(f"{side}.mid_block.resnets.1.", ch[-1], ch[-1])
    gn("encoder.conv_norm_out", ch[-1])
    conv("encoder.conv_out", 2 * cfg.latent_channels, ch[-1])
    conv("decoder.conv_in", ch[-1], cfg.latent_channels)
    rev = list(reversed(ch))
    cin = rev[0]
    for i, co in enumerate(rev):
        for j in range(cfg.layers_per_block + 1):
            res(f"decoder.up_blocks.{i}.resnets.{j}.", cin, co)
            cin = co
        if i + 1 < len(rev):
            conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", co, co)
    gn("decoder.conv_norm_out", ch[0])
    conv("decoder.conv_out", 3, ch[0])
    return w


def klvae_reference(cfg: KLVaeConfig, w, image: Optional[torch.Tensor] = None, latent: Optional[torch.Tensor] = None):
    """fp32 oracle.  image [3, H, W] in [-1, 1] -> scaled latent [C, H/8', W/8'];
    latent -> image [3, H, W]."""
    f = {k: v.float() for k, v in w.items()}
    gn = lambda v, p: F.group_norm(v, min(cfg.groups, v.shape[1]), f[p + ".weight"], f[p + ".bias"], cfg.eps)  # noqa
    conv = lambda v, p, pad=1: F.conv2d(v, f[p + ".weight"], f[p + ".bias"], padding=pad)  # noqa: E731

    def res(v, p):
        h = conv(F.silu(gn(v, p + "norm1")), p + "conv1")
        h = conv(F.silu(gn(h, p + "norm2")), p + "conv2")
        return h + (conv(v, p + "conv_shortcut", 0) if p + "conv_shortcut.weight" in f else v)

    def attn(v, p):
        N, Cc, H, W = v.shape
        h = gn(v, p + "group_norm").permute(0, 2, 3, 1).reshape(N, H * W, Cc)
        lin = lambda t, n: t @ f[p + n + ".weight"].t() + f[p + n + ".bias"]  # noqa: E731
        a = torch.softmax(lin(h, "to_q") @ lin(h, "to_k").transpose(1, 2) / math.sqrt(Cc), -1) @ lin(h, "to_v")
        return v + lin(a, "to_out.0").view(N, H, W, Cc).permute(0, 3, 1, 2)

    def mid(v, s):
        v = res(v, f"{s}.mid_block.resnets.0.")
        v = attn(v, f"{s}.mid_block.attentions.0.")
        return res(v, f"{s}.mid_block.resnets.1.")

    ch = cfg.block_out_channels
    if image is not None:
        x = conv(image.float()[None], "encoder.conv_in")
        for i in range(len(ch)):
            for j in range(cfg.layers_per_block):
                x = res(x, f"encoder.down_blocks.{i}.resnets.{j}.")
            if i + 1 < len(ch):
                p = f"encoder.down_blocks.{i}.downsamplers.0.conv"
                x = F.conv2d(F.pad(x, (0, 1, 0, 1)), f[p + ".weight"], f[p + ".bias"], stride=2)
        x = mid(x, "encoder")
        x = conv(F.silu(gn(x, "encoder.conv_norm_out")), "encoder.conv_out")
        mean = x[0, :cfg.latent_channels]
        return (mean - cfg.shift_factor) * cfg.scaling_factor
    z = latent.float()[None] / cfg.scaling_factor + cfg.shift_factor
    x = conv(z, "decoder.conv_in")
    x = mid(x, "decoder")
    for i in range(len(ch)):
        for j in range(cfg.layers_per_block + 1):
            x = res(x, f"decoder.up_blocks.{i}.resnets.{j}.")
        if i + 1 < len(ch):
            x = conv(F.interpolate(x, scale_factor=2, mode="nearest"), f"decoder.up_blocks.{i}.upsamplers.0.conv")
    return conv(F.silu(gn(x, "decoder.conv_norm_out")), "decoder.conv_out")[0]


class KLVae(WanVAE):
    """AutoEncoderKL on the VAE kernels (NHWC, im2col + tcgen05 GEMM)."""

    prefixes = ("encoder.", "decoder.")
    attn_prefixes = ("encoder.mid_block.attentions.0.", "decoder.mid_block.attentions.0.")

    def __init__(self, cfg: KLVaeConfig, device=None):
        super().__init__(VaeConfig(groups=cfg.groups, eps=cfg.eps), device)
        self.kl = cfg

    def random_init(self, seed: int = 0) -> None:
        self.load(klvae_random_weights(self.kl, seed, self.device))

    def _mid(self, x, side):
        x = self._res(x, f"{side}.mid_block.resnets.0.")
        x = self._attn(x, f"{side}.mid_block.attentions.0.")
        return self._res(x, f"{side}.mid_block.resnets.1.")

    def encode(self, image: torch.Tensor) -> torch.Tensor:
        """image f32 [3, H, W] in [-1, 1] -> scaled latent f32 [C, H/s, W/s]."""
        cfg = self.kl
        ch = cfg.block_out_channels
        x3 = image.to(self.device, torch.float32).permute(1, 2, 0)
        x = torch.zeros(1, x3.shape[0], x3.shape[1], 8, dtype=torch.bfloat16, device=self.device)
        x[0, :, :, :3] = x3.to(torch.bfloat16)  # 3 channels zero-padded to 8 for the 16-byte gathers
        x = self._conv3(x, "encoder.conv_in")
        for i in range(len(ch)):
            for j in range(cfg.layers_per_block):
                x = self._res(x, f"encoder.down_blocks.{i}.resnets.{j}.")
            if i + 1 < len(ch):
                x = self._conv3(x, f"encoder.down_blocks.{i}.downsamplers.0.conv", stride=2, pads=(0, 1, 0, 1))
        x = self._mid(x, "encoder")
        x = self._conv3(x, "encoder.conv_out", norm=(self._stats(x), "encoder.conv_norm_out."))
        mean = x[0, :, :, :cfg.latent_channels].float().permute(2, 0, 1)
        return ((mean - cfg.shift_factor) * cfg.scaling_factor).contiguous()

    def decode_image(self, latent: torch.Tensor, rgb: bool = True) -> torch.Tensor:
        """scaled latent [C, h, w] -> u8 [H, W, 3] (rgb=False: bf16 [H, W, 3])."""
        cfg = self.kl
        ch = cfg.block_out_channels
        z = (latent.to(self.device).float() / cfg.scaling_factor + cfg.shift_factor)
        x = z.permute(1, 2, 0)[None].to(torch.bfloat16).contiguous()
        x = self._conv3(x, "decoder.conv_in")
        x = self._mid(x, "decoder")
        for i in range(len(ch)):
            for j in range(cfg.layers_per_block + 1):
                x = self._res(x, f"decoder.up_blocks.{i}.resnets.{j}.")
            if i + 1 < len(ch):
                x = self._conv3(x, f"decoder.up_blocks.{i}.upsamplers.0.conv", up=2)
        out = self._conv3(x, "decoder.conv_out", norm=(self._stats(x), "decoder.conv_norm_out."))
        return self._to_rgb(out, rgb)[0]

    def load(self, full: Dict[str, torch.Tensor]) -> None:
        full = dict(full)
        w = full["encoder.conv_in.weight"]
        if w.shape[1] == 3:  # input channels padded to 8 like the gathered image
            full["encoder.conv_in.weight"] = torch.cat([w, torch.zeros(w.shape[0], 5, *w.shape[2:], device=w.device,
                                                                       dtype=w.dtype)], 1)
        super().load(full)


# ---------------------------------------------------------------- draft edit
class LongCatEditPipeline:
    """One-pass draft image edit (run_draft_image_edit): image + prompt
    embeddings -> edited image."""

    def __init__(self, transformer: LongCatTransformer, vae: KLVae, strength: float = 0.12,
                 max_delta_rms_ratio: float = 1.0):
        self.tr, self.vae = transformer, vae
        self.strength, self.ratio = strength, max_delta_rms_ratio

    @staticmethod
    def from_presets(transformer: str = "tiny-longcat", vae: str = "tiny", seed: int = 0, device=None):
        t = LongCatTransformer(longcat_preset(transformer), device)
        t.random_init(seed)
        v = KLVae(klvae_preset(vae), device)
        v.random_init(seed + 1)
        return LongCatEditPipeline(t, v)

    def edit(self, image_u8: torch.Tensor, prompt_embeds: torch.Tensor, rgb: bool = True) -> torch.Tensor:
        """image_u8 [H, W, 3] (H, W multiples of 16) -> edited u8 [H, W, 3]."""
        img = image_u8.to(self.vae.device).float().permute(2, 0, 1) / 127.5 - 1.0
        lat = self.vae.encode(img)  # [C, h, w]
        Cl, h, w = lat.shape
        packed = pack_latents(lat)
        out = self.tr.forward(packed, prompt_embeds, 0.5, (h // 2, w // 2)).float()
        delta = unpack_latents(out, Cl, h, w)
        lr, dr = lat.pow(2).mean().sqrt(), delta.pow(2).mean().sqrt()
        scale = torch.where(dr > 1e-6, torch.clamp(lr / dr, max=self.ratio), torch.zeros_like(dr))
        edited = lat + self.strength * delta * scale
        return self.vae.decode_image(edited, rgb)


def _C():
    from .._ext import cuda

    return cuda()
