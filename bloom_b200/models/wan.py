"""Wan 2.1 text-to-video diffusion transformer (DiT) on the B200 kernels.

Architecture (executor/wan/dit.rs): a 1x2x2 patch embedding of the
16-channel video latent, a sinusoidal timestep embedding -> MLP -> six AdaLN
rows per block, a text embedding MLP over the umT5 features, then N blocks of

    x += gate_sa * SelfAttn(LN(x) * (1 + scale_sa) + shift_sa)   (q/k RMSNorm, 3-D RoPE)
    x += CrossAttn(LN_affine(x), text)                             (q/k RMSNorm)
    x += gate_ff * FFN(LN(x) * (1 + scale_ff) + shift_ff)          (GELU-tanh)

and a modulated head whose output is un-patchified into the velocity field.

On the GPU (`WanDiT`):
  * every projection is a tcgen05 GEMM with the bias (and GELU) fused in the
    epilogue;
  * self attention runs the paged tcgen05 prefill kernel with causal masking
    off over a scratch page set written by `wan_qkv_norm_rope` (q/k RMSNorm
    over the model dim and the 3-D RoPE fused into the page write);
  * the cross-attention K / V of the text depend on neither the latent nor
    the timestep, so they are computed once per generation and kept as pages
    for every denoising step;
  * the residual stream stays fp32 and one `wan_residual_norm` kernel per
    sub-layer applies the gate, adds the residual and produces the next
    GEMM's normalised / modulated bf16 input;
  * classifier-free guidance runs the conditional and unconditional passes
    as one batch of two, and the un-patchify, guidance combine and Euler
    flow-matching update are one kernel.

Two deliberate departures from the reference's code, both to the published
Wan 2.1 definition: the RMSNorm divides by sqrt(mean(x^2) + eps) (the
reference's WanRMSNorm omits the square root, dit.rs:334-346) and the Euler
step is x + (sigma_next - sigma) * v (scheduler.rs:91 adds dt as a scalar).
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from .. import ops


@dataclass
class WanConfig:
    patch_size: Tuple[int, int, int] = (1, 2, 2)
    text_len: int = 512
    in_dim: int = 16
    dim: int = 1536
    ffn_dim: int = 8960
    freq_dim: int = 256
    text_dim: int = 4096
    out_dim: int = 16
    num_heads: int = 12
    num_layers: int = 30
    qk_norm: bool = True
    cross_attn_norm: bool = True
    eps: float = 1e-6
    name: str = ""

    @property
    def head_dim(self) -> int:
        return self.dim // self.num_heads


WAN_PRESETS = {
    # Wan2.1-T2V-1.3B (executor/wan/dit.rs:131-150)
    "wan2.1-t2v-1.3b": WanConfig(name="wan2.1-t2v-1.3b"),
    # test size: head_dim 128 like the real model
    "tiny-wan": WanConfig(text_len=24, dim=256, ffn_dim=512, freq_dim=64, text_dim=256, num_heads=2, num_layers=2,
                          name="tiny-wan"),
}


def wan_preset(name: str) -> WanConfig:
    if name not in WAN_PRESETS:
        raise KeyError(f"unknown Wan preset {name!r}; known: {sorted(WAN_PRESETS)}")
    return dataclasses.replace(WAN_PRESETS[name])


def rope_axes(head_dim: int) -> Tuple[int, int, int]:
    """Head dims rotated with the frame / row / column index (dit.rs:212-214)."""
    c_h = head_dim // 3
    return head_dim - 2 * c_h, c_h, c_h


def rope_table(head_dim: int, positions: int = 1024, theta: float = 10000.0) -> torch.Tensor:
    """[positions, head_dim / 2, 2] f32 (cos, sin) of pair p at position n:
    n * theta^(-2 i / axis_dim), i the pair's index within its axis."""
    ct, ch, cw = rope_axes(head_dim)
    inv = []
    for c in (ct, ch, cw):
        inv.append(1.0 / theta ** (torch.arange(c // 2, dtype=torch.float64) * 2 / c))
    inv = torch.cat(inv)
    ang = torch.arange(positions, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.stack([ang.cos(), ang.sin()], -1).float().contiguous()


def sinusoidal(dim: int, t: torch.Tensor) -> torch.Tensor:
    """[B, dim] = [cos | sin](t * 10000^(-i / (dim/2))) in float64 (dit.rs:153-168)."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    a = t.double().cpu()[:, None] * freqs[None, :]
    return torch.cat([a.cos(), a.sin()], 1)


def sampling_sigmas(num_steps: int, shift: float) -> List[float]:
    """Shifted flow-matching schedule (scheduler.rs:11-23): t from 1 to 0."""
    out = []
    for i in range(num_steps + 1):
        t = 1.0 - i / num_steps
        out.append(t if shift == 1.0 else shift * t / (1.0 + (shift - 1.0) * t))
    return out


def wan_random_weights(cfg: WanConfig, seed: int = 0, std: float = 0.02, device="cpu") -> Dict[str, torch.Tensor]:
    """Checkpoint-named random DiT weights (bf16 matrices, f32 norms / modulation)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    D, F = cfg.dim, cfg.ffn_dim

    def rn(*s, scale=std):
        return (torch.randn(*s, generator=g) * scale).to(torch.bfloat16).to(device)

    def f32(*s, base=0.0, scale=0.1):
        return (base + torch.randn(*s, generator=g) * scale).float().to(device)

    w = {"patch_embedding.weight": rn(D, cfg.in_dim, *cfg.patch_size, scale=0.1), "patch_embedding.bias": rn(D),
         "text_embedding.0.weight": rn(D, cfg.text_dim, scale=0.05), "text_embedding.0.bias": rn(D),
         "text_embedding.2.weight": rn(D, D, scale=0.05), "text_embedding.2.bias": rn(D),
         "time_embedding.0.weight": rn(D, cfg.freq_dim, scale=0.05), "time_embedding.0.bias": rn(D),
         "time_embedding.2.weight": rn(D, D, scale=0.05), "time_embedding.2.bias": rn(D),
         "time_projection.1.weight": rn(6 * D, D, scale=0.02), "time_projection.1.bias": rn(6 * D),
         "head.head.weight": rn(cfg.out_dim * 4, D, scale=0.05), "head.head.bias": rn(cfg.out_dim * 4),
         "head.modulation": f32(1, 2, D, scale=0.05)}
    for i in range(cfg.num_layers):
        p = f"blocks.{i}."
        for att in ("self_attn", "cross_attn"):
            for n in "qkvo":
                w[f"{p}{att}.{n}.weight"] = rn(D, D, scale=0.04)
                w[f"{p}{att}.{n}.bias"] = rn(D)
            w[f"{p}{att}.norm_q.weight"] = f32(D, base=1.0)
            w[f"{p}{att}.norm_k.weight"] = f32(D, base=1.0)
        w[p + "norm3.weight"] = f32(D, base=1.0)
        w[p + "norm3.bias"] = f32(D, scale=0.05)
        w[p + "ffn.0.weight"] = rn(F, D, scale=0.04)
        w[p + "ffn.0.bias"] = rn(F)
        w[p + "ffn.2.weight"] = rn(D, F, scale=0.04)
        w[p + "ffn.2.bias"] = rn(D)
        w[p + "modulation"] = f32(1, 6, D, scale=0.05)
    return w


# ---------------------------------------------------------------- fp32 oracle
def _gelu(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def wan_dit_reference(cfg: WanConfig, w: Dict[str, torch.Tensor], latent: torch.Tensor, t: torch.Tensor,
                      context: torch.Tensor) -> torch.Tensor:
    """fp32 DiT forward: latent [B, C, F, H, W], t [B], context [B, L, text_dim]
    -> velocity [B, C, F, H, W] (dit.rs WanModel::forward :938-996)."""
    f = {k: v.float() for k, v in w.items()}
    B, C, Fr, H, W = latent.shape
    D, nh, hd, eps = cfg.dim, cfg.num_heads, cfg.head_dim, cfg.eps
    H2, W2 = H // 2, W // 2
    S = Fr * H2 * W2
    dev = latent.device
    tok = latent.float().view(B, C, Fr, H2, 2, W2, 2).permute(0, 2, 3, 5, 1, 4, 6).reshape(B, S, C * 4)
    x = tok @ f["patch_embedding.weight"].reshape(D, -1).t() + f["patch_embedding.bias"]
    lin = lambda v, n: v @ f[n + ".weight"].t() + f[n + ".bias"]  # noqa: E731
    e = lin(torch.nn.functional.silu(lin(sinusoidal(cfg.freq_dim, t).float().to(dev), "time_embedding.0")),
            "time_embedding.2")
    e0 = lin(torch.nn.functional.silu(e), "time_projection.1").view(B, 6, D)
    ctx = lin(_gelu(lin(context.float(), "text_embedding.0")), "text_embedding.2")

    def ln(v, wt=None, b=None):
        y = torch.nn.functional.layer_norm(v, (D,), eps=eps)
        return y * wt + b if wt is not None else y

    def rms(v, wt):
        return v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps) * wt

    tab = rope_table(hd).to(dev)
    ct, ch, _ = rope_axes(hd)
    n = torch.arange(S, device=dev)
    pf, ph, pw = n // (H2 * W2), (n // W2) % H2, n % W2
    pidx = torch.arange(hd // 2, device=dev)
    pos = torch.where(pidx < ct // 2, pf[:, None], torch.where(pidx < (ct + ch) // 2, ph[:, None], pw[:, None]))
    cs = tab[pos, pidx[None, :]]  # [S, hd/2, 2]

    def rope(v):  # [B, S, nh, hd], interleaved pairs
        v2 = v.view(B, S, nh, hd // 2, 2)
        c, s = cs[None, :, None, :, 0], cs[None, :, None, :, 1]
        return torch.stack([v2[..., 0] * c - v2[..., 1] * s, v2[..., 0] * s + v2[..., 1] * c], -1).view(B, S, nh, hd)

    def attend(q, k, v):  # [B, Sq, nh, hd] x [B, Sk, nh, hd]
        a = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(hd)
        return torch.einsum("bhqk,bkhd->bqhd", a.softmax(-1), v).reshape(q.shape[0], q.shape[1], D)

    for i in range(cfg.num_layers):
        p = f"blocks.{i}."
        em = f[p + "modulation"] + e0  # [B, 6, D]
        y = ln(x) * (1 + em[:, 1:2]) + em[:, 0:1]
        q = rms(lin(y, p + "self_attn.q"), f[p + "self_attn.norm_q.weight"]).view(B, S, nh, hd)
        k = rms(lin(y, p + "self_attn.k"), f[p + "self_attn.norm_k.weight"]).view(B, S, nh, hd)
        v = lin(y, p + "self_attn.v").view(B, S, nh, hd)
        x = x + lin(attend(rope(q), rope(k), v), p + "self_attn.o") * em[:, 2:3]
        y = ln(x, f[p + "norm3.weight"], f[p + "norm3.bias"]) if cfg.cross_attn_norm else x
        L = ctx.shape[1]
        q = rms(lin(y, p + "cross_attn.q"), f[p + "cross_attn.norm_q.weight"]).view(B, S, nh, hd)
        k = rms(lin(ctx, p + "cross_attn.k"), f[p + "cross_attn.norm_k.weight"]).view(B, L, nh, hd)
        v = lin(ctx, p + "cross_attn.v").view(B, L, nh, hd)
        x = x + lin(attend(q, k, v), p + "cross_attn.o")
        y = ln(x) * (1 + em[:, 4:5]) + em[:, 3:4]
        x = x + lin(_gelu(lin(y, p + "ffn.0")), p + "ffn.2") * em[:, 5:6]
    hm = f["head.modulation"] + e[:, None, :]
    y = ln(x) * (1 + hm[:, 1:2]) + hm[:, 0:1]
    o = lin(y, "head.head").view(B, Fr, H2, W2, C, 2, 2)
    return o.permute(0, 4, 1, 2, 5, 3, 6).reshape(B, C, Fr, H, W)


# ---------------------------------------------------------------- B200 DiT
class WanDiT:
    """The DiT on one GPU; `denoise` runs a whole flow-matching generation."""

    def __init__(self, cfg: WanConfig, device=None):
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if cfg.patch_size != (1, 2, 2):
            raise ValueError("only the 1x2x2 patch embedding is supported")
        if cfg.head_dim != 128:
            raise ValueError("the paged attention kernels need head_dim 128")
        self.cfg = cfg
        self.device = dev
        self.w: Dict[str, torch.Tensor] = {}
        self.blocks: List[Dict[str, torch.Tensor]] = []
        self._meta: Dict[tuple, tuple] = {}

    def load(self, full: Dict[str, torch.Tensor]) -> None:
        cfg, dev = self.cfg, self.device
        bf = lambda n: full[n].to(dev, torch.bfloat16).contiguous()  # noqa: E731
        f32 = lambda n: full[n].to(dev, torch.float32).contiguous()  # noqa: E731
        D = cfg.dim
        self.w = {
            "patch_w": bf("patch_embedding.weight").reshape(D, -1).contiguous(),
            "patch_b": bf("patch_embedding.bias"),
            "txt0_w": bf("text_embedding.0.weight"), "txt0_b": bf("text_embedding.0.bias"),
            "txt2_w": bf("text_embedding.2.weight"), "txt2_b": bf("text_embedding.2.bias"),
            "t0_w": bf("time_embedding.0.weight"), "t0_b": bf("time_embedding.0.bias"),
            "t2_w": bf("time_embedding.2.weight"), "t2_b": bf("time_embedding.2.bias"),
            "tp_w": bf("time_projection.1.weight"), "tp_b": bf("time_projection.1.bias"),
            "head_w": bf("head.head.weight"), "head_b": bf("head.head.bias"),
            "head_mod": f32("head.modulation").reshape(2, D).contiguous(),
        }
        self.blocks = []
        for i in range(cfg.num_layers):
            p = f"blocks.{i}."
            cat = lambda names: torch.cat([bf(n) for n in names], 0).contiguous()  # noqa: E731
            self.blocks.append({
                "qkv_w": cat([p + f"self_attn.{n}.weight" for n in "qkv"]),
                "qkv_b": cat([p + f"self_attn.{n}.bias" for n in "qkv"]),
                "o_w": bf(p + "self_attn.o.weight"), "o_b": bf(p + "self_attn.o.bias"),
                "nq": f32(p + "self_attn.norm_q.weight"), "nk": f32(p + "self_attn.norm_k.weight"),
                "cq_w": bf(p + "cross_attn.q.weight"), "cq_b": bf(p + "cross_attn.q.bias"),
                "ckv_w": cat([p + "cross_attn.k.weight", p + "cross_attn.v.weight"]),
                "ckv_b": cat([p + "cross_attn.k.bias", p + "cross_attn.v.bias"]),
                "co_w": bf(p + "cross_attn.o.weight"), "co_b": bf(p + "cross_attn.o.bias"),
                "cnq": f32(p + "cross_attn.norm_q.weight"), "cnk": f32(p + "cross_attn.norm_k.weight"),
                "n3_w": f32(p + "norm3.weight"), "n3_b": f32(p + "norm3.bias"),
                "f0_w": bf(p + "ffn.0.weight"), "f0_b": bf(p + "ffn.0.bias"),
                "f2_w": bf(p + "ffn.2.weight"), "f2_b": bf(p + "ffn.2.bias"),
                "mod": f32(p + "modulation").reshape(6, D).contiguous(),
            })
        self.rope = rope_table(cfg.head_dim).to(dev)

    def random_init(self, seed: int = 0) -> None:
        self.load(wan_random_weights(self.cfg, seed, device=self.device))

    # ---------------------------------------------------------------- pieces
    def _attn_meta(self, Sq, Sk, B, bpb):
        """Block table, lengths and prefill tiles of B samples (cached per shape)."""
        key = (Sq, Sk, B, bpb)
        m = self._meta.get(key)
        if m is None:
            dev = self.device
            bt = (torch.arange(B, dtype=torch.int32, device=dev)[:, None] * bpb
                  + torch.arange(bpb, dtype=torch.int32, device=dev)[None, :]).contiguous()
            cu = [b * Sq for b in range(B + 1)]
            ts, tst = ops.prefill_tiles(cu, [Sk] * B)
            m = (bt, torch.full((B,), Sk, dtype=torch.int32, device=dev),
                 torch.tensor(cu, dtype=torch.int32, device=dev), ts.to(dev), tst.to(dev))
            self._meta[key] = m
        return m

    def _attention(self, q, kv, Sq, Sk, B, bpb):
        """Non-causal attention of B samples: q [B*Sq, nh, hd] over pages
        kv (sample b's keys in pages [b*bpb, b*bpb + ceil(Sk/16)))."""
        bt, lens, cu, ts, tst = self._attn_meta(Sq, Sk, B, bpb)
        out = torch.empty_like(q)
        ops.paged_prefill_attention(q, kv, 0, bt, lens, cu, ts, tst, out, scale=1.0 / math.sqrt(self.cfg.head_dim),
                                    causal=False)
        return out

    def encode_text(self, context: torch.Tensor):
        """context [B, L, text_dim] -> per-block cross-attention K / V pages
        (computed once per generation) and the page geometry."""
        cfg, C = self.cfg, _media()
        B, L, _ = context.shape
        D, nh, hd = cfg.dim, cfg.num_heads, cfg.head_dim
        c = context.to(self.device, torch.bfloat16).reshape(B * L, -1).contiguous()
        h = ops.gemm(c, self.w["txt0_w"], bias=self.w["txt0_b"], epi=ops.EPI_GELU_TANH)
        ctx = ops.gemm(h, self.w["txt2_w"], bias=self.w["txt2_b"])
        bpb = (L + 15) // 16
        pages = []
        for blk in self.blocks:
            kvp = ops.gemm(ctx, blk["ckv_w"], bias=blk["ckv_b"])
            kv = torch.zeros(1, B * bpb, 2, nh, 16, hd, dtype=torch.bfloat16, device=self.device)
            C.wan_qkv_norm_rope(kvp, -1, 0, D, nh, hd, None, blk["cnk"], cfg.eps, None, 0, 0, 1, 1, L, L, None, kv,
                                bpb)
            pages.append(kv)
        ops._count(len(self.blocks) + 2)
        return {"pages": pages, "L": L, "bpb": bpb, "B": B}

    def _time(self, t: float, B: int):
        """e [B, D] f32 and the block modulation source e0 [B, 6, D] f32."""
        st = sinusoidal(self.cfg.freq_dim, torch.full((B,), float(t))).to(torch.bfloat16).to(self.device)
        C = _media()
        h = ops.gemm(st, self.w["t0_w"], bias=self.w["t0_b"])
        C.silu_bf16(h, h)
        e = ops.gemm(h, self.w["t2_w"], bias=self.w["t2_b"], epi=ops.EPI_F32)
        es = e.to(torch.bfloat16)
        C.silu_bf16(es, es)
        e0 = ops.gemm(es, self.w["tp_w"], bias=self.w["tp_b"], epi=ops.EPI_F32)
        ops._count(2)
        return e.contiguous(), e0.contiguous()

    def velocity_tokens(self, latent_b: torch.Tensor, t: float, text) -> torch.Tensor:
        """Head output bf16 [B * S, C * 4] for latent_b f32 [B, C, F, H, W]."""
        cfg, C = self.cfg, _media()
        B, Cin, Fr, H, W = latent_b.shape
        D, nh, hd, eps = cfg.dim, cfg.num_heads, cfg.head_dim, cfg.eps
        H2, W2 = H // 2, W // 2
        S = Fr * H2 * W2
        T = B * S
        dev = self.device
        tok = torch.empty(T, Cin * 4, dtype=torch.bfloat16, device=dev)
        C.wan_patchify(latent_b.contiguous(), tok)
        xb = ops.gemm(tok, self.w["patch_w"], bias=self.w["patch_b"])
        x = xb.float()
        e, e0 = self._time(t, B)
        y = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
        bpb = (S + 15) // 16
        kv = torch.zeros(1, B * bpb, 2, nh, 16, hd, dtype=torch.bfloat16, device=dev)
        ct, ch, _ = rope_axes(hd)
        six = 6 * D
        # block 0's modulated norm1
        C.wan_residual_norm(x, None, None, None, -1, 0, 0, 2, None, None, self.blocks[0]["mod"], e0, 0, 1, six, D, S,
                            eps, y)
        nlaunch = 3
        for i, blk in enumerate(self.blocks):
            qkv = ops.gemm(y, blk["qkv_w"], bias=blk["qkv_b"])
            q = torch.empty(T, nh, hd, dtype=torch.bfloat16, device=dev)
            C.wan_qkv_norm_rope(qkv, 0, D, 2 * D, nh, hd, blk["nq"], blk["nk"], eps, self.rope, ct // 2, ch // 2,
                                Fr, H2, W2, S, q, kv, bpb)
            a = self._attention(q, kv, S, S, B, bpb)
            o = ops.gemm(a.view(T, D), blk["o_w"], bias=blk["o_b"])
            # x += gate_sa * o; y = norm3(x) (affine) or x
            C.wan_residual_norm(x, o, blk["mod"], e0, 2, six, D, 1 if cfg.cross_attn_norm else 0,
                                blk["n3_w"] if cfg.cross_attn_norm else None,
                                blk["n3_b"] if cfg.cross_attn_norm else None, None, None, 0, 0, six, D, S, eps, y)
            cq = ops.gemm(y, blk["cq_w"], bias=blk["cq_b"])
            qc = torch.empty(T, nh, hd, dtype=torch.bfloat16, device=dev)
            C.wan_qkv_norm_rope(cq, 0, -1, -1, nh, hd, blk["cnq"], None, eps, None, 0, 0, Fr, H2, W2, S, qc, None, 0)
            ca = self._attention(qc, text["pages"][i], S, text["L"], B, text["bpb"])
            co = ops.gemm(ca.view(T, D), blk["co_w"], bias=blk["co_b"])
            # x += co; y = LN(x) * (1 + scale_ff) + shift_ff
            C.wan_residual_norm(x, co, None, None, -1, 0, 0, 2, None, None, blk["mod"], e0, 3, 4, six, D, S, eps, y)
            h = ops.gemm(y, blk["f0_w"], bias=blk["f0_b"], epi=ops.EPI_GELU_TANH)
            fo = ops.gemm(h, blk["f2_w"], bias=blk["f2_b"])
            # x += gate_ff * fo; y = next block's modulated norm1, or the head's
            if i + 1 < len(self.blocks):
                C.wan_residual_norm(x, fo, blk["mod"], e0, 5, six, D, 2, None, None, self.blocks[i + 1]["mod"], e0, 0,
                                    1, six, D, S, eps, y)
            else:
                C.wan_residual_norm(x, fo, blk["mod"], e0, 5, six, D, 2, None, None, self.w["head_mod"], e, 0, 1, D, 0,
                                    S, eps, y)
            nlaunch += 6
        ops._count(nlaunch)
        return ops.gemm(y, self.w["head_w"], bias=self.w["head_b"])

    def denoise(self, latent: torch.Tensor, text, num_steps: int = 50, guidance: float = 5.0, shift: float = 5.0,
                progress=None) -> torch.Tensor:
        """Flow-matching Euler sampling in place on latent f32 [C, F, H, W].
        With guidance > 1, `text` holds the conditional (sample 0) and
        unconditional (sample 1) contexts and both run as one batch."""
        sig = sampling_sigmas(num_steps, shift)
        preds = 2 if guidance > 1.0 else 1
        if text["B"] != preds:
            raise ValueError(f"text context batch {text['B']} != {preds} (guidance {guidance})")
        C = _media()
        for s in range(num_steps):
            lb = latent.unsqueeze(0).expand(preds, *latent.shape).contiguous()
            ho = self.velocity_tokens(lb, sig[s] * 1000.0, text)
            C.wan_unpatchify_step(ho, preds, float(guidance), float(sig[s + 1] - sig[s]), latent)
            ops._count(1)
            if progress is not None:
                progress(s + 1, num_steps)
        return latent


def _media():
    from .._ext import cuda

    return cuda()
