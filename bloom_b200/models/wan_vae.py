"""Wan 2.1 VAE decoder (the reference's frame-wise 2-D decoder) on the B200.

Structure (executor/wan/vae.rs VaeDecoder :65-76, build_decoder :218-276):
conv_in 3x3 (16 -> 384), mid block (res, one-head self attention over the
pixels of each frame, res), four up blocks over channel multipliers
[4, 4, 2, 1] x 96 with two residual blocks each and a nearest x2 upsample +
conv3x3 after every block but the first, GroupNorm(32) -> SiLU -> conv_out
3x3 -> RGB bytes.  Residual block: GN -> SiLU -> conv3x3 -> GN -> SiLU ->
conv3x3, plus a 1x1 shortcut when the channel count changes.

Kernels: activations are NHWC bf16 with all frames of a chunk stacked, so
every convolution is one tcgen05 GEMM over (frames x pixels) rows; the
GroupNorm statistics come from `vae_gn_stats` and the normalisation, SiLU
and nearest upsampling are applied while `vae_im2col3x3` gathers the taps.
Bias and shortcut are added in the GEMM epilogue.  The attention is the
wide tensor-core kernel (head_dim 384, causal masking off) over per-frame
page sets.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from .. import ops


@dataclass
class VaeConfig:
    latent_channels: int = 16
    base_channels: int = 96
    channel_mult: List[int] = field(default_factory=lambda: [1, 2, 4, 4])
    num_res_blocks: int = 2
    temporal_stride: int = 4
    spatial_stride: int = 8
    groups: int = 32
    eps: float = 1e-6


def vae_preset(name: str = "wan2.1") -> VaeConfig:
    if name == "wan2.1":
        return VaeConfig()
    if name == "tiny":  # the real channel widths (the attention kernel needs head_dim 384), one res block per level
        return VaeConfig(num_res_blocks=1)
    raise KeyError(f"unknown VAE preset {name!r}")


def _levels(cfg: VaeConfig):
    """[(in_ch, out_ch, upsample)] of the up blocks (vae.rs:248-256)."""
    cur = cfg.base_channels * cfg.channel_mult[-1]
    out = []
    for level, mult in enumerate(reversed(cfg.channel_mult)):
        oc = cfg.base_channels * mult
        out.append((cur, oc, level > 0))
        cur = oc
    return out


def vae_random_weights(cfg: VaeConfig, seed: int = 0, device="cpu") -> Dict[str, torch.Tensor]:
    g = torch.Generator(device="cpu").manual_seed(seed)

    def conv(co, ci, k):
        return (torch.randn(co, ci, k, k, generator=g) / math.sqrt(ci * k * k)).to(device)

    def vec(n, base=0.0, s=0.05):
        return (base + s * torch.randn(n, generator=g)).to(device)

    w = {}
    top = cfg.base_channels * cfg.channel_mult[-1]

    def res(p, ci, co):
        w[p + "norm1.weight"], w[p + "norm1.bias"] = vec(ci, 1.0, 0.1), vec(ci)
        w[p + "conv1.weight"], w[p + "conv1.bias"] = conv(co, ci, 3), vec(co)
        w[p + "norm2.weight"], w[p + "norm2.bias"] = vec(co, 1.0, 0.1), vec(co)
        w[p + "conv2.weight"], w[p + "conv2.bias"] = conv(co, co, 3), vec(co)
        if ci != co:
            w[p + "conv_shortcut.weight"], w[p + "conv_shortcut.bias"] = conv(co, ci, 1), vec(co)

    w["decoder.conv_in.weight"], w["decoder.conv_in.bias"] = conv(top, cfg.latent_channels, 3), vec(top)
    res("decoder.mid_block.resnets.0.", top, top)
    a = "decoder.mid_block.attentions.0."
    w[a + "group_norm.weight"], w[a + "group_norm.bias"] = vec(top, 1.0, 0.1), vec(top)
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        w[a + n + ".weight"] = torch.randn(top, top, generator=g).to(device) / math.sqrt(top)
        w[a + n + ".bias"] = vec(top)
    res("decoder.mid_block.resnets.1.", top, top)
    for level, (ci, co, up) in enumerate(_levels(cfg)):
        c = ci
        for i in range(cfg.num_res_blocks):
            res(f"decoder.up_blocks.{level}.resnets.{i}.", c, co)
            c = co
        if up:
            p = f"decoder.up_blocks.{level}.upsamplers.0.conv."
            w[p + "weight"], w[p + "bias"] = conv(co, co, 3), vec(co)
    w["decoder.norm_out.weight"], w["decoder.norm_out.bias"] = vec(cfg.base_channels, 1.0, 0.1), vec(cfg.base_channels)
    w["decoder.conv_out.weight"], w["decoder.conv_out.bias"] = conv(3, cfg.base_channels, 3), vec(3)
    return w


# ---------------------------------------------------------------- fp32 oracle
def vae_decode_reference(cfg: VaeConfig, w: Dict[str, torch.Tensor], latent: torch.Tensor) -> torch.Tensor:
    """latent [C, F, H, W] -> frames [F, 3, 8H, 8W] in [-1, 1]-ish (fp32)."""
    f = {k: v.float() for k, v in w.items()}
    x = latent.float().permute(1, 0, 2, 3)  # [F, C, H, W]

    def gn(v, p):
        return F.group_norm(v, min(cfg.groups, v.shape[1]), f[p + "weight"], f[p + "bias"], cfg.eps)

    def conv(v, p, pad=1):
        return F.conv2d(v, f[p + "weight"], f[p + "bias"], padding=pad)

    def res(v, p):
        h = conv(F.silu(gn(v, p + "norm1.")), p + "conv1.")
        h = conv(F.silu(gn(h, p + "norm2.")), p + "conv2.")
        sc = conv(v, p + "conv_shortcut.", 0) if p + "conv_shortcut.weight" in f else v
        return h + sc

    x = conv(x, "decoder.conv_in.")
    x = res(x, "decoder.mid_block.resnets.0.")
    a = "decoder.mid_block.attentions.0."
    Fn, C, H, W = x.shape
    h = gn(x, a + "group_norm.").permute(0, 2, 3, 1).reshape(Fn, H * W, C)
    lin = lambda v, n: v @ f[a + n + ".weight"].t() + f[a + n + ".bias"]  # noqa: E731
    att = torch.softmax(lin(h, "to_q") @ lin(h, "to_k").transpose(1, 2) / math.sqrt(C), -1) @ lin(h, "to_v")
    x = x + lin(att, "to_out.0").view(Fn, H, W, C).permute(0, 3, 1, 2)
    x = res(x, "decoder.mid_block.resnets.1.")
    for level, (ci, co, up) in enumerate(_levels(cfg)):
        for i in range(cfg.num_res_blocks):
            x = res(x, f"decoder.up_blocks.{level}.resnets.{i}.")
        if up:
            x = conv(F.interpolate(x, scale_factor=2, mode="nearest"), f"decoder.up_blocks.{level}.upsamplers.0.conv.")
    return conv(F.silu(gn(x, "decoder.norm_out.")), "decoder.conv_out.")


def frames_to_rgb(frames: torch.Tensor) -> torch.Tensor:
    """[F, 3, H, W] in [-1, 1] -> u8 [F, H, W, 3] (vae.rs tensor_to_rgb_frame :573-606)."""
    return ((frames.float() * 0.5 + 0.5) * 255.0).clamp(0, 255).to(torch.uint8).permute(0, 2, 3, 1).contiguous()


# ---------------------------------------------------------------- B200 decoder
class WanVAE:
    """Frame-wise VAE decoder on one GPU: `decode(latent)` -> u8 frames."""

    def __init__(self, cfg: VaeConfig, device=None, max_im2col_bytes: int = 8 << 30):
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.cfg = cfg
        self.device = dev
        self.max_im2col_bytes = max_im2col_bytes
        self.p: Dict[str, torch.Tensor] = {}

    prefixes = ("decoder.",)
    attn_prefixes = ("decoder.mid_block.attentions.0.",)

    def load(self, full: Dict[str, torch.Tensor]) -> None:
        """Conv weights [Co, Ci, kh, kw] become GEMM rows [Co, kh * kw * Ci]
        (tap-major, matching vae_im2col3x3); outputs narrower than 16
        channels are zero-padded to 16 rows (sliced off after the GEMM)."""
        dev = self.device
        p = {}
        self.out_ch: Dict[str, int] = {}
        for k, v in full.items():
            if not k.startswith(self.prefixes):
                continue
            v = v.to(dev)
            if k.endswith(".weight") and v.dim() == 4:
                co = v.shape[0]
                v = v.permute(0, 2, 3, 1).reshape(co, -1)
                if co < 16:
                    self.out_ch[k[:-len(".weight")]] = co
                    v = torch.cat([v, torch.zeros(16 - co, v.shape[1], device=dev, dtype=v.dtype)], 0)
                p[k] = v.to(torch.bfloat16).contiguous()
            elif k.endswith(".bias") and k[:-len(".bias")] + ".weight" in full and full[k[:-len(".bias")] + ".weight"].dim() == 4 \
                    and v.numel() < 16:
                p[k] = torch.cat([v, torch.zeros(16 - v.numel(), device=dev, dtype=v.dtype)]).to(torch.bfloat16)
            elif "norm" in k.rsplit(".", 2)[-2] or "group_norm" in k:
                p[k] = v.float().contiguous()
            else:
                p[k] = v.to(torch.bfloat16).contiguous()
        for a in self.attn_prefixes:
            p[a + "qkv.weight"] = torch.cat([p[a + n + ".weight"] for n in ("to_q", "to_k", "to_v")], 0).contiguous()
            p[a + "qkv.bias"] = torch.cat([p[a + n + ".bias"] for n in ("to_q", "to_k", "to_v")], 0).contiguous()
        self.p = p

    def random_init(self, seed: int = 0) -> None:
        self.load(vae_random_weights(self.cfg, seed, self.device))

    # ---------------------------------------------------------------- pieces
    def _stats(self, x: torch.Tensor) -> torch.Tensor:
        G = min(self.cfg.groups, x.shape[3])
        st = torch.empty(x.shape[0], G, 2, dtype=torch.float32, device=self.device)
        _C().vae_gn_stats(x, G, self.cfg.eps, st)
        ops._count(2)
        return st

    def _conv3(self, x, name, up=1, norm=None, resid=None, stride=1, pads=(1, 1, 1, 1)):
        """3x3 conv of NHWC x (optionally GN+SiLU first, nearest x`up`,
        stride 2 with pads (top, bottom, left, right)) -> NHWC bf16."""
        N, H, W, C = x.shape
        pt, pb, pl, pr = pads
        Ho, Wo = (H * up + pt + pb - 3) // stride + 1, (W * up + pl + pr - 3) // stride + 1
        cols = torch.empty(N * Ho * Wo, 9 * C, dtype=torch.bfloat16, device=self.device)
        if norm is not None:
            st, pn = norm
            _C().vae_im2col3x3(x, up, st, self.p[pn + "weight"], self.p[pn + "bias"], st.shape[1], True, cols,
                               stride, pt, pb, pl, pr)
        else:
            _C().vae_im2col3x3(x, up, None, None, None, 0, False, cols, stride, pt, pb, pl, pr)
        ops._count()
        w, b = self.p[name + ".weight"], self.p[name + ".bias"]
        if resid is not None:
            y = ops.gemm(cols, w, bias=b, resid=resid.view(N * Ho * Wo, -1), epi=ops.EPI_RESIDUAL)
        else:
            y = ops.gemm(cols, w, bias=b)
        return y.view(N, Ho, Wo, -1)

    def _res(self, x, p):
        h = self._conv3(x, p + "conv1", norm=(self._stats(x), p + "norm1."))
        if p + "conv_shortcut.weight" in self.p:
            N, H, W, C = x.shape
            sc = ops.gemm(x.view(N * H * W, C), self.p[p + "conv_shortcut.weight"], bias=self.p[p + "conv_shortcut.bias"])
        else:
            sc = x
        return self._conv3(h, p + "conv2", norm=(self._stats(h), p + "norm2."), resid=sc)

    def _attn(self, x, a="decoder.mid_block.attentions.0."):
        N, H, W, C = x.shape
        P = H * W
        st = self._stats(x)
        xn = torch.empty_like(x)
        _C().vae_gn_apply(x, st, self.p[a + "group_norm.weight"], self.p[a + "group_norm.bias"], st.shape[1], False,
                          xn)
        qkv = ops.gemm(xn.view(N * P, C), self.p[a + "qkv.weight"], bias=self.p[a + "qkv.bias"])
        bpb = (P + 15) // 16
        q = torch.empty(N * P, 1, C, dtype=torch.bfloat16, device=self.device)
        kv = torch.zeros(N * bpb, 2 * 16 * C, dtype=torch.bfloat16, device=self.device)
        _C().vae_pack_attn(qkv, N, C, q, kv)
        bt = (torch.arange(N, dtype=torch.int32)[:, None] * bpb + torch.arange(bpb, dtype=torch.int32)[None, :])
        cu = [n * P for n in range(N + 1)]
        ts, tst = ops.prefill_tiles(cu, [P] * N)
        o = torch.empty_like(q)
        dev = self.device
        ops.wide_prefill_attention(q, kv, 1, bt.to(dev), torch.full((N,), P, dtype=torch.int32, device=dev),
                                   torch.tensor(cu, dtype=torch.int32, device=dev), ts.to(dev), tst.to(dev), o,
                                   scale=1.0 / math.sqrt(C), causal=False)
        ops._count(2)
        y = ops.gemm(o.view(N * P, C), self.p[a + "to_out.0.weight"], bias=self.p[a + "to_out.0.bias"],
                     resid=x.view(N * P, C), epi=ops.EPI_RESIDUAL)
        return y.view(N, H, W, C)

    def _decode_chunk(self, z: torch.Tensor, rgb: bool = True) -> torch.Tensor:
        """z NHWC bf16 [N, h, w, 16] -> u8 [N, 8h, 8w, 3] (rgb=False: the
        decoder's bf16 output [N, 8h, 8w, 3] before the byte conversion)."""
        cfg = self.cfg
        x = self._conv3(z, "decoder.conv_in")
        x = self._res(x, "decoder.mid_block.resnets.0.")
        x = self._attn(x)
        x = self._res(x, "decoder.mid_block.resnets.1.")
        for level, (ci, co, up) in enumerate(_levels(cfg)):
            for i in range(cfg.num_res_blocks):
                x = self._res(x, f"decoder.up_blocks.{level}.resnets.{i}.")
            if up:
                x = self._conv3(x, f"decoder.up_blocks.{level}.upsamplers.0.conv", up=2)
        out = self._conv3(x, "decoder.conv_out", norm=(self._stats(x), "decoder.norm_out."))
        return self._to_rgb(out, rgb)

    def _to_rgb(self, out: torch.Tensor, rgb: bool) -> torch.Tensor:
        N, H, W, _ = out.shape
        if not rgb:
            return out[..., :3]
        rgb = torch.empty(N * H * W, 3, dtype=torch.uint8, device=self.device)
        _C().vae_rgb(out.view(N * H * W, -1), rgb)
        ops._count()
        return rgb.view(N, H, W, 3)

    def frames_per_chunk(self, h: int, w: int) -> int:
        """Frames decoded together so the largest im2col stays under the byte cap."""
        s = self.cfg.spatial_stride  # the full-resolution convolutions read base_channels
        worst = (h * s) * (w * s) * 9 * self.cfg.base_channels * 2
        return max(1, int(self.max_im2col_bytes // max(worst, 1)))

    def decode(self, latent: torch.Tensor, rgb: bool = True) -> torch.Tensor:
        """latent f32 [C, F, h, w] -> u8 frames [F, 8h, 8w, 3] on the device."""
        C, Fr, h, w = latent.shape
        z = latent.to(self.device).permute(1, 2, 3, 0).to(torch.bfloat16).contiguous()  # NHWC
        step = self.frames_per_chunk(h, w)
        outs = [self._decode_chunk(z[i:i + step].contiguous(), rgb) for i in range(0, Fr, step)]
        return outs[0] if len(outs) == 1 else torch.cat(outs, 0)


def _C():
    from .._ext import cuda

    return cuda()
