"""Qwen3-VL: vision tower + Qwen3 text decoder with interleaved M-RoPE and
deepstack feature injection, on this repository's sm_100a kernels.

Vision tower (per image, N patches of 3 x 2 x 16 x 16 pixels, merge order):
    x = gemm(patches, W_patch) + b                     tcgen05 GEMM, bias epilogue
    x += bilinear(pos_embed grid -> h x w)             learned 2-D position table
    per block:  h = layernorm(x);  qkv = gemm(h) + b
                q, k rotated by the 2-D (row, column) rotary table
                a = attention(q, k, v) over all patches of the image (non-causal,
                    the paged prefill kernel on a scratch page table)
                x += gemm(a, W_proj) + b
                x += gemm(gelu_tanh(gemm(layernorm(x)) + b)) + b
                deepstack layers: feature_l = merger_l(x) (norm after the 2x2 shuffle)
    tokens = merger(x): layernorm, 2 x 2 patches -> one token, gemm + gelu, gemm
Text decoder: Qwen3 (q/k RMSNorm, SwiGLU) whose image-pad tokens take the
vision tokens as embeddings; positions are three planes (temporal, height,
width) combined per rotary frequency in the interleaved pattern (frequency
i takes the height plane when i % 3 == 1, width when i % 3 == 2, within the
24/20/20 sections) and applied by the CUDA M-RoPE kernel; after decoder
layer l < len(deepstack) the image positions' hidden states add deepstack
feature l.  Generation runs one request on a scratch paged KV cache
(prefill: paged prefill attention, decode: paged decode attention).

Weight names follow the HF Qwen3-VL checkpoints (model.visual.*,
model.language_model.*, lm_head.weight).  Reference: crates/engine/src/
executor/qwen3_vl.rs:24-1570 (the same vision / text structure; that
executor also pools the vision tokens to 512 with an extra attention pool,
which the HF model family does not have and this one does not add).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from .config import ModelConfig


@dataclass
class VisionConfig:
    depth: int = 24
    hidden_size: int = 1024
    num_heads: int = 16
    intermediate_size: int = 4096
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    in_channels: int = 3
    out_hidden_size: int = 2048
    num_position_embeddings: int = 2304
    deepstack_visual_indexes: Tuple[int, ...] = (5, 11, 17)
    layer_norm_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def patch_features(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2


@dataclass
class Qwen3VLConfig:
    text: ModelConfig
    vision: VisionConfig
    image_token_id: int = 151655
    vision_start_token_id: int = 151652
    vision_end_token_id: int = 151653
    mrope_section: Tuple[int, int, int] = (24, 20, 20)
    name: str = "qwen3-vl"


def _text(**kw) -> ModelConfig:
    base = dict(arch="qwen3", qk_norm=True, rms_norm_eps=1e-6, rope_theta=5_000_000.0,
                max_position_embeddings=262144, eos_token_ids=[151645, 151643], tie_word_embeddings=True)
    base.update(kw)
    return ModelConfig(**base)


PRESETS: Dict[str, Qwen3VLConfig] = {
    # Qwen3-VL-2B-Instruct shapes
    "qwen3-vl-2b": Qwen3VLConfig(
        _text(vocab_size=151936, hidden_size=2048, num_layers=28, num_heads=16, num_kv_heads=8, head_dim=128,
              intermediate_size=6144, name="qwen3-vl-2b"),
        VisionConfig(depth=24, hidden_size=1024, num_heads=16, intermediate_size=4096, out_hidden_size=2048,
                     num_position_embeddings=2304, deepstack_visual_indexes=(5, 11, 17)),
        name="qwen3-vl-2b"),
    # tiny shape for tests (vision head_dim 64, text head_dim 128)
    "tiny-qwen3-vl": Qwen3VLConfig(
        _text(vocab_size=512, hidden_size=256, num_layers=3, num_heads=4, num_kv_heads=2, head_dim=128,
              intermediate_size=512, max_position_embeddings=4096, eos_token_ids=[2], tie_word_embeddings=False,
              rope_theta=10000.0, name="tiny-qwen3-vl"),
        VisionConfig(depth=3, hidden_size=128, num_heads=2, intermediate_size=256, out_hidden_size=256,
                     num_position_embeddings=64, deepstack_visual_indexes=(0, 1)),
        image_token_id=500, vision_start_token_id=498, vision_end_token_id=499, name="tiny-qwen3-vl"),
}


def vl_preset(name: str) -> Qwen3VLConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown Qwen3-VL preset {name!r} ({', '.join(PRESETS)})")
    return PRESETS[name]


# ---------------------------------------------------------------- positions
def mrope_positions(ids: Sequence[int], grid_thw: Optional[Tuple[int, int, int]], image_token_id: int,
                    merge: int = 2) -> Tuple[torch.Tensor, int]:
    """Three position planes [3, T] for a prompt with at most one image, and
    the next text position.  Text tokens advance all planes together; the
    image's merged tokens share a temporal start and take (row, column)
    offsets; text after the image continues past the largest image offset."""
    T = len(ids)
    pos = torch.zeros(3, T, dtype=torch.long)
    nxt, st = 0, 0
    if grid_thw is not None and image_token_id in ids:
        ed = list(ids).index(image_token_id)
        pos[:, :ed] = torch.arange(ed)
        nxt = ed
        gt, gh, gw = grid_thw[0], grid_thw[1] // merge, grid_thw[2] // merge
        n = gt * gh * gw
        tt = torch.arange(gt).view(-1, 1, 1).expand(gt, gh, gw).reshape(-1)
        hh = torch.arange(gh).view(1, -1, 1).expand(gt, gh, gw).reshape(-1)
        ww = torch.arange(gw).view(1, 1, -1).expand(gt, gh, gw).reshape(-1)
        pos[0, ed:ed + n] = nxt + tt
        pos[1, ed:ed + n] = nxt + hh
        pos[2, ed:ed + n] = nxt + ww
        nxt = nxt + max(gt - 1, gh - 1, gw - 1) + 1
        st = ed + n
    pos[:, st:] = torch.arange(T - st) + nxt
    nxt += T - st
    return pos, nxt


def interleaved_mrope_cos_sin(pos: torch.Tensor, head_dim: int, theta: float, sections: Sequence[int], device):
    """cos, sin [T, head_dim] fp32: frequency i rotates by the height plane when
    i % 3 == 1 and i < 3 * sections[1], the width plane when i % 3 == 2 and
    i < 3 * sections[2], the temporal plane otherwise."""
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) * 2 / head_dim))
    plane = torch.zeros(half, dtype=torch.long)
    i = torch.arange(half)
    plane[(i % 3 == 1) & (i < 3 * sections[1])] = 1
    plane[(i % 3 == 2) & (i < 3 * sections[2])] = 2
    p = pos.to(torch.float64)  # [3, T]
    ang = p[plane, :].t() * inv  # [T, half]: column i from plane[i]
    emb = torch.cat([ang, ang], -1)
    return emb.cos().float().to(device), emb.sin().float().to(device)


# ---------------------------------------------------------------- vision helpers
def vision_rotary(grid_thw: Tuple[int, int, int], head_dim: int, theta: float, merge: int, device):
    """cos, sin [N, head_dim] of the 2-D rotary: half the rotary pairs follow
    the patch row, half the column (patches in merge-block order)."""
    gt, gh, gw = grid_thw
    quarter = head_dim // 4
    inv = 1.0 / (theta ** (torch.arange(0, 2 * quarter, 2, dtype=torch.float64) / (2 * quarter)))
    rows, cols = [], []
    for _ in range(gt):
        for bh in range(gh // merge):
            for bw in range(gw // merge):
                for ih in range(merge):
                    for iw in range(merge):
                        rows.append(bh * merge + ih)
                        cols.append(bw * merge + iw)
    r = torch.tensor(rows, dtype=torch.float64).view(-1, 1) * inv
    c = torch.tensor(cols, dtype=torch.float64).view(-1, 1) * inv
    emb = torch.cat([r, c], -1)
    emb = torch.cat([emb, emb], -1)
    return emb.cos().float().to(device), emb.sin().float().to(device)


def pos_embed_interp(table: torch.Tensor, grid_thw: Tuple[int, int, int], merge: int) -> torch.Tensor:
    """Bilinear interpolation of the square learned position grid to h x w,
    repeated over t, in merge-block order: [N, hidden] (table's dtype)."""
    gt, gh, gw = grid_thw
    side = int(round(math.sqrt(table.shape[0])))
    hv = torch.linspace(0, side - 1, gh, dtype=torch.float64)
    wv = torch.linspace(0, side - 1, gw, dtype=torch.float64)
    h0, w0 = hv.floor().long(), wv.floor().long()
    h1, w1 = (h0 + 1).clamp(max=side - 1), (w0 + 1).clamp(max=side - 1)
    dh, dw = (hv - h0).view(-1, 1), (wv - w0).view(1, -1)
    idx = [(h0.view(-1, 1) * side + w0.view(1, -1)), (h0.view(-1, 1) * side + w1.view(1, -1)),
           (h1.view(-1, 1) * side + w0.view(1, -1)), (h1.view(-1, 1) * side + w1.view(1, -1))]
    wts = [(1 - dh) * (1 - dw), (1 - dh) * dw, dh * (1 - dw), dh * dw]
    tf = table.float()
    acc = torch.zeros(gh * gw, table.shape[1], dtype=torch.float32, device=table.device)
    for ix, wt in zip(idx, wts):
        acc += tf.index_select(0, ix.reshape(-1).to(table.device)) * wt.reshape(-1, 1).float().to(table.device)
    acc = acc.view(gh // merge, merge, gw // merge, merge, -1).permute(0, 2, 1, 3, 4).reshape(gh * gw, -1)
    return acc.repeat(gt, 1).to(table.dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], -1)


# ---------------------------------------------------------------- model
class Qwen3VL:
    """Weights and forward of a Qwen3-VL model on one GPU."""

    def __init__(self, cfg: Qwen3VLConfig, device=None):
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.w: Dict[str, torch.Tensor] = {}

    # ------------------------------------------------------------ weights
    @staticmethod
    def weight_shapes(cfg: Qwen3VLConfig) -> Dict[str, Tuple[int, ...]]:
        v, t = cfg.vision, cfg.text
        hv, hd = v.hidden_size, t.head_dim
        s: Dict[str, Tuple[int, ...]] = {
            "model.visual.patch_embed.proj.weight": (hv, v.in_channels, v.temporal_patch_size, v.patch_size,
                                                     v.patch_size),
            "model.visual.patch_embed.proj.bias": (hv,),
            "model.visual.pos_embed.weight": (v.num_position_embeddings, hv),
        }
        for i in range(v.depth):
            p = f"model.visual.blocks.{i}."
            s.update({p + "norm1.weight": (hv,), p + "norm1.bias": (hv,), p + "norm2.weight": (hv,),
                      p + "norm2.bias": (hv,), p + "attn.qkv.weight": (3 * hv, hv), p + "attn.qkv.bias": (3 * hv,),
                      p + "attn.proj.weight": (hv, hv), p + "attn.proj.bias": (hv,),
                      p + "mlp.linear_fc1.weight": (v.intermediate_size, hv),
                      p + "mlp.linear_fc1.bias": (v.intermediate_size,),
                      p + "mlp.linear_fc2.weight": (hv, v.intermediate_size), p + "mlp.linear_fc2.bias": (hv,)})
        m4 = hv * v.spatial_merge_size ** 2
        for pfx, nsz in [("model.visual.merger.", hv)] + [
                (f"model.visual.deepstack_merger_list.{j}.", m4) for j in range(len(v.deepstack_visual_indexes))]:
            s.update({pfx + "norm.weight": (nsz,), pfx + "norm.bias": (nsz,), pfx + "linear_fc1.weight": (m4, m4),
                      pfx + "linear_fc1.bias": (m4,), pfx + "linear_fc2.weight": (v.out_hidden_size, m4),
                      pfx + "linear_fc2.bias": (v.out_hidden_size,)})
        L = "model.language_model."
        s[L + "embed_tokens.weight"] = (t.vocab_size, t.hidden_size)
        s[L + "norm.weight"] = (t.hidden_size,)
        if not t.tie_word_embeddings:
            s["lm_head.weight"] = (t.vocab_size, t.hidden_size)
        for i in range(t.num_layers):
            p = f"{L}layers.{i}."
            s.update({p + "input_layernorm.weight": (t.hidden_size,),
                      p + "post_attention_layernorm.weight": (t.hidden_size,),
                      p + "self_attn.q_proj.weight": (t.num_heads * hd, t.hidden_size),
                      p + "self_attn.k_proj.weight": (t.num_kv_heads * hd, t.hidden_size),
                      p + "self_attn.v_proj.weight": (t.num_kv_heads * hd, t.hidden_size),
                      p + "self_attn.o_proj.weight": (t.hidden_size, t.num_heads * hd),
                      p + "self_attn.q_norm.weight": (hd,), p + "self_attn.k_norm.weight": (hd,),
                      p + "mlp.gate_proj.weight": (t.intermediate_size, t.hidden_size),
                      p + "mlp.up_proj.weight": (t.intermediate_size, t.hidden_size),
                      p + "mlp.down_proj.weight": (t.hidden_size, t.intermediate_size)})
        return s

    @staticmethod
    def random_weights(cfg: Qwen3VLConfig, seed: int = 0, std: float = 0.05, device="cpu") -> Dict[str, torch.Tensor]:
        """N(0, std) matrices, norms 1 (+ small noise), biases small; fp32."""
        g = torch.Generator().manual_seed(seed)
        out = {}
        for k, shp in Qwen3VL.weight_shapes(cfg).items():
            if k.endswith("norm.weight") or "norm1.weight" in k or "norm2.weight" in k or \
                    k.endswith("layernorm.weight") or "q_norm" in k or "k_norm" in k:
                out[k] = 1.0 + 0.05 * torch.randn(*shp, generator=g)
            elif k.endswith("bias"):
                out[k] = 0.02 * torch.randn(*shp, generator=g)
            elif k.endswith("pos_embed.weight"):
                out[k] = 0.5 * torch.randn(*shp, generator=g)
            else:
                out[k] = std * torch.randn(*shp, generator=g)
        return {k: v.to(device) for k, v in out.items()}

    def load(self, full: Dict[str, torch.Tensor]) -> None:
        """Install HF-named weights in the kernels' layouts (bf16)."""
        from .llama import DecoderLM

        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        v = cfg.vision

        def put(k, src=None):
            self.w[k] = (src if src is not None else full[k]).to(dev, bf).contiguous()

        put("patch_w", full["model.visual.patch_embed.proj.weight"].reshape(v.hidden_size, -1))
        put("patch_b", full["model.visual.patch_embed.proj.bias"])
        put("pos_embed", full["model.visual.pos_embed.weight"])
        for k, t in full.items():
            if k.startswith("model.visual.blocks.") or k.startswith("model.visual.merger.") or \
                    k.startswith("model.visual.deepstack_merger_list."):
                put(k[len("model.visual."):], t)
        # text decoder: the LLM path's layout (fused qkv, interleaved gate/up)
        L = "model.language_model."
        hf = {("model." + k[len(L):] if k.startswith(L) else k): t for k, t in full.items() if not k.startswith(
            "model.visual.")}
        if "lm_head.weight" not in hf:
            hf["lm_head.weight"] = hf["model.embed_tokens.weight"]
        self.text = DecoderLM(cfg.text, None, dev)
        self.text.shard_full(hf)

    # ------------------------------------------------------------ vision
    def _layernorm(self, x, pfx, eps):
        return ops.layernorm(x.contiguous(), self.w[pfx + "weight"], self.w[pfx + "bias"], eps)

    def _merger(self, x: torch.Tensor, pfx: str, post: bool) -> torch.Tensor:
        v = self.cfg.vision
        m4 = v.hidden_size * v.spatial_merge_size ** 2
        if post:
            x = self._layernorm(x.reshape(-1, m4), pfx + "norm.", v.layer_norm_eps)
        else:
            x = self._layernorm(x, pfx + "norm.", v.layer_norm_eps).reshape(-1, m4)
        x = ops.gemm(x, self.w[pfx + "linear_fc1.weight"], bias=self.w[pfx + "linear_fc1.bias"], epi=ops.EPI_GELU)
        return ops.gemm(x, self.w[pfx + "linear_fc2.weight"], bias=self.w[pfx + "linear_fc2.bias"])

    def _vision_attention(self, qkv: torch.Tensor, cos, sin) -> torch.Tensor:
        """Non-causal attention of all N patches: q, k rotated, K / V laid out
        as pages of a scratch cache, the paged prefill kernel with causal off."""
        v = self.cfg.vision
        N, nh, hd = qkv.shape[0], v.num_heads, v.head_dim
        x = qkv.view(N, 3, nh, hd)
        q, k, val = x[:, 0].float(), x[:, 1].float(), x[:, 2]
        c, s = cos.view(N, 1, hd), sin.view(N, 1, hd)
        q = (q * c + rotate_half(q) * s).to(torch.bfloat16).contiguous()
        k = (k * c + rotate_half(k) * s).to(torch.bfloat16)
        NB = (N + 15) // 16
        kv = torch.zeros(1, NB, 2, nh, 16, hd, dtype=torch.bfloat16, device=qkv.device)
        pad = NB * 16 - N
        kp = F.pad(k, (0, 0, 0, 0, 0, pad)).view(NB, 16, nh, hd).transpose(1, 2)
        vp = F.pad(val, (0, 0, 0, 0, 0, pad)).view(NB, 16, nh, hd).transpose(1, 2)
        kv[0, :, 0] = kp
        kv[0, :, 1] = vp
        bt = torch.arange(NB, dtype=torch.int32, device=qkv.device).view(1, NB)
        ctx = torch.tensor([N], dtype=torch.int32, device=qkv.device)
        cu = torch.tensor([0, N], dtype=torch.int32, device=qkv.device)
        ts, tst = ops.prefill_tiles([0, N], [N])
        out = torch.empty(N, nh, hd, dtype=torch.bfloat16, device=qkv.device)
        ops.paged_prefill_attention(q, kv, 0, bt, ctx, cu, ts.to(qkv.device), tst.to(qkv.device), out,
                                    scale=1.0 / math.sqrt(hd), causal=False)
        return out.view(N, nh * hd)

    def encode_image(self, patches: torch.Tensor, grid_thw: Tuple[int, int, int]):
        """patches [N, C*T*P*P] (merge-block order) -> (tokens [N/4, out_hidden],
        deepstack features: list of [N/4, out_hidden])."""
        v = self.cfg.vision
        w = self.w
        x = ops.gemm(patches.to(self.device, torch.bfloat16).contiguous(), w["patch_w"], bias=w["patch_b"])
        x = (x.float() + pos_embed_interp(w["pos_embed"], grid_thw, v.spatial_merge_size).float()).to(torch.bfloat16)
        cos, sin = vision_rotary(grid_thw, v.head_dim, v.rope_theta, v.spatial_merge_size, self.device)
        feats = []
        for i in range(v.depth):
            p = f"blocks.{i}."
            h = self._layernorm(x, p + "norm1.", v.layer_norm_eps)
            qkv = ops.gemm(h, w[p + "attn.qkv.weight"], bias=w[p + "attn.qkv.bias"])
            a = self._vision_attention(qkv, cos, sin)
            x = (x.float() + ops.gemm(a, w[p + "attn.proj.weight"], bias=w[p + "attn.proj.bias"]).float()
                 ).to(torch.bfloat16)
            h = self._layernorm(x, p + "norm2.", v.layer_norm_eps)
            h = ops.gemm(h, w[p + "mlp.linear_fc1.weight"], bias=w[p + "mlp.linear_fc1.bias"], epi=ops.EPI_GELU_TANH)
            x = (x.float() + ops.gemm(h, w[p + "mlp.linear_fc2.weight"], bias=w[p + "mlp.linear_fc2.bias"]).float()
                 ).to(torch.bfloat16)
            if i in v.deepstack_visual_indexes:
                j = list(v.deepstack_visual_indexes).index(i)
                feats.append(self._merger(x, f"deepstack_merger_list.{j}.", post=True))
        return self._merger(x, "merger.", post=False), feats

    # ------------------------------------------------------------ text
    def _text_layers(self, x_res: torch.Tensor, pos3: torch.Tensor, slots: torch.Tensor, kv: torch.Tensor,
                     ctx_len: int, n_new: int, img_mask: Optional[torch.Tensor], feats: List[torch.Tensor]):
        t, m = self.cfg.text, self.text
        T = x_res.shape[0]
        nq, nkv, hd = m.nq, m.nkv, t.head_dim
        eps = t.rms_norm_eps
        cos, sin = interleaved_mrope_cos_sin(pos3, hd, t.rope_theta, self.cfg.mrope_section, self.device)
        cos3 = cos.view(1, 1, T, hd).expand(3, 1, T, hd)
        sin3 = sin.view(1, 1, T, hd).expand(3, 1, T, hd)
        NB = kv.shape[1]
        bt = torch.arange(NB, dtype=torch.int32, device=self.device).view(1, NB)
        blk, off = (slots // 16).long(), (slots % 16).long()
        x = ops.rmsnorm(x_res, m.layers[0]["ln1"], eps)
        for li, lay in enumerate(m.layers):
            qkv = ops.gemm(x, lay["qkv"])
            q = ops.rmsnorm(qkv[:, :nq * hd].contiguous().view(T * nq, hd), lay["q_norm"], eps).view(T, nq, hd)
            k = ops.rmsnorm(qkv[:, nq * hd:(nq + nkv) * hd].contiguous().view(T * nkv, hd), lay["k_norm"],
                            eps).view(T, nkv, hd)
            vv = qkv[:, (nq + nkv) * hd:].view(T, nkv, hd)
            qr, kr = ops.mrope(q.permute(1, 0, 2).unsqueeze(0), k.permute(1, 0, 2).unsqueeze(0), cos3, sin3,
                               sections=(hd // 2, 0, 0))
            q = qr[0].permute(1, 0, 2).contiguous()
            kv[li, blk, 0, :, off, :] = kr[0].permute(1, 0, 2)
            kv[li, blk, 1, :, off, :] = vv
            attn = torch.empty(T, nq, hd, dtype=torch.bfloat16, device=self.device)
            if T == 1:
                ops.paged_decode_attention(q, kv, li, bt, torch.tensor([ctx_len], dtype=torch.int32,
                                                                       device=self.device), attn,
                                           q_len=1, splits=1, workspace=None, scale=m.scale)
            else:
                ts, tst = ops.prefill_tiles([0, T], [ctx_len])
                ops.paged_prefill_attention(q, kv, li, bt, torch.tensor([ctx_len], dtype=torch.int32,
                                                                        device=self.device),
                                            torch.tensor([0, T], dtype=torch.int32, device=self.device),
                                            ts.to(self.device), tst.to(self.device), attn, scale=m.scale, causal=True)
            x = ops.add_rmsnorm(ops.gemm(attn.view(T, nq * hd), lay["o"]), x_res, lay["ln2"], eps)
            act = ops.gemm(x, lay["gate_up"], epi=ops.EPI_SWIGLU)
            nxt = m.layers[li + 1]["ln1"] if li + 1 < len(m.layers) else m.final_norm
            x = ops.add_rmsnorm(ops.gemm(act, lay["down"]), x_res, nxt, eps)
            if img_mask is not None and li < len(feats):
                x_res[img_mask] = (x_res[img_mask].float() + feats[li].float()).to(torch.bfloat16)
                x = ops.rmsnorm(x_res, nxt, eps)
        return x

    # ------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, ids: List[int], patches: Optional[torch.Tensor] = None,
                 grid_thw: Optional[Tuple[int, int, int]] = None, max_tokens: int = 16, eos: Sequence[int] = (),
                 on_token=None) -> List[int]:
        """Greedy generation of one request; `ids` holds the image-pad tokens
        (one per merged vision token) between vision start / end markers."""
        t, m = self.cfg.text, self.text
        if not hasattr(self, "text"):
            raise RuntimeError("load weights first")
        T = len(ids)
        max_len = T + max_tokens + 1
        NB = (max_len + 15) // 16
        kv = torch.zeros(t.num_layers, NB, 2, m.nkv, 16, t.head_dim, dtype=torch.bfloat16, device=self.device)
        ids_t = torch.tensor(ids, dtype=torch.int32, device=self.device)
        x_res = ops.embedding(ids_t, m.embed)
        img_mask, feats = None, []
        if patches is not None:
            toks, feats = self.encode_image(patches, grid_thw)
            img_mask = ids_t == self.cfg.image_token_id
            n_img = int(img_mask.sum().item())
            if n_img != toks.shape[0]:
                raise ValueError(f"prompt has {n_img} image-pad tokens but the image gives {toks.shape[0]}")
            x_res[img_mask] = toks
        pos3, nxt = mrope_positions(ids, grid_thw, self.cfg.image_token_id, self.cfg.vision.spatial_merge_size)
        slots = torch.arange(T, dtype=torch.int32, device=self.device)
        h = self._text_layers(x_res, pos3, slots, kv, T, T, img_mask, feats)
        out: List[int] = []
        tok = int(ops.argmax(ops.gemm(h[-1:].contiguous(), m.lm_head))[0].item())
        for step in range(max_tokens):
            out.append(tok)
            if on_token is not None:
                on_token(tok)
            if tok in eos or step == max_tokens - 1:
                break
            p = T + step
            x_res = ops.embedding(torch.tensor([tok], dtype=torch.int32, device=self.device), m.embed)
            pos = torch.full((3, 1), nxt + step, dtype=torch.long)
            h = self._text_layers(x_res, pos, torch.tensor([p], dtype=torch.int32, device=self.device), kv, p + 1,
                                  1, None, [])
            tok = int(ops.argmax(ops.gemm(h, m.lm_head))[0].item())
        return out

    def prompt_ids(self, text_ids: List[int], n_image_tokens: int, prefix: Sequence[int] = (),
                   suffix: Sequence[int] = ()) -> List[int]:
        c = self.cfg
        img = [c.vision_start_token_id] + [c.image_token_id] * n_image_tokens + [c.vision_end_token_id] \
            if n_image_tokens else []
        return list(prefix) + img + list(text_ids) + list(suffix)


# ---------------------------------------------------------------- fp32 oracle
def reference_logits(cfg: Qwen3VLConfig, w: Dict[str, torch.Tensor], ids: List[int],
                     patches: Optional[torch.Tensor], grid_thw) -> torch.Tensor:
    """Plain PyTorch fp32 restatement of the same model: logits [T, V]."""
    toks, feats = reference_vision(cfg, w, patches, grid_thw) if patches is not None else (None, [])
    return _reference_text(cfg, w, ids, grid_thw, toks, feats)


def reference_vision(cfg: Qwen3VLConfig, w: Dict[str, torch.Tensor], patches: torch.Tensor, grid_thw):
    """fp32 vision tower: (merged tokens [N/4, out], deepstack features)."""
    v = cfg.vision
    f = {k: x.float().cpu() for k, x in w.items() if k.startswith("model.visual.")}

    def ln(x, p, n):
        return F.layer_norm(x, (n,), f[p + "weight"], f[p + "bias"], v.layer_norm_eps)

    def lin(x, p):
        return x @ f[p + "weight"].t() + f[p + "bias"]

    def merger(x, p, post):
        m4 = v.hidden_size * v.spatial_merge_size ** 2
        x = ln(x.reshape(-1, m4), p + "norm.", m4) if post else ln(x, p + "norm.", v.hidden_size).reshape(-1, m4)
        return lin(F.gelu(lin(x, p + "linear_fc1.")), p + "linear_fc2.")

    feats, toks = [], None
    if True:
        V = "model.visual."
        x = patches.float().cpu() @ f[V + "patch_embed.proj.weight"].reshape(v.hidden_size, -1).t() + \
            f[V + "patch_embed.proj.bias"]
        x = x + pos_embed_interp(f[V + "pos_embed.weight"], grid_thw, v.spatial_merge_size)
        cos, sin = vision_rotary(grid_thw, v.head_dim, v.rope_theta, v.spatial_merge_size, "cpu")
        N, nh, hd = x.shape[0], v.num_heads, v.head_dim
        for i in range(v.depth):
            p = f"{V}blocks.{i}."
            h = ln(x, p + "norm1.", v.hidden_size)
            qkv = lin(h, p + "attn.qkv.").view(N, 3, nh, hd)
            q, k, vv = qkv[:, 0], qkv[:, 1], qkv[:, 2]
            c, s = cos.view(N, 1, hd), sin.view(N, 1, hd)
            q, k = q * c + rotate_half(q) * s, k * c + rotate_half(k) * s
            att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd), -1)
            a = torch.einsum("hqk,khd->qhd", att, vv).reshape(N, nh * hd)
            x = x + lin(a, p + "attn.proj.")
            x = x + lin(F.gelu(lin(ln(x, p + "norm2.", v.hidden_size), p + "mlp.linear_fc1."), approximate="tanh"),
                        p + "mlp.linear_fc2.")
            if i in v.deepstack_visual_indexes:
                j = list(v.deepstack_visual_indexes).index(i)
                feats.append(merger(x, f"{V}deepstack_merger_list.{j}.", True))
        toks = merger(x, f"{V}merger.", False)
    return toks, feats


def _reference_text(cfg: Qwen3VLConfig, w: Dict[str, torch.Tensor], ids: List[int], grid_thw, toks, feats):
    v, t = cfg.vision, cfg.text
    f = {k: x.float().cpu() for k, x in w.items() if not k.startswith("model.visual.")}
    L = "model.language_model."
    T = len(ids)
    idt = torch.tensor(ids)
    xr = f[L + "embed_tokens.weight"][idt].clone()
    mask = idt == cfg.image_token_id
    if toks is not None:
        xr[mask] = toks
    pos3, _ = mrope_positions(ids, grid_thw, cfg.image_token_id, v.spatial_merge_size)
    hd = t.head_dim
    cos, sin = interleaved_mrope_cos_sin(pos3, hd, t.rope_theta, cfg.mrope_section, "cpu")

    def rms(x, wt):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + t.rms_norm_eps) * wt

    G = t.num_heads // t.num_kv_heads
    causal = torch.full((T, T), float("-inf")).triu(1)
    for i in range(t.num_layers):
        p = f"{L}layers.{i}."
        h = rms(xr, f[p + "input_layernorm.weight"])
        q = (h @ f[p + "self_attn.q_proj.weight"].t()).view(T, t.num_heads, hd)
        k = (h @ f[p + "self_attn.k_proj.weight"].t()).view(T, t.num_kv_heads, hd)
        vv = (h @ f[p + "self_attn.v_proj.weight"].t()).view(T, t.num_kv_heads, hd)
        q, k = rms(q, f[p + "self_attn.q_norm.weight"]), rms(k, f[p + "self_attn.k_norm.weight"])
        c, s = cos.view(T, 1, hd), sin.view(T, 1, hd)
        q, k = q * c + rotate_half(q) * s, k * c + rotate_half(k) * s
        k, vv = k.repeat_interleave(G, 1), vv.repeat_interleave(G, 1)
        att = torch.softmax(torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd) + causal, -1)
        a = torch.einsum("hqk,khd->qhd", att, vv).reshape(T, -1)
        xr = xr + a @ f[p + "self_attn.o_proj.weight"].t()
        h = rms(xr, f[p + "post_attention_layernorm.weight"])
        xr = xr + (F.silu(h @ f[p + "mlp.gate_proj.weight"].t()) * (h @ f[p + "mlp.up_proj.weight"].t())) @ \
            f[p + "mlp.down_proj.weight"].t()
        if toks is not None and i < len(feats):
            xr[mask] = xr[mask] + feats[i]
    xr = rms(xr, f[L + "norm.weight"])
    head = f.get("lm_head.weight", f[L + "embed_tokens.weight"])
    return xr @ head.t()
