"""BERT-family sentence embedder (MiniLM / all-MiniLM-L6-v2 shape) on the GPU.

Sequences are packed without padding (cu_seqlens); per layer: fused QKV GEMM
(+bias) -> variable-length non-causal attention -> output GEMM (+bias) ->
LayerNorm(x + .) -> GEMM with bias+GELU epilogue -> GEMM (+bias) ->
LayerNorm(x + .); then mean pooling over each sequence and L2
normalisation in one kernel.  All linear layers run on the tcgen05 GEMM.

Reference: candle BertModel with a padded batch and masked mean pooling
(crates/engine/src/executor/candle.rs:177-264), L2 normalisation and
dimension truncation in the server (crates/server/src/embedding.rs:505-540).
"""
from __future__ import annotations

import json
import math
import os
from typing import Dict, List, Optional

import torch

from .. import ops
from .config import ModelConfig, from_hf_config, preset


def _strip(name: str) -> str:
    for p in ("bert.", "model.", "0.auto_model."):
        if name.startswith(p):
            name = name[len(p):]
    return name


class BertEmbedder:
    def __init__(self, cfg: ModelConfig, device="cuda", dtype=torch.bfloat16):
        """dtype bf16: tcgen05 GEMMs with fused bias / GELU and tensor-core
        attention.  dtype fp32: full precision end to end -- fp32 weights and
        activations, this repository's fp32 kernels for embeddings + LayerNorm,
        attention, residual LayerNorm, GELU and pooling, and fp32 SGEMM from
        cuBLAS (TF32 off) for the linear layers: tensor cores have no fp32
        mode, so the library GEMM is the full-precision path."""
        if dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("BertEmbedder dtype must be bf16 or fp32")
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.w: Dict[str, torch.Tensor] = {}
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.tokenizer = None

    # ------------------------------------------------------------ weights
    def load_state_dict(self, sd: Dict[str, torch.Tensor]) -> None:
        c, dev, bf = self.cfg, self.device, self.dtype
        sd = {_strip(k): v for k, v in sd.items()}

        def g(k):
            return sd[k].to(dev, bf).contiguous()

        self.w = {"word": g("embeddings.word_embeddings.weight"), "pos": g("embeddings.position_embeddings.weight"),
                  "type": g("embeddings.token_type_embeddings.weight"), "ln_w": g("embeddings.LayerNorm.weight"),
                  "ln_b": g("embeddings.LayerNorm.bias")}
        self.layers = []
        for i in range(c.num_layers):
            p = f"encoder.layer.{i}."
            qkv = torch.cat([sd[p + f"attention.self.{n}.weight"] for n in ("query", "key", "value")], 0)
            qkv_b = torch.cat([sd[p + f"attention.self.{n}.bias"] for n in ("query", "key", "value")], 0)
            self.layers.append({
                "qkv": qkv.to(dev, bf).contiguous(), "qkv_b": qkv_b.to(dev, bf).contiguous(),
                "o": g(p + "attention.output.dense.weight"), "o_b": g(p + "attention.output.dense.bias"),
                "ln1_w": g(p + "attention.output.LayerNorm.weight"), "ln1_b": g(p + "attention.output.LayerNorm.bias"),
                "i": g(p + "intermediate.dense.weight"), "i_b": g(p + "intermediate.dense.bias"),
                "out": g(p + "output.dense.weight"), "out_b": g(p + "output.dense.bias"),
                "ln2_w": g(p + "output.LayerNorm.weight"), "ln2_b": g(p + "output.LayerNorm.bias"),
            })

    @staticmethod
    def random_state_dict(cfg: ModelConfig, seed: int = 0, std: float = 0.02) -> Dict[str, torch.Tensor]:
        g = torch.Generator().manual_seed(seed)
        H, I = cfg.hidden_size, cfg.intermediate_size

        def rn(*s):
            return (torch.randn(*s, generator=g) * std).to(torch.bfloat16)

        def ones(n):
            return torch.ones(n, dtype=torch.bfloat16)

        def zeros(n):
            return torch.zeros(n, dtype=torch.bfloat16)

        sd = {"embeddings.word_embeddings.weight": rn(cfg.vocab_size, H),
              "embeddings.position_embeddings.weight": rn(cfg.max_position_embeddings, H),
              "embeddings.token_type_embeddings.weight": rn(cfg.type_vocab_size, H),
              "embeddings.LayerNorm.weight": ones(H), "embeddings.LayerNorm.bias": zeros(H)}
        for i in range(cfg.num_layers):
            p = f"encoder.layer.{i}."
            for n in ("query", "key", "value"):
                sd[p + f"attention.self.{n}.weight"] = rn(H, H)
                sd[p + f"attention.self.{n}.bias"] = rn(H)
            sd[p + "attention.output.dense.weight"] = rn(H, H)
            sd[p + "attention.output.dense.bias"] = rn(H)
            sd[p + "attention.output.LayerNorm.weight"] = ones(H)
            sd[p + "attention.output.LayerNorm.bias"] = zeros(H)
            sd[p + "intermediate.dense.weight"] = rn(I, H)
            sd[p + "intermediate.dense.bias"] = rn(I)
            sd[p + "output.dense.weight"] = rn(H, I)
            sd[p + "output.dense.bias"] = rn(H)
            sd[p + "output.LayerNorm.weight"] = ones(H)
            sd[p + "output.LayerNorm.bias"] = zeros(H)
        return sd

    @staticmethod
    def load(model: str, device="cuda") -> "BertEmbedder":
        from .config import PRESETS

        if model in PRESETS:
            cfg = preset(model)
            e = BertEmbedder(cfg, device)
            e.load_state_dict(BertEmbedder.random_state_dict(cfg))
            return e
        from ..formats.manifest import load_manifest
        from ..formats.safetensors_io import load_state_dict

        man = load_manifest(model)
        with open(os.path.join(man.root, "config.json")) as f:
            cfg = from_hf_config(json.load(f))
        e = BertEmbedder(cfg, device)
        e.load_state_dict(load_state_dict(man.root))
        tj = os.path.join(man.root, "tokenizer.json")
        if os.path.exists(tj):
            from tokenizers import Tokenizer

            e.tokenizer = Tokenizer.from_file(tj)
        return e

    # ------------------------------------------------------------ forward
    @torch.no_grad()
    def forward_ids(self, seqs: List[List[int]], normalize: bool = True) -> torch.Tensor:
        """Embeddings [S, H] f32 of token-id sequences (packed, no padding)."""
        c, dev = self.cfg, self.device
        lens = [min(len(s), c.max_position_embeddings) for s in seqs]
        T = sum(lens)
        ids = torch.tensor([t for s, L in zip(seqs, lens) for t in s[:L]], dtype=torch.int32)
        pos = torch.tensor([p for L in lens for p in range(L)], dtype=torch.int32)
        cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)
        ids, pos, cu = ids.to(dev, non_blocking=True), pos.to(dev, non_blocking=True), cu.to(dev, non_blocking=True)
        return self.forward_packed(ids, pos, cu, max(lens), normalize)

    def forward_packed(self, ids, pos, cu, max_len: int, normalize: bool = True) -> torch.Tensor:
        c = self.cfg
        w = self.w
        nh, hd = c.num_heads, c.hidden_size // c.num_heads
        scale = 1.0 / math.sqrt(hd)
        eps = c.layer_norm_eps
        x = ops.bert_embed_ln(ids, pos, None, w["word"], w["pos"], w["type"], w["ln_w"], w["ln_b"], eps)
        if self.dtype == torch.float32:
            return self._forward_f32(x, cu, max_len, nh, hd, scale, eps, normalize)
        for lay in self.layers:
            qkv = ops.gemm(x, lay["qkv"], bias=lay["qkv_b"])
            a = ops.varlen_attention(qkv, cu, nh, hd, max_len, scale)
            o = ops.gemm(a, lay["o"], bias=lay["o_b"])
            x = ops.layernorm(o, lay["ln1_w"], lay["ln1_b"], eps, resid=x)
            h = ops.gemm(x, lay["i"], epi=ops.EPI_GELU, bias=lay["i_b"])
            d = ops.gemm(h, lay["out"], bias=lay["out_b"])
            x = ops.layernorm(d, lay["ln2_w"], lay["ln2_b"], eps, resid=x)
        return ops.mean_pool_l2(x, cu, normalize)

    def _forward_f32(self, x, cu, max_len, nh, hd, scale, eps, normalize):
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            for lay in self.layers:
                qkv = torch.addmm(lay["qkv_b"], x, lay["qkv"].t())
                a = ops.varlen_attention(qkv, cu, nh, hd, max_len, scale)
                o = torch.addmm(lay["o_b"], a, lay["o"].t())
                x = ops.ln_residual_f32(o, x, lay["ln1_w"], lay["ln1_b"], eps)
                h = ops.gelu_f32_(torch.addmm(lay["i_b"], x, lay["i"].t()))
                d = torch.addmm(lay["out_b"], h, lay["out"].t())
                x = ops.ln_residual_f32(d, x, lay["ln2_w"], lay["ln2_b"], eps)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        return ops.mean_pool_l2(x, cu, normalize)

    def embed(self, texts: List[str], normalize: bool = True, dimensions: Optional[int] = None) -> List[List[float]]:
        if self.tokenizer is None:
            seqs = [[101] + [min(b + 1000, self.cfg.vocab_size - 1) for b in t.encode("utf-8")][:510] + [102]
                    for t in texts]
        else:
            seqs = [e.ids for e in self.tokenizer.encode_batch(texts, add_special_tokens=True)]
        out = self.forward_ids(seqs, normalize=normalize)
        if dimensions:
            out = out[:, :dimensions]
            out = out / out.norm(dim=1, keepdim=True).clamp_min(1e-12)
        return out.cpu().tolist()


def reference_embed(cfg: ModelConfig, sd: Dict[str, torch.Tensor], seqs: List[List[int]], normalize=True,
                    device="cpu") -> torch.Tensor:
    """fp32 PyTorch oracle: one sequence at a time (so no masking is involved)."""
    import torch.nn.functional as F

    sd = {_strip(k): v.float().to(device) for k, v in sd.items()}
    H, nh = cfg.hidden_size, cfg.num_heads
    hd = H // nh
    outs = []
    for s in seqs:
        L = len(s)
        ids = torch.tensor(s, device=device)
        x = sd["embeddings.word_embeddings.weight"][ids] + sd["embeddings.position_embeddings.weight"][:L] + \
            sd["embeddings.token_type_embeddings.weight"][0]
        x = F.layer_norm(x, (H,), sd["embeddings.LayerNorm.weight"], sd["embeddings.LayerNorm.bias"], cfg.layer_norm_eps)
        for i in range(cfg.num_layers):
            p = f"encoder.layer.{i}."

            def lin(t, n):
                return t @ sd[p + n + ".weight"].t() + sd[p + n + ".bias"]

            q = lin(x, "attention.self.query").view(L, nh, hd).transpose(0, 1)
            k = lin(x, "attention.self.key").view(L, nh, hd).transpose(0, 1)
            v = lin(x, "attention.self.value").view(L, nh, hd).transpose(0, 1)
            a = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(hd), -1) @ v
            a = a.transpose(0, 1).reshape(L, H)
            x = F.layer_norm(x + lin(a, "attention.output.dense"), (H,), sd[p + "attention.output.LayerNorm.weight"],
                             sd[p + "attention.output.LayerNorm.bias"], cfg.layer_norm_eps)
            h = F.gelu(lin(x, "intermediate.dense"))
            x = F.layer_norm(x + lin(h, "output.dense"), (H,), sd[p + "output.LayerNorm.weight"],
                             sd[p + "output.LayerNorm.bias"], cfg.layer_norm_eps)
        e = x.mean(0)
        if normalize:
            e = e / e.norm().clamp_min(1e-12)
        outs.append(e)
    return torch.stack(outs)
