"""Decoder-only transformer (Llama / Mistral / Qwen2 / Qwen3 and the MoE
variant) running on this repository's sm_100a kernels.

Per layer and step (T tokens: decode rows first, then chunked-prefill rows):

    qkv   = gemm(x, W_qkv) (+bias)                      tcgen05 GEMM
    q     = rope_kv_write(qkv) -> paged KV pages         RoPE (+q/k RMSNorm) fused with the KV write
    attn  = paged_decode_attention(q[:Bd*ql]) | paged_prefill_attention(q[Bd*ql:])
            (ql = 1 + proposals per sequence when verifying speculative tokens)
    o     = gemm(attn, W_o)                              (split-K fp32 partials on small batches)
    x     = add_rmsnorm(o -> residual)                   [tensor parallel: reduce across ranks]
    act   = gemm(x, W_gate_up, epilogue=SwiGLU)          gate/up rows interleaved, SwiGLU in the epilogue
    d     = gemm(act, W_down)
    x     = add_rmsnorm(d -> residual)

Weights live in the kernels' layout: fused QKV rows, interleaved gate/up
rows, nn.Linear [out, in] K-major matrices.  Tensor parallelism shards heads,
FFN columns and the vocabulary (Megatron column/row split); KV heads are
replicated when there are fewer KV heads than ranks.

Reference model semantics: candle-transformers llama/qwen2/qwen3 used by
crates/engine/src/executor/candle.rs:1461-1796 and the streaming Qwen model
(qwen_streaming.rs:300-801: RMSNorm, rotary, GQA attention, SwiGLU MLP,
last-position lm_head).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from .. import ops
from .config import ModelConfig

# Row-parallel GEMMs push their partial rows to the owning ranks from the
# epilogue (reduce-scatter fused into the GEMM); 0 keeps the pull variant.
_TP_PUSH = os.environ.get("BLOOM_TP_PUSH", "1") != "0"
# the fused all-gather leaves the wait for the peers' rows to the next GEMM
_TP_DEFER = os.environ.get("BLOOM_TP_DEFER", "1") != "0"


@dataclass
class StepInputs:
    """Device views of one engine step (see the scheduler's arena layout)."""

    input_ids: torch.Tensor  # [T] int32
    positions: torch.Tensor  # [T] int64
    slot_mapping: torch.Tensor  # [T] int32
    num_decode: int
    decode_block_table: Optional[torch.Tensor]  # [Bd, MB]
    decode_seq_lens: Optional[torch.Tensor]  # [Bd]
    decode_splits: int
    decode_workspace: Optional[torch.Tensor]
    num_prefill: int
    prefill_block_table: Optional[torch.Tensor]
    prefill_ctx_lens: Optional[torch.Tensor]
    prefill_cu_q: Optional[torch.Tensor]
    tile_seq: Optional[torch.Tensor]
    tile_start: Optional[torch.Tensor]
    logits_rows: torch.Tensor  # [NL] int32
    decode_q_len: int = 1


@dataclass
class TPInfo:
    rank: int = 0
    size: int = 1
    group: object = None
    comm: object = None  # bloom_b200.parallel.comm.Communicator


def _local_heads(cfg: ModelConfig, tp: int, rank: int):
    assert cfg.num_heads % tp == 0, "num_heads must divide by the TP size"
    nq = cfg.num_heads // tp
    if cfg.num_kv_heads >= tp:
        assert cfg.num_kv_heads % tp == 0
        nkv = cfg.num_kv_heads // tp
        kv0 = rank * nkv
    else:  # replicate KV heads: ranks sharing one KV head hold a copy
        assert tp % cfg.num_kv_heads == 0
        nkv = 1
        kv0 = rank // (tp // cfg.num_kv_heads)
    return nq, nkv, rank * nq, kv0


class DecoderLM:
    """Weights + forward of a decoder LM shard on one GPU."""

    def __init__(self, cfg: ModelConfig, tp: Optional[TPInfo] = None, device=None, pp=None):
        self.cfg = cfg
        self.tp = tp or TPInfo()
        # pipeline stage (parallel.pipeline.PPInfo): this process holds layers [l0, l1)
        self.pp = pp if (pp is not None and pp.stages > 1) else None
        self.l0, self.l1 = 0, cfg.num_layers
        if self.pp is not None:
            from ..parallel.pipeline import layer_range

            if self.tp.size != 1 or cfg.is_moe:
                raise ValueError("pipeline stages run dense models at TP=1")
            self.l0, self.l1 = layer_range(cfg.num_layers, self.pp.stage, self.pp.stages)
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.nq, self.nkv, self.q0, self.kv0 = _local_heads(cfg, self.tp.size, self.tp.rank)
        assert cfg.intermediate_size % (16 * self.tp.size) == 0 or cfg.is_moe
        self.inter = cfg.intermediate_size // self.tp.size
        self.vocab_local = cfg.vocab_size // self.tp.size
        assert cfg.vocab_size % self.tp.size == 0, "vocab must divide by the TP size"
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.embed: Optional[torch.Tensor] = None
        self.final_norm: Optional[torch.Tensor] = None
        self.lm_head: Optional[torch.Tensor] = None
        self.cos_sin: Optional[torch.Tensor] = None
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.moe = None  # set by qwen3_moe

    # ------------------------------------------------------------ weights
    def shard_full(self, full: Dict[str, torch.Tensor]) -> None:
        """Install weights from full (unsharded) HF-named tensors of one layer set.

        Expected names (HF Llama convention, layer index i):
          model.embed_tokens.weight, model.norm.weight, lm_head.weight,
          model.layers.{i}.input_layernorm.weight, .post_attention_layernorm.weight,
          .self_attn.{q,k,v,o}_proj.weight (+ q/k/v bias), .self_attn.{q,k}_norm.weight,
          .mlp.{gate,up,down}_proj.weight
        """
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        r, t = self.tp.rank, self.tp.size
        hd = cfg.head_dim

        def get(name):
            return full[name]

        self.embed = get("model.embed_tokens.weight").to(dev, bf).contiguous()
        self.final_norm = get("model.norm.weight").to(dev, bf).contiguous()
        lm = full.get("lm_head.weight", full["model.embed_tokens.weight"])
        V = cfg.vocab_size
        self.lm_head = lm[r * V // t:(r + 1) * V // t].to(dev, bf).contiguous()
        self.layers = []
        for i in range(self.l0, self.l1):
            p = f"model.layers.{i}."
            q = get(p + "self_attn.q_proj.weight")[self.q0 * hd:(self.q0 + self.nq) * hd]
            k = get(p + "self_attn.k_proj.weight")[self.kv0 * hd:(self.kv0 + self.nkv) * hd]
            v = get(p + "self_attn.v_proj.weight")[self.kv0 * hd:(self.kv0 + self.nkv) * hd]
            layer = {
                "ln1": get(p + "input_layernorm.weight").to(dev, bf).contiguous(),
                "ln2": get(p + "post_attention_layernorm.weight").to(dev, bf).contiguous(),
                "qkv": torch.cat([q, k, v], 0).to(dev, bf).contiguous(),
                "o": get(p + "self_attn.o_proj.weight")[:, self.q0 * hd:(self.q0 + self.nq) * hd].to(dev, bf)
                .contiguous(),
            }
            if cfg.qkv_bias:
                qb = get(p + "self_attn.q_proj.bias")[self.q0 * hd:(self.q0 + self.nq) * hd]
                kb = get(p + "self_attn.k_proj.bias")[self.kv0 * hd:(self.kv0 + self.nkv) * hd]
                vb = get(p + "self_attn.v_proj.bias")[self.kv0 * hd:(self.kv0 + self.nkv) * hd]
                layer["qkv_b"] = torch.cat([qb, kb, vb]).to(dev, bf).contiguous()
            if cfg.qk_norm:
                layer["q_norm"] = get(p + "self_attn.q_norm.weight").to(dev, bf).contiguous()
                layer["k_norm"] = get(p + "self_attn.k_norm.weight").to(dev, bf).contiguous()
            if not cfg.is_moe:
                I = self.inter
                g = get(p + "mlp.gate_proj.weight")[r * I:(r + 1) * I]
                u = get(p + "mlp.up_proj.weight")[r * I:(r + 1) * I]
                layer["gate_up"] = ops.interleave_gate_up(g.to(dev, bf), u.to(dev, bf))
                layer["down"] = get(p + "mlp.down_proj.weight")[:, r * I:(r + 1) * I].to(dev, bf).contiguous()
            self.layers.append(layer)
        if cfg.is_moe:
            from .qwen3_moe import MoEBlock

            self.moe = MoEBlock(self, full)
        self._finish()

    def load_gguf(self, path: str, quantized: bool = True) -> None:
        """Install a GGUF decoder (TP=1).  With `quantized`, the Q8_0 / Q4_0
        projection weights stay block-quantised in HBM (bit-exact GGUF blocks,
        rows reordered exactly as the float path: q/k RoPE rows un-permuted,
        q|k|v concatenated, gate/up interleaved); norms, embeddings and other
        types are dequantised to bf16."""
        import numpy as np

        from ..formats.gguf import GGUFFile, gguf_name_to_hf, unpermute_qk

        assert self.tp.size == 1, "quantised GGUF weights are served at TP=1"
        g = GGUFFile(path)
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        lin = ("q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight", "gate_proj.weight",
               "up_proj.weight", "down_proj.weight")
        rows: Dict[str, tuple] = {}
        full: Dict[str, torch.Tensor] = {}
        for name, t in g.tensors.items():
            hf = gguf_name_to_hf(name)
            if hf is None:
                continue
            if quantized and hf.endswith(lin) and t.type_name in ("Q8_0", "Q4_0"):
                N, K = t.shape
                r = torch.from_numpy(np.ascontiguousarray(g.raw(name))).view(N, -1)
                if g.arch == "llama" and (name.endswith("attn_q.weight") or name.endswith("attn_k.weight")):
                    r = unpermute_qk(r, g._heads_for(name)).contiguous()
                rows[hf] = (t.type_name, r, K)
            else:
                full[hf] = g.tensor(name)
        self.embed = full["model.embed_tokens.weight"].to(dev, bf).contiguous()
        self.final_norm = full["model.norm.weight"].to(dev, bf).contiguous()
        self.lm_head = full.get("lm_head.weight", full["model.embed_tokens.weight"]).to(dev, bf).contiguous()

        def weight(name):
            if name in rows:
                kind, r, K = rows[name]
                return ops.QWeight.from_rows(kind, r, K, dev)
            return full[name].to(dev, bf).contiguous()

        def cat_rows(names):
            if all(n in rows for n in names) and len({rows[n][0] for n in names}) == 1:
                kind, K = rows[names[0]][0], rows[names[0]][2]
                return ops.QWeight.from_rows(kind, torch.cat([rows[n][1] for n in names], 0), K, dev)
            return torch.cat([(weight(n).dequantize() if n in rows else weight(n)) for n in names], 0).contiguous()

        self.layers = []
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            layer = {"ln1": full[p + "input_layernorm.weight"].to(dev, bf).contiguous(),
                     "ln2": full[p + "post_attention_layernorm.weight"].to(dev, bf).contiguous(),
                     "qkv": cat_rows([p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                                      p + "self_attn.v_proj.weight"]),
                     "o": weight(p + "self_attn.o_proj.weight")}
            if cfg.qkv_bias:
                layer["qkv_b"] = torch.cat([full[p + f"self_attn.{x}_proj.bias"] for x in "qkv"]).to(dev, bf)
            if cfg.qk_norm:
                layer["q_norm"] = full[p + "self_attn.q_norm.weight"].to(dev, bf).contiguous()
                layer["k_norm"] = full[p + "self_attn.k_norm.weight"].to(dev, bf).contiguous()
            gn, un = p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"
            if gn in rows and un in rows and rows[gn][0] == rows[un][0]:
                kind, K = rows[gn][0], rows[gn][2]
                layer["gate_up"] = ops.QWeight.from_rows(kind, ops.interleave_gate_up(rows[gn][1], rows[un][1]), K, dev)
            else:
                gw = weight(gn)
                uw = weight(un)
                gw = gw.dequantize() if isinstance(gw, ops.QWeight) else gw
                uw = uw.dequantize() if isinstance(uw, ops.QWeight) else uw
                layer["gate_up"] = ops.interleave_gate_up(gw, uw)
            layer["down"] = weight(p + "mlp.down_proj.weight")
            self.layers.append(layer)
        self._finish()

    def quantize_weights(self, kind: str = "Q8_0") -> None:
        """Re-store the projection weights as GGUF blocks on the device (round
        to nearest), e.g. to serve a bf16 checkpoint in Q8_0 / Q4_0."""
        assert self.tp.size == 1
        for lay in self.layers:
            for k in ("qkv", "o", "gate_up", "down"):
                if k in lay and not isinstance(lay[k], ops.QWeight):
                    lay[k] = ops.QWeight.quantize(lay[k], kind, self.device)
        torch.cuda.empty_cache()

    def random_init(self, seed: int = 0, std: float = 0.02) -> None:
        """N(0, std) weights (norms = 1) generated as full tensors from one seeded
        stream and then sharded, so every TP size holds the same model."""
        cfg = self.cfg
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        bf = torch.bfloat16

        def randn(*shape):
            return (torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32) * std).to(bf)

        H, hd = cfg.hidden_size, cfg.head_dim
        full: Dict[str, torch.Tensor] = {}
        full["model.embed_tokens.weight"] = randn(cfg.vocab_size, H)
        full["model.norm.weight"] = torch.ones(H, dtype=bf, device=self.device)
        if not cfg.tie_word_embeddings:
            full["lm_head.weight"] = randn(cfg.vocab_size, H)
        self.layers = []
        # generate and install layer by layer to bound peak memory
        r, t = self.tp.rank, self.tp.size
        V = cfg.vocab_size
        self.embed = full["model.embed_tokens.weight"]
        self.final_norm = full["model.norm.weight"]
        lm = full.get("lm_head.weight", self.embed)
        self.lm_head = lm[r * V // t:(r + 1) * V // t].contiguous()
        if "lm_head.weight" in full:
            del full["lm_head.weight"]
        if cfg.is_moe:
            from .qwen3_moe import MoEBlock

            self.moe = MoEBlock(self)
        for i in range(cfg.num_layers):
            p = f"model.layers.{i}."
            lay = {
                p + "input_layernorm.weight": torch.ones(H, dtype=bf, device=self.device),
                p + "post_attention_layernorm.weight": torch.ones(H, dtype=bf, device=self.device),
                p + "self_attn.q_proj.weight": randn(cfg.q_size, H),
                p + "self_attn.k_proj.weight": randn(cfg.kv_size, H),
                p + "self_attn.v_proj.weight": randn(cfg.kv_size, H),
                p + "self_attn.o_proj.weight": randn(H, cfg.q_size),
            }
            if cfg.qkv_bias:
                lay[p + "self_attn.q_proj.bias"] = randn(cfg.q_size)
                lay[p + "self_attn.k_proj.bias"] = randn(cfg.kv_size)
                lay[p + "self_attn.v_proj.bias"] = randn(cfg.kv_size)
            if cfg.qk_norm:
                lay[p + "self_attn.q_norm.weight"] = torch.ones(hd, dtype=bf, device=self.device)
                lay[p + "self_attn.k_norm.weight"] = torch.ones(hd, dtype=bf, device=self.device)
            if cfg.is_moe:
                E, Im = cfg.num_experts, cfg.moe_intermediate_size
                lay[p + "mlp.gate.weight"] = randn(E, H)
                lay[p + "mlp.experts.gate_proj"] = randn(E, Im, H)
                lay[p + "mlp.experts.up_proj"] = randn(E, Im, H)
                lay[p + "mlp.experts.down_proj"] = randn(E, H, Im)
            else:
                lay[p + "mlp.gate_proj.weight"] = randn(cfg.intermediate_size, H)
                lay[p + "mlp.up_proj.weight"] = randn(cfg.intermediate_size, H)
                lay[p + "mlp.down_proj.weight"] = randn(H, cfg.intermediate_size)
            if self.l0 <= i < self.l1:  # every stage draws all layers: the same model at any stage count
                self._install_layer(i, lay, slot=i - self.l0)
            if cfg.is_moe:
                self.moe.add_layer(i, lay)
            del lay
        self._finish()

    def random_init_flat(self, seed: int = 0, std: float = 0.02) -> None:
        """N(0, std) weights (norms = 1) in this shard's final layout, drawn by
        ONE normal fill over a flat buffer that every projection is a view of
        (128-element aligned, so every view is a 16-byte aligned TMA operand).
        Three device launches in all, instead of several per tensor; the
        values differ from `random_init` and from one TP size to another.
        Dense decoders only."""
        if self.cfg.is_moe:
            raise NotImplementedError("random_init_flat covers dense decoders; use random_init for MoE")
        if self.pp is not None:
            raise NotImplementedError("pipeline stages load with random_init or shard_full")
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        H, hd = cfg.hidden_size, cfg.head_dim
        qkv_rows = (self.nq + 2 * self.nkv) * hd
        shapes = [("embed", (cfg.vocab_size, H))]
        if not cfg.tie_word_embeddings:
            shapes.append(("lm_head", (self.vocab_local, H)))
        per_layer = [("qkv", (qkv_rows, H)), ("o", (H, self.nq * hd)), ("gate_up", (2 * self.inter, H)),
                     ("down", (H, self.inter))]
        if cfg.qkv_bias:
            per_layer.append(("qkv_b", (qkv_rows,)))
        for i in range(cfg.num_layers):
            shapes += [(f"{i}.{n}", sh) for n, sh in per_layer]

        def numel(sh):
            n = 1
            for d in sh:
                n *= d
            return n

        align = 128
        total = sum((numel(sh) + align - 1) // align * align for _, sh in shapes)
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        flat = torch.empty(total, dtype=bf, device=dev).normal_(0.0, std, generator=g)
        views: Dict[str, torch.Tensor] = {}
        off = 0
        for name, sh in shapes:
            n = numel(sh)
            views[name] = flat[off:off + n].view(sh)
            off += (n + align - 1) // align * align
        nnorm = (2 * cfg.num_layers + 1) * H + (2 * cfg.num_layers * hd if cfg.qk_norm else 0)
        ones = torch.ones(nnorm, dtype=bf, device=dev)
        self._flat = (flat, ones)
        self.embed = views["embed"]
        self.lm_head = views["lm_head"] if "lm_head" in views else views["embed"][
            self.tp.rank * self.vocab_local:(self.tp.rank + 1) * self.vocab_local]
        o = 0

        def norm_w(n):
            nonlocal o
            t = ones[o:o + n]
            o += n
            return t

        self.final_norm = norm_w(H)
        self.layers = []
        for i in range(cfg.num_layers):
            lay = {"ln1": norm_w(H), "ln2": norm_w(H), "qkv": views[f"{i}.qkv"], "o": views[f"{i}.o"],
                   "gate_up": views[f"{i}.gate_up"], "down": views[f"{i}.down"]}
            if cfg.qkv_bias:
                lay["qkv_b"] = views[f"{i}.qkv_b"]
            if cfg.qk_norm:
                lay["q_norm"] = norm_w(hd)
                lay["k_norm"] = norm_w(hd)
            self.layers.append(lay)
        self._finish()

    def _install_layer(self, i: int, lay: Dict[str, torch.Tensor], slot: Optional[int] = None) -> None:
        """Install global layer i (weight names) at position `slot` (default i) of self.layers."""
        cfg, hd, bf = self.cfg, self.cfg.head_dim, torch.bfloat16
        r = self.tp.rank
        p = f"model.layers.{i}."
        q = lay[p + "self_attn.q_proj.weight"][self.q0 * hd:(self.q0 + self.nq) * hd]
        k = lay[p + "self_attn.k_proj.weight"][self.kv0 * hd:(self.kv0 + self.nkv) * hd]
        v = lay[p + "self_attn.v_proj.weight"][self.kv0 * hd:(self.kv0 + self.nkv) * hd]
        layer = {
            "ln1": lay[p + "input_layernorm.weight"].to(self.device, bf).contiguous(),
            "ln2": lay[p + "post_attention_layernorm.weight"].to(self.device, bf).contiguous(),
            "qkv": torch.cat([q, k, v], 0).to(self.device, bf).contiguous(),
            "o": lay[p + "self_attn.o_proj.weight"][:, self.q0 * hd:(self.q0 + self.nq) * hd]
            .to(self.device, bf).contiguous(),
        }
        if cfg.qkv_bias:
            layer["qkv_b"] = torch.cat([
                lay[p + "self_attn.q_proj.bias"][self.q0 * hd:(self.q0 + self.nq) * hd],
                lay[p + "self_attn.k_proj.bias"][self.kv0 * hd:(self.kv0 + self.nkv) * hd],
                lay[p + "self_attn.v_proj.bias"][self.kv0 * hd:(self.kv0 + self.nkv) * hd]]).to(self.device, bf)
        if cfg.qk_norm:
            layer["q_norm"] = lay[p + "self_attn.q_norm.weight"].to(self.device, bf).contiguous()
            layer["k_norm"] = lay[p + "self_attn.k_norm.weight"].to(self.device, bf).contiguous()
        if not cfg.is_moe:
            I = self.inter
            g = lay[p + "mlp.gate_proj.weight"][r * I:(r + 1) * I].to(self.device, bf)
            u = lay[p + "mlp.up_proj.weight"][r * I:(r + 1) * I].to(self.device, bf)
            layer["gate_up"] = ops.interleave_gate_up(g, u)
            layer["down"] = lay[p + "mlp.down_proj.weight"][:, r * I:(r + 1) * I].to(self.device, bf).contiguous()
        slot = i if slot is None else slot
        if len(self.layers) <= slot:
            self.layers.append(layer)
        else:
            self.layers[slot] = layer

    # ------------------------------------------------------------ layer placement
    def place_layers(self, gpu_layers: int) -> None:
        """Keep layers [0, gpu_layers) in HBM; the other layers' projection
        weights move to pinned host memory and are streamed, one layer ahead,
        into two HBM staging slots on a copy stream while the previous layer
        computes (every layer still runs on this GPU's kernels).  For models
        larger than the device memory left after the KV cache.  Reference:
        LayerPlacementStrategy (crates/engine/src/core/memory.rs:484-533),
        which computes the non-GPU layers on the CPU instead."""
        n = len(self.layers)
        g = max(0, min(int(gpu_layers), n))
        self.host_layers = list(range(g, n))
        if not self.host_layers:
            return
        keys = ("qkv", "o", "gate_up", "down")
        for i in self.host_layers:
            for k in keys:
                t = self.layers[i].get(k)
                if isinstance(t, torch.Tensor) and t.is_cuda:
                    self.layers[i][k] = t.cpu().pin_memory()
        ref = self.layers[self.host_layers[0]]
        self._slots = [{k: torch.empty_like(ref[k], device=self.device) for k in keys if k in ref} for _ in range(2)]
        self._copy_stream = torch.cuda.Stream(self.device)
        self._ready = [torch.cuda.Event() for _ in range(2)]
        self._done = [torch.cuda.Event() for _ in range(2)]
        self._pending = -1  # host layer whose copy was issued ahead
        torch.cuda.empty_cache()

    @property
    def offloaded(self) -> bool:
        return bool(getattr(self, "host_layers", None))

    def _stage(self, li: int) -> None:
        """Queue the copy of host layer li into its slot (after the slot's last user finished)."""
        j = self.host_layers.index(li)
        s = j & 1
        with torch.cuda.stream(self._copy_stream):
            self._copy_stream.wait_event(self._done[s])
            for k, dst in self._slots[s].items():
                dst.copy_(self.layers[li][k], non_blocking=True)
            self._ready[s].record(self._copy_stream)
        self._pending = li

    def _layer(self, li: int) -> Dict[str, torch.Tensor]:
        lay = self.layers[li]
        if not self.offloaded or li not in self.host_layers:
            return lay
        j = self.host_layers.index(li)
        s = j & 1
        if self._pending != li:
            self._stage(li)
        torch.cuda.current_stream(self.device).wait_event(self._ready[s])
        if j + 1 < len(self.host_layers):
            self._stage(self.host_layers[j + 1])
        return dict(lay, **self._slots[s])

    def _release(self, li: int) -> None:
        if self.offloaded and li in self.host_layers:
            self._done[self.host_layers.index(li) & 1].record(torch.cuda.current_stream(self.device))

    def _finish(self) -> None:
        cfg = self.cfg
        self.cos_sin = ops.rope_cos_sin(cfg.max_position_embeddings, cfg.head_dim, cfg.rope_theta, self.device,
                                        cfg.rope_scaling)

    @property
    def num_kv_layers(self) -> int:
        """Layers whose KV pages this process holds (a pipeline stage holds its own)."""
        return self.l1 - self.l0

    def gemm_shapes(self):
        """(N, K, swiglu) of every distinct projection, for the GEMM autotuner."""
        cfg = self.cfg
        hd = cfg.head_dim
        shapes = {((self.nq + 2 * self.nkv) * hd, cfg.hidden_size, False), (cfg.hidden_size, self.nq * hd, False),
                  (self.vocab_local, cfg.hidden_size, False)}
        if not cfg.is_moe:
            shapes |= {(2 * self.inter, cfg.hidden_size, True), (cfg.hidden_size, self.inter, False)}
        return sorted(shapes)

    def weight_bytes(self) -> int:
        n = 0
        for lay in self.layers:
            n += sum(t.nbytes() if isinstance(t, ops.QWeight) else t.numel() * t.element_size() for t in lay.values())
        for t in (self.embed, self.final_norm, self.lm_head):
            if t is not None:
                n += t.numel() * t.element_size()
        if self.moe is not None:
            n += self.moe.weight_bytes()
        return n

    # ------------------------------------------------------------ forward
    def _reduce(self, t: torch.Tensor) -> torch.Tensor:
        """Sum a row-parallel output across TP ranks (bf16 [T, H] or f32 partials)."""
        if self.tp.size == 1:
            return t
        return self.tp.comm.all_reduce(t)

    def _row_parallel_norm(self, inp: torch.Tensor, w_mat: torch.Tensor, residual: torch.Tensor,
                           norm_w: torch.Tensor, eps: float, wait=None, next_w=None):
        """x = rmsnorm(residual += inp @ w_mat^T summed over TP ranks) * norm_w.

        Returns (x, wait): with the fused collective and a bf16 `next_w` (the
        weight of the GEMM that reads x next), the all-gather is deferred and
        `wait` must be passed to that GEMM; otherwise wait is None."""
        fused = self.tp.comm.fused if (self.tp.size > 1 and self.tp.comm is not None) else None
        if fused is not None:
            T = inp.shape[0]
            push = _TP_PUSH and isinstance(w_mat, torch.Tensor)
            defer = _TP_DEFER and isinstance(next_w, torch.Tensor)
            ops.gemm(inp, w_mat, fused.partial(T), push=fused.push_args(T) if push else None, wait=wait)
            x = fused.allreduce_rmsnorm(T, residual, norm_w, eps, pushed=push, defer=defer)
            return x, (fused.wait_args() if defer else None)
        d = self._reduce(ops.gemm(inp, w_mat, wait=wait))
        return ops.add_rmsnorm(d, residual, norm_w, eps), None

    def forward(self, s: StepInputs, kv_cache: torch.Tensor) -> torch.Tensor:
        """Returns the final-normed hidden states of the logits rows [NL, H] (bf16)."""
        cfg = self.cfg
        T = s.input_ids.shape[0]
        Bd = s.num_decode
        Td = Bd * s.decode_q_len  # decode / verify token rows come first
        H = cfg.hidden_size
        eps = cfg.rms_norm_eps
        dev = self.device
        if self.pp is not None and not self.pp.first:  # the previous stage's residual stream
            residual = self.pp.recv_prev(torch.empty(T, H, dtype=torch.bfloat16, device=dev))
        else:
            residual = ops.embedding(s.input_ids, self.embed)
        x = ops.rmsnorm(residual, self.layers[0]["ln1"], eps)
        qkv_dim = (self.nq + 2 * self.nkv) * cfg.head_dim
        wait = None  # a deferred all-gather the next GEMM must wait for
        L = len(self.layers)
        for li in range(L):
            lay = self._layer(li)
            qkv = ops.gemm(x, lay["qkv"], bias=lay.get("qkv_b"), wait=wait)
            wait = None
            q = torch.empty(T, self.nq, cfg.head_dim, dtype=torch.bfloat16, device=dev)
            ops.rope_kv_write(qkv, s.positions, s.slot_mapping, self.cos_sin, q, kv_cache, li, self.nq, self.nkv,
                              lay.get("q_norm"), lay.get("k_norm"), eps)
            attn = torch.empty_like(q)
            if Bd > 0:
                ops.paged_decode_attention(q[:Td], kv_cache, li, s.decode_block_table, s.decode_seq_lens, attn[:Td],
                                           q_len=s.decode_q_len, splits=s.decode_splits,
                                           workspace=s.decode_workspace, scale=self.scale)
            if s.num_prefill > 0:
                ops.paged_prefill_attention(q[Td:], kv_cache, li, s.prefill_block_table, s.prefill_ctx_lens,
                                            s.prefill_cu_q, s.tile_seq, s.tile_start, attn[Td:], scale=self.scale)
            a2 = attn.view(T, self.nq * cfg.head_dim)
            moe_router = self.moe.layers[li].get("router") if self.moe is not None else None
            x, wait = self._row_parallel_norm(a2, lay["o"], residual, lay["ln2"], eps,
                                              next_w=lay.get("gate_up") if self.moe is None else moe_router)
            nxt = (self.layers[li + 1]["ln1"] if li + 1 < len(self.layers) else
                   self.final_norm if self.pp is None or self.pp.last else lay["ln1"])  # the next stage renormalises
            if self.moe is not None:
                fused = self.tp.comm.fused if (self.tp.size > 1 and self.tp.comm is not None) else None
                if fused is not None:
                    # the combine pushes each token's row to its owner (like the dense push
                    # epilogue); the collective then reduces local slots only
                    push = _TP_PUSH
                    self.moe.forward(li, x, out=fused.partial(T), push=fused.push_args(T) if push else None,
                                     wait=wait)
                    nq_w = self.layers[li + 1].get("qkv") if (li + 1 < L and not self.offloaded) else None
                    defer = _TP_DEFER and isinstance(nq_w, torch.Tensor)
                    x = fused.allreduce_rmsnorm(T, residual, nxt, eps, pushed=push, defer=defer)
                    wait = fused.wait_args() if defer else None
                else:
                    d = self._reduce(self.moe.forward(li, x, wait=wait))
                    wait = None
                    x = ops.add_rmsnorm(d, residual, nxt, eps)
            else:
                act = ops.gemm(x, lay["gate_up"], epi=ops.EPI_SWIGLU, wait=wait)
                wait = None
                # the next layer's qkv GEMM can take the wait unless its layer is streamed in
                nq_w = self.layers[li + 1].get("qkv") if (li + 1 < L and not self.offloaded) else None
                x, wait = self._row_parallel_norm(act, lay["down"], residual, nxt, eps, next_w=nq_w)
            self._release(li)
        if self.pp is not None and not self.pp.last:
            self.pp.send_next(residual)
            return None
        return x.index_select(0, s.logits_rows)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """Local vocab shard of the logits [NL, V/tp] (bf16)."""
        return ops.gemm(h, self.lm_head)
