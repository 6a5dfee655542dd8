"""Gemma4 text decoder on the paged engine (one GPU).

Per layer and step (executor/gemma4.rs DecoderLayer::forward :892-910):

    qkv  = gemm(y, W_qkv)                         q | k | v (no v rows when k = v)
    gemma_qkv_write: q/k RMSNorm * w, v RMSNorm, RoPE on the first `rot`
                     dims -> q, and K / V into this layer's KV pages
    attn = wide paged attention (head_dim 256 sliding / 512 global, scale 1,
           soft-capped scores, window of `sliding_window` keys on sliding layers)
    o    = gemm(attn, W_o)
    y    = residual_norm: x += rmsnorm(o) * w_post_attn;  y = rmsnorm(x) * w_pre_ff
    act  = gemm(y, W_gate_up) with the GeGLU epilogue (gelu_tanh(gate) * up)
    m    = gemm(act, W_down)
    y    = residual_norm: x = (x + rmsnorm(m) * w_post_ff) * layer_scalar;
           y = rmsnorm(x) * (next layer's input norm, or the final norm)

The embedding is scaled by sqrt(hidden) (Model::forward :1043), the lm_head
is the tied embedding and the logits are soft-capped (:1055-1061).

KV cache: bf16 [L, NB, E] (E = the widest layer's 2 * KVH * 16 * D), so the
block tables, prefix cache, swap and KV export of the engine work unchanged;
each layer uses the first 2 * KVH_l * 16 * D_l elements of its slots.

Tensor parallelism is not supported for this family (the global layers have
a single KV head in the reference's defaults); the model runs on one GPU.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

from .. import ops
from .config import ModelConfig
from .llama import StepInputs, TPInfo
from .reference import GEMMA4_PREFIX


class Gemma4LM:
    """Weights + forward of a Gemma4 text model on one GPU."""

    wide_attention = True  # the runner leaves the KV layout and decode splits to the model

    def __init__(self, cfg: ModelConfig, tp: Optional[TPInfo] = None, device=None):
        if cfg.arch != "gemma4":
            raise ValueError(f"Gemma4LM needs a gemma4 config, not {cfg.arch!r}")
        self.tp = tp or TPInfo()
        if self.tp.size != 1:
            raise ValueError("Gemma4 runs on one GPU (tensor parallelism is not supported for this family)")
        dev = torch.device(device) if device is not None else torch.device("cuda")
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.cfg = cfg
        self.device = dev
        self.nq = cfg.num_heads
        self.nkv = cfg.num_kv_heads
        self.vocab_local = cfg.vocab_size
        self.moe = None
        self.offloaded = False
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.embed: Optional[torch.Tensor] = None
        self.final_norm: Optional[torch.Tensor] = None
        # per-layer geometry: (head_dim, kv heads, rotary dims, sliding window, k = v)
        self.geo = []
        for i in range(cfg.num_layers):
            d, kvh = cfg.layer_attn(i)
            sliding = cfg.is_sliding(i)
            rot = d if sliding else int(d * cfg.partial_rotary_factor)
            rot -= rot % 2
            self.geo.append((d, kvh, rot, cfg.sliding_window if sliding else 0,
                             bool(cfg.attention_k_eq_v and not sliding)))
        self.kv_elems = max(2 * kvh * 16 * d for d, kvh, *_ in self.geo)
        self.embed_scale = math.sqrt(cfg.hidden_size)
        self.cos_sin: Dict[int, torch.Tensor] = {}
        self._ws: Optional[torch.Tensor] = None
        self._max_kv = 0

    # ------------------------------------------------------------ KV layout (used by the runner)
    def kv_cache_shape(self, num_blocks: int):
        return (self.cfg.num_layers, num_blocks, self.kv_elems)

    def kv_block_bytes(self) -> int:
        return self.cfg.num_layers * self.kv_elems * 2

    def prepare_runner(self, max_num_seqs: int, q_len: int, max_blocks: int) -> None:
        """Size the split-K workspace of decode attention for the runner's
        largest decode step (allocated once, before any graph capture)."""
        self._max_kv = max_blocks * 16
        dev = self.device.index or 0
        need = 1
        for d, kvh, _, window, _ in set(self.geo):
            for b in range(1, max_num_seqs + 1):  # eager steps may have any decode count
                sb = ops.wide_decode_splits(b, self.nq, kvh, d, q_len, self._max_kv, window, dev)
                need = max(need, ops.wide_decode_workspace_numel(b, self.nq, kvh, d, q_len, sb))
        self._ws = torch.empty(need, dtype=torch.float32, device=self.device)

    # ------------------------------------------------------------ weights
    def _get(self, full: Dict[str, torch.Tensor], name: str) -> torch.Tensor:
        for pre in (GEMMA4_PREFIX, "model."):
            if pre + name in full:
                return full[pre + name]
        raise KeyError(f"missing Gemma4 weight {GEMMA4_PREFIX + name}")

    def shard_full(self, full: Dict[str, torch.Tensor]) -> None:
        """Install HF-named weights (model.language_model.* or model.*)."""
        cfg, dev, bf = self.cfg, self.device, torch.bfloat16
        g = lambda n: self._get(full, n).to(dev, bf).contiguous()  # noqa: E731
        self.embed = g("embed_tokens.weight")
        self.final_norm = g("norm.weight")
        self.layers = []
        for i in range(cfg.num_layers):
            p = f"layers.{i}."
            d, kvh, rot, window, k_eq_v = self.geo[i]
            rows = [g(p + "self_attn.q_proj.weight"), g(p + "self_attn.k_proj.weight")]
            if not k_eq_v:
                rows.append(g(p + "self_attn.v_proj.weight"))
            lay = {
                "qkv": torch.cat(rows, 0).contiguous(),
                "o": g(p + "self_attn.o_proj.weight"),
                "q_norm": g(p + "self_attn.q_norm.weight"),
                "k_norm": g(p + "self_attn.k_norm.weight"),
                "ln_in": g(p + "input_layernorm.weight"),
                "ln_post_attn": g(p + "post_attention_layernorm.weight"),
                "ln_pre_ff": g(p + "pre_feedforward_layernorm.weight"),
                "ln_post_ff": g(p + "post_feedforward_layernorm.weight"),
                "gate_up": ops.interleave_gate_up(g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")),
                "down": g(p + "mlp.down_proj.weight"),
            }
            try:
                lay["scalar"] = float(self._get(full, p + "layer_scalar").float().reshape(-1)[0])
            except KeyError:
                lay["scalar"] = 1.0
            self.layers.append(lay)
        self._finish()

    def random_init(self, seed: int = 0, std: float = 0.02) -> None:
        from .reference import gemma4_random_weights

        self.shard_full(gemma4_random_weights(self.cfg, seed, std, self.device))

    def _finish(self) -> None:
        cfg = self.cfg
        for d, kvh, rot, window, _ in self.geo:
            key = (rot, d, window > 0)
            if key not in self.cos_sin:
                theta = cfg.rope_local_theta if window > 0 else cfg.rope_theta
                self.cos_sin[key] = ops.wide_cos_sin(cfg.max_position_embeddings, rot, d, theta, self.device)

    def gemm_shapes(self):
        cfg, H = self.cfg, self.cfg.hidden_size
        shapes = {(self.vocab_local, H, False), (2 * cfg.intermediate_size, H, True), (H, cfg.intermediate_size, False)}
        for d, kvh, _, _, k_eq_v in self.geo:
            shapes |= {((self.nq + kvh * (1 if k_eq_v else 2)) * d, H, False), (H, self.nq * d, False)}
        return sorted(shapes)

    def weight_bytes(self) -> int:
        n = sum(t.numel() * t.element_size() for lay in self.layers for t in lay.values()
                if isinstance(t, torch.Tensor))
        return n + sum(t.numel() * t.element_size() for t in (self.embed, self.final_norm) if t is not None)

    # ------------------------------------------------------------ forward
    def _workspace(self, need: int) -> torch.Tensor:
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.float32, device=self.device)
        return self._ws

    def forward(self, s: StepInputs, kv_cache: torch.Tensor, trace=None) -> torch.Tensor:
        """Final-normed hidden states of the logits rows [NL, H] (bf16).
        trace: an optional list that receives the residual stream after every
        sub-layer (debugging against the oracle)."""
        cfg = self.cfg
        T = s.input_ids.shape[0]
        Bd, ql = s.num_decode, s.decode_q_len
        Td = Bd * ql
        eps = cfg.rms_norm_eps
        cap = float(cfg.attn_logit_softcapping or 0.0)
        emb = ops.embedding(s.input_ids, self.embed)
        x = torch.empty_like(emb)
        y = ops.residual_norm(emb, x, None, self.layers[0]["ln_in"], in_scale=self.embed_scale, eps=eps)
        max_kv = s.decode_block_table.shape[1] * 16 if Bd else 0
        for li, lay in enumerate(self.layers):
            d, kvh, rot, window, k_eq_v = self.geo[li]
            kv = kv_cache[li]
            qkv = ops.gemm(y, lay["qkv"])
            q = torch.empty(T, self.nq, d, dtype=torch.bfloat16, device=self.device)
            ops.gemma_qkv_write(qkv, s.positions, s.slot_mapping, self.cos_sin[(rot, d, window > 0)], q, kv, self.nq,
                                kvh, rot, lay["q_norm"], lay["k_norm"], eps, k_eq_v)
            attn = torch.empty_like(q)
            if Bd > 0:
                splits = ops.wide_decode_splits(Bd, self.nq, kvh, d, ql, max_kv, window, self.device.index or 0)
                ws = None
                if splits > 1:
                    ws = self._workspace(ops.wide_decode_workspace_numel(Bd, self.nq, kvh, d, ql, splits))
                ops.wide_decode_attention(q[:Td], kv, kvh, s.decode_block_table, s.decode_seq_lens, attn[:Td],
                                          q_len=ql, window=window, scale=1.0, softcap=cap, splits=splits,
                                          workspace=ws)
            if s.num_prefill > 0:
                ops.wide_prefill_attention(q[Td:], kv, kvh, s.prefill_block_table, s.prefill_ctx_lens,
                                           s.prefill_cu_q, s.tile_seq, s.tile_start, attn[Td:], window=window,
                                           scale=1.0, softcap=cap)
            o = ops.gemm(attn.view(T, self.nq * d), lay["o"])
            y = ops.residual_norm(o, x, lay["ln_post_attn"], lay["ln_pre_ff"], eps=eps)
            if trace is not None:
                trace.append(x.float().clone())
            act = ops.gemm(y, lay["gate_up"], epi=ops.EPI_GEGLU)
            m = ops.gemm(act, lay["down"])
            nxt = self.layers[li + 1]["ln_in"] if li + 1 < len(self.layers) else self.final_norm
            y = ops.residual_norm(m, x, lay["ln_post_ff"], nxt, out_scale=lay["scalar"], eps=eps)
            if trace is not None:
                trace.append(x.float().clone())
        return y.index_select(0, s.logits_rows)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """[NL, V] bf16, soft-capped when the config asks for it."""
        out = ops.gemm(h, self.embed)
        if self.cfg.final_logit_softcapping:
            ops.softcap_(out, float(self.cfg.final_logit_softcapping))
        return out
