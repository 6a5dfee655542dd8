"""Sparse MoE feed-forward (Qwen3-MoE: top-k softmax router, SwiGLU experts).

Per layer and step, on every rank (experts sharded over the expert-parallel
group = the tensor-parallel ranks; E_local = E / ranks):
    logits = gemm(x, W_router) f32                     (router replicated)
    route:   softmax -> top-k -> renormalise -> slots of this rank's experts
    plan:    expert row offsets + grouped-GEMM tile lists (on the device)
    gather:  routed token rows into per-expert segments
    act  = grouped gemm(x_sorted, W_gate_up[e]) with SwiGLU epilogue
    y    = grouped gemm(act, W_down[e])
    out  = combine: sum_k w_k * y  -> this rank's partial of the MoE output
The partials of all ranks are summed by the same fused reduce-scatter +
residual + RMSNorm + all-gather kernel the dense layers use.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch

from .. import ops
from .._ext import cuda as _C


class MoEBlock:
    def __init__(self, model, full: Optional[Dict[str, torch.Tensor]] = None):
        cfg = model.cfg
        self.model = model
        self.cfg = cfg
        self.E = cfg.num_experts
        self.K = cfg.num_experts_per_tok
        self.I = cfg.moe_intermediate_size
        self.H = cfg.hidden_size
        ep = model.tp.size
        assert self.E % ep == 0, "experts must divide by the expert-parallel size"
        self.El = self.E // ep
        self.e0 = model.tp.rank * self.El
        self.dev = model.device
        self.layers: List[Dict[str, torch.Tensor]] = []
        self.counts = torch.zeros(self.El, dtype=torch.int32, device=self.dev)
        self.offsets = torch.zeros(self.El + 1, dtype=torch.int32, device=self.dev)
        self.n_gu = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.n_d = torch.zeros(1, dtype=torch.int32, device=self.dev)
        if full is not None:
            for i in range(cfg.num_layers):
                self.add_layer(i, full)

    def add_layer(self, i: int, full: Dict[str, torch.Tensor]) -> None:
        p = f"model.layers.{i}.mlp."
        bf, dev = torch.bfloat16, self.dev
        e0, e1 = self.e0, self.e0 + self.El
        g = full[p + "experts.gate_proj"][e0:e1].to(dev, bf)  # [El, I, H]
        u = full[p + "experts.up_proj"][e0:e1].to(dev, bf)
        gu = torch.stack([ops.interleave_gate_up(g[e], u[e]) for e in range(self.El)])  # [El, 2I, H]
        d = full[p + "experts.down_proj"][e0:e1].to(dev, bf)  # [El, H, I]
        lay = {"router": full[p + "gate.weight"].to(dev, bf).contiguous(),
               "gate_up": gu.reshape(self.El * 2 * self.I, self.H).contiguous(),
               "down": d.reshape(self.El * self.H, self.I).contiguous()}
        while len(self.layers) <= i:
            self.layers.append({})
        self.layers[i] = lay

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for lay in self.layers for t in lay.values())

    @staticmethod
    def _bn(avg_rows: float) -> int:
        for b in (16, 32, 64, 128):
            if avg_rows <= b:
                return b
        return 256

    def forward(self, li: int, x: torch.Tensor, out: Optional[torch.Tensor] = None, push=None,
                wait=None) -> torch.Tensor:
        """Routed expert FFN of `x` for this rank's experts.  push=(peer
        buffers, rank, rows) stores each token's combined row straight into
        its owner rank's slot over NVLink (see parallel.fused.push_args);
        wait=(flag block, timeout) makes the router GEMM wait for a deferred
        all-gather of `x` first."""
        lay = self.layers[li]
        T = x.shape[0]
        C = _C()
        st = ops.status(self.dev.index)
        logits = ops.gemm(x, lay["router"], epi=ops.EPI_F32, wait=wait)
        K = self.K
        topk_ids = torch.empty(T, K, dtype=torch.int32, device=self.dev)
        topk_w = torch.empty(T, K, dtype=torch.float32, device=self.dev)
        slot = torch.empty(T, K, dtype=torch.int32, device=self.dev)
        bn = self._bn(T * K / self.E)
        ft_gu = (2 * self.I + 127) // 128
        ft_d = (self.H + 127) // 128
        max_tiles = ((T * K + bn - 1) // bn + self.El) * max(ft_gu, ft_d)
        tiles_gu = torch.empty(max_tiles, 4, dtype=torch.int32, device=self.dev)
        tiles_d = torch.empty(max_tiles, 4, dtype=torch.int32, device=self.dev)
        C.moe_route(logits, K, self.cfg.norm_topk_prob, self.e0, self.El, topk_ids, topk_w, slot, self.counts)
        C.moe_plan(self.counts, self.offsets, bn, ft_gu, ft_d, tiles_gu, self.n_gu, tiles_d, self.n_d)
        R = T * K
        xs = torch.empty(R, self.H, dtype=torch.bfloat16, device=self.dev)
        pos = torch.empty(T, K, dtype=torch.int32, device=self.dev)
        C.moe_gather(x, self.e0, self.El, topk_ids, slot, self.offsets, pos, xs)
        act = torch.empty(R, self.I, dtype=torch.bfloat16, device=self.dev)
        C.gemm_grouped_out(xs, lay["gate_up"], act, ops.EPI_SWIGLU, tiles_gu, self.n_gu, 2 * self.I, bn, st)
        ys = torch.empty(R, self.H, dtype=torch.bfloat16, device=self.dev)
        C.gemm_grouped_out(act, lay["down"], ys, ops.EPI_BF16, tiles_d, self.n_d, self.H, bn, st)
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.dev)
        if push is not None:
            ptrs, rank, rows = push
            C.moe_combine(ys, pos, topk_w, out, list(ptrs), int(rank), int(rows))
        else:
            C.moe_combine(ys, pos, topk_w, out)
        ops._count(6)
        return out
