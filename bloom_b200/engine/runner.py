"""Model runner: one GPU's share of an engine step.

The C++ scheduler writes the step's metadata into a pinned arena; the runner
copies the used part to the device in one transfer, runs the forward (a CUDA
graph replay for decode-only steps padded to a batch bucket, eager kernels
otherwise), samples on the GPU and reads back one int32 per sampling row
plus the kernels' status word (the OR over all tensor-parallel ranks), in
one device-to-host copy.  A nonzero status means the step's outputs cannot be
trusted: the engine fails the step's requests instead of emitting tokens.

Tensor parallel ranks run identical schedulers on identical inputs; sampled
tokens are made identical across ranks (greedy: distributed argmax over the
vocabulary shards; stochastic: all-gathered logits with the same Philox
stream), so no per-step metadata broadcast is needed.
"""
from __future__ import annotations

import math
import time
from typing import Dict, List, Optional

import torch

from .. import ops
from .._ext import runtime as _rt
from ..models.llama import DecoderLM, StepInputs

DEFAULT_BUCKETS = [1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512]


def kv_block_bytes(model: DecoderLM, block_size: int = 16, kv_dtype: str = "bf16") -> int:
    """Bytes of one KV block over all layers: bf16 pages, or int8 pages plus
    one fp32 scale per token and head (ops.kv_q8_block_bytes)."""
    cfg = model.cfg
    if hasattr(model, "kv_block_bytes"):  # models that lay out their own KV slots (wide heads)
        return model.kv_block_bytes()
    L = getattr(model, "num_kv_layers", cfg.num_layers)  # a pipeline stage holds its own layers
    if kv_dtype == "int8":
        return L * ops.kv_q8_block_bytes(model.nkv, cfg.head_dim)
    return L * 2 * model.nkv * block_size * cfg.head_dim * 2


class ModelRunner:
    def __init__(
        self,
        model: DecoderLM,
        num_blocks: int,
        max_num_seqs: int = 256,
        max_num_batched_tokens: int = 8192,
        max_model_len: int = 4096,
        use_cuda_graphs: bool = True,
        graph_buckets: Optional[List[int]] = None,
        spec_len: int = 0,
        kv_dtype: str = "bf16",
    ):
        self.model = model
        self.cfg = model.cfg
        self.device = model.device
        self.block_size = 16
        self.max_num_seqs = max_num_seqs
        self.q_len = spec_len + 1  # token rows per decode sequence (verify rows when speculating)
        self.max_tokens = max(max_num_batched_tokens, max_num_seqs * self.q_len)
        # verify rows may run spec_len positions past the last token
        self.max_blocks = (max_model_len + spec_len + self.block_size - 1) // self.block_size
        self.num_blocks = num_blocks
        cfg = self.cfg
        # zero-filled: masked tail slots of a page are multiplied by p = 0, which must not meet NaN bit patterns
        if kv_dtype not in ("bf16", "int8"):
            raise ValueError(f"kv cache dtype must be bf16 or int8, not {kv_dtype!r}")
        self.kv_dtype = kv_dtype
        self.wide = bool(getattr(model, "wide_attention", False))
        if self.wide:
            if kv_dtype != "bf16":
                raise ValueError(f"{cfg.arch} keeps a bf16 KV cache")
            self.kv_cache = torch.zeros(model.kv_cache_shape(num_blocks), dtype=torch.bfloat16, device=self.device)
        elif kv_dtype == "int8":
            self.kv_cache = torch.zeros(getattr(model, "num_kv_layers", cfg.num_layers), num_blocks,
                                        ops.kv_q8_block_bytes(model.nkv, cfg.head_dim), dtype=torch.uint8,
                                        device=self.device)
        else:
            self.kv_cache = torch.zeros(getattr(model, "num_kv_layers", cfg.num_layers), num_blocks, 2, model.nkv,
                                        self.block_size, cfg.head_dim, dtype=torch.bfloat16, device=self.device)
        rt = _rt()
        worst = rt.arena_layout(self.max_tokens, max_num_seqs, max_num_seqs,
                                self.max_tokens // 64 + max_num_seqs, self.max_tokens + max_num_seqs,
                                self.max_blocks)
        self.arena_words = worst.used_words
        self.arena_host = torch.zeros(self.arena_words, dtype=torch.int32).pin_memory()
        self.arena_dev = torch.zeros(self.arena_words, dtype=torch.int32, device=self.device)
        self.sampled_host = torch.zeros(self.max_tokens + max_num_seqs + 1, dtype=torch.int32).pin_memory()
        self.last_status = 0
        self.buckets = [b for b in (graph_buckets or DEFAULT_BUCKETS) if b <= max_num_seqs]
        if max_num_seqs not in self.buckets:
            self.buckets.append(max_num_seqs)
        # streamed (host-placed) layers order copies across two streams: eager steps only
        # (pipeline stages exchange activations with NCCL point-to-point calls: eager steps)
        self.pp = getattr(model, "pp", None)
        self.use_cuda_graphs = use_cuda_graphs and not getattr(model, "offloaded", False) and self.pp is None
        # decode attention split-K workspace, sized for the largest need over buckets
        ws = 1
        self.decode_splits: Dict[int, int] = {}
        self.head_chunks = 1
        if self.wide:  # the model sizes its own decode attention workspace
            model.prepare_runner(max_num_seqs, self.q_len, self.max_blocks)
        else:
            self.head_chunks = ops.decode_head_chunks(model.nq, model.nkv, self.q_len)
            if self.head_chunks == 0:
                raise ValueError(f"speculation length {spec_len} does not fit the decode attention kernel")
            vkh = model.nkv * self.head_chunks  # CTAs per sequence and split
            for b in range(1, max_num_seqs + 1):  # eager steps may have any decode count
                s = ops.decode_attention_splits(b, vkh, self.max_blocks, self.device.index)
                self.decode_splits[b] = s
                ws = max(ws, ops.decode_workspace_numel(b, vkh, s))
        self.decode_ws = torch.empty(ws, dtype=torch.float32, device=self.device)
        self.graphs: Dict[tuple, tuple] = {}  # (decode rows, q_len) -> captured step
        self.last_logits: Optional[torch.Tensor] = None
        import os as _os

        self.check_finite = _os.environ.get("BLOOM_CHECK_FINITE", "0") == "1"
        self.graph_pool = None
        self.l2 = None
        self.stats = {"steps": 0, "graph_steps": 0, "eager_steps": 0, "tokens": 0, "h2d_bytes": 0, "d2h_bytes": 0}

    # ------------------------------------------------------------ CacheMesh tiers
    def kv_block_bytes(self) -> int:
        return kv_block_bytes(self.model, self.block_size, self.kv_dtype)

    def _block_slots(self, buf: torch.Tensor, slots: int) -> torch.Tensor:
        """A host byte buffer seen as `slots` KV blocks shaped like kv_cache[:, blk]."""
        kv = self.kv_cache
        return buf.view(kv.dtype).view(slots, kv.shape[0], *kv.shape[2:])

    def enable_cachemesh(self, scheduler, l2_bytes: int, l3_dir: str = "", l3_max_blocks: int = 0,
                         namespace: str = "default") -> None:
        """Pinned host slots (L2) and optional files (L3) below the HBM prefix
        cache; the scheduler queues the block copies, `apply_kv_copies` issues them."""
        bb = self.kv_block_bytes()
        slots = max(1, int(l2_bytes) // bb)
        self.l2 = torch.empty(slots * bb, dtype=torch.uint8).pin_memory()
        self.l2_view = self._block_slots(self.l2, slots)
        scheduler.enable_cachemesh(self.l2, bb, l3_dir, int(l3_max_blocks), namespace)

    def apply_kv_copies(self, restores, offloads) -> None:
        """Host -> HBM restores first (a slot may be reused by an offload of
        the same step), then HBM -> host offloads; both on the step's stream,
        ahead of the forward that may overwrite an offloaded block."""
        for blk, slot in restores:
            self.kv_cache[:, blk].copy_(self.l2_view[slot], non_blocking=True)
        for blk, slot in offloads:
            self.l2_view[slot].copy_(self.kv_cache[:, blk], non_blocking=True)
        self.stats["kv_restores"] = self.stats.get("kv_restores", 0) + len(restores)
        self.stats["kv_offloads"] = self.stats.get("kv_offloads", 0) + len(offloads)

    # ------------------------------------------------------------ swap preemption
    def enable_swap(self, slots: int) -> None:
        """Pinned host slots (one KV block each, all layers) for swap preemption."""
        bb = self.kv_block_bytes()
        self.swap = torch.empty(max(1, slots) * bb, dtype=torch.uint8).pin_memory()
        self.swap_view = self._block_slots(self.swap, max(1, slots))

    def apply_swaps(self, swap_ins, swap_outs) -> None:
        """Swap-ins (host slot -> block) before swap-outs (block -> slot): a
        slot freed by a swap-in may be reused by a swap-out of the same step.
        Both are queued on the step's stream ahead of its forward, so a block
        freed by a swap-out is copied before a new owner overwrites it."""
        for blk, slot in swap_ins:
            self.kv_cache[:, blk].copy_(self.swap_view[slot], non_blocking=True)
        for blk, slot in swap_outs:
            self.swap_view[slot].copy_(self.kv_cache[:, blk], non_blocking=True)
        self.stats["swap_ins"] = self.stats.get("swap_ins", 0) + len(swap_ins)
        self.stats["swap_outs"] = self.stats.get("swap_outs", 0) + len(swap_outs)

    # ------------------------------------------------------------ views
    def _v(self, off: int, n: int, dtype=torch.int32) -> torch.Tensor:
        if dtype == torch.int32 or dtype == torch.float32:
            t = self.arena_dev[off:off + n]
            return t if dtype == torch.int32 else t.view(torch.float32)
        return self.arena_dev[off:off + 2 * n].view(torch.int64)

    def views(self, m) -> StepInputs:
        T, Bd, Sp, NT, NL = m.num_tokens, m.num_decode, m.num_prefill, m.num_tiles, m.num_logits
        MB = self.max_blocks
        splits = 1
        if Bd and not self.wide:
            splits = self.decode_splits.get(Bd) or ops.decode_attention_splits(
                Bd, self.model.nkv * self.head_chunks, MB, self.device.index)
        return StepInputs(
            input_ids=self._v(m.off_input_ids, T),
            positions=self._v(m.off_positions, T, torch.int64),
            slot_mapping=self._v(m.off_slot_mapping, T),
            num_decode=Bd,
            decode_block_table=self._v(m.off_decode_block_table, Bd * MB).view(Bd, MB) if Bd else None,
            decode_seq_lens=self._v(m.off_decode_seq_lens, Bd) if Bd else None,
            decode_splits=splits,
            decode_workspace=self.decode_ws,
            num_prefill=Sp,
            prefill_block_table=self._v(m.off_prefill_block_table, Sp * MB).view(Sp, MB) if Sp else None,
            prefill_ctx_lens=self._v(m.off_prefill_ctx_lens, Sp) if Sp else None,
            prefill_cu_q=self._v(m.off_prefill_cu_q, Sp + 1) if Sp else None,
            tile_seq=self._v(m.off_tile_seq, NT) if Sp else None,
            tile_start=self._v(m.off_tile_start, NT) if Sp else None,
            logits_rows=self._v(m.off_logits_rows, NL),
            decode_q_len=m.decode_q_len,
        )

    def sampling_views(self, m):
        NL = m.num_logits
        draft = self._v(m.off_draft_ids, NL) if m.decode_q_len > 1 else None
        return (self._v(m.off_temperature, NL, torch.float32), self._v(m.off_top_p, NL, torch.float32),
                self._v(m.off_top_k, NL), self._v(m.off_seeds, NL, torch.int64), self._v(m.off_offsets, NL, torch.int64),
                draft)

    # ------------------------------------------------------------ sampling
    def _sample(self, logits: Optional[torch.Tensor], m, greedy: bool) -> torch.Tensor:
        """int32 [NL + 1]: sampled tokens, then the (rank-combined) status word."""
        if self.pp is not None:
            # the last stage samples; every stage gets its tokens and the worst status of all stages
            NL = m.num_logits
            out = torch.empty(NL + 1, dtype=torch.int32, device=self.device)
            st = ops.status(self.device.index)[:1].clone()
            self.pp.max_status(st)
            if self.pp.last:
                if greedy:
                    ops.argmax(logits, out=out[:NL])
                else:
                    ops.sample(logits, *self.sampling_views(m), out=out[:NL])
                out[NL:].copy_(st)
            return self.pp.broadcast_from_last(out)
        tp = self.model.tp
        if tp.size == 1:
            NL = logits.shape[0]
            out = torch.empty(NL + 1, dtype=torch.int32, device=logits.device)
            if greedy:
                ops.argmax(logits, out=out[:NL])
            else:
                ops.sample(logits, *self.sampling_views(m), out=out[:NL])
            out[NL:].copy_(ops.status(self.device.index)[:1])
            return out
        return tp.comm.sample_vocab_parallel(logits, greedy, self.sampling_views(m) if not greedy else None,
                                             self.model.vocab_local)

    def _forward_logits(self, s: StepInputs) -> Optional[torch.Tensor]:
        h = self.model.forward(s, self.kv_cache)
        return None if h is None else self.model.logits(h)  # None: a pipeline stage before the last

    # ------------------------------------------------------------ graphs
    def capture_graphs(self, buckets: Optional[List[int]] = None) -> None:
        if not self.use_cuda_graphs:
            return
        rt = _rt()
        buckets = sorted(buckets or self.buckets, reverse=True)
        # a valid dummy step: every row reads one page of block 0, writes no KV.
        # With speculation both verify steps (q_len rows per sequence) and plain
        # decode steps (one row: no proposal this step) get graphs.
        shapes = [(B, self.q_len) for B in buckets] + ([(B, 1) for B in buckets] if self.q_len > 1 else [])
        for B, ql in shapes:
            T = B * ql
            m = rt.arena_layout(T, B, 0, 0, T, self.max_blocks, ql)
            h = self.arena_host
            h[:m.used_words].zero_()  # regions of the previous bucket's layout must not leak in
            h[m.off_slot_mapping:m.off_slot_mapping + T] = -1
            h[m.off_decode_seq_lens:m.off_decode_seq_lens + B] = ql
            pos = h[m.off_positions:m.off_positions + 2 * T].view(torch.int64)
            pos.copy_(torch.arange(ql, dtype=torch.int64).repeat(B))
            h[m.off_logits_rows:m.off_logits_rows + T] = torch.arange(T, dtype=torch.int32)
            h[m.off_draft_ids:m.off_draft_ids + T] = -1
            self.arena_dev[:m.used_words].copy_(self.arena_host[:m.used_words])
            s = self.views(m)
            torch.cuda.synchronize(self.device)
            # warm-up on a side stream (lazy kernel attribute setup, allocator)
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                self._forward_logits(s)
            torch.cuda.current_stream(self.device).wait_stream(side)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            n0 = ops.LAUNCHES[0]
            with torch.cuda.graph(g, pool=self.graph_pool):
                logits = self._forward_logits(s)
            if self.graph_pool is None:
                self.graph_pool = g.pool()
            self.graphs[(B, ql)] = (g, logits, m, ops.LAUNCHES[0] - n0)
        torch.cuda.synchronize(self.device)

    def release_graphs(self) -> None:
        self.graphs.clear()
        self.graph_pool = None

    # ------------------------------------------------------------ step
    def execute(self, m) -> torch.Tensor:
        """Run one scheduled step; returns host int32 sampled tokens [num_logits]."""
        return self.finish(m, self.launch(m))

    def launch(self, m) -> torch.Tensor:
        """Queue the step's arena copy and forward on the GPU; returns the
        logits tensor without waiting (the host may prepare token masks meanwhile)."""
        used = m.used_words
        self.arena_dev[:used].copy_(self.arena_host[:used], non_blocking=True)
        graph = (self.graphs.get((m.num_decode, m.decode_q_len)) if (m.num_prefill == 0 and m.num_decode > 0)
                 else None)
        if graph is not None and graph[2].used_words == used:
            g, logits, _, nlaunch = graph
            g.replay()
            ops.LAUNCHES[0] += nlaunch
            self.stats["graph_steps"] += 1
        else:
            logits = self._forward_logits(self.views(m))
            self.stats["eager_steps"] += 1
        if self.check_finite and m.num_logits and logits is not None:
            bad = (~torch.isfinite(logits[:m.num_real_logits].float())).any(dim=1)
            if bool(bad.any()):
                rows = bad.nonzero().flatten().tolist()
                raise FloatingPointError(f"non-finite logits in rows {rows} (T={m.num_tokens}, decode={m.num_decode}, "
                                         f"prefill={m.num_prefill})")
        self.last_logits = logits
        return logits

    def finish(self, m, logits: torch.Tensor, token_mask=None) -> torch.Tensor:
        """Optional constrained-decoding masks (rows int32 [R], mask int32
        [R, words] on the device), sampling, and the one device-to-host read
        of the tokens and the status word."""
        if token_mask is not None and logits is not None:
            rows, mask = token_mask
            ops.apply_token_mask(logits, rows, mask, self.model.tp.rank * self.model.vocab_local)
        toks = self._sample(logits, m, m.all_greedy)
        NL = m.num_logits
        self.sampled_host[:NL + 1].copy_(toks[:NL + 1], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        self.last_status = int(self.sampled_host[NL])
        self.stats["steps"] += 1
        self.stats["tokens"] += m.num_tokens
        self.stats["h2d_bytes"] += 4 * m.used_words
        self.stats["d2h_bytes"] += 4 * (NL + 1)
        return self.sampled_host
