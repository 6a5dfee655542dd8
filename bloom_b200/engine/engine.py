"""LLMEngine: the public generation API.

    eng = LLMEngine.from_preset("llama3-8b")            # or LLMEngine(model_path)
    outs = eng.generate([[1, 2, 3], [4, 5]], SamplingParams(max_tokens=16))

An engine step = C++ scheduler decision (decode rows + chunked prefill with
the leftover token budget, prefix reuse, preemption) -> one batched forward
on the GPU -> GPU sampling -> scheduler update (stop conditions, KV frees).
Every running request advances by one token per step (in-flight batching).

Reference surface: InferencePipeline::{run, run_stream, run_embedding_batch}
(crates/engine/src/core/pipeline.rs:375-405), InferenceScheduler::{submit,
step, cancel_request} (scheduler/mod.rs:1479-1845), GenerationParams
defaults (max_tokens 128, temperature 0.7, top_p 0.9; crates/core/src/types.rs:242-260).
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterator, List, Optional

import torch

from .._ext import runtime as _rt
from ..models.config import ModelConfig, preset
from ..models.llama import DecoderLM, TPInfo
from .runner import ModelRunner, kv_block_bytes


@dataclass
class SamplingParams:
    max_tokens: int = 128
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int = 0
    seed: Optional[int] = None
    min_tokens: int = 0
    ignore_eos: bool = False
    stop_token_ids: List[int] = field(default_factory=list)
    json_mode: bool = False

    def to_native(self, default_seed: int):
        sp = _rt().SamplingParams()
        sp.max_tokens = int(self.max_tokens)
        sp.temperature = float(self.temperature)
        sp.top_p = float(self.top_p)
        sp.top_k = int(self.top_k)
        sp.seed = int(self.seed if self.seed is not None else default_seed)
        sp.min_tokens = int(self.min_tokens)
        sp.ignore_eos = bool(self.ignore_eos)
        sp.stop_token_ids = [int(t) for t in self.stop_token_ids]
        return sp


GREEDY = SamplingParams(temperature=0.0, top_p=1.0)

FINISH_REASONS = {0: None, 1: "stop", 2: "length", 3: "abort", 4: "error"}

# Status-word bits (csrc/include/bloom/common.cuh StatusBits).
STATUS_NAMES = {1: "GEMM pipeline wait timed out", 2: "attention wait timed out", 4: "cross-GPU wait timed out",
                8: "bad kernel argument", 16: "MoE buffer overflow", 32: "communicator poisoned"}


def describe_status(bits: int) -> str:
    names = [n for b, n in STATUS_NAMES.items() if bits & b]
    return f"kernel status 0x{bits:x} ({', '.join(names) or 'unknown'})"


@dataclass
class RequestOutput:
    request_id: int
    prompt_token_ids: List[int]
    token_ids: List[int] = field(default_factory=list)
    finished: bool = False
    finish_reason: Optional[str] = None
    arrival_time: float = 0.0
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    num_cached_tokens: int = 0
    error: Optional[str] = None  # set when finish_reason == "error"


@dataclass
class EngineConfig:
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    max_model_len: int = 4096
    gpu_memory_utilization: float = 0.85
    num_blocks: Optional[int] = None
    enable_prefix_caching: bool = True
    chunked_prefill: bool = True
    use_cuda_graphs: bool = True
    autotune: bool = True
    seed: int = 0
    # speculative decoding: proposals verified per sequence and step (0 = off);
    # attach a proposer with LLMEngine.attach_speculator / make_speculator
    spec_len: int = 0
    # CacheMesh: pinned host bytes for evicted prefix blocks (0 = off) and an
    # optional directory of block files below it
    cachemesh_l2_bytes: int = 0
    cachemesh_l3_dir: str = ""
    cachemesh_l3_blocks: int = 0
    cachemesh_namespace: Optional[str] = None
    # long-context policy: "full", "sliding_window:<tokens>",
    # "context_shift:<max_context_tokens>:<shift_tokens>" or
    # "compact_inactive:<target_free_blocks>"
    long_context_policy: str = "full"


LONG_CONTEXT_POLICIES = {"full": 0, "sliding_window": 1, "context_shift": 2, "compact_inactive": 3}


def apply_long_context_policy(sc, spec: str) -> None:
    """Parse a policy string into the scheduler config's lc_* fields."""
    parts = (spec or "full").strip().lower().split(":")
    kind = parts[0]
    if kind not in LONG_CONTEXT_POLICIES:
        raise ValueError(f"unknown long-context policy {spec!r} (full, sliding_window:N, context_shift:MAX:SHIFT, "
                         "compact_inactive:N)")
    args = [int(a) for a in parts[1:]]
    need = {"full": 0, "sliding_window": 1, "context_shift": 2, "compact_inactive": 1}[kind]
    if len(args) != need or any(a < 0 for a in args):
        raise ValueError(f"long-context policy {spec!r} takes {need} non-negative integer argument(s)")
    sc.lc_policy = LONG_CONTEXT_POLICIES[kind]
    if kind == "sliding_window":
        if args[0] == 0:
            raise ValueError("sliding_window needs a window of at least one token")
        sc.lc_window_tokens = args[0]
    elif kind == "context_shift":
        sc.lc_max_context, sc.lc_shift = args
    elif kind == "compact_inactive":
        sc.lc_target_free = args[0]


class LLMEngine:
    def __init__(self, model: DecoderLM, config: Optional[EngineConfig] = None):
        self.model = model
        self.cfg = model.cfg
        self.econf = config or EngineConfig()
        ec = self.econf
        rt = _rt()
        dev = model.device
        if ec.num_blocks is None:
            torch.cuda.synchronize(dev)
            free, total = torch.cuda.mem_get_info(dev)
            reserve = int(total * (1.0 - ec.gpu_memory_utilization)) + (4 << 30)  # activations, graphs
            budget = max(free - reserve, 64 * kv_block_bytes(model))
            need = ec.max_num_seqs * ((ec.max_model_len + 15) // 16) + 64
            ec.num_blocks = int(min(budget // kv_block_bytes(model), max(need, 1024)))
        sc = rt.SchedulerConfig()
        sc.max_num_seqs = ec.max_num_seqs
        sc.max_num_batched_tokens = ec.max_num_batched_tokens
        sc.max_model_len = ec.max_model_len
        sc.chunked_prefill = ec.chunked_prefill
        sc.eos_token_ids = list(self.cfg.eos_token_ids)
        sc.spec_len = int(ec.spec_len)
        apply_long_context_policy(sc, ec.long_context_policy)
        self.scheduler = rt.Scheduler(sc, ec.num_blocks, 16, ec.enable_prefix_caching)
        self.runner = ModelRunner(model, ec.num_blocks, ec.max_num_seqs, ec.max_num_batched_tokens,
                                  ec.max_model_len, ec.use_cuda_graphs, spec_len=int(ec.spec_len))
        if ec.autotune and dev.type == "cuda":
            from .. import ops

            ql = self.runner.q_len
            ops.gemm_autotune(model.gemm_shapes(), [b * ql for b in self.runner.buckets + [ec.max_num_seqs]], dev)
        self.scheduler.set_arena(self.runner.arena_host, self.runner.max_tokens, ec.max_num_seqs,
                                 self.runner.max_blocks)
        if ec.cachemesh_l2_bytes > 0:
            self.runner.enable_cachemesh(self.scheduler, ec.cachemesh_l2_bytes, ec.cachemesh_l3_dir,
                                         ec.cachemesh_l3_blocks, ec.cachemesh_namespace or self._namespace())
        if ec.use_cuda_graphs:
            self.scheduler.set_decode_buckets(sorted(self.runner.buckets))
            self.runner.capture_graphs()
        self.requests: Dict[int, RequestOutput] = {}
        self.constraints: Dict[int, object] = {}
        self.tokenizer = None  # set by the pipeline; needed for JSON-mode constraints
        self._seed_counter = ec.seed
        self.step_times: List[float] = []
        self.failures: List[dict] = []  # steps failed by a kernel status error
        self.speculator = None

    def attach_speculator(self, spec) -> None:
        if int(spec.k) != int(self.econf.spec_len):
            raise ValueError(f"speculator proposes {spec.k} tokens but the engine verifies {self.econf.spec_len}")
        self.speculator = spec

    # ------------------------------------------------------------ construction helpers
    @staticmethod
    def from_preset(name: str, tp: Optional[TPInfo] = None, config: Optional[EngineConfig] = None, seed: int = 0,
                    device=None) -> "LLMEngine":
        cfg = preset(name)
        model = DecoderLM(cfg, tp, device)
        model.random_init(seed)
        return LLMEngine(model, config)

    @staticmethod
    def from_pretrained(path: str, tp: Optional[TPInfo] = None, config: Optional[EngineConfig] = None,
                        device=None) -> "LLMEngine":
        from ..formats.loader import load_decoder

        model = load_decoder(path, tp, device)
        return LLMEngine(model, config)

    # ------------------------------------------------------------ requests
    def add_request(self, prompt_token_ids: List[int], params: Optional[SamplingParams] = None,
                    priority: int = 0) -> int:
        params = params or SamplingParams()
        self._seed_counter += 1
        rid = self.scheduler.add_request([int(t) for t in prompt_token_ids], params.to_native(self._seed_counter),
                                         priority)
        self.requests[rid] = RequestOutput(rid, list(prompt_token_ids), arrival_time=time.perf_counter())
        if params.json_mode and self.tokenizer is not None:
            from .structured import JsonConstraint, vocab_strings

            self.constraints[rid] = JsonConstraint(vocab_strings(self.tokenizer, self.cfg.vocab_size),
                                                   list(params.stop_token_ids) + list(self.cfg.eos_token_ids))
        return rid

    def abort(self, request_id: int) -> bool:
        self.constraints.pop(request_id, None)
        if self.speculator is not None:
            self.speculator.forget(request_id)
        ok = self.scheduler.abort(request_id)
        r = self.requests.get(request_id)
        if ok and r is not None:
            r.finished = True
            r.finish_reason = "abort"
            r.finish_time = time.perf_counter()
        return ok

    def has_unfinished(self) -> bool:
        return self.scheduler.has_unfinished()

    def step(self) -> List[RequestOutput]:
        """One engine step; returns the requests that received a token."""
        t0 = time.perf_counter()
        if self.speculator is not None:
            self.speculator.propose(self)
            for rid in self.constraints:
                self.scheduler.set_draft(rid, [])
        meta = self.scheduler.schedule()
        if self.runner.l2 is not None:
            self.runner.apply_kv_copies(self.scheduler.take_restores(), self.scheduler.take_offloads())
        if meta.num_tokens == 0:
            return []
        sampled = self.runner.execute(meta)
        if self.runner.last_status:
            return self._fail_step(self.runner.last_status)
        if self.constraints:
            self._apply_constraints(sampled, meta)
        events = self.scheduler.update(sampled, meta.num_real_logits)
        now = time.perf_counter()
        out = []
        for rid, tok, finished, reason in events:
            r = self.requests.get(rid)
            if r is None:
                continue
            if r.first_token_time is None:
                r.first_token_time = now
                r.num_cached_tokens = 0
            r.token_ids.append(tok)
            c = self.constraints.get(rid)
            if c is not None:
                c.advance(tok)
            if finished:
                self.constraints.pop(rid, None)
                if self.speculator is not None:
                    self.speculator.forget(rid)
                r.finished = True
                r.finish_reason = FINISH_REASONS.get(reason, "stop")
                r.finish_time = now
            out.append(r)
        self.step_times.append(now - t0)
        return out

    def _fail_step(self, bits: int) -> List[RequestOutput]:
        """A kernel of the step reported an error (the status word, combined over
        all tensor-parallel ranks, so every rank takes this path in the same
        step): no token of the step is emitted; every request the step
        scheduled finishes with finish_reason "error" and releases its KV
        blocks; requests outside the step continue.  A cross-GPU timeout also
        drops the fused communicator (later steps run on NCCL) and re-captures
        the CUDA graphs.  Reference: fail_scheduled_requests
        (crates/engine/src/scheduler/mod.rs:1862-1907)."""
        from .. import ops

        msg = describe_status(bits)
        ops.status(self.model.device.index).zero_()
        now = time.perf_counter()
        out = []
        for rid in self.scheduler.fail_scheduled():
            self.constraints.pop(rid, None)
            if self.speculator is not None:
                self.speculator.forget(rid)
            r = self.requests.get(rid)
            if r is None:
                continue
            r.finished = True
            r.finish_reason = "error"
            r.error = msg
            r.finish_time = now
            out.append(r)
        self.failures.append({"time": now, "status": bits, "message": msg, "requests": [r.request_id for r in out]})
        comm = self.model.tp.comm
        if comm is not None and bits & comm.COMM_BITS and comm.poison():
            self.runner.release_graphs()
            if self.econf.use_cuda_graphs:
                self.runner.capture_graphs()
        return out

    def _apply_constraints(self, sampled, meta) -> None:
        """JSON mode: replace the sampled token of constrained rows by the best
        candidate (top-256 logits) that keeps the output valid JSON."""
        ids = self.scheduler.sampling_ids()
        # first row of each request only (constrained requests get no proposals)
        rows = [(i, sid) for i, sid in enumerate(ids) if sid in self.constraints and (i == 0 or ids[i - 1] != sid)]
        if not rows or self.runner.last_logits is None or self.model.tp.size > 1:
            return
        logits = self.runner.last_logits
        idx = torch.tensor([i for i, _ in rows], device=logits.device)
        sel = logits.index_select(0, idx).float()
        top = torch.topk(sel, k=min(256, logits.shape[1]), dim=1).indices.cpu()
        for j, ((row, sid), cand) in enumerate(zip(rows, top.tolist())):
            full = (lambda j=j: torch.argsort(sel[j], descending=True).cpu().tolist())
            sampled[row] = self.constraints[sid].choose(cand, int(sampled[row]), full)

    def generate(self, prompts: List[List[int]], params: Optional[SamplingParams] = None,
                 on_token: Optional[Callable[[RequestOutput], None]] = None) -> List[RequestOutput]:
        ids = [self.add_request(p, params) for p in prompts]
        while self.has_unfinished():
            for r in self.step():
                if on_token is not None:
                    on_token(r)
        res = [self.requests.pop(i) for i in ids]
        return res

    def stream(self, prompt: List[int], params: Optional[SamplingParams] = None) -> Iterator[int]:
        rid = self.add_request(prompt, params)
        seen = 0
        while True:
            self.step()
            r = self.requests[rid]
            while seen < len(r.token_ids):
                yield r.token_ids[seen]
                seen += 1
            if r.finished:
                self.requests.pop(rid, None)
                return

    def kv_metrics(self) -> dict:
        d = dict(self.scheduler.kv_metrics())
        mesh = dict(self.scheduler.cachemesh_metrics())
        if mesh:
            d["cachemesh"] = mesh
        return d

    def _namespace(self) -> str:
        """Model + KV layout + a fingerprint of the weights: L3 files of another
        model or another set of weights never match."""
        import hashlib

        m, cfg = self.model, self.cfg
        h = hashlib.sha256()
        for lay in m.layers[:4]:
            w = lay["qkv"]
            w = w.scales if hasattr(w, "scales") else w
            h.update(w.reshape(-1)[:256].float().cpu().numpy().tobytes())
        h.update(m.embed.reshape(-1)[:256].float().cpu().numpy().tobytes())
        return (f"{cfg.name or cfg.arch}-L{cfg.num_layers}-kv{m.nkv}-hd{cfg.head_dim}-tp{m.tp.rank}of{m.tp.size}-"
                f"{h.hexdigest()[:16]}")

    def shutdown(self) -> None:
        self.runner.release_graphs()
