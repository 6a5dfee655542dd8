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
    json_mode: bool = False  # constrain the output to a JSON object
    json_schema: Optional[dict] = None  # ... that satisfies this JSON Schema (see engine.structured)

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
    # speculation pauses (plain one-row decode, no draft work) while the
    # acceptance rate of its proposals stays below this; 0 = always speculate
    spec_min_acceptance: float = field(
        default_factory=lambda: float(os.environ.get("BLOOM_SPEC_MIN_ACCEPTANCE", "0.1")))
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
    # preemption when the KV pool cannot grow a running sequence: victim policy
    # (newest, priority, oldest, kv_cost, aegaeon, lru, largest_first), a cap on
    # preemptions per request (0 = none), priority preemption after a waiting
    # request has waited this long (ms, < 0 = off), and the KV utilisation at
    # which no new request is admitted (1.0 = off)
    preemption_policy: str = "newest"
    max_preemptions_per_request: int = 0
    priority_preemption_ms: float = -1.0
    kv_admission_threshold: float = 1.0
    # swap preemption: pinned host bytes that preempted sequences' KV blocks are
    # copied into (resumed without recompute); 0 = recompute preemption only
    swap_space_bytes: int = 0
    # deterministic replay: write every scheduler call, its clock and its
    # result to this JSON-lines file ("{rank}" expands to the TP rank; also
    # BLOOM_STEP_LOG); `python -m bloom_b200.engine.replay <file>` re-runs it
    step_log: str = ""
    # KV cache element type: "bf16" or "int8" (per-token, per-head symmetric
    # scale; halves the KV bytes decode attention reads).  BLOOM_KV_CACHE_DTYPE
    # sets the default.
    kv_cache_dtype: str = field(default_factory=lambda: os.environ.get("BLOOM_KV_CACHE_DTYPE", "bf16"))


VICTIM_POLICIES = {"newest": 0, "priority": 1, "oldest": 2, "kv_cost": 3, "aegaeon": 4, "lru": 5, "largest_first": 6}

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
            budget = max(free - reserve, 64 * kv_block_bytes(model, 16, ec.kv_cache_dtype))
            need = ec.max_num_seqs * ((ec.max_model_len + 15) // 16) + 64
            ec.num_blocks = int(min(budget // kv_block_bytes(model, 16, ec.kv_cache_dtype), max(need, 1024)))
        sc = rt.SchedulerConfig()
        sc.max_num_seqs = ec.max_num_seqs
        sc.max_num_batched_tokens = ec.max_num_batched_tokens
        sc.max_model_len = ec.max_model_len
        sc.chunked_prefill = ec.chunked_prefill
        sc.eos_token_ids = list(self.cfg.eos_token_ids)
        sc.spec_len = int(ec.spec_len)
        apply_long_context_policy(sc, ec.long_context_policy)
        if ec.preemption_policy not in VICTIM_POLICIES:
            raise ValueError(f"unknown preemption policy {ec.preemption_policy!r} ({', '.join(VICTIM_POLICIES)})")
        if not 0.0 < ec.kv_admission_threshold <= 1.0:
            raise ValueError("kv_admission_threshold must be in (0, 1]")
        sc.victim_policy = VICTIM_POLICIES[ec.preemption_policy]
        sc.max_preemptions_per_request = int(ec.max_preemptions_per_request)
        sc.priority_preempt_ms = float(ec.priority_preemption_ms)
        sc.kv_admission_threshold = float(ec.kv_admission_threshold)
        swap_slots = (int(ec.swap_space_bytes) // kv_block_bytes(model, 16, ec.kv_cache_dtype)
                      if ec.swap_space_bytes > 0 else 0)
        sc.swap_slots = swap_slots
        self.scheduler = rt.Scheduler(sc, ec.num_blocks, 16, ec.enable_prefix_caching)
        log = ec.step_log or os.environ.get("BLOOM_STEP_LOG", "")
        if log:
            from .replay import SchedulerRecorder

            rank = model.tp.rank if getattr(model, "tp", None) is not None else 0
            self.scheduler = SchedulerRecorder(self.scheduler, log.replace("{rank}", str(rank)), sc, ec.num_blocks,
                                               16, ec.enable_prefix_caching)
        self.runner = ModelRunner(model, ec.num_blocks, ec.max_num_seqs, ec.max_num_batched_tokens,
                                  ec.max_model_len, ec.use_cuda_graphs, spec_len=int(ec.spec_len),
                                  kv_dtype=ec.kv_cache_dtype)
        if ec.autotune and dev.type == "cuda":
            from .. import ops

            ql = self.runner.q_len
            ops.gemm_autotune(model.gemm_shapes(), [b * ql for b in self.runner.buckets + [ec.max_num_seqs]], dev)
        self.scheduler.set_arena(self.runner.arena_host, self.runner.max_tokens, ec.max_num_seqs,
                                 self.runner.max_blocks)
        if swap_slots > 0:
            self.runner.enable_swap(swap_slots)
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
        self._mask_host = None  # constrained decoding: pinned token masks of one step
        self.speculator = None

    def attach_speculator(self, spec) -> None:
        if int(spec.k) != int(self.econf.spec_len):
            raise ValueError(f"speculator proposes {spec.k} tokens but the engine verifies {self.econf.spec_len}")
        if getattr(spec, "gate", None) is None and self.econf.spec_min_acceptance > 0.0:
            from .speculative import AdaptiveGate

            spec.gate = AdaptiveGate(self.econf.spec_min_acceptance)
        self.speculator = spec

    # ------------------------------------------------------------ construction helpers
    @staticmethod
    def from_preset(name: str, tp: Optional[TPInfo] = None, config: Optional[EngineConfig] = None, seed: int = 0,
                    device=None) -> "LLMEngine":
        from ..models import build_decoder

        cfg = preset(name)
        model = build_decoder(cfg, tp, device)
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
        ids = [int(t) for t in prompt_token_ids]
        V = self.cfg.vocab_size
        bad = [t for t in ids if t < 0 or t >= V]
        if bad:
            raise ValueError(f"prompt token ids outside the vocabulary [0, {V}): {bad[:5]}")
        self._seed_counter += 1
        rid = self.scheduler.add_request(ids, params.to_native(self._seed_counter), priority)
        self.requests[rid] = RequestOutput(rid, list(prompt_token_ids), arrival_time=time.perf_counter())
        if (params.json_mode or params.json_schema is not None) and self.tokenizer is not None:
            from .structured import SchemaConstraint, TokenVocab

            vocab = TokenVocab.get(self.tokenizer, self.cfg.vocab_size)
            self.constraints[rid] = SchemaConstraint(vocab, params.json_schema,
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
        from ..utils.tracing import enabled, span

        if enabled():
            with span("engine.step", running=self.scheduler.num_running, waiting=self.scheduler.num_waiting):
                return self._step()
        return self._step()

    def _step(self) -> List[RequestOutput]:
        t0 = time.perf_counter()
        if self.speculator is not None:
            gate = getattr(self.speculator, "gate", None)
            if gate is None or gate.allow(self.scheduler):
                self.speculator.propose(self)
                for rid in self.constraints:
                    self.scheduler.set_draft(rid, [])
        meta = self.scheduler.schedule()
        if self.runner.l2 is not None:
            self.runner.apply_kv_copies(self.scheduler.take_restores(), self.scheduler.take_offloads())
        if self.econf.swap_space_bytes > 0:
            ins, outs = self.scheduler.take_swap_ins(), self.scheduler.take_swap_outs()
            if ins or outs:
                self.runner.apply_swaps(ins, outs)
        if meta.num_tokens == 0:
            return []
        if self.constraints:
            logits = self.runner.launch(meta)
            sampled = self.runner.finish(meta, logits, self._constraint_masks())  # masks built while the GPU runs
        else:
            sampled = self.runner.execute(meta)
        if self.runner.last_status:
            return self._fail_step(self.runner.last_status)
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

    def _constraint_masks(self):
        """Allowed-token masks of this step's constrained sampling rows:
        (rows int32 [R], mask int32 [R, words]) on the device, or None.  Each
        constrained request has exactly one sampling row (it gets no
        speculative proposals).  Host work: one cached trie walk per row."""
        ids = self.scheduler.sampling_ids()
        rows = [(i, sid) for i, sid in enumerate(ids) if sid in self.constraints and (i == 0 or ids[i - 1] != sid)]
        if not rows:
            return None
        words = next(iter(self.constraints.values())).words
        R = len(rows)
        if self._mask_host is None or self._mask_host.shape[0] < R or self._mask_host.shape[1] != words:
            n = max(R, self.econf.max_num_seqs)
            self._mask_host = torch.zeros(n, words, dtype=torch.int32).pin_memory()
            self._mask_rows_host = torch.zeros(n, dtype=torch.int32).pin_memory()
            self._mask_dev = torch.zeros(n, words, dtype=torch.int32, device=self.model.device)
            self._mask_rows_dev = torch.zeros(n, dtype=torch.int32, device=self.model.device)
        for j, (row, sid) in enumerate(rows):
            self.constraints[sid].mask_into(self._mask_host[j])
            self._mask_rows_host[j] = row
        self._mask_dev[:R].copy_(self._mask_host[:R], non_blocking=True)
        self._mask_rows_dev[:R].copy_(self._mask_rows_host[:R], non_blocking=True)
        self.runner.stats["h2d_bytes"] += 4 * R * (words + 1)
        return self._mask_rows_dev[:R], self._mask_dev[:R]

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

    # ------------------------------------------------------------ KV state export / import
    _BLOB_MAGIC = b"BLOOMKV1"

    def export_state(self, request_id: int) -> bytes:
        """Serialise a live request's KV cache and tokens (between steps) into
        a blob: magic, header length, JSON header (model fingerprint, layout,
        tokens, sampling parameters), then the request's KV pages in the cache's
        own layout: bf16 [blocks, layers, 2, kv_heads, 16, head_dim], or for an
        int8 cache the per-layer block bytes [blocks, layers, bytes] (this
        rank's heads under tensor parallelism).  `import_state` on an engine with the same model
        and layout resumes it without recomputing the prefix.  Reference:
        Model::export_state / import_state and StateBlob
        (crates/engine/src/core/model.rs:11-21,215-238)."""
        import json as _json
        import struct

        st = self.scheduler.export_sequence(int(request_id))
        blocks = list(st["blocks"])
        torch.cuda.synchronize(self.model.device)
        if blocks:
            idx = torch.tensor(blocks, dtype=torch.long, device=self.model.device)
            pages = self.runner.kv_cache.index_select(1, idx).transpose(0, 1).contiguous().cpu()
        else:
            pages = torch.empty(0, dtype=self.runner.kv_cache.dtype)
        sp = st["params"]
        r = self.requests.get(int(request_id))
        hdr = {"kind": "kv_cache", "model": self._namespace(), "num_layers": self.cfg.num_layers,
               "kv_heads": self.model.nkv, "head_dim": self.cfg.head_dim, "block_size": 16,
               "dtype": self.runner.kv_dtype,
               "tp": [self.model.tp.rank, self.model.tp.size], "tokens": list(st["tokens"]),
               "num_prompt": st["num_prompt"], "num_computed": st["num_computed"], "num_blocks": len(blocks),
               "priority": st["priority"],
               "params": {"max_tokens": sp.max_tokens, "temperature": sp.temperature, "top_p": sp.top_p,
                          "top_k": sp.top_k, "seed": sp.seed, "min_tokens": sp.min_tokens,
                          "ignore_eos": sp.ignore_eos, "stop_token_ids": list(sp.stop_token_ids)},
               "arrival": r.arrival_time if r is not None else None}
        h = _json.dumps(hdr, separators=(",", ":")).encode()
        return self._BLOB_MAGIC + struct.pack("<I", len(h)) + h + pages.view(torch.uint8).numpy().tobytes()

    def import_state(self, blob: bytes, params: Optional[SamplingParams] = None) -> int:
        """Resume a request exported by `export_state`; returns its new id.
        The blob's model fingerprint and KV layout must match this engine."""
        import json as _json
        import struct

        if not blob.startswith(self._BLOB_MAGIC):
            raise ValueError("not a bloom KV state blob")
        n = struct.unpack("<I", blob[8:12])[0]
        hdr = _json.loads(blob[12:12 + n])
        want = {"model": self._namespace(), "num_layers": self.cfg.num_layers, "kv_heads": self.model.nkv,
                "head_dim": self.cfg.head_dim, "block_size": 16, "dtype": self.runner.kv_dtype,
                "tp": [self.model.tp.rank, self.model.tp.size]}
        for k, v in want.items():
            if hdr.get(k) != v:
                raise ValueError(f"KV state blob does not match this engine: {k} {hdr.get(k)!r} != {v!r}")
        nb = int(hdr["num_blocks"])
        payload = memoryview(blob)[12 + n:]
        kv = self.runner.kv_cache
        shape = (nb, kv.shape[0], *kv.shape[2:])
        numel = 1
        for d in shape:
            numel *= d
        if len(payload) != numel * kv.element_size():
            raise ValueError(f"KV state blob payload has {len(payload)} bytes, expected {numel * kv.element_size()}")
        if params is None:
            p = hdr["params"]
            params = SamplingParams(max_tokens=p["max_tokens"], temperature=p["temperature"], top_p=p["top_p"],
                                    top_k=p["top_k"], seed=p["seed"], min_tokens=p["min_tokens"],
                                    ignore_eos=p["ignore_eos"], stop_token_ids=list(p["stop_token_ids"]))
        self._seed_counter += 1
        tokens = [int(t) for t in hdr["tokens"]]
        rid, table = self.scheduler.import_sequence(tokens, int(hdr["num_prompt"]), int(hdr["num_computed"]),
                                                    params.to_native(self._seed_counter), int(hdr["priority"]))
        if nb:
            pages = torch.frombuffer(bytearray(payload), dtype=kv.dtype).view(shape)
            dev_pages = pages.to(self.model.device, non_blocking=False)
            k = min(nb, len(table))
            idx = torch.tensor(list(table[:k]), dtype=torch.long, device=self.model.device)
            self.runner.kv_cache.index_copy_(1, idx, dev_pages[:k].transpose(0, 1).contiguous())
        P = int(hdr["num_prompt"])
        self.requests[rid] = RequestOutput(rid, tokens[:P], token_ids=tokens[P:], arrival_time=time.perf_counter())
        return rid

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
