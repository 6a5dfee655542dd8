"""Speculative decoding: proposers and the engine hook.

Every engine step with speculation on turns each decoding sequence into a
verify group of q_len = k + 1 token rows (its last sampled token plus k
proposals) inside the ONE batched forward of the step.  The target's logits
at every row are sampled on the GPU (greedy: argmax; stochastic: the
rejection-sampling verify kernel, which accepts a proposal d with
probability p(d) and otherwise draws from p with d removed); the C++
scheduler accepts the longest agreeing prefix plus one corrected / bonus
token and moves the sequence's KV length back over rejected rows (no copy:
the paged block table is trimmed and the rows are overwritten later).

Proposers:
  * n-gram (prompt lookup): the longest suffix of the sequence of length
    order..1 that occurred earlier proposes the tokens that followed it
    (C++, csrc/runtime/scheduler.cpp ngram_propose).
  * draft model: a small decoder with its own paged KV cache and scheduler
    keeps one mirror sequence per target sequence; per step the mirrors are
    re-synchronised with the target (set_tail: keep the agreed prefix, append
    the corrected token) and the draft runs k batched greedy decode steps
    (CUDA-graph replays).  Unlike a re-prefill of the whole context per
    proposal, the draft's KV survives across steps and only rejected rows are
    recomputed.  With tensor parallelism the draft runs on the first rank
    and its proposals are broadcast, so all ranks verify identical tokens.

Proposals are deterministic (greedy draft / lookup), i.e. the proposal
distribution q is one-hot; rejection sampling with such a q keeps the
target distribution exact for any temperature / top-k / top-p.

Reference behaviour: crates/engine/src/executor/speculative.rs:15-70
(SpeculativeStrategy), :78-180 (n-gram), :184-560 (draft model),
:638-753 (verify_with_rejection_sampling), :756-840 (modes and
BLOOM_SPECULATIVE / BLOOM_DRAFT_MODEL / BLOOM_NUM_SPECULATIVE_TOKENS /
BLOOM_SPECULATIVE_NGRAM_ORDER), :871-889 (greedy verification).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional

import torch


class AdaptiveGate:
    """Pauses speculation while it does not pay.  After every verify step the
    gate reads the scheduler's cumulative (proposed, accepted) counters -- the
    same on every tensor-parallel rank, so every rank decides alike -- and
    keeps an exponential average of the acceptance rate.  Below
    `min_acceptance` it pauses proposing for `backoff` steps (doubling up to
    `max_backoff` while it stays low); a paused step schedules plain one-row
    decode, so neither the draft nor the verify width costs anything.  After
    a pause it proposes again to re-measure."""

    def __init__(self, min_acceptance: float = 0.1, alpha: float = 0.25, backoff: int = 16, max_backoff: int = 512):
        self.min_acceptance = float(min_acceptance)
        self.alpha = float(alpha)
        self.backoff0 = self.backoff = int(backoff)
        self.max_backoff = int(max_backoff)
        self.rate: Optional[float] = None
        self.paused = 0
        self.last = (0, 0)
        self.pauses = 0
        self.probing = False

    def allow(self, scheduler) -> bool:
        if self.min_acceptance <= 0.0:
            return True
        st = scheduler.spec_stats()
        prop, acc = int(st["proposed"]), int(st["accepted"])
        dp, da = prop - self.last[0], acc - self.last[1]
        self.last = (prop, acc)
        if dp > 0:
            r = da / dp
            self.rate = r if self.rate is None or self.probing else (1 - self.alpha) * self.rate + self.alpha * r
            self.probing = False
            if self.rate < self.min_acceptance:
                self.paused = self.backoff
                self.backoff = min(self.backoff * 2, self.max_backoff)
                self.pauses += 1
            else:
                self.backoff = self.backoff0
        if self.paused > 0:
            self.paused -= 1
            if self.paused == 0:
                self.probing = True  # the next verify step re-measures from scratch
            return False
        return True


class Speculator:
    """Engine hook: `propose(engine)` sets the next step's proposals on the
    engine's scheduler; `stats()` reports acceptance."""

    k: int = 0
    gate: Optional[AdaptiveGate] = None

    def propose(self, engine) -> None:  # pragma: no cover - interface
        raise NotImplementedError

    def forget(self, request_id: int) -> None:
        pass

    def stats(self, engine) -> dict:
        d = dict(engine.scheduler.spec_stats())
        d["acceptance_rate"] = d["accepted"] / d["proposed"] if d["proposed"] else 0.0
        d["tokens_per_verify"] = ((d["accepted"] + d["verify_groups"]) / d["verify_groups"]
                                  if d["verify_groups"] else 0.0)
        d["num_speculative_tokens"] = self.k
        if self.gate is not None:
            d["gate_pauses"] = self.gate.pauses
            d["gate_acceptance"] = self.gate.rate
        return d


class NgramSpeculator(Speculator):
    def __init__(self, k: int = 5, max_order: int = 4, min_order: int = 1):
        self.k = int(k)
        self.max_order = int(max_order)
        self.min_order = int(min_order)

    def propose(self, engine) -> None:
        engine.scheduler.propose_ngram(self.max_order, self.min_order)


class DraftModelSpeculator(Speculator):
    """Greedy proposals from a small draft decoder (see module docstring)."""

    def __init__(self, draft_engine, k: int = 4, tp=None):
        self.k = int(k)
        self.draft = draft_engine  # None on ranks that only receive proposals
        self.tp = tp
        self.mirror: Dict[int, int] = {}  # target request id -> draft request id
        self.synced: Dict[int, int] = {}  # target request id -> tokens known equal
        from .engine import SamplingParams

        self._params = SamplingParams(max_tokens=1 << 30, temperature=0.0, top_p=1.0, ignore_eos=True)

    # -- helpers
    def _mirror_tokens(self, mid: int) -> List[int]:
        r = self.draft.requests[mid]
        return r.prompt_token_ids + r.token_ids

    def _drop(self, tid: int) -> None:
        mid = self.mirror.pop(tid, None)
        self.synced.pop(tid, None)
        if mid is not None and self.draft is not None:
            self.draft.abort(mid)
            self.draft.requests.pop(mid, None)

    def forget(self, request_id: int) -> None:
        self._drop(request_id)

    def _local_proposals(self, engine, cands: List[int]) -> Dict[int, List[int]]:
        d = self.draft
        k = self.k
        live = set(cands)
        for tid in list(self.mirror):
            if tid not in live:
                self._drop(tid)
        targets: Dict[int, List[int]] = {}
        limit = d.econf.max_model_len - k - 2
        for tid in cands:
            r = engine.requests.get(tid)
            if r is None:
                continue
            full = r.prompt_token_ids + r.token_ids
            if len(full) >= limit:
                self._drop(tid)
                continue
            targets[tid] = full
            mid = self.mirror.get(tid)
            if mid is None:
                self.mirror[tid] = d.add_request(full, self._params)
                self.synced[tid] = 0
                continue
            m = self._mirror_tokens(mid)
            c = self.synced[tid]
            n = min(len(m), len(full))
            while c < n and m[c] == full[c]:
                c += 1
            if c < len(m) or c < len(full):
                if not d.scheduler.set_tail(mid, c, full[c:]):
                    self._drop(tid)
                    self.mirror[tid] = d.add_request(full, self._params)
                    self.synced[tid] = 0
                    continue
                dr = d.requests[mid]
                keep = c - len(dr.prompt_token_ids)
                dr.token_ids = dr.token_ids[:keep] + full[c:]
            self.synced[tid] = len(full)
        # k greedy draft tokens past the target's end for every mirror (a new
        # mirror first prefills its context, possibly over several chunks)
        for _ in range(k + 4):
            if all(len(self._mirror_tokens(self.mirror[t])) >= len(f) + k
                   for t, f in targets.items() if t in self.mirror):
                break
            if not d.has_unfinished():
                break
            d.step()
        out: Dict[int, List[int]] = {}
        for tid, full in targets.items():
            mid = self.mirror.get(tid)
            if mid is None:
                continue
            m = self._mirror_tokens(mid)
            out[tid] = m[len(full):len(full) + k]
        return out

    def propose(self, engine) -> None:
        cands = list(engine.scheduler.decode_candidates())
        if not cands:
            return
        tp = self.tp
        if tp is None or tp.size == 1:
            props = self._local_proposals(engine, cands)
            for tid, p in props.items():
                if p:
                    engine.scheduler.set_draft(tid, p)
            return
        # tensor parallel: the first rank drafts, every rank receives the same proposals
        import torch.distributed as dist

        buf = torch.full((len(cands), self.k), -1, dtype=torch.int32, device=engine.model.device)
        if tp.rank == 0:
            props = self._local_proposals(engine, cands)
            host = torch.full((len(cands), self.k), -1, dtype=torch.int32)
            for i, tid in enumerate(cands):
                p = props.get(tid, [])
                if p:
                    host[i, :len(p)] = torch.tensor(p, dtype=torch.int32)
            buf.copy_(host)
        group = tp.comm.group
        dist.broadcast(buf, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        rows = buf.cpu().tolist()
        for tid, row in zip(cands, rows):
            p = [t for t in row if t >= 0]
            if p:
                engine.scheduler.set_draft(tid, p)


def speculative_mode_from_env() -> dict:
    """BLOOM_SPECULATIVE (none|ngram|draft), BLOOM_DRAFT_MODEL,
    BLOOM_NUM_SPECULATIVE_TOKENS (5), BLOOM_SPECULATIVE_NGRAM_ORDER (4)."""
    mode = os.environ.get("BLOOM_SPECULATIVE", "none").strip().lower() or "none"
    if mode not in ("none", "ngram", "draft", "mtp"):
        raise ValueError(f"BLOOM_SPECULATIVE must be none|ngram|draft, got {mode!r}")
    if mode == "mtp":
        raise ValueError("multi-token-prediction heads are not supported by the B200 decoder; use ngram or draft")
    return {"mode": mode, "draft_model": os.environ.get("BLOOM_DRAFT_MODEL"),
            "k": int(os.environ.get("BLOOM_NUM_SPECULATIVE_TOKENS", "5")),
            "ngram_order": int(os.environ.get("BLOOM_SPECULATIVE_NGRAM_ORDER", "4"))}


def build_draft_engine(draft_model: str, target_engine, k: int, seed: int = 0):
    """Draft LLMEngine on the target's device: a preset name (random init) or
    a model path.  Prefix caching is off so rollbacks never meet shared blocks."""
    from ..models.config import PRESETS, preset
    from ..models.llama import DecoderLM
    from .engine import EngineConfig, LLMEngine

    te = target_engine.econf
    dev = target_engine.model.device
    if draft_model in PRESETS:
        dm = DecoderLM(preset(draft_model), None, dev)
        dm.random_init(seed)
    else:
        from ..formats.loader import load_decoder

        dm = load_decoder(draft_model, None, dev)
    if dm.cfg.vocab_size != target_engine.cfg.vocab_size:
        raise ValueError(f"draft vocabulary {dm.cfg.vocab_size} != target vocabulary {target_engine.cfg.vocab_size}")
    ec = EngineConfig(max_num_seqs=te.max_num_seqs, max_num_batched_tokens=te.max_num_batched_tokens,
                      max_model_len=te.max_model_len + k + 4, enable_prefix_caching=False,
                      use_cuda_graphs=te.use_cuda_graphs, autotune=te.autotune,
                      gpu_memory_utilization=te.gpu_memory_utilization)
    return LLMEngine(dm, ec)


def make_speculator(kind: str, llm, draft_model: Optional[str], nspec: int, ngram_order: int = 4):
    """Attach a speculator to an engine built with EngineConfig.spec_len == nspec."""
    if kind == "ngram":
        spec = NgramSpeculator(nspec, ngram_order)
    elif kind == "draft":
        if not draft_model:
            raise ValueError("--speculative draft needs --draft-model")
        tp = llm.model.tp
        draft = build_draft_engine(draft_model, llm, nspec) if (tp.size == 1 or tp.rank == 0) else None
        spec = DraftModelSpeculator(draft, nspec, tp if tp.size > 1 else None)
    else:
        raise ValueError(f"unknown speculative mode {kind!r}")
    llm.attach_speculator(spec)
    return spec
