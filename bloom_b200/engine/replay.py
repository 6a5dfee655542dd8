"""Deterministic record / replay of the scheduler step log.

`SchedulerRecorder` wraps the C++ runtime scheduler of an engine and writes
one JSON line per call that changes its state: the configuration first, then
add_request (prompt, native sampling parameters, priority), abort, set_draft,
schedule (with a fingerprint of the step it produced: the StepMeta fields and
the arena words it wrote), update (the sampled tokens it was given and the
events it returned), fail_scheduled and the KV copy / swap queues.  Before
every call the scheduler clock is pinned to the wall clock and the value is
logged, so clock-dependent policies (priority preemption, LRU / oldest
victims, arrival order) see the same times on replay.

`replay(path)` builds a fresh scheduler from the logged configuration, an
arena of the logged size, and feeds it the logged calls with the logged
clock values; it compares every result with the log and returns the first
divergence (None when the run reproduces exactly).  Sampled tokens come from
the log, so no model and no GPU are needed: a step sequence seen on a GPU
run can be re-run and bisected on any host.

Enable with EngineConfig.step_log = "<path>" (or BLOOM_STEP_LOG=<path>).
The reference has no equivalent; its scheduler tests drive fixed request
sequences (crates/engine/src/scheduler/scheduler_test.rs).
"""
from __future__ import annotations

import hashlib
import json
import time
from typing import Any, Dict, List, Optional

import torch

from .._ext import runtime as _rt

META_FIELDS = ("num_tokens", "num_decode", "decode_q_len", "num_real_decode", "num_prefill", "num_tiles",
               "num_logits", "num_real_logits", "max_decode_blocks", "num_preempted", "all_greedy", "used_words")
CONFIG_SKIP = ("__class__",)


def _config_dict(sc) -> Dict[str, Any]:
    d = {}
    for k in dir(sc):
        if k.startswith("_"):
            continue
        v = getattr(sc, k)
        if callable(v):
            continue
        d[k] = list(v) if isinstance(v, (list, tuple)) else v
    return d


def _params_dict(p) -> Dict[str, Any]:
    return _config_dict(p)


def _make_config(d: Dict[str, Any]):
    sc = _rt().SchedulerConfig()
    for k, v in d.items():
        setattr(sc, k, v)
    return sc


def _make_params(d: Dict[str, Any]):
    p = _rt().SamplingParams()
    for k, v in d.items():
        setattr(p, k, v)
    return p


def step_fingerprint(meta, arena: torch.Tensor) -> str:
    h = hashlib.sha1()
    h.update(json.dumps([int(getattr(meta, f)) for f in META_FIELDS]).encode())
    n = int(meta.used_words)
    if n > 0:
        h.update(arena[:n].contiguous().numpy().tobytes())
    return h.hexdigest()


def _events(ev) -> List[List[int]]:
    return [[int(x) for x in e] for e in ev]


class SchedulerRecorder:
    """Forwards every attribute to the wrapped scheduler; state-changing calls
    are logged as JSON lines (flushed per step)."""

    _LOGGED_QUEUES = ("take_restores", "take_offloads", "take_swap_ins", "take_swap_outs")

    def __init__(self, sched, path: str, config, num_blocks: int, block_size: int, prefix_caching: bool):
        object.__setattr__(self, "_s", sched)
        object.__setattr__(self, "_f", open(path, "w"))
        object.__setattr__(self, "_arena", None)
        self._write({"m": "config", "sched": _config_dict(config), "num_blocks": int(num_blocks),
                     "block_size": int(block_size), "prefix": bool(prefix_caching)})

    # ---------------------------------------------------------------- helpers
    def _write(self, rec: Dict[str, Any]) -> None:
        self._f.write(json.dumps(rec, separators=(",", ":")) + "\n")

    def _pin(self) -> float:
        t = time.monotonic() * 1000.0
        self._s.set_clock_ms(t)
        return t

    def __getattr__(self, name):
        attr = getattr(self._s, name)
        if name in self._LOGGED_QUEUES:
            def q(*args):
                r = attr(*args)
                self._write({"m": name, "r": [list(map(int, x)) if isinstance(x, (list, tuple)) else int(x)
                                              for x in r]})
                return r
            return q
        return attr

    def close(self) -> None:
        self._f.close()

    # ---------------------------------------------------------------- logged calls
    def set_arena(self, arena, max_tokens, max_seqs, max_blocks):
        object.__setattr__(self, "_arena", arena)
        self._write({"m": "set_arena", "n": int(arena.numel()), "args": [int(max_tokens), int(max_seqs),
                                                                          int(max_blocks)]})
        return self._s.set_arena(arena, max_tokens, max_seqs, max_blocks)

    def enable_cachemesh(self, l2, block_bytes, l3_dir, l3_max_blocks, ns):
        self._write({"m": "enable_cachemesh", "n": int(l2.numel()), "bb": int(block_bytes), "l3": bool(l3_dir),
                     "l3n": int(l3_max_blocks), "ns": str(ns)})
        return self._s.enable_cachemesh(l2, block_bytes, l3_dir, l3_max_blocks, ns)

    def set_decode_buckets(self, buckets):
        self._write({"m": "set_decode_buckets", "b": [int(b) for b in buckets]})
        return self._s.set_decode_buckets(buckets)

    def add_request(self, prompt, params, priority=0):
        t = self._pin()
        rid = self._s.add_request(prompt, params, priority)
        self._write({"m": "add", "t": t, "prompt": [int(x) for x in prompt], "params": _params_dict(params),
                     "prio": int(priority), "r": int(rid)})
        return rid

    def import_sequence(self, tokens, num_prompt, num_computed, params, priority=0):
        t = self._pin()
        r = self._s.import_sequence(tokens, num_prompt, num_computed, params, priority)
        rid, table = r
        self._write({"m": "import", "t": t, "tokens": [int(x) for x in tokens], "np": int(num_prompt),
                     "nc": int(num_computed), "params": _params_dict(params), "prio": int(priority),
                     "r": [int(rid), [int(b) for b in table]]})
        return r

    def abort(self, rid):
        t = self._pin()
        ok = self._s.abort(rid)
        self._write({"m": "abort", "t": t, "rid": int(rid), "r": bool(ok)})
        return ok

    def set_draft(self, rid, tokens):
        self._write({"m": "set_draft", "rid": int(rid), "tokens": [int(x) for x in tokens]})
        return self._s.set_draft(rid, tokens)

    def schedule(self):
        t = self._pin()
        meta = self._s.schedule()
        self._write({"m": "schedule", "t": t, "fp": step_fingerprint(meta, self._arena)})
        return meta

    def update(self, sampled, n):
        ev = self._s.update(sampled, n)
        self._write({"m": "update", "sampled": [int(x) for x in sampled[: max(int(n), 0)].tolist()], "n": int(n),
                     "r": _events(ev)})
        self._f.flush()
        return ev

    def fail_scheduled(self):
        r = self._s.fail_scheduled()
        self._write({"m": "fail", "r": [int(x) for x in r]})
        self._f.flush()
        return r


def replay(path: str) -> Optional[Dict[str, Any]]:
    """Re-run a step log through a fresh scheduler; None when every result
    matches, else {"line", "call", "expected", "got"} of the first mismatch."""
    rt = _rt()
    with open(path) as f:
        recs = [json.loads(line) for line in f if line.strip()]
    if not recs or recs[0].get("m") != "config":
        raise ValueError(f"{path} does not start with a scheduler configuration record")
    c = recs[0]
    s = rt.Scheduler(_make_config(c["sched"]), int(c["num_blocks"]), int(c["block_size"]), bool(c["prefix"]))
    arena = None

    def diff(i, rec, got):
        return {"line": i + 1, "call": rec["m"], "expected": rec.get("r", rec.get("fp")), "got": got}

    import tempfile

    keep = []
    for i, rec in enumerate(recs[1:], start=1):
        m = rec["m"]
        if "t" in rec:
            s.set_clock_ms(float(rec["t"]))
        if m == "enable_cachemesh":
            l2 = torch.zeros(int(rec["n"]), dtype=torch.uint8)
            l3 = tempfile.mkdtemp(prefix="bloom-replay-l3-") if rec["l3"] else ""
            keep.append(l2)
            s.enable_cachemesh(l2, rec["bb"], l3, rec["l3n"], rec["ns"])
        elif m == "set_arena":
            arena = torch.zeros(int(rec["n"]), dtype=torch.int32)
            s.set_arena(arena, *rec["args"])
        elif m == "set_decode_buckets":
            s.set_decode_buckets(rec["b"])
        elif m == "add":
            got = int(s.add_request(rec["prompt"], _make_params(rec["params"]), int(rec["prio"])))
            if got != rec["r"]:
                return diff(i, rec, got)
        elif m == "import":
            rid, table = s.import_sequence(rec["tokens"], rec["np"], rec["nc"], _make_params(rec["params"]),
                                           int(rec["prio"]))
            got = [int(rid), [int(b) for b in table]]
            if got != rec["r"]:
                return diff(i, rec, got)
        elif m == "abort":
            got = bool(s.abort(int(rec["rid"])))
            if got != rec["r"]:
                return diff(i, rec, got)
        elif m == "set_draft":
            s.set_draft(int(rec["rid"]), rec["tokens"])
        elif m == "schedule":
            got = step_fingerprint(s.schedule(), arena)
            if got != rec["fp"]:
                return diff(i, rec, got)
        elif m == "update":
            sampled = torch.tensor(rec["sampled"] or [0], dtype=torch.int32)
            got = _events(s.update(sampled, int(rec["n"])))
            if got != rec["r"]:
                return diff(i, rec, got)
        elif m == "fail":
            got = [int(x) for x in s.fail_scheduled()]
            if got != rec["r"]:
                return diff(i, rec, got)
        elif m in SchedulerRecorder._LOGGED_QUEUES:
            got = [list(map(int, x)) if isinstance(x, (list, tuple)) else int(x) for x in getattr(s, m)()]
            if got != rec["r"]:
                return diff(i, rec, got)
        else:
            raise ValueError(f"{path}:{i + 1}: unknown call {m!r}")
    return None


def main(argv=None) -> int:
    import argparse

    ap = argparse.ArgumentParser(description="replay a scheduler step log and report the first divergence")
    ap.add_argument("log")
    a = ap.parse_args(argv)
    d = replay(a.log)
    print(json.dumps({"reproduced": d is None, "divergence": d}))
    return 0 if d is None else 1


if __name__ == "__main__":
    raise SystemExit(main())
