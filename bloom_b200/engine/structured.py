"""Structured output: JSON mode (response_format json_object / json_schema).

Each constrained request carries a JSON recogniser (C++ `JsonDfa` in
bloom_b200._runtime).  After the GPU forward of a step, the top-256 logits of
the constrained rows are read back; the first candidate that keeps the
output a valid JSON prefix is emitted, end-of-sequence only once the document
is complete; if no top candidate qualifies the whole vocabulary is searched
in logit order, and end-of-sequence closes the output when nothing fits
(reference: executor/candle.rs:2584-3243 -- autocomplete_json, JsonDfa,
filter_logits_by_grammar with top-256 candidates and EOS gating).
`repair_json` closes an unfinished document (open strings and containers)
when generation stops on the token limit.
"""
from __future__ import annotations

import json
from typing import Dict, List, Optional

from .._ext import runtime as _rt

TOPK = 256
_VOCAB_CACHE: Dict[int, List[str]] = {}


def vocab_strings(tokenizer, n: int) -> List[str]:
    key = id(tokenizer)
    v = _VOCAB_CACHE.get(key)
    if v is None or len(v) < n:
        v = [tokenizer.decode([i], skip_special_tokens=False) for i in range(n)]
        _VOCAB_CACHE[key] = v
    return v


class JsonConstraint:
    def __init__(self, vocab: List[str], eos: List[int]):
        self.dfa = _rt().JsonDfa()
        self.vocab = vocab
        self.eos = list(eos)

    def choose(self, candidates: List[int], fallback: int, full_order=None) -> int:
        """First candidate that keeps the document a valid JSON prefix.  When
        none of the top candidates qualifies, `full_order()` (the whole
        vocabulary by descending logit) is searched; if still nothing fits,
        the document is ended with the first end-of-sequence id."""
        t = self.dfa.pick(candidates, self.vocab, self.eos)
        if t < 0 and full_order is not None:
            t = self.dfa.pick(full_order(), self.vocab, self.eos)
        if t < 0:
            return self.eos[0] if self.eos else fallback
        return t

    def advance(self, token: int) -> None:
        if token in self.eos or not (0 <= token < len(self.vocab)):
            return
        self.dfa.feed(self.vocab[token])


def constrain_params(params, response_format: dict, pipeline) -> None:
    params.json_mode = True


def repair_json(text: str) -> str:
    """Close an unfinished JSON document; valid documents are returned unchanged."""
    try:
        json.loads(text)
        return text
    except ValueError:
        pass
    stack: List[str] = []
    in_str = esc = False
    start = text.find("{") if "{" in text else text.find("[")
    if start < 0:
        return "{}"
    body = text[start:]
    for c in body:
        if in_str:
            if esc:
                esc = False
            elif c == "\\":
                esc = True
            elif c == '"':
                in_str = False
            continue
        if c == '"':
            in_str = True
        elif c in "{[":
            stack.append("}" if c == "{" else "]")
        elif c in "}]" and stack:
            stack.pop()
    out = body + ('"' if in_str else "")
    out = out.rstrip().rstrip(",").rstrip(":")
    if out.endswith(","):
        out = out[:-1]
    out += "".join(reversed(stack))
    try:
        json.loads(out)
        return out
    except ValueError:
        return "{}"
