"""Text side of generation: tokenizer wrapper, incremental detokenisation,
stop-sequence filtering.

* `Detokenizer` emits text deltas for streaming without re-decoding the whole
  output every step (the reference re-decodes all generated tokens per step,
  executor/candle.rs:1870-1887); it decodes a small window and holds back
  incomplete UTF-8.
* `StopSequenceFilter` withholds text that could be the start of a stop
  string until it is decided, so a stop sequence split across deltas never
  leaks (reference StopSequenceFilter, crates/server/src/helpers.rs:155-237).
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple


class ByteTokenizer:
    """Fallback tokenizer for packages without a vocabulary: one token per UTF-8 byte
    (ids 3..258; 0/1/2 = pad/bos/eos)."""

    bos_id, eos_id = 1, 2

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        return [b + 3 for b in text.encode("utf-8")]

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return bytes([i - 3 for i in ids if 3 <= i < 259]).decode("utf-8", errors="replace")

    def token_to_id(self, s: str) -> Optional[int]:
        return None

    @property
    def vocab_size(self) -> int:
        return 259


class Tokenizer:
    """Thin wrapper over `tokenizers.Tokenizer` (or the byte fallback)."""

    def __init__(self, tok=None):
        self._t = tok if tok is not None else ByteTokenizer()
        self.is_hf = tok is not None

    def encode(self, text: str, add_special_tokens: bool = False) -> List[int]:
        if self.is_hf:
            return self._t.encode(text, add_special_tokens=add_special_tokens).ids
        return self._t.encode(text)

    def decode(self, ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        if self.is_hf:
            return self._t.decode(list(ids), skip_special_tokens=skip_special_tokens)
        return self._t.decode(ids)

    def token_to_id(self, s: str) -> Optional[int]:
        return self._t.token_to_id(s) if self.is_hf else None

    def vocab_strings(self, n: int) -> List[str]:
        return [self.decode([i], skip_special_tokens=False) for i in range(n)]


class Detokenizer:
    """Incremental decoding: text(ids[:k+1]) - text(ids[:k]) without O(n^2) work."""

    def __init__(self, tokenizer: Tokenizer, prefix_window: int = 6):
        self.tok = tokenizer
        self.ids: List[int] = []
        self.prefix_offset = 0
        self.read_offset = 0
        self.window = prefix_window

    def add(self, token: int) -> str:
        self.ids.append(int(token))
        prefix = self.tok.decode(self.ids[self.prefix_offset:self.read_offset])
        full = self.tok.decode(self.ids[self.prefix_offset:])
        if full.endswith("�"):
            return ""  # incomplete UTF-8 sequence: wait for more bytes
        delta = full[len(prefix):]
        self.prefix_offset = max(0, len(self.ids) - self.window)
        self.read_offset = len(self.ids)
        if self.prefix_offset > self.read_offset:
            self.prefix_offset = self.read_offset
        return delta

    def text(self) -> str:
        return self.tok.decode(self.ids)


class StopSequenceFilter:
    """Stream filter that cuts output at the first stop string."""

    def __init__(self, stops: Sequence[str]):
        self.stops = [s for s in stops if s]
        self.pending = ""
        self.stopped = False

    def push(self, delta: str) -> Tuple[str, bool]:
        """Returns (text safe to emit now, stopped)."""
        if self.stopped:
            return "", True
        self.pending += delta
        if not self.stops:
            out, self.pending = self.pending, ""
            return out, False
        first = None
        for s in self.stops:
            i = self.pending.find(s)
            if i >= 0 and (first is None or i < first):
                first = i
        if first is not None:
            out = self.pending[:first]
            self.pending = ""
            self.stopped = True
            return out, True
        # hold back the longest suffix that is a proper prefix of some stop string
        hold = 0
        for s in self.stops:
            for k in range(min(len(s) - 1, len(self.pending)), 0, -1):
                if self.pending.endswith(s[:k]):
                    hold = max(hold, k)
                    break
        out = self.pending[:len(self.pending) - hold]
        self.pending = self.pending[len(self.pending) - hold:]
        return out, False

    def flush(self) -> str:
        out, self.pending = ("" if self.stopped else self.pending), ""
        return out
