"""Vision-language pipeline: multimodal requests (text, token and image
blocks) through a Qwen3-VL model, one request at a time with streamed text.

A request is a list of blocks in the reference's DataBlock form:
    {"Text": "..."}, {"Tokens": [ids]}, {"Image": {"bytes": [...] | base64, "mime": "image/png"}}
Images are decoded and cut into patches by engine.processor; each image
becomes vision-start, one image-pad token per merged vision token, and
vision-end in the prompt (at most one image per request, as in the
reference's upload route).  When the tokenizer knows the ChatML markers the
prompt is wrapped as a user turn followed by the assistant header.
Reference: crates/server/src/handlers.rs:4502-4600 (multimodal stream and
upload), crates/engine/src/executor/qwen3_vl.rs (request assembly).
"""
from __future__ import annotations

import base64
from typing import Any, Dict, Iterator, List, Optional, Tuple

from .processor import ProcessorError, decode_image, qwen_vl_patches
from .text import Detokenizer, Tokenizer


def parse_blocks(blocks: Any) -> List[Tuple[str, Any]]:
    """Validated (kind, value) pairs; image bytes decoded from a list or base64."""
    if not isinstance(blocks, list) or not blocks:
        raise ProcessorError("blocks must be a non-empty array")
    out = []
    for b in blocks:
        if not isinstance(b, dict) or len(b) != 1:
            raise ProcessorError("each block must be an object with exactly one of Text, Tokens, Image")
        kind, v = next(iter(b.items()))
        if kind == "Text" and isinstance(v, str):
            out.append(("Text", v))
        elif kind == "Tokens" and isinstance(v, list) and all(isinstance(t, int) and t >= 0 for t in v):
            out.append(("Tokens", v))
        elif kind == "Image" and isinstance(v, dict):
            raw = v.get("bytes")
            data = base64.b64decode(raw) if isinstance(raw, str) else bytes(raw or [])
            if not data:
                raise ProcessorError("Image block without bytes")
            out.append(("Image", (data, str(v.get("mime", "")))))
        else:
            raise ProcessorError(f"unsupported block {kind!r}")
    if sum(1 for k, _ in out if k == "Image") > 1:
        raise ProcessorError("Only one image attachment is supported per request.")
    return out


class VisionLanguagePipeline:
    engine_name = "qwen3-vl"
    is_embedding = False
    accepts_images = True
    template = "chatml"

    def __init__(self, model, tokenizer: Optional[Tokenizer] = None, context_size: int = 4096, max_pixels: int = 1 << 20):
        self.model = model
        self.cfg = model.cfg.text
        self.tokenizer = tokenizer or Tokenizer(None)
        self.context_size = context_size
        self.max_pixels = max_pixels
        self.last_generated_tokens = 0

    @staticmethod
    def from_preset(name: str, device: str = "cuda", seed: int = 0, **kw) -> "VisionLanguagePipeline":
        from ..models.qwen3_vl import Qwen3VL, vl_preset

        cfg = vl_preset(name)
        m = Qwen3VL(cfg, device)
        m.load(Qwen3VL.random_weights(cfg, seed=seed))
        return VisionLanguagePipeline(m, **kw)

    def eos_ids(self) -> List[int]:
        return list(self.cfg.eos_token_ids)

    def _marker(self, s: str) -> Optional[int]:
        try:
            return self.tokenizer.token_to_id(s)
        except Exception:
            return None

    def build(self, blocks) -> Tuple[List[int], Any, Any]:
        """(prompt ids, patches or None, grid or None)."""
        vc = self.model.cfg
        ids: List[int] = []
        patches = grid = None
        for kind, v in parse_blocks(blocks):
            if kind == "Text":
                ids += self.tokenizer.encode(v)
            elif kind == "Tokens":
                ids += [int(t) for t in v]
            else:
                img = decode_image(*v)
                patches, grid = qwen_vl_patches(img, vc.vision, max_pixels=self.max_pixels)
                n = grid[0] * grid[1] * grid[2] // vc.vision.spatial_merge_size ** 2
                ids += [vc.vision_start_token_id] + [vc.image_token_id] * n + [vc.vision_end_token_id]
        s, e = self._marker("<|im_start|>"), self._marker("<|im_end|>")
        if s is not None and e is not None:
            ids = [s] + self.tokenizer.encode("user\n") + ids + [e] + self.tokenizer.encode("\n") + [s] + \
                self.tokenizer.encode("assistant\n")
        if len(ids) >= self.context_size:
            raise ProcessorError(f"prompt has {len(ids)} tokens; the context window is {self.context_size}")
        return ids, patches, grid

    def run_multimodal(self, blocks, params) -> Iterator[str]:
        """Streams text deltas of a greedy continuation."""
        import queue
        import threading

        ids, patches, grid = self.build(blocks)
        q: "queue.Queue" = queue.Queue()
        detok = Detokenizer(self.tokenizer)
        eos = set(self.eos_ids()) | set(getattr(params, "stop_token_ids", []) or [])
        max_tokens = min(int(getattr(params, "max_tokens", 64)), self.context_size - len(ids) - 1)
        err: List[BaseException] = []

        def work():
            try:
                out = self.model.generate(ids, patches, grid, max_tokens=max(1, max_tokens), eos=tuple(eos),
                                          on_token=q.put)
                self.last_generated_tokens = len(out)
            except BaseException as ex:  # surfaced to the caller below
                err.append(ex)
            q.put(None)

        threading.Thread(target=work, daemon=True).start()
        while True:
            tok = q.get()
            if tok is None:
                break
            if tok in eos:
                continue
            d = detok.add(tok)
            if d:
                yield d
        if err:
            raise err[0]

    def run_stream(self, messages, params, raw: bool = False, stop=None, prompt_ids=None) -> Iterator[str]:
        text = messages if isinstance(messages, str) else "\n".join(m.get("content", "") for m in messages)
        blocks = [{"Tokens": list(prompt_ids)}] if prompt_ids else [{"Text": text}]
        yield from self.run_multimodal(blocks, params)
