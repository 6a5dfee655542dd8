"""Text prompt encoder of the LongCat image-edit pipeline: the Qwen2-family
language stack of Qwen2.5-VL run once over the edit-instruction chat
template, its final-normed hidden states being the transformer's prompt
embeddings.

Reference behaviour: executor/longcat_native.rs prompt_context_tensor
:1533-1609 (token embeddings, the decoder layers under a causal mask, the
final RMSNorm, no lm_head) and longcat_qwen_prompt_ids :1778-1792 (the
system instruction and the vision-slot placeholders of the chat template).
Here the stack is the paged serving decoder (`DecoderLM`, tcgen05 GEMMs,
fused RoPE + KV write, paged prefill attention) driven with one prefill
sequence whose every row is an output row.  The Qwen2.5-VL vision tower is
not part of this module: image placeholders are left out of the template
(`image_tokens=0`), so the context is the text-only prompt.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .. import ops
from .config import ModelConfig
from .llama import DecoderLM, StepInputs

# The instruction text has to be the one the transformer was trained with,
# so it is kept verbatim.
EDIT_SYSTEM = ("As an image editing expert, first analyze the content and attributes of the input image(s). "
               "Then, based on the user's editing instructions, clearly and precisely determine how to modify "
               "the given image(s), ensuring that only the specified parts are altered and all other aspects "
               "remain consistent with the original(s).")

BLOCK = 16  # KV block size of the paged cache


def edit_prompt_text(prompt: str, image_tokens: int = 0) -> str:
    """Chat-template text of one edit instruction; `image_tokens` placeholder
    slots go between the vision markers (none: the markers are dropped)."""
    vision = ("<|vision_start|>" + "<|image_pad|>" * image_tokens + "<|vision_end|>") if image_tokens else ""
    return (f"<|im_start|>system\n{EDIT_SYSTEM}<|im_end|>\n<|im_start|>user\n{vision}{prompt}<|im_end|>\n"
            "<|im_start|>assistant\n")


class TextPromptEncoder:
    """[T] token ids -> [T, hidden] bf16 final-normed hidden states."""

    def __init__(self, model: DecoderLM):
        if getattr(model, "wide_attention", False):
            raise ValueError("the prompt encoder runs standard-width attention decoders")
        self.model = model
        self.cfg: ModelConfig = model.cfg
        self.device = model.device

    @staticmethod
    def random(cfg: ModelConfig, seed: int = 0, device=None) -> "TextPromptEncoder":
        m = DecoderLM(cfg, device=device)
        m.random_init(seed)
        return TextPromptEncoder(m)

    def encode_ids(self, ids: Sequence[int]) -> torch.Tensor:
        T = len(ids)
        if T == 0:
            raise ValueError("empty prompt")
        cfg, dev = self.cfg, self.device
        nb = (T + BLOCK - 1) // BLOCK
        kv = torch.zeros(cfg.num_layers, nb, 2, self.model.nkv, BLOCK, cfg.head_dim, dtype=torch.bfloat16,
                         device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        cu = torch.tensor([0, T], dtype=torch.int32)
        ctx = torch.tensor([T], dtype=torch.int32)
        ts, tst = ops.prefill_tiles(cu, ctx)
        s = StepInputs(
            input_ids=torch.as_tensor(list(ids), **i32),
            positions=torch.arange(T, dtype=torch.int64, device=dev),
            slot_mapping=torch.arange(T, **i32),
            num_decode=0, decode_block_table=None, decode_seq_lens=None, decode_splits=1, decode_workspace=None,
            num_prefill=1,
            prefill_block_table=torch.arange(nb, **i32).view(1, nb),
            prefill_ctx_lens=ctx.to(dev), prefill_cu_q=cu.to(dev),
            tile_seq=ts.to(dev), tile_start=tst.to(dev),
            logits_rows=torch.arange(T, **i32),
        )
        return self.model.forward(s, kv)

    def encode(self, prompt: str, tokenizer, max_len: Optional[int] = None) -> torch.Tensor:
        """Prompt text -> hidden states of its edit-template tokens."""
        enc = tokenizer.encode(edit_prompt_text(prompt))
        ids: List[int] = list(enc.ids if hasattr(enc, "ids") else enc)
        if max_len is not None:
            ids = ids[:max_len]
        return self.encode_ids([int(t) % self.cfg.vocab_size for t in ids])


def reference_hidden(cfg: ModelConfig, w, ids: Sequence[int]) -> torch.Tensor:
    """fp32 oracle of `TextPromptEncoder.encode_ids`: the oracle decoder up
    to and including the final RMSNorm."""
    from .reference import forward_logits

    # forward_logits multiplies the normed states by the lm_head: an identity
    # head of width H returns the normed states themselves
    ww = dict(w)
    ww["lm_head.weight"] = torch.eye(cfg.hidden_size, device=w["model.norm.weight"].device)
    return forward_logits(cfg, ww, list(ids))
