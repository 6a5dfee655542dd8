"""Chat prompt templates, selected by token contract (templates are never executed).

The prompt strings of each family are the families' own token contracts, so
they are reproduced exactly (reference: crates/server/src/chat_template.rs:12-213,
crates/engine/src/bin/bloom_infer.rs:431-560): ChatML (Qwen, generic),
SmolLM2 (ChatML with a default system turn), Qwen3 with thinking disabled,
Llama-2 [INST], Llama-3 header ids, Gemma turns.  A Jinja `chat_template`
found in tokenizer_config.json or GGUF metadata is only *classified* by the
special tokens it mentions (reference manifest.rs:669-698).
"""
from __future__ import annotations

from typing import Dict, List, Optional

IM_START, IM_END = "<|im_start|>", "<|im_end|>"


def _chatml(messages: List[Dict[str, str]]) -> str:
    out = "".join(f"{IM_START}{m['role']}\n{m['content']}{IM_END}\n" for m in messages)
    return out + f"{IM_START}assistant\n"


def _smollm2(messages):
    pre = ""
    if not messages or messages[0]["role"] != "system":
        pre = f"{IM_START}system\nYou are a helpful AI assistant named SmolLM, trained by Hugging Face{IM_END}\n"
    return pre + _chatml(messages)


def _qwen3_no_think(messages):
    return _chatml(messages) + "<think>\n\n</think>\n\n"


def _llama2(messages):
    out = "<s>"
    i = 0
    if messages and messages[0]["role"] == "system":
        sysm = messages[0]["content"]
        if len(messages) > 1 and messages[1]["role"] == "user":
            out += f"[INST] <<SYS>>\n{sysm}\n<</SYS>>\n\n{messages[1]['content']} [/INST]"
            i = 2
        else:
            out += f"[INST] <<SYS>>\n{sysm}\n<</SYS>> [/INST]"
            i = 1
    for m in messages[i:]:
        if m["role"] == "user":
            out += f"<s>[INST] {m['content']} [/INST]"
        elif m["role"] == "assistant":
            out += f" {m['content']} </s>"
        else:
            out += f"[INST] {m['content']} [/INST]"
    return out


def _llama3(messages):
    out = "<|begin_of_text|>"
    for m in messages:
        out += f"<|start_header_id|>{m['role']}<|end_header_id|>\n\n{m['content']}<|eot_id|>"
    return out + "<|start_header_id|>assistant<|end_header_id|>\n\n"


def _gemma(messages):
    out = "".join(f"<start_of_turn>{m['role']}\n{m['content']}<end_of_turn>\n" for m in messages)
    return out + "<start_of_turn>model\n"


def _legacy(messages):
    parts = []
    for m in messages:
        parts.append(f"{m['role'].capitalize()}: {m['content']}")
    return "\n".join(parts) + "\nAssistant:"


TEMPLATES = {"chatml": _chatml, "qwen": _chatml, "generic": _chatml, "smollm2": _smollm2,
             "qwen3-no-think": _qwen3_no_think, "llama2": _llama2, "llama": _llama2, "llama3": _llama3,
             "gemma": _gemma, "legacy": _legacy}

STOP_TOKENS = {"chatml": ["<|im_end|>"], "qwen": ["<|im_end|>"], "generic": ["<|im_end|>"],
               "smollm2": ["<|im_end|>"], "qwen3-no-think": ["<|im_end|>"], "llama2": ["</s>"],
               "llama": ["</s>"], "llama3": ["<|eot_id|>", "<|end_of_text|>"], "gemma": ["<end_of_turn>"],
               "legacy": []}


def classify_template(jinja: Optional[str]) -> Optional[str]:
    """Template kind from the special tokens a Jinja chat template mentions."""
    if not jinja:
        return None
    if "<|start_header_id|>" in jinja:
        return "llama3"
    if "<start_of_turn>" in jinja:
        return "gemma"
    if "[INST]" in jinja:
        return "llama2"
    if "<|im_start|>" in jinja:
        if "SmolLM" in jinja:
            return "smollm2"
        return "chatml"
    return None


def select_template(family: str = "", architecture: Optional[str] = None, kind: Optional[str] = None) -> str:
    fam = (family or "").lower()
    if fam == "qwen" and (architecture or "").lower() == "qwen3":
        return "qwen3-no-think"
    if kind and kind.lower() in TEMPLATES:
        return kind.lower()
    return {"qwen": "chatml", "llama": "llama2", "gemma": "gemma"}.get(fam, "generic")


def render(messages: List[Dict[str, str]], kind: str) -> str:
    return TEMPLATES.get(kind, _chatml)(messages)
