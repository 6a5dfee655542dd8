"""Load a model package (bloom.json / HF directory / GGUF) into this engine.

Decoder weights are read on the host (memory-mapped safetensors or GGUF
blocks), sharded for the local tensor-parallel rank and moved to the GPU as
bf16 in the kernels' layout.  GGUF Q8_0/Q4_0 blocks are dequantised on the
host (C++ kernels of bloom_b200._runtime) before upload.
"""
from __future__ import annotations

import json
import os
from typing import Optional

import torch

from ..models.config import ModelConfig, from_hf_config
from .manifest import ModelManifest, load_manifest


def model_config(man: ModelManifest) -> ModelConfig:
    gg = [f for f in man.files if f.format == "Gguf"]
    if gg:
        from .gguf import GGUFFile, config_from_gguf

        return config_from_gguf(GGUFFile(os.path.join(man.root, gg[0].name)))
    with open(os.path.join(man.root, "config.json")) as f:
        return from_hf_config(json.load(f))


def load_weights(man: ModelManifest, device=None) -> dict:
    gg = [f for f in man.files if f.format == "Gguf"]
    if gg:
        from .gguf import GGUFFile, load_hf_weights

        return load_hf_weights(GGUFFile(os.path.join(man.root, gg[0].name)))
    from .quant_config import QuantizationConfig, dequantize_checkpoint
    from .safetensors_io import load_state_dict

    sd = load_state_dict(man.root)
    # AWQ / GPTQ / bitsandbytes 4-bit checkpoints: packed layers -> bf16 weights
    sd = dequantize_checkpoint(sd, QuantizationConfig.from_model_dir(man.root), device)
    # HF checkpoints of MoE models keep experts as separate tensors: stack them
    out = {}
    experts = {}
    for k, v in sd.items():
        if ".mlp.experts." in k and k.endswith(".weight"):
            pre, rest = k.split(".mlp.experts.")
            e, proj, _ = rest.split(".")
            experts.setdefault((pre, proj), {})[int(e)] = v
        else:
            out[k] = v
    for (pre, proj), d in experts.items():
        out[f"{pre}.mlp.experts.{proj}"] = torch.stack([d[i] for i in sorted(d)])
    return out


def load_decoder(path: str, tp=None, device=None, pp=None):
    from ..utils.tracing import span

    with span("model.load", path=str(path)):
        return _load_decoder(path, tp, device, pp)


def _load_decoder(path: str, tp=None, device=None, pp=None):
    from ..models import build_decoder

    man = load_manifest(path)
    cfg = model_config(man)
    model = build_decoder(cfg, tp, device, pp=pp)
    gg = [f for f in man.files if f.format == "Gguf"]
    if gg and (tp is None or tp.size == 1) and man.primary_dtype in ("Q8", "Q4") and hasattr(model, "load_gguf"):
        # Q8_0 / Q4_0 projections stay block-quantised on the GPU (qgemv / dequant + tcgen05)
        model.load_gguf(os.path.join(man.root, gg[0].name), quantized=True)
        return model
    w = load_weights(man, device if torch.cuda.is_available() else None)
    model.shard_full(w)
    return model


def load_tokenizer(path: str):
    """HF `tokenizers.Tokenizer` from tokenizer.json, or synthesised from GGUF metadata."""
    from tokenizers import Tokenizer

    man = load_manifest(path)
    tj = os.path.join(man.root, "tokenizer.json")
    if os.path.exists(tj):
        return Tokenizer.from_file(tj)
    gg = [f for f in man.files if f.format == "Gguf"]
    if gg:
        from .gguf import GGUFFile, tokenizer_json_from_gguf

        d = tokenizer_json_from_gguf(GGUFFile(os.path.join(man.root, gg[0].name)))
        if d is not None:
            return Tokenizer.from_str(json.dumps(d))
    return None
