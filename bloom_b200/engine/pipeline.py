"""InferencePipeline: load a model package and run requests (CLI, server, C ABI).

Reference semantics (crates/engine/src/core/pipeline.rs):
  * DEFAULT_CONTEXT_SIZE 2048 (:13); the context is clamped to the model's
    limit (:119-129);
  * OOM degradation ladder unless strict: halve the context down to 512, then
    fall back to the CPU engine, then context 128; at most 5 attempts
    (:133-259); BLOOM_STRICT_MEMORY_BUDGET=1 refuses any change (:261-277);
  * hash verification with BLOOM_ALLOW_HASH_MISMATCH (:99-117);
  * run / run_stream / run_embedding_batch / tokenize / detokenize (:375-483).
A model argument may also be a preset name (random-initialised weights of a
named architecture, used by benchmarks and tests).
"""
from __future__ import annotations

import os
import statistics
import time
from typing import Dict, Iterator, List, Optional

import torch

from ..models.config import PRESETS, ModelConfig, preset
from .chat_template import STOP_TOKENS, classify_template, render, select_template
from .registry import FALLBACK, NATIVE, default_registry
from .text import Detokenizer, StopSequenceFilter, Tokenizer

DEFAULT_CONTEXT_SIZE = 2048


def _is_oom(e: BaseException) -> bool:
    s = str(e).lower()
    return isinstance(e, torch.cuda.OutOfMemoryError) or "out of memory" in s or "cuda error: out of memory" in s


class InferencePipeline:
    def __init__(self, engine_name: str, cfg: ModelConfig, tokenizer: Tokenizer, template: str, context_size: int,
                 llm=None, cpu=None, embedder=None, manifest=None, device: str = "gpu", spec=None):
        self.engine_name = engine_name
        self.cfg = cfg
        self.tokenizer = tokenizer
        self.template = template
        self.context_size = context_size
        self.llm = llm
        self.cpu = cpu
        self.embedder = embedder
        self.manifest = manifest
        self.device = device
        self.spec = spec
        self.last_generated_tokens = 0
        self.stop_strings = STOP_TOKENS.get(template, [])

    # ------------------------------------------------------------ loading
    @property
    def is_embedding(self) -> bool:
        return self.cfg.arch == "bert"

    @staticmethod
    def inspect(model: str, context_size: int = DEFAULT_CONTEXT_SIZE, registry=None, tp: int = 1) -> dict:
        """Metadata-only description (loads no weights): keys of the reference's
        --inspect output (bloom_infer.rs:1183-1231)."""
        from ..formats.manifest import estimate_memory, load_manifest

        reg = registry or default_registry()
        if model in PRESETS:
            cfg = preset(model)
            man = {"id": model, "family": cfg.arch, "primary_dtype": "BF16", "parameters": cfg.__dict__}
            return {"model_path": model, "selected_engine": "b200", "selected_engine_maturity": "Beta",
                    "context_size": min(context_size, cfg.max_position_embeddings), "manifest": man,
                    "memory_estimate": None, "engines": reg.describe(), "notes": ["preset: random-initialised weights"]}
        man = load_manifest(model)
        fmt = man.files[0].format if man.files else "Unknown"
        fam = man.family if isinstance(man.family, str) else list(man.family.values())[0]
        eng, lvl = reg.route(fam, fmt, man.primary_dtype, "gpu" if torch.cuda.is_available() else "cpu")
        ctx = min(context_size, int(man.parameters.get("max_position_embeddings", context_size)))
        est = estimate_memory(man, ctx, tp=tp)
        notes = []
        if lvl == FALLBACK:
            notes.append(f"{man.primary_dtype} weights run on the {eng} engine through a fallback path")
        if man.is_embedding:
            notes.append("embedding model: use the HTTP server's /v1/embeddings")
        cap = reg.get(eng) if eng else None
        return {"model_path": os.path.abspath(model), "selected_engine": eng,
                "selected_engine_maturity": cap.maturity if cap else None, "context_size": ctx,
                "manifest": man.to_dict(), "memory_estimate": est.to_dict(), "engines": reg.describe(),
                "notes": notes}

    @staticmethod
    def load(model: str, device: str = "gpu", context_size: int = DEFAULT_CONTEXT_SIZE, tp: int = 1,
             use_cuda_graphs: bool = True, template: Optional[str] = None, strict: Optional[bool] = None,
             speculative: str = "none", draft_model: Optional[str] = None, num_speculative_tokens: int = 5,
             ngram_order: int = 4, max_num_seqs: int = 64, tp_info=None, gpu_layers: Optional[int] = None,
             pp_info=None,
             max_num_batched_tokens: Optional[int] = None, threads: Optional[int] = None) -> "InferencePipeline":
        """`gpu_layers`: layers kept in HBM (the rest stream from pinned host
        memory; default all, or BLOOM_GPU_LAYERS); `max_num_batched_tokens`:
        tokens per engine step (the prefill chunk); `threads`: host CPU threads
        of the native kernels."""
        if threads:
            from .._ext import runtime as _rt

            _rt().set_num_threads(int(threads))
        if gpu_layers is None and os.environ.get("BLOOM_GPU_LAYERS"):
            gpu_layers = int(os.environ["BLOOM_GPU_LAYERS"])
        if strict is None:
            strict = os.environ.get("BLOOM_STRICT_MEMORY_BUDGET", "0") == "1"
        attempts = 0
        ctx = context_size
        dev = device
        last = None
        while attempts < 5:
            attempts += 1
            try:
                return InferencePipeline._load_once(model, dev, ctx, tp, use_cuda_graphs, template, speculative,
                                                    draft_model, num_speculative_tokens, ngram_order, max_num_seqs,
                                                    tp_info, gpu_layers, max_num_batched_tokens, pp_info)
            except Exception as e:  # degradation ladder on OOM only
                if not _is_oom(e) or strict:
                    raise
                last = e
                torch.cuda.empty_cache()
                if dev == "gpu" and ctx > 512:
                    ctx = max(512, ctx // 2)
                elif dev == "gpu":
                    dev = "cpu"
                elif ctx > 128:
                    ctx = 128
                else:
                    break
        raise RuntimeError(f"could not load {model} within the memory budget: {last}")

    @staticmethod
    def _load_once(model, device, ctx, tp, use_cuda_graphs, template, speculative, draft_model, nspec, ngram_order,
                   max_num_seqs, tp_info, gpu_layers=None, max_num_batched_tokens=None, pp_info=None):
        from ..formats.loader import load_tokenizer, load_weights, model_config
        from ..formats.manifest import load_manifest, verify_hashes

        if model == "echo":
            return EchoPipeline()
        if model in PRESETS:
            cfg = preset(model)
            man = None
            tok = Tokenizer(None)
            weights = None
        else:
            man = load_manifest(model)
            verify_hashes(man)
            cfg = model_config(man)
            hf_tok = load_tokenizer(model)
            tok = Tokenizer(hf_tok)
            weights = None
        ctx = min(ctx, cfg.max_position_embeddings)
        kind = template
        if kind is None:
            jinja = None
            if man is not None:
                tc = os.path.join(man.root, "tokenizer_config.json")
                if os.path.exists(tc):
                    import json

                    with open(tc) as f:
                        jinja = json.load(f).get("chat_template")
                if jinja is None and man.files and man.files[0].format == "Gguf":
                    from ..formats.gguf import GGUFFile

                    jinja = GGUFFile(os.path.join(man.root, man.files[0].name)).metadata.get("tokenizer.chat_template")
            fam = {"llama": "llama", "qwen2": "qwen", "qwen3": "qwen", "qwen3_moe": "qwen"}.get(cfg.arch, "")
            kind = select_template(fam, cfg.arch, classify_template(jinja))
            if cfg.arch == "llama" and jinja is None and cfg.vocab_size >= 128000:
                kind = "llama3"
        if cfg.arch == "bert":
            from ..models.bert import BertEmbedder

            emb = BertEmbedder.load(model, device="cuda" if device == "gpu" else "cpu")
            return InferencePipeline("b200", cfg, tok, kind, ctx, embedder=emb, manifest=man, device=device)
        if device == "cpu":
            from .cpu_engine import CpuDecoder

            if man is not None and man.files and man.files[0].format == "Gguf":
                cpu = CpuDecoder.from_gguf(os.path.join(man.root, man.files[0].name))
            else:
                from ..models.reference import random_weights

                w = load_weights(man) if man is not None else random_weights(cfg)
                cpu = CpuDecoder.from_weights(cfg, w)
            return InferencePipeline("cpu", cfg, tok, kind, ctx, cpu=cpu, manifest=man, device="cpu")
        from .engine import EngineConfig, LLMEngine
        from ..models.llama import DecoderLM

        if man is None:
            from ..models import build_decoder

            dm = build_decoder(cfg, tp_info, None, pp=pp_info)
            dm.random_init(0)
        else:
            from ..formats.loader import load_decoder

            dm = load_decoder(model, tp_info, None, pp=pp_info)
        if gpu_layers is not None and gpu_layers < cfg.num_layers:
            dm.place_layers(gpu_layers)
        spec_len = nspec if speculative in ("ngram", "draft") else 0
        budget = int(max_num_batched_tokens) if max_num_batched_tokens else max(ctx, 2048)
        llm = LLMEngine(dm, EngineConfig(max_num_seqs=max_num_seqs, max_num_batched_tokens=budget,
                                         max_model_len=ctx, use_cuda_graphs=use_cuda_graphs, spec_len=spec_len))
        llm.tokenizer = tok
        spec = None
        if speculative in ("ngram", "draft"):
            from .speculative import make_speculator

            spec = make_speculator(speculative, llm, draft_model, nspec, ngram_order)
        return InferencePipeline("b200", cfg, tok, kind, ctx, llm=llm, manifest=man, device="gpu", spec=spec)

    # ------------------------------------------------------------ text helpers
    def tokenize(self, text: str) -> List[int]:
        return self.tokenizer.encode(text)

    def detokenize(self, ids: List[int]) -> str:
        return self.tokenizer.decode(ids)

    def prompt_ids(self, messages, raw: bool = False) -> List[int]:
        if isinstance(messages, str):
            text = messages if raw else render([{"role": "user", "content": messages}], self.template)
        else:
            text = "\n".join(m["content"] for m in messages) if raw else render(messages, self.template)
        ids = self.tokenizer.encode(text)
        if not ids:
            ids = [self.cfg.bos_token_id or 1]
        return ids

    def eos_ids(self) -> List[int]:
        ids = list(self.cfg.eos_token_ids)
        for s in self.stop_strings:
            t = self.tokenizer.token_to_id(s)
            if t is not None and t not in ids:
                ids.append(t)
        return ids

    # ------------------------------------------------------------ generation
    def run_stream(self, messages, params, raw: bool = False, stop: Optional[List[str]] = None,
                   prompt_ids: Optional[List[int]] = None) -> Iterator[str]:
        ids = prompt_ids if prompt_ids is not None else self.prompt_ids(messages, raw)
        if len(ids) + 1 >= self.context_size:
            raise ValueError(f"prompt of {len(ids)} tokens does not fit the context of {self.context_size}")
        max_new = min(params.max_tokens, self.context_size - len(ids) - 1)
        detok = Detokenizer(self.tokenizer)
        filt = StopSequenceFilter(list(stop or []))
        eos = self.eos_ids()
        self.last_generated_tokens = 0
        if self.cpu is not None:
            toks = self.cpu.generate(ids, max_new, params.temperature, params.top_p, params.seed, eos,
                                     params.ignore_eos)
        else:  # speculation, when configured, is attached to the engine itself
            from dataclasses import replace

            p2 = replace(params, max_tokens=max_new, stop_token_ids=list(set(params.stop_token_ids) | set(eos)))
            toks = self.llm.stream(ids, p2)
        for t in toks:
            self.last_generated_tokens += 1
            if t in eos and not params.ignore_eos:
                break
            out, stopped = filt.push(detok.add(t))
            if out:
                yield out
            if stopped:
                return
        tail = filt.flush()
        if tail:
            yield tail

    def run(self, messages, params, raw: bool = False, stop=None) -> str:
        from ..utils.tracing import span

        with span("pipeline.run", engine=self.engine_name):
            return "".join(self.run_stream(messages, params, raw, stop))

    def run_embedding_batch(self, texts: List[str]) -> List[List[float]]:
        if self.embedder is None:
            raise ValueError("not an embedding model")
        return self.embedder.embed(texts)

    def benchmark(self, messages, params, repetitions: int = 3, warmup: int = 1, raw: bool = False) -> dict:
        """bloom_bench-style single-request benchmark (reference bloom_bench.rs:257-800):
        TTFT at the first delta, TBT = (duration - TTFT) / (generated - 1)."""
        for _ in range(warmup):
            for _ in self.run_stream(messages, params, raw):
                pass
        runs = []
        for _ in range(repetitions):
            t0 = time.perf_counter()
            ttft = None
            for _ in self.run_stream(messages, params, raw):
                if ttft is None:
                    ttft = time.perf_counter() - t0
            dur = time.perf_counter() - t0
            n = self.last_generated_tokens
            runs.append((ttft or dur, dur, n))
        ttft = statistics.mean(r[0] for r in runs)
        dur = statistics.mean(r[1] for r in runs)
        n = statistics.mean(r[2] for r in runs)
        return {"engine": self.engine_name, "device": self.device, "ttft_ms": ttft * 1e3,
                "tbt_ms": (dur - ttft) / max(n - 1, 1) * 1e3, "tokens_per_second": n / dur if dur > 0 else 0.0,
                "generated_tokens": n, "total_duration_ms": dur * 1e3, "repetitions": repetitions, "warmup": warmup,
                "prompt_tokens": len(self.prompt_ids(messages, raw))}


class EchoPipeline(InferencePipeline):
    """Deterministic test model: streams "echo: " + the prompt (reference EchoTextModel,
    crates/engine/src/core/model.rs:339-375)."""

    def __init__(self):
        from ..models.config import ModelConfig

        super().__init__("echo", ModelConfig(arch="llama", name="echo", vocab_size=259), Tokenizer(None), "legacy",
                         DEFAULT_CONTEXT_SIZE, device="cpu")

    def run_stream(self, messages, params, raw: bool = False, stop=None, prompt_ids=None) -> Iterator[str]:
        text = messages if isinstance(messages, str) else messages[-1]["content"]
        out = "echo: " + text
        words = out.split(" ")
        n = min(len(words), max(1, params.max_tokens))
        self.last_generated_tokens = n
        filt = StopSequenceFilter(list(stop or []))
        for i in range(n):
            piece = words[i] if i == 0 else " " + words[i]
            o, stopped = filt.push(piece)
            if o:
                yield o
            if stopped:
                return
        tail = filt.flush()
        if tail:
            yield tail

    accepts_images = True

    def run_multimodal(self, blocks, params) -> Iterator[str]:
        """Echo of a multimodal request: its text, and each image's size."""
        from .processor import decode_image
        from .vl_pipeline import parse_blocks

        parts = []
        for kind, v in parse_blocks(blocks):
            if kind == "Text":
                parts.append(v)
            elif kind == "Tokens":
                parts.append(self.tokenizer.decode(v))
            else:
                img = decode_image(*v)
                parts.append(f"[image {img.shape[1]}x{img.shape[0]}]")
        words = ("echo: " + " ".join(parts)).split(" ")
        n = min(len(words), max(1, getattr(params, "max_tokens", 128)))
        self.last_generated_tokens = n
        for i in range(n):
            yield words[i] if i == 0 else " " + words[i]

