"""bloom_infer: run one prompt through a model package.

    python -m bloom_b200.cli.infer --model PATH|PRESET --prompt "..." [--stream]
    python -m bloom_b200.cli.infer --model PATH --inspect          (metadata-only JSON, loads no weights)

Flags and defaults follow the reference CLI (crates/engine/src/bin/
bloom_infer.rs:88-287): -m/--model, -p/--prompt ('-' reads stdin),
--prompt-file, --system-prompt, --max-tokens/--num-predict 128,
--temperature/--temp 0.7, --top-p 0.9, --seed, --stream, --device cpu|gpu,
--context-size/--ctx-size 2048, --speculative none|ngram|draft,
--draft-model, --num-speculative-tokens 5, --speculative-ngram-order 4,
-i/--interactive, --list-engines, --bench, --inspect, --repetitions,
--warmup, --bench-json, --quiet, --config, --init-config; B200 additions:
--tp, --no-cuda-graphs, --template.  Precedence: CLI > config file
(~/.bloom/config.json or BLOOM_CONFIG, section "infer") > defaults.
Text goes to stdout, metrics to stderr; --bench-json prints a BenchmarkResult.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from typing import List, Optional

DEFAULTS = {"max_tokens": 128, "temperature": 0.7, "top_p": 0.9, "context_size": 2048, "device": "gpu",
            "num_speculative_tokens": 5, "speculative_ngram_order": 4, "speculative": "none", "repetitions": 3,
            "warmup": 1}


def config_path() -> str:
    return os.environ.get("BLOOM_CONFIG") or os.path.join(os.path.expanduser("~"), ".bloom", "config.json")


def load_config(path: Optional[str] = None) -> dict:
    p = path or config_path()
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def example_config() -> dict:
    return {"infer": {"max_tokens": 128, "temperature": 0.7, "top_p": 0.9, "context_size": 2048, "device": "gpu"},
            "server": {"host": "127.0.0.1", "port": 3000, "max_concurrent": 4, "context_size": 2048},
            "bench": {"repetitions": 3, "warmup": 1}}


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="bloom_infer", description="Run a prompt through a model (B200 engine)")
    ap.add_argument("-m", "--model", help="model directory, bloom.json, .gguf file or preset name")
    ap.add_argument("-p", "--prompt", help="prompt text ('-' reads stdin)")
    ap.add_argument("--prompt-file")
    ap.add_argument("--system-prompt")
    ap.add_argument("--max-tokens", "--num-predict", dest="max_tokens", type=int)
    ap.add_argument("--temperature", "--temp", dest="temperature", type=float)
    ap.add_argument("--top-p", dest="top_p", type=float)
    ap.add_argument("--top-k", dest="top_k", type=int, default=0)
    ap.add_argument("--seed", type=int)
    ap.add_argument("--stream", action="store_true")
    ap.add_argument("--device", choices=["cpu", "gpu"])
    ap.add_argument("--backend", "--engine", dest="backend", default=None)
    ap.add_argument("--dtype", default=None)
    ap.add_argument("--context-size", "--ctx-size", dest="context_size", type=int)
    ap.add_argument("--threads", type=int, help="host CPU threads of the native kernels")
    ap.add_argument("--batch-size", type=int, help="tokens per engine step (the prefill chunk)")
    ap.add_argument("--gpu-layers", type=int,
                    help="layers kept in HBM; the others stream from pinned host memory each step")
    ap.add_argument("--speculative", choices=["none", "ngram", "draft", "mtp"])
    ap.add_argument("--draft-model")
    ap.add_argument("--num-speculative-tokens", type=int)
    ap.add_argument("--speculative-ngram-order", type=int)
    ap.add_argument("--image", help="PNG / PPM image for a vision-language model (a Qwen3-VL preset or package)")
    ap.add_argument("-i", "--interactive", action="store_true")
    ap.add_argument("--list-engines", action="store_true")
    ap.add_argument("--bench", action="store_true")
    ap.add_argument("--inspect", action="store_true")
    ap.add_argument("--repetitions", type=int)
    ap.add_argument("--warmup", type=int)
    ap.add_argument("--bench-json", action="store_true")
    ap.add_argument("--quiet", action="store_true")
    ap.add_argument("--config")
    ap.add_argument("--init-config", action="store_true")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--no-cuda-graphs", action="store_true")
    ap.add_argument("--template", default=None, help="chat template override (chatml, llama3, llama2, gemma, ...)")
    ap.add_argument("--raw", action="store_true", help="do not apply a chat template")
    # text-to-video (--backend wan; bloom_infer.rs VideoGeneration arguments)
    ap.add_argument("--negative-prompt", default=None)
    ap.add_argument("--width", type=int, default=832)
    ap.add_argument("--height", type=int, default=480)
    ap.add_argument("--num-frames", type=int, default=81)
    ap.add_argument("--fps", type=float, default=16.0)
    ap.add_argument("--guidance-scale", type=float, default=5.0)
    ap.add_argument("--num-steps", type=int, default=50)
    ap.add_argument("-o", "--output", default=None, help="video output: .gif, or a directory / .png for PNG frames")
    return ap


def resolve(args, cfg: dict) -> dict:
    sec = cfg.get("infer", {})
    out = {}
    for k, d in DEFAULTS.items():
        v = getattr(args, k, None)
        out[k] = v if v is not None else sec.get(k, d)
    return out


def read_prompt(args) -> Optional[str]:
    if args.prompt_file:
        with open(args.prompt_file) as f:
            return f.read()
    if args.prompt == "-":
        return sys.stdin.read()
    return args.prompt


def run_image_edit(args) -> int:
    """LongCat draft image edit: --image input (PNG / PPM), --output PNG.
    --model names 'transformer[:vae]' presets (random weights: no checkpoint
    download here); the prompt embeddings are a deterministic function of the
    prompt bytes until a text encoder checkpoint is loaded."""
    import torch

    from ..engine.processor import decode_image
    from ..models.longcat import LongCatEditPipeline

    if not args.image:
        print("error: --backend longcat needs --image", file=sys.stderr)
        return 2
    parts = (args.model or "tiny-longcat").split(":")
    tr = parts[0]
    vae = parts[1] if len(parts) > 1 else ("tiny" if tr.startswith("tiny") else "flux")
    pipe = LongCatEditPipeline.from_presets(tr, vae, seed=0)
    with open(args.image, "rb") as f:
        img = decode_image(f.read())
    h, w = (img.shape[0] // 16) * 16, (img.shape[1] // 16) * 16
    img_t = torch.from_numpy(img[:h, :w, :3].copy())
    g = torch.Generator().manual_seed(sum((args.prompt or "").encode()) + 1)
    emb = torch.randn(max(1, len((args.prompt or "").encode())), pipe.tr.cfg.joint_attention_dim, generator=g)
    out = pipe.edit(img_t, emb).cpu()
    files = []
    if args.output:
        from .._ext import runtime

        with open(args.output, "wb") as f:
            f.write(runtime().encode_png(out.contiguous().numpy().tobytes(), out.shape[0], out.shape[1]))
        files = [args.output]
    print(json.dumps({"width": int(out.shape[1]), "height": int(out.shape[0]), "files": files}))
    return 0


def run_video(args) -> int:
    """Text-to-video with the Wan 2.1 pipeline.  --model names a preset pair
    'dit[:vae[:t5]]' of random-weight shapes (no checkpoint download here)."""
    from ..engine.video import WanVideoPipeline

    parts = (args.model or "tiny-wan").split(":")
    dit = parts[0]
    vae = parts[1] if len(parts) > 1 else ("tiny" if dit.startswith("tiny") else "wan2.1")
    t5 = parts[2] if len(parts) > 2 else ("tiny" if dit.startswith("tiny") else "umt5-xxl")
    pipe = WanVideoPipeline.from_presets(dit, vae, t5, seed=0)
    total = [0]

    def progress(step, n):
        total[0] = n
        if not args.quiet:
            print(f"diffusion step {step}/{n}", file=sys.stderr)

    out = pipe.generate(args.prompt or "", negative_prompt=args.negative_prompt, width=args.width,
                        height=args.height, num_frames=args.num_frames, fps=args.fps,
                        guidance_scale=args.guidance_scale, num_steps=args.num_steps, seed=args.seed,
                        progress=progress)
    files = out.save(args.output) if args.output else []
    print(json.dumps({"width": out.width, "height": out.height, "fps": out.fps, "frame_count": out.frame_count,
                      "steps": total[0], "files": files, "timings": {k: round(v, 4) for k, v in out.timings.items()}}))
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    args = build_parser().parse_args(argv)
    if args.init_config:
        p = args.config or config_path()
        os.makedirs(os.path.dirname(p), exist_ok=True)
        if not os.path.exists(p):
            with open(p, "w") as f:
                json.dump(example_config(), f, indent=2)
        print(p)
        return 0
    from ..engine.registry import default_registry

    reg = default_registry()
    if args.list_engines:
        print(json.dumps(reg.describe(), indent=2))
        return 0
    if not args.model:
        print("error: --model is required", file=sys.stderr)
        return 2
    opts = resolve(args, load_config(args.config))
    from ..engine.pipeline import InferencePipeline

    if args.inspect:
        print(json.dumps(InferencePipeline.inspect(args.model, opts["context_size"], reg, tp=args.tp), indent=2))
        return 0
    t0 = time.perf_counter()
    if args.backend == "wan":
        return run_video(args)
    if args.backend == "longcat":
        return run_image_edit(args)
    if args.image:
        return run_image(args, opts)
    if args.backend in ("llamacpp", "script"):
        from ..engine.external import ExternalPipeline, ExternalScriptEngine, ExternalServerEngine

        eng = (ExternalServerEngine(args.model, device=opts["device"], context_size=opts["context_size"],
                                    threads=args.threads) if args.backend == "llamacpp" else
               ExternalScriptEngine(args.model))
        pipe = ExternalPipeline(eng, template=args.template or "chatml", context_size=opts["context_size"])
    else:
        pipe = None
    if pipe is None:
        pipe = InferencePipeline.load(args.model, device=opts["device"], context_size=opts["context_size"], tp=args.tp,
                                      use_cuda_graphs=not args.no_cuda_graphs, template=args.template,
                                      speculative=opts["speculative"], draft_model=args.draft_model,
                                      num_speculative_tokens=opts["num_speculative_tokens"],
                                      ngram_order=opts["speculative_ngram_order"], gpu_layers=args.gpu_layers,
                                      max_num_batched_tokens=args.batch_size, threads=args.threads)
    load_s = time.perf_counter() - t0
    if pipe.is_embedding:
        print("error: embedding models are served by the HTTP server (/v1/embeddings), not bloom_infer",
              file=sys.stderr)
        return 2
    from ..engine.engine import SamplingParams

    sp = SamplingParams(max_tokens=opts["max_tokens"], temperature=opts["temperature"], top_p=opts["top_p"],
                        top_k=args.top_k, seed=args.seed)
    if args.interactive:
        return interactive(pipe, sp, args)
    prompt = read_prompt(args)
    if prompt is None:
        print("error: --prompt, --prompt-file or --interactive is required", file=sys.stderr)
        return 2
    messages = ([{"role": "system", "content": args.system_prompt}] if args.system_prompt else []) + \
        [{"role": "user", "content": prompt}]
    if args.bench or args.bench_json:
        res = pipe.benchmark(messages, sp, repetitions=opts["repetitions"], warmup=opts["warmup"], raw=args.raw)
        res["load_time_ms"] = load_s * 1e3
        print(json.dumps(res, indent=2))
        return 0
    t1 = time.perf_counter()
    ttft = None
    n = 0
    text_parts = []
    for delta in pipe.run_stream(messages, sp, raw=args.raw):
        if ttft is None:
            ttft = time.perf_counter() - t1
        n += 1
        if args.stream:
            sys.stdout.write(delta)
            sys.stdout.flush()
        else:
            text_parts.append(delta)
    dur = time.perf_counter() - t1
    if not args.stream:
        sys.stdout.write("".join(text_parts))
    sys.stdout.write("\n")
    if not args.quiet:
        gen = pipe.last_generated_tokens
        tps = gen / dur if dur > 0 else 0.0
        print(f"[load {load_s * 1e3:.0f} ms | ttft {(ttft or 0) * 1e3:.1f} ms | {gen} tokens | {tps:.2f} tok/s]",
              file=sys.stderr)
    return 0


def run_image(args, opts) -> int:
    """Text + one image through the vision-language pipeline (streamed)."""
    from ..engine.engine import SamplingParams
    from ..engine.vl_pipeline import VisionLanguagePipeline
    from ..models.qwen3_vl import PRESETS

    if args.model not in PRESETS:
        print(f"error: --image needs a vision-language model ({', '.join(PRESETS)})", file=sys.stderr)
        return 2
    t0 = time.perf_counter()
    pipe = VisionLanguagePipeline.from_preset(args.model, context_size=opts["context_size"])
    load_s = time.perf_counter() - t0
    with open(args.image, "rb") as f:
        data = f.read()
    blocks = [{"Image": {"bytes": list(data), "mime": ""}}, {"Text": read_prompt(args) or ""}]
    sp = SamplingParams(max_tokens=opts["max_tokens"], temperature=0.0)
    t1 = time.perf_counter()
    for d in pipe.run_multimodal(blocks, sp):
        sys.stdout.write(d)
        sys.stdout.flush()
    sys.stdout.write("\n")
    if not args.quiet:
        print(f"[load {load_s * 1e3:.0f} ms | {pipe.last_generated_tokens} tokens in "
              f"{(time.perf_counter() - t1) * 1e3:.0f} ms]", file=sys.stderr)
    return 0


def interactive(pipe, sp, args) -> int:
    history = [{"role": "system", "content": args.system_prompt}] if args.system_prompt else []
    while True:
        try:
            line = input("> ")
        except EOFError:
            return 0
        if line.strip() in ("/exit", "/quit"):
            return 0
        history.append({"role": "user", "content": line})
        parts = []
        for d in pipe.run_stream(history, sp, raw=args.raw):
            sys.stdout.write(d)
            sys.stdout.flush()
            parts.append(d)
        sys.stdout.write("\n")
        history.append({"role": "assistant", "content": "".join(parts)})


if __name__ == "__main__":
    sys.exit(main())
