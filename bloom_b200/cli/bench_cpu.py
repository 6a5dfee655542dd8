"""CPU decoding benchmark: SmolLM2-135M-shape decoder as a Q8_0 GGUF.

    python -m bloom_b200.cli.bench_cpu [--tokens 128] [--prompt 32] [--repeats 3]

Writes a random-init (N(0, 0.02), seed 0) SmolLM2-135M-shape model (hidden
576, 30 layers, 9 heads / 3 KV heads, FFN 1536, vocab 49152, tied
embeddings) to a GGUF with Q8_0 blocks, loads it through the public
pipeline API on the CPU, and decodes one prompt of 32 uniform-random token
ids for 128 greedy tokens (EOS ignored): non-streamed (pipeline.run, wall
time of the call) and streamed (the pipeline's token stream, time to the
first token and between tokens).  Prints one JSON line; medians over
--repeats runs after one warm-up run.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import tempfile
import time


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--threads", type=int, default=0,
                    help="PyTorch intra-op threads (0: the CPU decoder's default, one; its matmuls use the native pool)")
    args = ap.parse_args()
    import torch

    if args.threads:
        torch.set_num_threads(args.threads)
    from ..engine.engine import SamplingParams
    from ..engine.pipeline import InferencePipeline
    from ..formats.gguf import GGML_Q8_0, write_decoder_gguf
    from ..models.config import preset
    from ..models.reference import random_weights

    cfg = preset("smollm2-135m")
    d = tempfile.mkdtemp(prefix="bloom-bench-cpu-")
    path = os.path.join(d, "smollm2-135m-q8_0.gguf")
    write_decoder_gguf(path, cfg, random_weights(cfg, seed=0, std=0.02), GGML_Q8_0)
    t0 = time.perf_counter()
    pipe = InferencePipeline.load(path, device="cpu", context_size=512)
    load_s = time.perf_counter() - t0
    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, cfg.vocab_size, (args.prompt,), generator=g).tolist()
    sp = SamplingParams(max_tokens=args.tokens, temperature=0.0, top_p=1.0, ignore_eos=True)

    def non_streamed():
        t = time.perf_counter()
        "".join(pipe.run_stream(None, sp, prompt_ids=prompt))
        dt = time.perf_counter() - t
        return dt, pipe.last_generated_tokens

    def streamed():
        t = time.perf_counter()
        stamps = []
        for _ in pipe.cpu.generate(prompt, args.tokens, 0.0, 1.0, None, None, True):
            stamps.append(time.perf_counter())
        ttft = stamps[0] - t
        tbt = (stamps[-1] - stamps[0]) / max(1, len(stamps) - 1)
        return ttft, tbt, len(stamps) / (stamps[-1] - t)

    non_streamed()
    ns = [non_streamed() for _ in range(args.repeats)]
    st = [streamed() for _ in range(args.repeats)]
    n = ns[0][1]
    line = {
        "metric": "CPU decode tok/s, TTFT and TBT, SmolLM2-135M-shape Q8_0 GGUF",
        "value": round(n / statistics.median(x[0] for x in ns), 2),
        "unit": "output tokens/s (non-streamed, wall clock of pipeline.run)",
        "streamed": {"tok_s": round(statistics.median(x[2] for x in st), 2),
                     "ttft_ms": round(1e3 * statistics.median(x[0] for x in st), 2),
                     "tbt_ms": round(1e3 * statistics.median(x[1] for x in st), 3)},
        "tokens": n, "prompt_tokens": args.prompt, "repeats": args.repeats, "load_s": round(load_s, 2),
        "data": "synthetic (uniform-random prompt ids, random-init N(0,0.02) weights seed 0)",
        "host": {"cpu": platform.processor() or platform.machine(), "cores": os.cpu_count(),
                 "torch_threads": torch.get_num_threads()},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
