#!/usr/bin/env python
"""Headline serving benchmark: Llama-3-8B-shape, bf16, tensor parallel over N GPUs.

Workload (one benchmark "step" = one complete serving run):
  256 concurrent requests submitted at t0, prompt lengths uniform in
  [512, 2048], uniform-random token ids, 256 greedy output tokens each
  (EOS ignored), paged KV cache with 16-token blocks, in-flight batching
  (decode rows + chunked prefill with the leftover token budget per step).
  Model: Llama-3-8B shape (hidden 4096, 32 layers, 32 heads, 8 KV heads,
  FFN 14336, vocab 128256, RoPE theta 5e5), random N(0, 0.02) weights, seed 0.

Reported
  value          output tokens/s for the whole box (all N GPUs), device-timed
                 with CUDA events around each run, max over ranks
  p50_ttft_ms    median time to first token over the 256 requests
  e2e            the same metric through the public API (LLMEngine.generate:
                 prompts from host lists, per engine step one H2D copy of the
                 step arena from pinned memory and one D2H read of the sampled
                 tokens), timed by the host clock around the call

    python bench.py [--gpus N] [--steps K] [--warmup W]          (N > 1: launch with torchrun)
    python bench.py --impl reference ...                          reference arm
"""
from __future__ import annotations

import argparse
import json
import os

# the fused collectives use plain peer loads / stores only: no NVLink multicast object
os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
import statistics
import sys
import threading
import time

BASELINE_TOKS = None  # the reference publishes no GPU number for this config


def reference_arm(args):
    """The reference is a Rust Cargo workspace (candle + cudarc).  This arm
    looks for what building it would need -- a Rust toolchain, a vendored
    crate registry, or an installed reference under baseline/_ref -- and
    reports what it found; with none of them it prints the `unavailable`
    line and exits 0."""
    import glob
    import shutil

    here = os.path.dirname(os.path.abspath(__file__))
    found = {tool: shutil.which(tool) for tool in ("cargo", "rustc")}
    registry = [p for p in (os.path.expanduser("~/.cargo/registry"), os.path.join(here, "baseline", "_ref", "vendor"))
                if os.path.isdir(p)]
    ref = os.path.join(here, "baseline", "_ref")
    ref_files = sorted(os.path.basename(p) for p in glob.glob(os.path.join(ref, "*")))[:8]
    engine_bins = [p for p in glob.glob(os.path.join(ref, "**", "bloom_infer*"), recursive=True) if os.access(p, os.X_OK)]
    probe = (f"cargo={found['cargo'] or 'absent'}, rustc={found['rustc'] or 'absent'}, "
             f"crate registry={'present' if registry else 'absent'}, "
             f"baseline/_ref={'[' + ', '.join(ref_files) + ']' if ref_files else 'empty or absent'}, "
             f"bloom_infer binary={'present' if engine_bins else 'absent'}")
    rank = int(os.environ.get("RANK", "0"))
    if engine_bins or (found["cargo"] and registry):
        reason = ("a Rust toolchain or reference binary was found, but this arm has no driver for the reference's "
                  "engine on this metric (it has no tensor-parallel CUDA path to run): " + probe)
    else:
        reason = ("reference is a Rust workspace (Cargo, candle 0.10, cudarc 0.19) and cannot be built here; "
                  "pip install of it fails (not a Python project); probe: " + probe)
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
    return 0


class ClockSampler:
    """Samples SM clock and throttle reasons via NVML while the timed region runs."""

    def __init__(self, device_index: int, period_s: float = 0.2):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        names = {
            "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
            "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
            "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
        }
        while not self._stop.is_set():
            try:
                util = nv.nvmlDeviceGetUtilizationRates(self.h).gpu
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except Exception:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                if util > 50:
                    self.samples.append(mhz)
                for n, bit in names.items():
                    if r & bit and n != "gpu_idle":
                        self.reasons.add(n)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self):
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def make_workload(n_req, lo, hi, vocab, seed):
    import random

    rng = random.Random(seed)
    prompts = []
    for _ in range(n_req):
        L = rng.randint(lo, hi)
        prompts.append([rng.randrange(0, vocab) for _ in range(L)])
    return prompts


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="bloom_b200", choices=["bloom_b200", "reference"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--prompt-min", type=int, default=512)
    ap.add_argument("--prompt-max", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--max-batched-tokens", type=int, default=8192)
    ap.add_argument("--comm", default=os.environ.get("BLOOM_COMM", "fused"), choices=["nccl", "fused"])
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--profile", default="",
                    help="after the timed runs, profile one more (untimed) run with torch.profiler and write the "
                         "per-kernel device-time table of every rank to PROFILE.rank<r>.json")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)

    import torch
    import torch.distributed as dist

    from bloom_b200 import ops
    from bloom_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from bloom_b200.models.config import preset
    from bloom_b200.models.llama import DecoderLM, TPInfo
    from bloom_b200.parallel.comm import Communicator, init_distributed

    rank, world, local = init_distributed("nccl")
    if world != args.gpus:
        if rank == 0:
            print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}; using {world}", file=sys.stderr)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = dist.group.WORLD if world > 1 else None
    comm = Communicator(rank, world, dev, group, mode=args.comm, max_tokens=max(args.max_batched_tokens, args.requests),
                        hidden=preset(args.model).hidden_size)
    tp = TPInfo(rank=rank, size=world, group=group, comm=comm)

    cfg = preset(args.model)
    model = DecoderLM(cfg, tp, dev)
    model.random_init(seed=0)
    max_len = args.prompt_max + args.output_len + 16
    ec = EngineConfig(max_num_seqs=args.requests, max_num_batched_tokens=args.max_batched_tokens,
                      max_model_len=max_len, use_cuda_graphs=not args.no_graphs, enable_prefix_caching=False,
                      gpu_memory_utilization=0.90)
    t_init = time.perf_counter()
    eng = LLMEngine(model, ec)
    init_s = time.perf_counter() - t_init
    prompts = make_workload(args.requests, args.prompt_min, args.prompt_max, cfg.vocab_size, seed=1234)
    sp = SamplingParams(max_tokens=args.output_len, temperature=0.0, top_p=1.0, ignore_eos=True)

    def barrier():
        if world > 1:
            dist.barrier()

    def one_run():
        """One serving run; returns (device ms, host ms, outputs, arena bytes, d2h bytes, launches)."""
        st = eng.runner.stats
        h0, d0, l0 = st["h2d_bytes"], st["d2h_bytes"], ops.LAUNCHES[0]
        barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        ev0.record()
        outs = eng.generate(prompts, sp)
        ev1.record()
        torch.cuda.synchronize()
        host_ms = (time.perf_counter() - t0) * 1e3
        barrier()
        dev_ms = ev0.elapsed_time(ev1)
        return dev_ms, host_ms, outs, st["h2d_bytes"] - h0, st["d2h_bytes"] - d0, ops.LAUNCHES[0] - l0

    for _ in range(args.warmup):
        one_run()
    ops.status().zero_()
    results = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            results.append(one_run())
    st_bits = int(ops.status()[0].item())

    dev_ms = torch.tensor([r[0] for r in results], device=dev)
    host_ms = torch.tensor([r[1] for r in results], device=dev)
    if world > 1:
        dist.all_reduce(dev_ms, op=dist.ReduceOp.MAX)
        dist.all_reduce(host_ms, op=dist.ReduceOp.MAX)
    total_dev_s = dev_ms.sum().item() / 1e3
    total_host_s = host_ms.sum().item() / 1e3
    out_tokens = sum(len(o.token_ids) for r in results for o in r[2])
    per_step_tokens = out_tokens / len(results)
    ttfts = [(o.first_token_time - o.arrival_time) * 1e3 for r in results for o in r[2]]
    tbts = []
    for r in results:
        for o in r[2]:
            if len(o.token_ids) > 1:
                tbts.append((o.finish_time - o.first_token_time) * 1e3 / (len(o.token_ids) - 1))
    value = out_tokens / total_dev_s
    e2e = out_tokens / total_host_s
    line = {
        "metric": ("decode tok/s/box (max over ranks) & p50 TTFT, Llama-3-8B-shape bf16, TP=1/2/4/8"
                   if args.model == "llama3-8b" else
                   f"decode tok/s/box (max over ranks) & p50 TTFT, {args.model} bf16, "
                   f"{'EP' if cfg.is_moe else 'TP'}={world}"),
        "value": round(value, 1),
        "unit": "output tokens/s (whole box)",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms.mean().item(), 2),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (uniform-random token ids, random-init N(0,0.02) weights seed 0)",
        "p50_ttft_ms": round(statistics.median(ttfts), 1),
        "p90_ttft_ms": round(sorted(ttfts)[int(0.9 * (len(ttfts) - 1))], 1),
        "mean_tbt_ms": round(statistics.mean(tbts), 2) if tbts else None,
        "config": {
            "model": (f"{args.model} (hidden {cfg.hidden_size}, {cfg.num_layers} layers, {cfg.num_heads}/"
                      f"{cfg.num_kv_heads} heads, " + (f"{cfg.num_experts} experts top-{cfg.num_experts_per_tok} "
                                                       f"FFN {cfg.moe_intermediate_size}" if cfg.is_moe else
                                                       f"FFN {cfg.intermediate_size}") + f", vocab {cfg.vocab_size})"),
            "global_batch": args.requests,
            "seq_len": f"prompt U[{args.prompt_min},{args.prompt_max}] + {args.output_len} output",
            "parallelism": (f"ep{world}+tp{world}-attention" if cfg.is_moe and world > 1 else f"tp{world}"),
            "comm": args.comm if world > 1 else "none",
            "step": f"one full serving run of the {args.requests}-request workload",
            "cache": "inputs larger than L2 (16 GB weights / tp, tens of GB of KV pages per run)",
            "kv_block": 16,
            "max_num_batched_tokens": args.max_batched_tokens,
            "cuda_graphs": not args.no_graphs,
        },
        "e2e": {
            "value": round(e2e, 1),
            "unit": "output tokens/s via LLMEngine.generate (host clock)",
            "h2d_bytes_per_step": int(sum(r[3] for r in results) / len(results)),
            "d2h_bytes_per_step": int(sum(r[4] for r in results) / len(results)),
        },
        "gpu_launches": int(sum(r[5] for r in results)),
        "clocks": clk.summary(),
        "kernel_status": st_bits,
        "init_s": round(init_s, 1),
        "engine_steps_per_run": eng.runner.stats["steps"] // max(1, args.steps + args.warmup),
        "output_tokens_per_step": per_step_tokens,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if args.profile:
        from bloom_b200.utils.step_profile import profile_call

        table = profile_call(one_run, dev)
        table.update({"rank": rank, "n_gpus": world, "config": line["config"]})
        with open(f"{args.profile}.rank{rank}.json", "w") as f:
            json.dump(table, f, indent=1)
    eng.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
