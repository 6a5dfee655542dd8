"""Per-kernel device-time breakdown of one call, for finding what limits a step.

`profile_call(fn, device)` runs `fn()` once under torch.profiler (CUPTI
kernel records, graph replays included) and returns a table: device time and
launch count per kernel name, the same grouped into classes (GEMM, attention,
collectives, norm/RoPE, sampling, MoE, copies, other), the wall time of the
call and the device-busy fraction (kernel time / wall time -- the rest is host
overhead, synchronisation and launch gaps).  A number taken under the
profiler is for shares only, never a benchmark value.
"""
from __future__ import annotations

import time
from typing import Callable, Dict

CLASSES = (
    ("collective", ("tp_", "nccl", "allreduce", "allgather", "ncclDevKernel")),
    ("moe", ("moe_",)),
    ("gemm", ("gemm", "qgemv", "qdequant")),
    ("attention", ("attn", "attention", "decode_combine")),
    ("norm_rope", ("rmsnorm", "rope", "embedding", "norm_kernel")),
    ("sampling", ("argmax", "sample", "verify")),
    ("copy", ("memcpy", "memset", "copy", "Memcpy", "Memset")),
)


def classify(name: str) -> str:
    for cls, keys in CLASSES:
        if any(k in name for k in keys):
            return cls
    return "other"


def profile_call(fn: Callable[[], object], device) -> Dict:
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        fn()
        torch.cuda.synchronize(device)
    wall_ms = (time.perf_counter() - t0) * 1e3
    kernels: Dict[str, Dict[str, float]] = {}
    for e in prof.events():
        dt = getattr(e, "device_type", None)
        if dt is None or "CUDA" not in str(dt):
            continue
        us = float(getattr(e, "device_time", 0.0) or getattr(e, "cuda_time", 0.0) or 0.0)
        k = kernels.setdefault(e.name, {"us": 0.0, "count": 0})
        k["us"] += us
        k["count"] += 1
    total_us = sum(k["us"] for k in kernels.values())
    by_class: Dict[str, Dict[str, float]] = {}
    for name, k in kernels.items():
        c = by_class.setdefault(classify(name), {"us": 0.0, "count": 0})
        c["us"] += k["us"]
        c["count"] += k["count"]
    top = sorted(kernels.items(), key=lambda kv: -kv[1]["us"])[:40]
    return {
        "wall_ms_under_profiler": round(wall_ms, 2),
        "kernel_ms": round(total_us / 1e3, 2),
        "device_busy_fraction": round(total_us / 1e3 / wall_ms, 3) if wall_ms else None,
        "by_class": {c: {"ms": round(v["us"] / 1e3, 2), "count": v["count"],
                         "share": round(v["us"] / total_us, 3) if total_us else 0.0}
                     for c, v in sorted(by_class.items(), key=lambda kv: -kv[1]["us"])},
        "top_kernels": [{"name": n[:160], "ms": round(v["us"] / 1e3, 3), "count": v["count"],
                         "avg_us": round(v["us"] / max(1, v["count"]), 2)} for n, v in top],
    }
