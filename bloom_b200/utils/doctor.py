"""Side-effect-free deployment checks (`bloom_server --doctor`, `bloom_infer --doctor`).

Report shape follows the reference (crates/server/src/doctor.rs:46-160,
object "bloom.server_doctor", schema_version 1, checks with PASS / WARN /
FAIL and a remediation), with B200 checks: native extensions built for
sm_100a, a Blackwell device, HBM headroom, NVLink peer access and
multicast (NVLS) for tensor parallelism, NCCL, the model package and its
memory estimate for 180 GB per GPU, and the speculative configuration.
Nothing is loaded onto a GPU and no setting is changed.
"""
from __future__ import annotations

import glob
import os
import time
from typing import Dict, List, Optional

SCHEMA_VERSION = 1
VERSION = "0.1.0"


def _check(cid: str, status: str, message: str, remediation: Optional[str] = None) -> Dict[str, str]:
    d = {"id": cid, "status": status, "message": message}
    if remediation:
        d["remediation"] = remediation
    return d


def _extensions() -> Dict[str, str]:
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    found = {}
    for stem in ("_C", "_runtime"):
        hits = glob.glob(os.path.join(root, stem + ".*.so"))
        if hits:
            found[stem] = hits[0]
    return found


def doctor_report(model: Optional[str] = None, tp: int = 1, speculative: str = "none",
                  draft_model: Optional[str] = None, context_size: int = 2048, max_concurrent: int = 4,
                  host: str = "127.0.0.1", api_keys: Optional[List[str]] = None) -> Dict[str, object]:
    checks: List[Dict[str, str]] = []
    ext = _extensions()
    if "_C" in ext and "_runtime" in ext:
        checks.append(_check("native_extensions", "pass", "CUDA kernels and the C++ runtime are built in-tree."))
    else:
        missing = [k for k in ("_C", "_runtime") if k not in ext]
        checks.append(_check("native_extensions", "fail", f"missing native extension(s): {', '.join(missing)}",
                             "Run `python setup.py build_ext --inplace` (nvcc for sm_100a)."))
    if host not in ("127.0.0.1", "localhost", "::1") and not api_keys:
        checks.append(_check("network", "fail", f"non-loopback bind {host} without an API key",
                             "Pass --api-key or bind to 127.0.0.1."))
    else:
        checks.append(_check("network", "pass", f"bind address {host} is allowed."))
    if max_concurrent < 1 or context_size < 16:
        checks.append(_check("arguments", "fail", "max_concurrent must be >= 1 and context_size >= 16",
                             "Correct the reported flags."))
    else:
        checks.append(_check("arguments", "pass", "Numeric limits are consistent."))
    try:
        import torch

        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # noqa: BLE001
        n = 0
    if n == 0:
        checks.append(_check("device", "warn", "no CUDA device visible; only the CPU engine can run",
                             "Run on a B200 host, or use --device cpu."))
    else:
        import torch

        p = torch.cuda.get_device_properties(0)
        if (p.major, p.minor) == (10, 0):
            checks.append(_check("device", "pass", f"{n} x {p.name} (sm_100), {p.total_memory / 2**30:.0f} GiB HBM, "
                                 f"{p.multi_processor_count} SMs."))
        else:
            checks.append(_check("device", "fail", f"{p.name} is sm_{p.major}{p.minor}; kernels target sm_100a",
                                 "Run on a B200 (compute capability 10.0)."))
        if tp > 1:
            if tp > n:
                checks.append(_check("tensor_parallel", "fail", f"tp={tp} but only {n} GPU(s) visible",
                                     "Lower --tp or expose more GPUs."))
            else:
                ok = all(torch.cuda.can_device_access_peer(i, j) for i in range(tp) for j in range(tp) if i != j)
                from .probe_gpu import multicast_supported

                mc = all(multicast_supported(i) for i in range(tp))
                checks.append(_check("tensor_parallel", "pass" if ok else "fail",
                                     f"peer access among {tp} GPUs: {ok}; NVLink multicast: {mc}",
                                     None if ok else "The fused NVLink kernels need P2P; use --comm nccl."))
    try:
        import torch

        v = ".".join(str(x) for x in torch.cuda.nccl.version())
        checks.append(_check("nccl", "pass", f"NCCL {v} available."))
    except Exception:  # noqa: BLE001
        checks.append(_check("nccl", "warn", "NCCL not available", "Multi-GPU runs need torch built with NCCL."))
    if model:
        from ..models.config import PRESETS

        if model in PRESETS or model == "echo":
            checks.append(_check("startup_model", "pass", f"preset {model!r} (random-init weights)."))
        elif not os.path.exists(model):
            checks.append(_check("startup_model", "fail", f"model path {model!r} does not exist",
                                 "Pass a model directory, a .gguf file, or a preset name."))
        else:
            try:
                from ..formats.manifest import estimate_memory, load_manifest

                man = load_manifest(model)
                est = estimate_memory(man, context_size, concurrent_seqs=max_concurrent, tp=tp)
                st = "pass" if est.fits else "fail"
                checks.append(_check("startup_model", st,
                                     f"{man.family} {man.primary_dtype}: {est.per_gpu_bytes / 2**30:.1f} GiB per GPU "
                                     f"at context {context_size} x {max_concurrent}",
                                     None if est.fits else "Lower --context-size / --max-concurrent or raise --tp."))
            except Exception as e:  # noqa: BLE001
                checks.append(_check("startup_model", "fail", f"model package rejected: {e}",
                                     "Check config.json / bloom.json / GGUF header."))
    else:
        checks.append(_check("startup_model", "warn", "no startup model configured",
                             "Pass --model PATH|PRESET."))
    if speculative == "draft" and not draft_model:
        checks.append(_check("speculative", "fail", "draft speculation without --draft-model",
                             "Pass --draft-model PATH|PRESET or use --speculative ngram."))
    else:
        checks.append(_check("speculative", "pass", f"speculative mode {speculative}."))
    summary = {"passed": sum(c["status"] == "pass" for c in checks),
               "warnings": sum(c["status"] == "warn" for c in checks),
               "failures": sum(c["status"] == "fail" for c in checks)}
    status = "fail" if summary["failures"] else ("warn" if summary["warnings"] else "pass")
    return {"schema_version": SCHEMA_VERSION, "object": "bloom.server_doctor", "created": int(time.time()),
            "bloom_version": VERSION, "status": status, "summary": summary, "checks": checks}


def render_text(report: Dict[str, object]) -> str:
    out = [f"Bloom server doctor {report['bloom_version']}", f"Result: {str(report['status']).upper()}", ""]
    for c in report["checks"]:
        out.append(f"[{c['status'].upper()}] {c['id']}: {c['message']}")
        if c.get("remediation"):
            out.append(f"       Next: {c['remediation']}")
    s = report["summary"]
    out.append("")
    out.append(f"Summary: {s['passed']} passed, {s['warnings']} warning(s), {s['failures']} failure(s)")
    return "\n".join(out) + "\n"
