"""Model packages: bloom.json manifests, manifest inference, memory estimation.

`ModelManifest` keeps the reference's bloom.json field names
(crates/core/src/manifest.rs:86-111; schema examples/manifest/
model-manifest.schema.json): id, family, version, license, io_schema,
memory_profile, files (name, format, size_bytes, hash_sha256, required),
parameters, runtime_hints, primary_dtype, quantization, processors.

`load_manifest(path)` accepts a bloom.json, a Hugging Face directory
(config.json + tokenizer.json + safetensors), a single .gguf file or a
directory holding exactly one .gguf (reference load_manifest,
crates/engine/src/core/manifest.rs:858-943).

`estimate_memory` restates the reference estimator (manifest.rs:148-363: KV
bytes per token = 2 * layers * kv_heads * head_dim * dtype bytes; temporary
tensors = max(weights / 10, ctx * hidden * 2)) and re-derives it for a B200:
weights and KV are divided by the tensor/expert-parallel degree, and the
device budget is the HBM of one GPU (180 GB), not a desktop VRAM size.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

HBM_BYTES_PER_GPU = 183_359 * 1024 * 1024  # B200 (nvidia-smi 183,359 MiB)
GIB = 1 << 30

FAMILIES = {"llama": "Llama", "mistral": "Llama", "qwen2": "Qwen", "qwen3": "Qwen", "qwen3_moe": "Qwen",
            "bert": "Bert", "gemma": "Gemma", "gemma4": "Gemma", "gemma4_text": "Gemma", "gemma4_unified": "Gemma"}
DTYPE_BYTES = {"F32": 4.0, "F16": 2.0, "BF16": 2.0, "Q8": 34 / 32, "Q4": 18 / 32, "I8": 1.0, "U8": 1.0, "I4": 0.5,
               "NF4": 0.5}


class ManifestError(ValueError):
    pass


@dataclass
class ModelFile:
    name: str
    format: str  # Safetensors | Gguf | OpenVinoIr | TensorRtEngine | Unknown
    size_bytes: int
    hash_sha256: Optional[str] = None
    required: bool = True


@dataclass
class ModelManifest:
    id: str
    family: Any
    version: str
    io_schema: Dict[str, List[str]]
    memory_profile: Dict[str, int]
    primary_dtype: str
    files: List[ModelFile] = field(default_factory=list)
    parameters: Dict[str, Any] = field(default_factory=dict)
    runtime_hints: Dict[str, Any] = field(default_factory=dict)
    license: Optional[str] = None
    description: Optional[str] = None
    source_url: Optional[str] = None
    quantization: Optional[Dict[str, Any]] = None
    processors: List[Dict[str, Any]] = field(default_factory=list)
    schema_version: str = "1"
    root: str = ""  # directory the files are relative to (not serialised)

    def to_dict(self) -> dict:
        d = dataclasses.asdict(self)
        d.pop("root", None)
        return d

    def to_json(self, indent: int = 2) -> str:
        return json.dumps(self.to_dict(), indent=indent)

    @property
    def is_embedding(self) -> bool:
        return self.family == "Bert" or "Embedding" in self.io_schema.get("outputs", [])


def validate_manifest(d: dict) -> None:
    req = ["id", "family", "version", "io_schema", "memory_profile", "primary_dtype"]
    for k in req:
        if k not in d:
            raise ManifestError(f"manifest missing required field {k!r}")
    if not isinstance(d["id"], str) or not d["id"]:
        raise ManifestError("manifest id must be a non-empty string")
    io = d["io_schema"]
    if not isinstance(io, dict) or not io.get("inputs") or not io.get("outputs"):
        raise ManifestError("io_schema needs non-empty inputs and outputs")
    if d["primary_dtype"] not in DTYPE_BYTES:
        raise ManifestError(f"unknown primary_dtype {d['primary_dtype']!r}")
    for f in d.get("files", []):
        for k in ("name", "format", "size_bytes", "required"):
            if k not in f:
                raise ManifestError(f"file entry missing {k!r}")
        if f["format"] not in ("Safetensors", "Gguf", "OpenVinoIr", "TensorRtEngine", "Unknown"):
            raise ManifestError(f"unknown file format {f['format']!r}")
        h = f.get("hash_sha256")
        if h is not None and (len(h) != 64 or any(c not in "0123456789abcdefABCDEF" for c in h)):
            raise ManifestError(f"bad sha256 for {f['name']}")
        if ".." in f["name"].replace("\\", "/").split("/") or os.path.isabs(f["name"]):
            raise ManifestError(f"file name escapes the package: {f['name']}")


def manifest_from_dict(d: dict, root: str = "") -> ModelManifest:
    validate_manifest(d)
    files = [ModelFile(**{k: v for k, v in f.items() if k in ("name", "format", "size_bytes", "hash_sha256",
                                                                "required")}) for f in d.get("files", [])]
    return ModelManifest(id=d["id"], family=d["family"], version=d["version"], io_schema=d["io_schema"],
                         memory_profile=d["memory_profile"], primary_dtype=d["primary_dtype"], files=files,
                         parameters=d.get("parameters", {}), runtime_hints=d.get("runtime_hints", {}),
                         license=d.get("license"), description=d.get("description"),
                         source_url=d.get("source_url"), quantization=d.get("quantization"),
                         processors=d.get("processors", []), schema_version=str(d.get("schema_version", "1")),
                         root=root)


def _find_gguf(path: str) -> Optional[str]:
    if os.path.isfile(path) and path.endswith(".gguf"):
        return path
    if os.path.isdir(path):
        g = [f for f in os.listdir(path) if f.endswith(".gguf")]
        if len(g) == 1:
            return os.path.join(path, g[0])
        if len(g) > 1 and not os.path.exists(os.path.join(path, "config.json")):
            raise ManifestError(f"{path}: more than one .gguf file; pass the file explicitly")
    return None


def load_manifest(path: str) -> ModelManifest:
    path = os.path.abspath(path)
    if os.path.isdir(path) and os.path.exists(os.path.join(path, "bloom.json")):
        with open(os.path.join(path, "bloom.json")) as f:
            return manifest_from_dict(json.load(f), root=path)
    if path.endswith("bloom.json") and os.path.isfile(path):
        with open(path) as f:
            return manifest_from_dict(json.load(f), root=os.path.dirname(path))
    g = _find_gguf(path)
    if g is not None and not (os.path.isdir(path) and os.path.exists(os.path.join(path, "config.json"))):
        return manifest_from_gguf(g)
    if os.path.isdir(path) and os.path.exists(os.path.join(path, "config.json")):
        return manifest_from_hf_dir(path)
    raise ManifestError(f"{path}: not a bloom.json package, Hugging Face directory or GGUF file")


def manifest_from_hf_dir(path: str) -> ModelManifest:
    from .safetensors_io import resolve_shards

    with open(os.path.join(path, "config.json")) as f:
        cfg = json.load(f)
    if not os.path.exists(os.path.join(path, "tokenizer.json")):
        raise ManifestError(f"{path}: missing tokenizer.json")
    shards = resolve_shards(path)
    mt = (cfg.get("model_type") or "llama").lower()
    family = FAMILIES.get(mt, {"Custom": mt})
    files = [ModelFile(os.path.basename(s), "Safetensors", os.path.getsize(s)) for s in shards]
    files.append(ModelFile("config.json", "Unknown", os.path.getsize(os.path.join(path, "config.json"))))
    files.append(ModelFile("tokenizer.json", "Unknown", os.path.getsize(os.path.join(path, "tokenizer.json"))))
    dt = {"bfloat16": "BF16", "float16": "F16", "float32": "F32"}.get(str(cfg.get("torch_dtype", "bfloat16")), "BF16")
    is_bert = mt == "bert"
    params = {k: cfg[k] for k in ("num_hidden_layers", "hidden_size", "intermediate_size", "num_attention_heads",
                                  "num_key_value_heads", "vocab_size", "max_position_embeddings", "head_dim",
                                  "num_experts", "num_experts_per_tok", "moe_intermediate_size") if k in cfg}
    if "head_dim" not in params and "hidden_size" in cfg and "num_attention_heads" in cfg:
        params["head_dim"] = cfg["hidden_size"] // cfg["num_attention_heads"]
    w = sum(f.size_bytes for f in files if f.format == "Safetensors")
    return ModelManifest(
        id=os.path.basename(path.rstrip("/")), family=family, version="1", primary_dtype=dt,
        io_schema={"inputs": ["Text"], "outputs": ["Embedding" if is_bert else "Text"]},
        memory_profile={"min_ram_bytes": 0, "min_vram_bytes": w, "recommended_ram_bytes": 0,
                        "recommended_vram_bytes": int(w * 1.2)},
        files=files, parameters=params, runtime_hints={"preferred_backends": ["b200"], "supports_mmap": True,
                                                       "requires_streaming": False},
        processors=[{"name": "tokenizer", "kind": "TextTokenizer", "version": "1"}], root=path)


def manifest_from_gguf(path: str) -> ModelManifest:
    from .gguf import GGUFFile

    g = GGUFFile(path)
    m, a = g.metadata, g.arch
    prim = g.primary_dtype()
    dt = {"Q8_0": "Q8", "Q4_0": "Q4", "F16": "F16", "BF16": "BF16", "F32": "F32"}.get(prim, "Q4")
    params = {"num_hidden_layers": int(m.get(f"{a}.block_count", 0)),
              "hidden_size": int(m.get(f"{a}.embedding_length", 0)),
              "intermediate_size": int(m.get(f"{a}.feed_forward_length", 0)),
              "num_attention_heads": int(m.get(f"{a}.attention.head_count", 0)),
              "num_key_value_heads": int(m.get(f"{a}.attention.head_count_kv", m.get(f"{a}.attention.head_count", 0))),
              "max_position_embeddings": int(m.get(f"{a}.context_length", 2048)),
              "vocab_size": len(m.get("tokenizer.ggml.tokens", [])) or int(m.get(f"{a}.vocab_size", 0))}
    if params["num_attention_heads"]:
        params["head_dim"] = int(m.get(f"{a}.attention.key_length",
                                       params["hidden_size"] // params["num_attention_heads"]))
    size = os.path.getsize(path)
    family = FAMILIES.get({"qwen3moe": "qwen3_moe"}.get(a, a), {"Custom": a})
    return ModelManifest(
        id=os.path.splitext(os.path.basename(path))[0], family=family, version="1", primary_dtype=dt,
        io_schema={"inputs": ["Text"], "outputs": ["Text"]},
        memory_profile={"min_ram_bytes": size, "min_vram_bytes": size, "recommended_ram_bytes": int(size * 1.2),
                        "recommended_vram_bytes": int(size * 1.2)},
        files=[ModelFile(os.path.basename(path), "Gguf", size)], parameters=params,
        runtime_hints={"preferred_backends": ["b200", "cpu"], "supports_mmap": True, "requires_streaming": False},
        quantization={"scheme": prim, "bits": 8 if dt == "Q8" else (4 if dt == "Q4" else 16), "group_size": 32}
        if dt in ("Q8", "Q4") else None,
        processors=[{"name": "tokenizer", "kind": "TextTokenizer", "version": "1"}], root=os.path.dirname(path))


def verify_hashes(man: ModelManifest, allow_mismatch: Optional[bool] = None) -> List[str]:
    """Check sha256 of files that declare one (BLOOM_ALLOW_HASH_MISMATCH=1 downgrades to warnings)."""
    if allow_mismatch is None:
        allow_mismatch = os.environ.get("BLOOM_ALLOW_HASH_MISMATCH", "0") == "1"
    bad = []
    for f in man.files:
        if not f.hash_sha256:
            continue
        p = os.path.join(man.root, f.name)
        if not os.path.exists(p):
            if f.required:
                bad.append(f"{f.name}: missing")
            continue
        h = hashlib.sha256()
        with open(p, "rb") as fh:
            for chunk in iter(lambda: fh.read(1 << 20), b""):
                h.update(chunk)
        if h.hexdigest().lower() != f.hash_sha256.lower():
            bad.append(f"{f.name}: sha256 mismatch")
    if bad and not allow_mismatch:
        raise ManifestError("; ".join(bad))
    return bad


@dataclass
class MemoryEstimate:
    weights_bytes: int
    kv_cache_bytes: int
    temp_bytes: int
    total_bytes: int
    per_gpu_bytes: int
    kv_bytes_per_token: int
    fits: bool
    device_budget_bytes: int
    notes: List[str] = field(default_factory=list)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def estimate_memory(man: ModelManifest, context_size: int, concurrent_seqs: int = 1, tp: int = 1, ep: int = 1,
                    device: str = "gpu", kv_dtype_bytes: int = 2, gpu_util: float = 0.9) -> MemoryEstimate:
    p = man.parameters
    weights = sum(f.size_bytes for f in man.files if f.format in ("Safetensors", "Gguf"))
    if weights == 0:
        L = int(p.get("num_hidden_layers", 0))
        H = int(p.get("hidden_size", 0))
        I = int(p.get("intermediate_size", 4 * H))
        V = int(p.get("vocab_size", 32000))
        params = L * (4 * H * H + 3 * H * I) + 2 * V * H
        weights = int(params * DTYPE_BYTES.get(man.primary_dtype, 2.0)) or GIB
    if device == "gpu" and man.primary_dtype in ("Q8", "Q4"):
        # GGUF blocks are dequantised to bf16 on the GPU path
        weights = int(weights * 2.0 / DTYPE_BYTES[man.primary_dtype])
    L = int(p.get("num_hidden_layers", 32))
    kvh = int(p.get("num_key_value_heads", p.get("num_attention_heads", 8)))
    hd = int(p.get("head_dim", 128))
    H = int(p.get("hidden_size", 4096))
    kv_tok = 0 if man.is_embedding else 2 * L * kvh * hd * (kv_dtype_bytes if device == "gpu" else 4)
    kv = kv_tok * context_size * max(1, concurrent_seqs)
    temp = max(weights // 10, context_size * H * 2)
    total = weights + kv + temp
    shards = max(1, tp) * max(1, ep)
    # KV heads shard over TP (replicated when kv_heads < tp)
    kv_div = min(max(1, tp), kvh) if kvh else 1
    per_gpu = weights // shards + kv // kv_div + temp // max(1, tp)
    budget = int(HBM_BYTES_PER_GPU * gpu_util) if device == "gpu" else _host_ram()
    notes = []
    if per_gpu > budget:
        need = (per_gpu + budget - 1) // budget
        notes.append(f"does not fit one GPU: needs about {need}x the per-GPU budget; raise --tp or lower context")
    return MemoryEstimate(weights, kv, temp, total, per_gpu, kv_tok, per_gpu <= budget, budget, notes)


def _host_ram() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 16 * GIB
