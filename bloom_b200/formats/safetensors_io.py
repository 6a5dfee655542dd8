"""Safetensors reading/writing with the reference's shard validation rules.

Single file: `model.safetensors`.  Sharded: `model.safetensors.index.json`
whose `weight_map` names canonical shards `model-XXXXX-of-YYYYY.safetensors`;
every shard must exist, be referenced, and hold exactly the tensors the index
assigns to it (reference: crates/engine/src/core/manifest.rs:1731 header
parsing, :1886-2027 shard resolver).  Headers are validated before any data
is touched: 8-byte little-endian length, JSON object, dtype/shape/offsets
consistent and inside the file, no overlapping or out-of-order ranges.
"""
from __future__ import annotations

import json
import os
import re
import struct
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

DTYPES = {"F32": (np.float32, 4), "F16": (np.float16, 2), "BF16": (np.uint16, 2), "I64": (np.int64, 8),
          "I32": (np.int32, 4), "I16": (np.int16, 2), "I8": (np.int8, 1), "U8": (np.uint8, 1), "BOOL": (np.bool_, 1),
          "F64": (np.float64, 8)}
MAX_HEADER = 100 * 1024 * 1024
SHARD_RE = re.compile(r"^model-(\d{5})-of-(\d{5})\.safetensors$")


class SafetensorsError(ValueError):
    pass


def read_header(path: str) -> Tuple[Dict[str, dict], int]:
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise SafetensorsError(f"{path}: truncated header length")
        (n,) = struct.unpack("<Q", raw)
        if n == 0 or n > MAX_HEADER or 8 + n > size:
            raise SafetensorsError(f"{path}: invalid header length {n}")
        hdr = json.loads(f.read(n).decode("utf-8"))
    if not isinstance(hdr, dict):
        raise SafetensorsError(f"{path}: header is not a JSON object")
    data_start = 8 + n
    data_len = size - data_start
    ranges = []
    out = {}
    for name, info in hdr.items():
        if name == "__metadata__":
            continue
        dt = info.get("dtype")
        if dt not in DTYPES:
            raise SafetensorsError(f"{path}: tensor {name} has unsupported dtype {dt}")
        shape = info.get("shape")
        offs = info.get("data_offsets")
        if not isinstance(shape, list) or not isinstance(offs, list) or len(offs) != 2:
            raise SafetensorsError(f"{path}: tensor {name} lacks shape/data_offsets")
        b, e = int(offs[0]), int(offs[1])
        nbytes = int(np.prod(shape)) * DTYPES[dt][1] if shape else DTYPES[dt][1]
        if b < 0 or e < b or e > data_len or e - b != nbytes:
            raise SafetensorsError(f"{path}: tensor {name} has inconsistent offsets")
        ranges.append((b, e, name))
        out[name] = {"dtype": dt, "shape": tuple(int(s) for s in shape), "begin": data_start + b,
                     "end": data_start + e}
    ranges.sort()
    for (b0, e0, n0), (b1, e1, n1) in zip(ranges, ranges[1:]):
        if b1 < e0:
            raise SafetensorsError(f"{path}: tensors {n0} and {n1} overlap")
    return out, data_start


class SafetensorsFile:
    def __init__(self, path: str):
        self.path = path
        self.tensors, self.data_start = read_header(path)
        self._mm = None

    def keys(self) -> List[str]:
        return list(self.tensors)

    def get(self, name: str):
        import torch

        info = self.tensors[name]
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        raw = self._mm[info["begin"]:info["end"]]
        npdt = DTYPES[info["dtype"]][0]
        arr = np.frombuffer(raw, dtype=npdt).reshape(info["shape"])
        t = torch.from_numpy(arr.copy())
        if info["dtype"] == "BF16":
            t = t.view(torch.bfloat16)
        return t


def resolve_shards(model_dir: str) -> List[str]:
    """Safetensors files of a HF model directory (single file or a validated shard set)."""
    single = os.path.join(model_dir, "model.safetensors")
    index = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            idx = json.load(f)
        wm = idx.get("weight_map")
        if not isinstance(wm, dict) or not wm:
            raise SafetensorsError("index has no weight_map")
        shards = sorted(set(wm.values()))
        totals = set()
        for s in shards:
            m = SHARD_RE.match(s)
            if not m:
                raise SafetensorsError(f"non-canonical shard name {s}")
            totals.add(int(m.group(2)))
            if not os.path.exists(os.path.join(model_dir, s)):
                raise SafetensorsError(f"missing shard {s}")
        if len(totals) != 1 or len(shards) != totals.pop():
            raise SafetensorsError("shard set is incomplete or inconsistent")
        for s in shards:
            names, _ = read_header(os.path.join(model_dir, s))
            want = {k for k, v in wm.items() if v == s}
            if set(names) != want:
                raise SafetensorsError(f"shard {s} does not hold exactly the tensors the index assigns")
        return [os.path.join(model_dir, s) for s in shards]
    if os.path.exists(single):
        read_header(single)
        return [single]
    raise SafetensorsError(f"{model_dir}: no model.safetensors or model.safetensors.index.json")


def load_state_dict(model_dir: str, names: Optional[Iterable[str]] = None) -> Dict[str, object]:
    out = {}
    want = set(names) if names is not None else None
    for path in resolve_shards(model_dir):
        f = SafetensorsFile(path)
        for k in f.keys():
            if want is None or k in want:
                out[k] = f.get(k)
    return out


def load_file(path: str) -> Dict[str, object]:
    """All tensors of one .safetensors file."""
    f = SafetensorsFile(path)
    return {k: f.get(k) for k in f.keys()}


def save_file(tensors: Dict[str, object], path: str, metadata: Optional[Dict[str, str]] = None) -> None:
    import torch

    hdr: Dict[str, object] = {}
    if metadata:
        hdr["__metadata__"] = metadata
    blobs = []
    off = 0
    rev = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.int64: "I64",
           torch.int32: "I32", torch.int8: "I8", torch.uint8: "U8"}
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        dt = rev[t.dtype]
        b = (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).numpy().tobytes()
        hdr[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def save_sharded(tensors: Dict[str, object], model_dir: str, max_shard_bytes: int) -> List[str]:
    """Write canonical shards + index (model-00001-of-0000N.safetensors)."""
    groups: List[Dict[str, object]] = [{}]
    size = 0
    for k, t in tensors.items():
        nb = t.numel() * t.element_size()
        if groups[-1] and size + nb > max_shard_bytes:
            groups.append({})
            size = 0
        groups[-1][k] = t
        size += nb
    n = len(groups)
    wm = {}
    names = []
    for i, g in enumerate(groups):
        fn = f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_file(g, os.path.join(model_dir, fn))
        names.append(fn)
        for k in g:
            wm[k] = fn
    with open(os.path.join(model_dir, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": sum(t.numel() * t.element_size() for t in tensors.values())},
                   "weight_map": wm}, f)
    return names
