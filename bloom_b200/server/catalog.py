"""Model catalog for the operator API: the model packages under a models
directory (a subdirectory with config.json / bloom.json / safetensors, or a
.gguf file), with their manifest summary and size.  Subset of the
reference's catalog (crates/server/src/lib.rs model-management routes):
list, preflight (memory estimate for 180 GB per GPU), switch, unload and
remove.  Downloads and imports need a network and are not offered.
"""
from __future__ import annotations

import os
import shutil
from typing import Dict, List, Optional


def _size(path: str) -> int:
    if os.path.isfile(path):
        return os.path.getsize(path)
    total = 0
    for root, _, files in os.walk(path):
        for f in files:
            try:
                total += os.path.getsize(os.path.join(root, f))
            except OSError:
                pass
    return total


class ModelCatalog:
    def __init__(self, root: Optional[str]):
        self.root = os.path.abspath(root) if root else None

    def entries(self) -> List[Dict[str, object]]:
        from ..formats.manifest import load_manifest

        out = []
        if not self.root or not os.path.isdir(self.root):
            return out
        for name in sorted(os.listdir(self.root)):
            if name.startswith("."):  # store metadata, quarantine, imports in progress
                continue
            path = os.path.join(self.root, name)
            if not (os.path.isdir(path) or name.endswith(".gguf")):
                continue
            try:
                man = load_manifest(path)
                out.append({"id": name, "path": path, "family": man.family, "primary_dtype": man.primary_dtype,
                            "format": man.files[0].format if man.files else None, "size_bytes": _size(path),
                            "valid": True})
            except Exception as e:  # noqa: BLE001 - listed as invalid, not hidden
                out.append({"id": name, "path": path, "valid": False, "error": str(e), "size_bytes": _size(path)})
        return out

    def find(self, model_id: str) -> Optional[Dict[str, object]]:
        for e in self.entries():
            if e["id"] == model_id:
                return e
        return None

    def preflight(self, model_id: str, context_size: int, concurrent: int, tp: int = 1) -> Dict[str, object]:
        from ..formats.manifest import estimate_memory, load_manifest

        e = self.find(model_id)
        if e is None:
            raise KeyError(model_id)
        if not e.get("valid"):
            return {"model": model_id, "fits": False, "error": e.get("error")}
        est = estimate_memory(load_manifest(e["path"]), context_size, concurrent_seqs=concurrent, tp=tp)
        d = est.to_dict()
        d.update(model=model_id, fits=bool(est.fits))
        return d

    def remove(self, model_id: str) -> None:
        e = self.find(model_id)
        if e is None:
            raise KeyError(model_id)
        p = str(e["path"])
        if not p.startswith(self.root + os.sep):
            raise PermissionError("refusing to remove a path outside the models directory")
        if os.path.isdir(p):
            shutil.rmtree(p)
        else:
            os.remove(p)
