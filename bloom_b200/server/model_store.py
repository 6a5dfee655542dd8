"""Offline model acquisition: checksummed import, integrity verification with
quarantine, and inventory export / reconcile for the models directory.

Layout under the models root:
    <id>/ or <id>.gguf                  installed packages (what the catalog lists)
    .bloom/provenance/<id>.json         per package: sha256 digest, files with
                                        size and sha256, source, import time
    .bloom/quarantine/<id>[.N]          packages whose re-hash did not match
A package digest is the SHA-256 of its sorted "<path>\\t<size>\\t<sha256>\\n"
lines (a single-file package: the file's own SHA-256).  Hashing is the C++
`hash_files` (parallel files, large reads).

Import copies a local file or package directory into a temporary name
inside the root, validates it as a model package, hashes it, checks an
expected digest if one was given, and renames it into place with its
provenance record -- a failed import leaves nothing behind.  Verification
re-hashes an installed package against its provenance; on a mismatch the
package moves to quarantine (the catalog stops listing it) unless
`quarantine=False`.  Downloads need a network and are not offered.
Reference: crates/server/src/model_import.rs, model_integrity.rs,
model_inventory.rs.
"""
from __future__ import annotations

import json
import os
import shutil
import threading
import time
import uuid
from typing import Dict, List, Optional

from .._ext import runtime as _rt

_ID_OK = set("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789._-")


class StoreError(ValueError):
    pass


def _valid_id(model_id: str) -> str:
    if not model_id or len(model_id) > 128 or model_id.startswith(".") or any(c not in _ID_OK for c in model_id):
        raise StoreError(f"invalid model id {model_id!r} (1-128 of [A-Za-z0-9._-], not starting with '.')")
    return model_id


def _files_of(path: str) -> List[str]:
    if os.path.isfile(path):
        return [path]
    out = []
    for root, dirs, files in os.walk(path):
        dirs[:] = sorted(d for d in dirs if not d.startswith("."))
        for f in sorted(files):
            p = os.path.join(root, f)
            if os.path.islink(p):
                raise StoreError(f"symbolic links are not allowed in a model package: {p}")
            out.append(p)
    return out


def hash_package(path: str, threads: int = 8, progress=None) -> Dict:
    """{"sha256", "size_bytes", "files": [{"filename", "size", "sha256"}]}."""
    files = _files_of(path)
    res = _rt().hash_files(files, threads, progress) if progress else _rt().hash_files(files, threads)
    entries = []
    for r in res:
        if r["error"]:
            raise StoreError(r["error"])
        rel = os.path.basename(path) if os.path.isfile(path) else os.path.relpath(r["path"], path)
        entries.append({"filename": rel.replace(os.sep, "/"), "size": int(r["size"]), "sha256": r["sha256"]})
    entries.sort(key=lambda e: e["filename"])
    if os.path.isfile(path):
        digest = entries[0]["sha256"]
    else:
        lines = "".join(f"{e['filename']}\t{e['size']}\t{e['sha256']}\n" for e in entries)
        digest = _rt().sha256_bytes(lines.encode())
    return {"sha256": digest, "size_bytes": sum(e["size"] for e in entries), "files": entries}


class ModelStore:
    def __init__(self, root: str):
        self.root = os.path.abspath(root)
        self.meta = os.path.join(self.root, ".bloom")
        self.prov_dir = os.path.join(self.meta, "provenance")
        self.quarantine_dir = os.path.join(self.meta, "quarantine")
        self._lock = threading.Lock()
        self.status: Dict = {"phase": "idle", "model_id": None, "checked_bytes": 0, "total_bytes": None,
                             "expected_sha256": None, "actual_sha256": None, "matches_expected": None,
                             "verified_at": None, "error": None}

    # ------------------------------------------------------------ provenance
    def _prov_path(self, model_id: str) -> str:
        return os.path.join(self.prov_dir, _valid_id(model_id) + ".json")

    def provenance(self, model_id: str) -> Optional[Dict]:
        try:
            with open(self._prov_path(model_id)) as f:
                return json.load(f)
        except FileNotFoundError:
            return None

    def _write_prov(self, model_id: str, rec: Dict) -> None:
        os.makedirs(self.prov_dir, exist_ok=True)
        tmp = self._prov_path(model_id) + f".tmp{uuid.uuid4().hex[:8]}"
        with open(tmp, "w") as f:
            json.dump(rec, f, indent=1, sort_keys=True)
        os.replace(tmp, self._prov_path(model_id))

    def path_of(self, model_id: str) -> str:
        p = os.path.join(self.root, _valid_id(model_id))
        if not os.path.exists(p):
            raise StoreError(f"model {model_id!r} is not installed")
        return p

    # ------------------------------------------------------------ import
    def import_package(self, source: str, model_id: Optional[str] = None,
                       expected_sha256: Optional[str] = None) -> Dict:
        from ..formats.manifest import load_manifest

        src = os.path.abspath(source)
        if not os.path.exists(src):
            raise StoreError(f"source {source!r} does not exist")
        if src == self.root or src.startswith(self.root + os.sep):
            raise StoreError("the source is already inside the models directory")
        model_id = _valid_id(model_id or os.path.basename(src.rstrip(os.sep)))
        dest = os.path.join(self.root, model_id)
        if os.path.exists(dest):
            raise StoreError(f"model {model_id!r} is already installed")
        os.makedirs(self.root, exist_ok=True)
        tmp = os.path.join(self.root, f".import-{uuid.uuid4().hex[:12]}" + (".gguf" if src.endswith(".gguf") else ""))
        try:
            if os.path.isdir(src):
                _files_of(src)  # rejects symlinks before copying
                shutil.copytree(src, tmp)
            else:
                shutil.copy2(src, tmp)
            try:
                load_manifest(tmp)
            except Exception as e:  # noqa: BLE001
                raise StoreError(f"not a loadable model package: {e}") from None
            h = hash_package(tmp)
            if expected_sha256 and h["sha256"] != expected_sha256.lower():
                raise StoreError(f"checksum mismatch: expected {expected_sha256}, got {h['sha256']}")
            if not os.path.isdir(tmp):  # single files keep their own name (the catalog lists *.gguf)
                h["files"][0]["filename"] = model_id
            os.replace(tmp, dest)
            rec = {"id": model_id, "sha256": h["sha256"], "size_bytes": h["size_bytes"], "files": h["files"],
                   "kind": "package" if os.path.isdir(dest) else "file", "source": src,
                   "imported_at": time.time(), "verified_at": time.time()}
            self._write_prov(model_id, rec)
            return rec
        finally:
            if os.path.isdir(tmp):
                shutil.rmtree(tmp, ignore_errors=True)
            elif os.path.exists(tmp):
                os.remove(tmp)

    def record(self, model_id: str, source: str = "local") -> Dict:
        """Adopt an already-installed package: hash it and record its provenance."""
        p = self.path_of(model_id)
        h = hash_package(p)
        rec = {"id": model_id, "sha256": h["sha256"], "size_bytes": h["size_bytes"], "files": h["files"],
               "kind": "package" if os.path.isdir(p) else "file", "source": source, "imported_at": time.time(),
               "verified_at": time.time()}
        self._write_prov(model_id, rec)
        return rec

    # ------------------------------------------------------------ integrity
    def verify(self, model_id: str, quarantine: bool = True) -> Dict:
        with self._lock:
            if self.status["phase"] == "verifying":
                raise StoreError(f"verification of {self.status['model_id']!r} is already running")
            rec = self.provenance(model_id)
            if rec is None:
                raise StoreError("No verified acquisition checksum is recorded for this model.")
            self.status = {"phase": "verifying", "model_id": model_id, "checked_bytes": 0,
                           "total_bytes": rec["size_bytes"], "expected_sha256": rec["sha256"], "actual_sha256": None,
                           "matches_expected": None, "verified_at": None, "error": None}
        try:
            p = self.path_of(model_id)
            on_disk = {os.path.relpath(f, p).replace(os.sep, "/") if os.path.isdir(p) else model_id
                       for f in _files_of(p)}
            expected = {e["filename"] for e in rec["files"]}
            if rec["kind"] == "package" and on_disk != expected:
                raise StoreError(f"package files changed: missing {sorted(expected - on_disk)[:5]}, "
                                 f"unexpected {sorted(on_disk - expected)[:5]}")

            def progress(done):
                self.status["checked_bytes"] = int(done)
                return True

            h = hash_package(p, progress=progress)
            ok = h["sha256"] == rec["sha256"]
            st = dict(self.status, phase="complete", checked_bytes=h["size_bytes"], actual_sha256=h["sha256"],
                      matches_expected=ok, verified_at=time.time())
            if ok:
                rec["verified_at"] = st["verified_at"]
                self._write_prov(model_id, rec)
            elif quarantine:
                st["quarantined_to"] = self.quarantine(model_id, f"checksum mismatch: {h['sha256']}")
            self.status = st
            return st
        except Exception as e:  # noqa: BLE001
            st = dict(self.status, phase="error", error=str(e), matches_expected=False)
            if quarantine and isinstance(e, StoreError) and "files changed" in str(e):
                st["quarantined_to"] = self.quarantine(model_id, str(e))
            self.status = st
            return st

    def quarantine(self, model_id: str, reason: str) -> str:
        p = self.path_of(model_id)
        os.makedirs(self.quarantine_dir, exist_ok=True)
        dest = os.path.join(self.quarantine_dir, model_id)
        n = 1
        while os.path.exists(dest):
            dest = os.path.join(self.quarantine_dir, f"{model_id}.{n}")
            n += 1
        os.replace(p, dest)
        with open(dest.rstrip(os.sep) + ".reason.json", "w") as f:
            json.dump({"id": model_id, "reason": reason, "at": time.time()}, f)
        return dest

    def quarantined(self) -> List[Dict]:
        if not os.path.isdir(self.quarantine_dir):
            return []
        out = []
        for name in sorted(os.listdir(self.quarantine_dir)):
            if name.endswith(".reason.json"):
                with open(os.path.join(self.quarantine_dir, name)) as f:
                    d = json.load(f)
                d["path"] = os.path.join(self.quarantine_dir, name[:-len(".reason.json")])
                out.append(d)
        return out

    # ------------------------------------------------------------ inventory
    def inventory(self) -> Dict:
        """Installed packages with their recorded provenance (no hashing)."""
        models = []
        if os.path.isdir(self.root):
            for name in sorted(os.listdir(self.root)):
                if name.startswith("."):
                    continue
                p = os.path.join(self.root, name)
                rec = self.provenance(name) if all(c in _ID_OK for c in name) else None
                size = sum(os.path.getsize(f) for f in _files_of(p)) if os.path.exists(p) else 0
                models.append({"id": name, "size_bytes": size, "sha256": rec["sha256"] if rec else None,
                               "recorded": rec is not None, "size_matches": bool(rec) and rec["size_bytes"] == size,
                               "verified_at": rec.get("verified_at") if rec else None})
        return {"object": "bloom.inventory", "schema_version": 1, "root": self.root, "generated_at": time.time(),
                "models": models}

    def reconcile(self, inventory: Dict) -> Dict:
        """Compare an exported inventory with what is installed now."""
        want = {m["id"]: m for m in inventory.get("models", [])}
        have = {m["id"]: m for m in self.inventory()["models"]}
        changed = [i for i in want if i in have and want[i].get("sha256") and have[i].get("sha256") and
                   (want[i]["sha256"] != have[i]["sha256"] or want[i].get("size_bytes") != have[i]["size_bytes"])]
        return {"object": "bloom.inventory.reconcile", "missing": sorted(set(want) - set(have)),
                "unexpected": sorted(set(have) - set(want)), "changed": sorted(changed),
                "unrecorded": sorted(i for i, m in have.items() if not m["recorded"]),
                "in_sync": set(want) == set(have) and not changed}
