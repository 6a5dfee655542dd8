"""Native engine plugins (shared libraries with the CBloomEngine table of
csrc/plugin/bloom_plugin.h), described by a plugin manifest JSON:

    {"metadata": {"name": "com.acme.echo", "version": "1.0.0", "description": "...",
                  "author": "...", "license": "MIT", "platforms": ["linux-x86_64"],
                  "min_runtime_version": "0.1.0"},
     "entry_point": {"type": "native", "path": "libecho.so"},
     "supported_families": ["Llama"], "supported_modalities": ["Text"], ...}

Validation follows the reference (crates/engine/src/plugin/mod.rs:
load_manifest / validate_manifest / validate_entry_point): non-empty name,
version and platforms, the current platform listed, a known entry-point type
(native / wasm / remote / subprocess; only native is loadable), entry path
resolved against the manifest's directory, names on the security allowlist
when BLOOM_STRICT_SECURITY=1 (BLOOM_ALLOWED_PLUGINS, comma-separated).
"""
from __future__ import annotations

import json
import os
import platform
from dataclasses import dataclass, field
from typing import Iterator, List, Optional

from .._ext import runtime as _rt

ENTRY_TYPES = ("native", "wasm", "remote", "subprocess")
MODALITIES = {0: "Text", 1: "Audio", 2: "Vision", 3: "Embedding"}
DEVICES = {0: "cpu", 1: "cuda", 2: "metal", 3: "npu"}


class PluginError(Exception):
    pass


def current_platform() -> str:
    m = platform.machine().lower()
    arch = {"x86_64": "x86_64", "amd64": "x86_64", "aarch64": "aarch64", "arm64": "aarch64"}.get(m, m)
    osn = {"linux": "linux", "darwin": "macos", "windows": "windows"}.get(platform.system().lower(), "unknown")
    return f"{osn}-{arch}"


@dataclass
class PluginManifest:
    name: str
    version: str
    platforms: List[str]
    entry_type: str
    entry_path: str
    base_dir: str
    description: str = ""
    supported_families: List[str] = field(default_factory=list)
    supported_modalities: List[str] = field(default_factory=list)
    supported_devices: List[str] = field(default_factory=list)
    supports_streaming: Optional[bool] = None
    raw: dict = field(default_factory=dict)

    @property
    def library_path(self) -> str:
        p = self.entry_path
        return p if os.path.isabs(p) else os.path.join(self.base_dir, p)


def load_manifest(path: str) -> PluginManifest:
    try:
        with open(path) as f:
            d = json.load(f)
    except (OSError, ValueError) as e:
        raise PluginError(f"failed to read plugin manifest {path}: {e}") from e
    md = d.get("metadata") or {}
    ep = d.get("entry_point") or {}
    man = PluginManifest(name=md.get("name", ""), version=md.get("version", ""), platforms=list(md.get("platforms", [])),
                         entry_type=ep.get("type", ""), entry_path=ep.get("path", ""),
                         base_dir=os.path.dirname(os.path.abspath(path)), description=md.get("description", ""),
                         supported_families=list(d.get("supported_families", [])),
                         supported_modalities=list(d.get("supported_modalities", [])),
                         supported_devices=list(d.get("supported_devices", [])),
                         supports_streaming=d.get("supports_streaming"), raw=d)
    validate_manifest(man)
    return man


def validate_manifest(m: PluginManifest) -> None:
    if not m.name:
        raise PluginError("Plugin name cannot be empty")
    if os.environ.get("BLOOM_STRICT_SECURITY", "0") == "1":
        allowed = [x.strip() for x in os.environ.get("BLOOM_ALLOWED_PLUGINS", "").split(",") if x.strip()]
        if m.name not in allowed:
            raise PluginError(f"plugin {m.name!r} is not on the strict-security allowlist")
    if not m.version:
        raise PluginError("Plugin version cannot be empty")
    if not m.platforms:
        raise PluginError("Plugin platforms list cannot be empty")
    cur = current_platform()
    if not cur.startswith("unknown") and cur not in m.platforms:
        raise PluginError(f"Plugin '{m.name}' is not compatible with current platform '{cur}'. "
                          f"Supported platforms: {m.platforms}")
    if not m.entry_path:
        raise PluginError("Plugin entry point path cannot be empty")
    if m.entry_type not in ENTRY_TYPES:
        raise PluginError(f"Invalid entry point type: {m.entry_type}")


class PluginEngine:
    """A loaded native plugin; `load(model_path, device)` gives a PluginModel."""

    def __init__(self, manifest: PluginManifest):
        if manifest.entry_type != "native":
            raise PluginError("Only 'native' entry point type is supported for engine plugins")
        if not os.path.exists(manifest.library_path):
            raise PluginError(f"Native plugin entry point does not exist: {manifest.library_path}")
        self.manifest = manifest
        self.lib = _rt().NativePlugin(manifest.library_path)

    @property
    def name(self) -> str:
        return self.lib.name()

    def supported_modalities(self) -> List[str]:
        return [MODALITIES.get(c, str(c)) for c in self.lib.supported_modalities()]

    def supported_devices(self) -> List[str]:
        return [DEVICES.get(c, str(c)) for c in self.lib.supported_devices()]

    def load(self, model_path: str, device: str = "cpu") -> "PluginModel":
        code = {v: k for k, v in DEVICES.items()}.get({"gpu": "cuda"}.get(device, device), 0)
        return PluginModel(self, self.lib.load_model(model_path, code))


class PluginModel:
    def __init__(self, engine: PluginEngine, handle: int):
        self.engine = engine
        self.handle = handle

    def metadata(self) -> dict:
        return json.loads(self.engine.lib.metadata(self.handle) or "{}")

    def infer(self, model_input: dict) -> dict:
        return json.loads(self.engine.lib.infer(self.handle, json.dumps(model_input)))

    def infer_stream(self, model_input: dict) -> Iterator[object]:
        chunks: List[object] = []
        self.engine.lib.infer_stream(self.handle, json.dumps(model_input),
                                     lambda c: chunks.append(json.loads(c)) is None)
        yield from chunks

    def run(self, prompt: str) -> str:
        out = self.infer({"Text": {"prompt": prompt}})
        return out.get("text") or ""

    def close(self) -> None:
        if self.handle:
            self.engine.lib.free_model(self.handle)
            self.handle = 0

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass


def discover(directory: str) -> List[PluginManifest]:
    """Manifests (*.json with metadata + entry_point) found directly in a directory."""
    out = []
    if not os.path.isdir(directory):
        return out
    for n in sorted(os.listdir(directory)):
        if n.endswith(".json"):
            try:
                out.append(load_manifest(os.path.join(directory, n)))
            except PluginError:
                continue
    return out
