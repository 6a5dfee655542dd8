"""Offline acquisition: checksummed import, integrity verification with
quarantine, inventory export / reconcile (reference: model_import.rs,
model_integrity.rs, model_inventory.rs), through the Python API and HTTP."""
import hashlib
import json
import os

import pytest
from fastapi.testclient import TestClient

from bloom_b200.server.model_store import ModelStore, StoreError, hash_package


@pytest.fixture()
def gguf(tmp_path):
    from bloom_b200.formats.gguf import GGML_Q8_0, write_decoder_gguf
    from bloom_b200.models.config import preset
    from bloom_b200.models.reference import random_weights

    cfg = preset("tiny-llama")
    src = tmp_path / "src"
    src.mkdir()
    p = src / "tiny.gguf"
    write_decoder_gguf(str(p), cfg, random_weights(cfg, seed=0, std=0.08), GGML_Q8_0)
    return p


def test_package_digest(tmp_path):
    d = tmp_path / "pkg"
    (d / "sub").mkdir(parents=True)
    (d / "a.bin").write_bytes(b"abc")
    (d / "sub" / "b.bin").write_bytes(b"x" * 5000)
    h = hash_package(str(d))
    lines = "".join(f"{n}\t{len(b)}\t{hashlib.sha256(b).hexdigest()}\n"
                    for n, b in sorted([("a.bin", b"abc"), ("sub/b.bin", b"x" * 5000)]))
    assert h["sha256"] == hashlib.sha256(lines.encode()).hexdigest() and h["size_bytes"] == 5003
    os.symlink(str(d / "a.bin"), str(d / "link"))
    with pytest.raises(StoreError, match="symbolic"):
        hash_package(str(d))


def test_import_verify_quarantine_inventory(tmp_path, gguf):
    root = tmp_path / "models"
    s = ModelStore(str(root))
    want = hashlib.sha256(gguf.read_bytes()).hexdigest()
    with pytest.raises(StoreError, match="checksum mismatch"):
        s.import_package(str(gguf), expected_sha256="0" * 64)
    assert not [n for n in os.listdir(root) if not n.startswith(".bloom")]  # nothing left behind
    rec = s.import_package(str(gguf), expected_sha256=want)
    assert rec["sha256"] == want and (root / "tiny.gguf").exists()
    with pytest.raises(StoreError, match="already installed"):
        s.import_package(str(gguf))
    st = s.verify("tiny.gguf")
    assert st["phase"] == "complete" and st["matches_expected"] and st["checked_bytes"] == rec["size_bytes"]
    inv = s.inventory()
    assert [m["id"] for m in inv["models"]] == ["tiny.gguf"] and inv["models"][0]["recorded"]
    assert s.reconcile(inv)["in_sync"]
    # tamper: flip a byte -> verification fails and the package is quarantined
    b = bytearray((root / "tiny.gguf").read_bytes())
    b[-1] ^= 0xFF
    (root / "tiny.gguf").write_bytes(bytes(b))
    st = s.verify("tiny.gguf")
    assert st["matches_expected"] is False and "quarantined_to" in st
    assert not (root / "tiny.gguf").exists() and s.quarantined()[0]["id"] == "tiny.gguf"
    r = s.reconcile(inv)
    assert r["missing"] == ["tiny.gguf"] and not r["in_sync"]
    with pytest.raises(StoreError, match="not a loadable"):
        (tmp_path / "junk.gguf").write_bytes(b"not gguf")
        s.import_package(str(tmp_path / "junk.gguf"))


def test_http_acquisition_routes(tmp_path, gguf):
    from bloom_b200.engine.pipeline import EchoPipeline
    from bloom_b200.server.app import ServerSettings, create_app

    root = tmp_path / "models"
    root.mkdir()
    app = create_app(EchoPipeline(), ServerSettings(model_id="echo", models_dir=str(root)))
    with TestClient(app) as c:
        r = c.post("/v1/model-management/import", json={"path": str(gguf)})
        assert r.status_code == 200, r.text
        ids = [e["id"] for e in c.get("/v1/model-management/models").json()["data"]]
        assert ids == ["tiny.gguf"]  # the .bloom metadata directory is not a catalog entry
        v = c.post("/v1/model-management/verify", json={"model": "tiny.gguf"}).json()
        assert v["matches_expected"] is True
        assert c.get("/v1/model-management/integrity").json()["phase"] == "complete"
        inv = c.get("/v1/model-management/inventory").json()
        assert c.post("/v1/model-management/inventory/reconcile", json={"inventory": inv}).json()["in_sync"]
        assert c.post("/v1/model-management/import", json={"path": str(tmp_path / "nope")}).status_code == 400
        assert c.get("/v1/model-management/quarantine").json()["data"] == []
