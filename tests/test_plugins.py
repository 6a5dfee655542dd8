"""Native engine plugins: manifest validation and a real C plugin loaded
through bloom_plugin_init (intent of the reference's plugin tests,
crates/engine/src/plugin/mod.rs:333-575)."""
import json
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PLUGIN_C = r'''
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "bloom_plugin.h"

static const char* name(void) { return "c-echo"; }
static int32_t mods(int32_t* out, size_t* n) { out[0] = 0; *n = 1; return 0; }
static int32_t devs(int32_t* out, size_t* n) { out[0] = 0; out[1] = 1; *n = 2; return 0; }
typedef struct { char path[256]; } Model;
static int32_t load(const char* p, int32_t dev, void** out) {
  Model* m = (Model*)calloc(1, sizeof(Model)); strncpy(m->path, p, 255); *out = m; return 0; }
static void free_model(void* m) { free(m); }
static char* dup(const char* s) { char* r = (char*)malloc(strlen(s) + 1); strcpy(r, s); return r; }
static int32_t meta(void* m, char** out) {
  char buf[512]; snprintf(buf, sizeof buf, "{\"path\": \"%s\"}", ((Model*)m)->path); *out = dup(buf); return 0; }
static int32_t infer(void* m, const char* in, char** out) {
  const char* p = strstr(in, "\"prompt\": \"");
  if (!p) return 3;
  p += 11; const char* e = strchr(p, '"'); char buf[512];
  snprintf(buf, sizeof buf, "{\"text\": \"plugin: %.*s\"}", (int)(e - p), p); *out = dup(buf); return 0; }
static int32_t stream(void* m, const char* in, CBloomStreamCallback cb, void* u) {
  if (cb(u, "{\"TextDelta\": \"a\"}") != 0) return 0;
  if (cb(u, "{\"TextDelta\": \"b\"}") != 0) return 0;
  cb(u, "\"End\""); return 0; }
static void free_string(char* s) { free(s); }
int32_t bloom_plugin_init(CBloomEngine* e) {
  e->name = name; e->supported_modalities = mods; e->supported_devices = devs; e->load_model = load;
  e->free_model = free_model; e->model_metadata = meta; e->model_infer = infer; e->model_infer_stream = stream;
  e->free_string = free_string; return 0; }
'''


@pytest.fixture(scope="module")
def plugin_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("plugin")
    (d / "echo.c").write_text(PLUGIN_C)
    subprocess.check_call(["gcc", "-std=c99", "-shared", "-fPIC", "-Wall", "-I", os.path.join(ROOT, "csrc", "plugin"),
                           str(d / "echo.c"), "-o", str(d / "libecho.so")])
    from bloom_b200.engine.plugins import current_platform

    man = {"metadata": {"name": "com.example.c-echo", "version": "1.0.0", "description": "test", "author": "t",
                        "license": "MIT", "platforms": [current_platform()], "min_runtime_version": "0.1.0"},
           "entry_point": {"type": "native", "path": "libecho.so"}, "supported_modalities": ["Text"]}
    (d / "echo.json").write_text(json.dumps(man))
    return d


def test_native_plugin_roundtrip(plugin_dir):
    from bloom_b200.engine.plugins import PluginEngine, discover, load_manifest

    man = load_manifest(str(plugin_dir / "echo.json"))
    eng = PluginEngine(man)
    assert eng.name == "c-echo"
    assert eng.supported_modalities() == ["Text"] and eng.supported_devices() == ["cpu", "cuda"]
    m = eng.load("/models/x", "gpu")
    assert m.metadata() == {"path": "/models/x"}
    assert m.run("hello") == "plugin: hello"
    assert list(m.infer_stream({"Text": {"prompt": "q"}})) == [{"TextDelta": "a"}, {"TextDelta": "b"}, "End"]
    m.close()
    assert [x.name for x in discover(str(plugin_dir))] == ["com.example.c-echo"]


def test_manifest_validation(plugin_dir, tmp_path, monkeypatch):
    from bloom_b200.engine.plugins import PluginEngine, PluginError, load_manifest

    good = json.loads((plugin_dir / "echo.json").read_text())

    def write(d):
        p = tmp_path / "m.json"
        p.write_text(json.dumps(d))
        return str(p)

    for mutate, msg in [(lambda d: d["metadata"].update(name=""), "name"),
                        (lambda d: d["metadata"].update(version=""), "version"),
                        (lambda d: d["metadata"].update(platforms=["plan9-mips"]), "not compatible"),
                        (lambda d: d["entry_point"].update(type="dll"), "Invalid entry point")]:
        d = json.loads(json.dumps(good))
        mutate(d)
        with pytest.raises(PluginError, match=msg):
            load_manifest(write(d))
    d = json.loads(json.dumps(good))
    d["entry_point"]["type"] = "wasm"
    with pytest.raises(PluginError, match="Only 'native'"):
        PluginEngine(load_manifest(write(d)))
    monkeypatch.setenv("BLOOM_STRICT_SECURITY", "1")
    with pytest.raises(PluginError, match="allowlist"):
        load_manifest(str(plugin_dir / "echo.json"))
    monkeypatch.setenv("BLOOM_ALLOWED_PLUGINS", "com.example.c-echo")
    load_manifest(str(plugin_dir / "echo.json"))


def test_library_without_init_is_rejected(tmp_path):
    from bloom_b200._ext import runtime

    (tmp_path / "x.c").write_text("int nothing(void) { return 0; }\n")
    subprocess.check_call(["gcc", "-shared", "-fPIC", str(tmp_path / "x.c"), "-o", str(tmp_path / "libx.so")])
    with pytest.raises(RuntimeError, match="bloom_plugin_init"):
        runtime().NativePlugin(str(tmp_path / "libx.so"))
