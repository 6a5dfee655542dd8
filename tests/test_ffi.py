"""C ABI (csrc/ffi/bloom.h, libbloom_ffi.so) on the mock engine, CPU only.

Intent follows the reference ABI tests (crates/ffi/tests/ffi_tests.rs and
header_smoke.c/.cpp): ABI version, length-delimited v2 buffers, stream
chunks, cancellation before and during a stream, strict UTF-8, stable
statuses for malformed / oversized input, NULL callbacks and a zero
context, plus a real C host linking the library."""
import ctypes
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FFI = os.path.join(ROOT, "csrc", "ffi")


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    sys.path.insert(0, FFI)
    import build as ffi_build  # csrc/ffi/build.py

    out = str(tmp_path_factory.mktemp("ffi") / "libbloom_ffi.so")
    ffi_build.build(out)
    from bloom_b200.ffi.client import open_library

    return open_library(out), out


def _sl(b):
    from bloom_b200.ffi.client import _slice

    return _slice(b)


PARAMS = b'{"max_tokens":10,"temperature":0.7,"top_p":0.9,"seed":null}'


def _load(L, engine=b"mock", ctx=2048):
    err = ctypes.create_string_buffer(512)
    p = L.bloom_pipeline_load_v2(_sl(b"."), _sl(engine), _sl(b"cpu"), ctx, err, len(err))
    return p, err


def test_header_smoke_compiles_as_c_and_cpp(tmp_path, lib):
    """Both smoke programs compile warning-free against the header and link
    against the built library (the C one takes the address of every export
    with its declared signature); running them checks statuses and layouts."""
    _, path = lib
    d = os.path.dirname(path)
    for src, cc, std in (("header_smoke.c", "gcc", "-std=c99"), ("header_smoke.cpp", "g++", "-std=c++17")):
        exe = str(tmp_path / src.replace(".", "_"))
        subprocess.check_call([cc, std, "-Wall", "-Werror", os.path.join(FFI, "tests", src), "-o", exe, f"-L{d}",
                               "-l:libbloom_ffi.so", f"-Wl,-rpath,{d}"])
        assert subprocess.call([exe]) == 0


def test_v2_run_uses_length_delimited_buffers(lib):
    from bloom_b200.ffi.client import BloomOwnedBuffer

    L, _ = lib
    assert L.bloom_abi_version() == 2
    p, err = _load(L)
    assert p, err.value
    out = BloomOwnedBuffer()
    st = L.bloom_pipeline_run_v2(p, _sl(b'{"Text":{"prompt":"Hello v2"}}'), _sl(PARAMS), ctypes.byref(out), err,
                                 len(err))
    assert st == 0, err.value
    assert json.loads(ctypes.string_at(out.data, out.len))["text"] == "echo: Hello v2"
    L.bloom_buffer_free(ctypes.byref(out))
    assert not out.data and out.len == 0
    L.bloom_pipeline_free(p)


def test_stream_chunks_and_cancellation(lib):
    from bloom_b200.ffi.client import CALLBACK_V2

    L, _ = lib
    p, err = _load(L)
    seen = []

    @CALLBACK_V2
    def cb(_u, data, n):
        seen.append(json.loads(ctypes.string_at(data, n)))

    st = L.bloom_pipeline_run_stream_v2(p, _sl(b'{"Text":{"prompt":"a b c"}}'), _sl(PARAMS), cb, None, None, err,
                                        len(err))
    assert st == 0
    assert "".join(c["TextDelta"] for c in seen if isinstance(c, dict) and "TextDelta" in c) == "echo: a b c"
    assert seen[-1] == "End" and any(isinstance(c, dict) and "Metrics" in c for c in seen)
    # cancelled before the call: no callback, CANCELLED
    tok = L.bloom_cancellation_token_new()
    assert L.bloom_cancellation_token_cancel(tok) == 0
    seen.clear()
    st = L.bloom_pipeline_run_stream_v2(p, _sl(b'{"Text":{"prompt":"x y"}}'), _sl(PARAMS), cb, None, tok, err,
                                        len(err))
    assert st == -8 and not seen and b"cancel" in err.value
    L.bloom_cancellation_token_free(tok)
    # cancelled from inside the first callback: exactly one chunk delivered
    tok2 = L.bloom_cancellation_token_new()
    count = [0]

    @CALLBACK_V2
    def cancel_cb(_u, data, n):
        count[0] += 1
        L.bloom_cancellation_token_cancel(tok2)

    st = L.bloom_pipeline_run_stream_v2(p, _sl(b'{"Text":{"prompt":"one two three"}}'), _sl(PARAMS), cancel_cb,
                                        None, tok2, err, len(err))
    assert st == -8 and count[0] == 1
    L.bloom_cancellation_token_free(tok2)
    assert L.bloom_cancellation_token_cancel(None) == -1
    L.bloom_pipeline_free(p)


def test_stable_statuses(lib):
    from bloom_b200.ffi.client import CALLBACK_V2, BloomOwnedBuffer, BloomSlice

    L, _ = lib
    p, err = _load(L)
    good = _sl(b'{"Text":{"prompt":"Hello"}}')
    bad_utf8 = b"\xff\xfe"
    huge = BloomSlice(ctypes.cast(ctypes.c_char_p(b"{}"), ctypes.c_void_p), 16 * 1024 * 1024 + 1)
    for inp, par, expected in [(_sl(b"{"), _sl(PARAMS), -3), (good, _sl(b"{"), -4), (huge, _sl(PARAMS), -1),
                               (_sl(bad_utf8), _sl(PARAMS), -2), (_sl(b'{"Audio":{}}'), _sl(PARAMS), -3)]:
        out = BloomOwnedBuffer()
        st = L.bloom_pipeline_run_v2(p, inp, par, ctypes.byref(out), err, len(err))
        assert st == expected, (st, expected, err.value)
        assert not out.data
    st = L.bloom_pipeline_run_stream_v2(p, good, _sl(PARAMS), CALLBACK_V2(), None, None, err, len(err))
    assert st == -1 and b"Null argument" in err.value
    L.bloom_pipeline_free(p)
    p0, err0 = _load(L, ctx=0)
    assert not p0 and b"context_size must be greater than zero" in err0.value
    p1, err1 = _load(L, engine=b"vulkan")
    assert not p1 and b"unknown engine" in err1.value


def test_revision1_symbols(lib):
    L, _ = lib
    L.bloom_pipeline_load.restype = ctypes.c_void_p
    L.bloom_pipeline_run.restype = ctypes.c_void_p
    L.bloom_pipeline_run.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                     ctypes.c_size_t]
    L.bloom_string_free.argtypes = [ctypes.c_void_p]
    err = ctypes.create_string_buffer(256)
    p = L.bloom_pipeline_load(b".", b"mock", b"cpu", ctypes.c_size_t(2048), err, ctypes.c_size_t(len(err)))
    assert p
    s = L.bloom_pipeline_run(p, b'{"Text":{"prompt":"v1"}}', PARAMS, err, len(err))
    assert json.loads(ctypes.string_at(s))["text"] == "echo: v1"
    L.bloom_string_free(s)
    L.bloom_pipeline_free(ctypes.c_void_p(p))


def test_c_host_program(lib, tmp_path):
    _, so = lib
    exe = str(tmp_path / "demo")
    subprocess.check_call(["gcc", "-std=c99", "-Wall", os.path.join(FFI, "examples", "demo.c"), "-I" + FFI,
                           so, "-Wl,-rpath," + os.path.dirname(so), "-o", exe])
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    import site

    env["PYTHONPATH"] += os.pathsep + os.pathsep.join(site.getsitepackages())
    r = subprocess.run([exe], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert 'output: {"text": "echo: Hello from C"' in r.stdout
    assert "stream status 0" in r.stdout


def test_python_client(lib):
    from bloom_b200.ffi.client import BloomClient

    _, so = lib
    with BloomClient.load(".", engine="mock", device="cpu", library=so) as c:
        assert c.run("hi there", max_tokens=8) == "echo: hi there"
        chunks = list(c.stream("p q", max_tokens=8))
        assert chunks[-1] == "End"
