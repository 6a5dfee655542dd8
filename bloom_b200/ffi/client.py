"""ctypes client of libbloom_ffi (the C ABI in csrc/ffi/bloom.h).

    from bloom_b200.ffi.client import BloomClient
    with BloomClient.load("model-dir-or-preset", engine="b200", device="gpu") as c:
        print(c.run("Hello", max_tokens=32))
        for chunk in c.stream("Hello"):
            ...

Mirrors the reference SDK surface (load / run / run_stream / cancellation)
over the same ABI a C or C++ host links against.
"""
from __future__ import annotations

import ctypes
import json
import os
import threading
from typing import Iterator, List, Optional

STATUS = {0: "OK", -1: "INVALID_ARGUMENT", -2: "INVALID_UTF8", -3: "INVALID_INPUT_JSON",
          -4: "INVALID_PARAMS_JSON", -5: "INFERENCE_ERROR", -6: "OUTPUT_ERROR", -7: "PANIC", -8: "CANCELLED"}


class BloomSlice(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("len", ctypes.c_size_t)]


class BloomOwnedBuffer(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("len", ctypes.c_size_t)]


CALLBACK_V2 = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint8), ctypes.c_size_t)


class BloomError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


def default_library() -> str:
    return os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbloom_ffi.so")


def open_library(path: Optional[str] = None) -> ctypes.CDLL:
    lib = ctypes.CDLL(path or default_library())
    lib.bloom_abi_version.restype = ctypes.c_uint32
    lib.bloom_pipeline_load_v2.restype = ctypes.c_void_p
    lib.bloom_pipeline_load_v2.argtypes = [BloomSlice, BloomSlice, BloomSlice, ctypes.c_size_t, ctypes.c_char_p,
                                           ctypes.c_size_t]
    lib.bloom_pipeline_run_v2.restype = ctypes.c_int32
    lib.bloom_pipeline_run_v2.argtypes = [ctypes.c_void_p, BloomSlice, BloomSlice, ctypes.POINTER(BloomOwnedBuffer),
                                          ctypes.c_char_p, ctypes.c_size_t]
    lib.bloom_pipeline_run_stream_v2.restype = ctypes.c_int32
    lib.bloom_pipeline_run_stream_v2.argtypes = [ctypes.c_void_p, BloomSlice, BloomSlice, CALLBACK_V2,
                                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
    lib.bloom_pipeline_free.argtypes = [ctypes.c_void_p]
    lib.bloom_buffer_free.argtypes = [ctypes.POINTER(BloomOwnedBuffer)]
    lib.bloom_cancellation_token_new.restype = ctypes.c_void_p
    lib.bloom_cancellation_token_cancel.restype = ctypes.c_int32
    lib.bloom_cancellation_token_cancel.argtypes = [ctypes.c_void_p]
    lib.bloom_cancellation_token_free.argtypes = [ctypes.c_void_p]
    return lib


def _slice(b: bytes) -> BloomSlice:
    return BloomSlice(ctypes.cast(ctypes.c_char_p(b), ctypes.c_void_p), len(b))


class CancellationToken:
    def __init__(self, lib):
        self.lib = lib
        self.ptr = lib.bloom_cancellation_token_new()

    def cancel(self) -> None:
        self.lib.bloom_cancellation_token_cancel(self.ptr)

    def __del__(self):
        if getattr(self, "ptr", None):
            self.lib.bloom_cancellation_token_free(self.ptr)
            self.ptr = None


class BloomClient:
    def __init__(self, lib, ptr):
        self.lib = lib
        self.ptr = ptr

    @classmethod
    def load(cls, model: str, engine: str = "auto", device: str = "gpu", context_size: int = 2048,
             library: Optional[str] = None) -> "BloomClient":
        lib = open_library(library)
        err = ctypes.create_string_buffer(1024)
        bufs = [model.encode(), engine.encode(), device.encode()]
        ptr = lib.bloom_pipeline_load_v2(_slice(bufs[0]), _slice(bufs[1]), _slice(bufs[2]), context_size, err,
                                         len(err))
        if not ptr:
            raise BloomError(-1, err.value.decode(errors="replace"))
        return cls(lib, ptr)

    @staticmethod
    def _params(max_tokens=128, temperature=0.7, top_p=0.9, seed=None) -> bytes:
        return json.dumps({"max_tokens": max_tokens, "temperature": temperature, "top_p": top_p,
                           "seed": seed}).encode()

    def run(self, prompt: str, **params) -> str:
        inp = json.dumps({"Text": {"prompt": prompt}}).encode()
        par = self._params(**params)
        out = BloomOwnedBuffer()
        err = ctypes.create_string_buffer(1024)
        st = self.lib.bloom_pipeline_run_v2(self.ptr, _slice(inp), _slice(par), ctypes.byref(out), err, len(err))
        if st != 0:
            raise BloomError(st, err.value.decode(errors="replace"))
        try:
            data = ctypes.string_at(out.data, out.len)
        finally:
            self.lib.bloom_buffer_free(ctypes.byref(out))
        return json.loads(data)["text"]

    def stream(self, prompt: str, cancel: Optional[CancellationToken] = None, **params) -> Iterator[dict]:
        """Runs the stream on a worker thread and yields the decoded chunks."""
        inp = json.dumps({"Text": {"prompt": prompt}}).encode()
        par = self._params(**params)
        chunks: List[dict] = []
        cv = threading.Condition()
        state = {"done": False, "status": 0, "err": ""}

        @CALLBACK_V2
        def on_chunk(_user, data, n):
            obj = json.loads(ctypes.string_at(data, n))
            with cv:
                chunks.append(obj)
                cv.notify()

        def work():
            err = ctypes.create_string_buffer(1024)
            st = self.lib.bloom_pipeline_run_stream_v2(self.ptr, _slice(inp), _slice(par), on_chunk, None,
                                                       cancel.ptr if cancel else None, err, len(err))
            with cv:
                state.update(done=True, status=st, err=err.value.decode(errors="replace"))
                cv.notify()

        th = threading.Thread(target=work, daemon=True)
        th.start()
        i = 0
        while True:
            with cv:
                while i >= len(chunks) and not state["done"]:
                    cv.wait()
                if i < len(chunks):
                    c = chunks[i]
                    i += 1
                else:
                    break
            yield c
        th.join()
        if state["status"] not in (0,):
            raise BloomError(state["status"], state["err"])

    def close(self) -> None:
        if self.ptr:
            self.lib.bloom_pipeline_free(self.ptr)
            self.ptr = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass
