"""External-runtime adapters: models served by another runtime process.

ExternalServerEngine
    Starts an OpenAI-compatible server binary for a GGUF (llama.cpp's
    `llama-server` by default: `-m <gguf> --host 127.0.0.1 --port <free port>
    --ctx-size N --no-webui --gpu-layers -1|0 [--threads T]`), waits (bounded)
    until its /health answers 200, and streams completions from its
    /v1/completions endpoint (server-sent events).  The binary comes from
    BLOOM_LLAMA_CPP_SERVER or PATH; the process is stopped on close().
ExternalScriptEngine
    Runs a bridge script or binary per request: one JSON request on stdin
    ({"prompt", "params"}), JSON lines on stdout ({"TextDelta": "..."} chunks
    and a final "End"), the reference's pattern for its OpenVINO / NPU / ASR
    bridges.
Both check the executable against the security allowlist first: under
BLOOM_STRICT_SECURITY=1 only names listed in BLOOM_ALLOWED_RUNNERS (binaries)
or BLOOM_ALLOWED_SCRIPTS (scripts) may run; otherwise a short list of known
runners is accepted silently and anything else with a warning.
Reference: crates/engine/src/executor/llamacpp.rs:28-320 (llama-server
adapter), core/security.rs:5-160 (validate_runner / validate_script),
executor/openvino.rs, intel_npu.rs, funasr.rs (script bridges).
"""
from __future__ import annotations

import json
import logging
import os
import shutil
import socket
import subprocess
import sys
import time
import urllib.error
import urllib.request
from typing import Dict, Iterator, List, Optional

log = logging.getLogger("bloom_b200.external")
KNOWN_RUNNERS = ("llama-server", "llama-cli", "ffmpeg", "nvidia-smi")


class ExternalError(RuntimeError):
    pass


def _allowed(path: str, env: str, known=()) -> None:
    name = os.path.basename(path)
    listed = [x.strip() for x in os.environ.get(env, "").split(",") if x.strip()]
    ok = any(a == name or a in path for a in listed)
    if os.environ.get("BLOOM_STRICT_SECURITY", "0") == "1":
        if not ok:
            raise ExternalError(f"Security Error: {path!r} is not in the allowlist ({env}); "
                                "BLOOM_STRICT_SECURITY=1 rejects this execution.")
    elif not ok and name not in known:
        log.warning("running external program %r, which is not allowlisted (set BLOOM_STRICT_SECURITY=1 and %s)",
                    path, env)


def validate_runner(path: str) -> None:
    _allowed(path, "BLOOM_ALLOWED_RUNNERS", KNOWN_RUNNERS)


def validate_script(path: str) -> None:
    _allowed(path, "BLOOM_ALLOWED_SCRIPTS")


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class ExternalServerEngine:
    engine_name = "llamacpp"

    def __init__(self, model_path: str, binary: Optional[str] = None, device: str = "gpu", context_size: int = 4096,
                 threads: Optional[int] = None, extra_args: Optional[List[str]] = None, ready_timeout_s: float = 120.0):
        gguf = model_path
        if os.path.isdir(model_path):
            cands = sorted(f for f in os.listdir(model_path) if f.endswith(".gguf"))
            if not cands:
                raise ExternalError(f"no .gguf file in {model_path}")
            gguf = os.path.join(model_path, cands[0])
        binary = binary or os.environ.get("BLOOM_LLAMA_CPP_SERVER") or shutil.which("llama-server")
        if not binary:
            raise ExternalError("llama-server was not found; set BLOOM_LLAMA_CPP_SERVER to its path")
        validate_runner(binary)
        self.port = _free_port()
        cmd = [binary, "-m", gguf, "--host", "127.0.0.1", "--port", str(self.port), "--ctx-size", str(context_size),
               "--no-webui", "--gpu-layers", "-1" if device == "gpu" else "0"]
        if threads:
            cmd += ["--threads", str(threads)]
        cmd += list(extra_args or [])
        quiet = os.environ.get("BLOOM_LLAMA_CPP_LOG", "0") not in ("1", "true", "yes")
        self.proc = subprocess.Popen(cmd, stdout=subprocess.DEVNULL if quiet else None,
                                     stderr=subprocess.DEVNULL if quiet else None)
        self.base = f"http://127.0.0.1:{self.port}"
        self._wait_ready(ready_timeout_s)

    def _wait_ready(self, timeout_s: float) -> None:
        t0 = time.time()
        while time.time() - t0 < timeout_s:
            if self.proc.poll() is not None:
                raise ExternalError(f"external server exited with code {self.proc.returncode} before it was ready")
            try:
                with urllib.request.urlopen(self.base + "/health", timeout=2) as r:
                    if r.status == 200:
                        return
            except (urllib.error.URLError, OSError):
                pass
            time.sleep(0.1)
        self.close()
        raise ExternalError(f"external server did not become ready within {timeout_s:.0f} s")

    def stream(self, prompt: str, params) -> Iterator[str]:
        body = {"prompt": prompt, "max_tokens": int(getattr(params, "max_tokens", 128)),
                "temperature": float(getattr(params, "temperature", 0.0)), "top_p": float(getattr(params, "top_p", 1.0)),
                "stream": True}
        if getattr(params, "seed", None) is not None:
            body["seed"] = int(params.seed)
        req = urllib.request.Request(self.base + "/v1/completions", data=json.dumps(body).encode(),
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=600) as r:
            for raw in r:
                line = raw.decode("utf-8", "replace").strip()
                if not line.startswith("data:"):
                    continue
                data = line[5:].strip()
                if data == "[DONE]":
                    return
                ev = json.loads(data)
                text = ev.get("choices", [{}])[0].get("text") or ev.get("content") or ""
                if text:
                    yield text

    def close(self) -> None:
        if self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()


class ExternalScriptEngine:
    engine_name = "script"

    def __init__(self, script: str, interpreter: Optional[str] = None, timeout_s: float = 600.0):
        if not os.path.exists(script):
            raise ExternalError(f"bridge script {script!r} does not exist")
        validate_script(script)
        self.cmd = ([interpreter or sys.executable] if script.endswith(".py") else []) + [script]
        self.timeout = timeout_s

    def stream(self, prompt: str, params) -> Iterator[str]:
        req = {"prompt": prompt, "params": {"max_tokens": int(getattr(params, "max_tokens", 128)),
                                            "temperature": float(getattr(params, "temperature", 0.0))}}
        p = subprocess.Popen(self.cmd, stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                             text=True)
        try:
            p.stdin.write(json.dumps(req) + "\n")
            p.stdin.close()
            t0 = time.time()
            for line in p.stdout:
                if time.time() - t0 > self.timeout:
                    raise ExternalError("bridge script timed out")
                line = line.strip()
                if not line:
                    continue
                ev = json.loads(line)
                if ev == "End":
                    break
                if isinstance(ev, dict) and "TextDelta" in ev:
                    yield str(ev["TextDelta"])
                elif isinstance(ev, dict) and "error" in ev:
                    raise ExternalError(f"bridge script error: {ev['error']}")
            rc = p.wait(timeout=max(1.0, self.timeout - (time.time() - t0)))
            if rc != 0:
                raise ExternalError(f"bridge script exited with code {rc}: {p.stderr.read()[-500:]}")
        finally:
            if p.poll() is None:
                p.kill()
                p.wait()

    def close(self) -> None:
        pass


class ExternalPipeline:
    """Pipeline surface (run_stream / run) over an external engine; prompts
    are rendered with the chat template of the model family when known."""

    is_embedding = False
    cfg = None

    def __init__(self, engine, template: str = "chatml", context_size: int = 4096):
        from .text import Tokenizer

        self.engine = engine
        self.engine_name = engine.engine_name
        self.template = template
        self.context_size = context_size
        self.tokenizer = Tokenizer(None)
        self.last_generated_tokens = 0

    def eos_ids(self):
        return []

    def run_stream(self, messages, params, raw: bool = False, stop=None, prompt_ids=None) -> Iterator[str]:
        from .chat_template import render

        if isinstance(messages, str):
            prompt = messages if raw else render([{"role": "user", "content": messages}], self.template)
        else:
            prompt = "\n".join(m["content"] for m in messages) if raw else render(messages, self.template)
        self.last_generated_tokens = 0
        for d in self.engine.stream(prompt, params):
            self.last_generated_tokens += 1
            yield d

    def run(self, messages, params, raw: bool = False, stop=None) -> str:
        return "".join(self.run_stream(messages, params, raw, stop))

    def close(self) -> None:
        self.engine.close()
