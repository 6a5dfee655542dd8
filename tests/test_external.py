"""External-runtime adapters with fake runtimes: an OpenAI-compatible server
binary (llama-server arguments, /health, streamed /v1/completions) and a JSON
bridge script; the security allowlist under strict mode (reference:
executor/llamacpp.rs, core/security.rs)."""
import json
import os
import stat
import sys
import textwrap

import pytest

from bloom_b200.engine.external import ExternalError, ExternalScriptEngine, ExternalServerEngine

FAKE_SERVER = textwrap.dedent(r'''
    #!PYTHON
    import json, sys, time
    from http.server import BaseHTTPRequestHandler, HTTPServer
    args = sys.argv[1:]
    port = int(args[args.index("--port") + 1])
    assert args[args.index("-m") + 1].endswith(".gguf") and "--no-webui" in args
    class H(BaseHTTPRequestHandler):
        def log_message(self, *a): pass
        def do_GET(self):
            self.send_response(200 if self.path == "/health" else 404); self.end_headers(); self.wfile.write(b"{}")
        def do_POST(self):
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            self.send_response(200); self.send_header("Content-Type", "text/event-stream"); self.end_headers()
            for w in ("ext:" + body["prompt"]).split(" ")[: body["max_tokens"]]:
                self.wfile.write(("data: " + json.dumps({"choices": [{"text": w + " "}]}) + "\n\n").encode())
            self.wfile.write(b"data: [DONE]\n\n")
    time.sleep(0.3)  # not ready at once
    HTTPServer(("127.0.0.1", port), H).serve_forever()
''').replace("#!PYTHON", "#!" + sys.executable).lstrip()

BRIDGE = textwrap.dedent(r'''
    import json, sys
    req = json.loads(sys.stdin.readline())
    for w in req["prompt"].split(" ")[: req["params"]["max_tokens"]]:
        print(json.dumps({"TextDelta": w.upper() + " "}), flush=True)
    print(json.dumps("End"))
''')


class P:
    max_tokens = 3
    temperature = 0.0
    top_p = 1.0
    seed = None


def _exe(path, text):
    path.write_text(text)
    path.chmod(path.stat().st_mode | stat.S_IEXEC)
    return str(path)


def test_external_server_adapter(tmp_path, monkeypatch):
    server = _exe(tmp_path / "llama-server", FAKE_SERVER)
    (tmp_path / "m.gguf").write_bytes(b"GGUF")
    eng = ExternalServerEngine(str(tmp_path), binary=server, device="cpu", ready_timeout_s=30)
    try:
        assert "".join(eng.stream("hello big world again", P())) == "ext:hello big world "
    finally:
        eng.close()
    assert eng.proc.poll() is not None
    monkeypatch.setenv("BLOOM_STRICT_SECURITY", "1")
    monkeypatch.setenv("BLOOM_ALLOWED_RUNNERS", "something-else")
    with pytest.raises(ExternalError, match="allowlist"):
        ExternalServerEngine(str(tmp_path / "m.gguf"), binary=server)
    dead = _exe(tmp_path / "dead-server", "#!/bin/sh\nexit 3\n")
    monkeypatch.setenv("BLOOM_ALLOWED_RUNNERS", "dead-server")
    with pytest.raises(ExternalError, match="exited with code 3"):
        ExternalServerEngine(str(tmp_path / "m.gguf"), binary=dead, ready_timeout_s=10)


def test_external_script_bridge(tmp_path, monkeypatch):
    script = tmp_path / "bridge.py"
    script.write_text(BRIDGE)
    eng = ExternalScriptEngine(str(script))
    assert "".join(eng.stream("one two three four", P())) == "ONE TWO THREE "
    bad = tmp_path / "bad.py"
    bad.write_text("import sys; sys.exit(4)\n")
    with pytest.raises(ExternalError, match="code 4"):
        list(ExternalScriptEngine(str(bad)).stream("x", P()))
    monkeypatch.setenv("BLOOM_STRICT_SECURITY", "1")
    with pytest.raises(ExternalError, match="BLOOM_ALLOWED_SCRIPTS"):
        ExternalScriptEngine(str(script))
    monkeypatch.setenv("BLOOM_ALLOWED_SCRIPTS", "bridge.py")
    assert ExternalScriptEngine(str(script)) is not None


def test_bloom_infer_script_backend(tmp_path, capsys):
    from bloom_b200.cli.infer import main

    script = tmp_path / "bridge.py"
    script.write_text(BRIDGE)
    rc = main(["-m", str(script), "--backend", "script", "-p", "alpha beta", "--raw", "--max-tokens", "8",
               "--device", "cpu", "--quiet"])
    assert rc == 0 and capsys.readouterr().out.strip() == "ALPHA BETA"
