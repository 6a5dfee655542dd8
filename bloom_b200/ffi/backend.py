"""Python side of the C ABI (csrc/ffi/bloom_ffi.cpp calls these functions).

JSON shapes are those of the reference ABI (crates/ffi/bloom.h and
crates/engine/src/core/io.rs): input is a ModelInput enum such as
{"Text": {"prompt": "..."}}, params a GenerationParams object such as
{"max_tokens": 10, "temperature": 0.7, "top_p": 0.9, "seed": null}; a run
returns a ModelOutput {"text": ..., "logits": null, "image": null,
"audio": null, "video": null}; a stream yields OutputChunk values
{"TextDelta": "..."} ... {"Metrics": {"compute_ms": n}} and "End".

Errors are raised as the exception classes below; the C++ layer maps each
to its BLOOM_STATUS_* code.
"""
from __future__ import annotations

import json
import time
from typing import Iterator


class InvalidArgument(Exception):
    pass


class InvalidInputJson(Exception):
    pass


class InvalidParamsJson(Exception):
    pass


class InferenceError(Exception):
    pass


_ENGINES = ("mock", "b200", "cpu", "auto")


class _Handle:
    def __init__(self, pipe, engine: str):
        self.pipe = pipe
        self.engine = engine


def load(model_path: str, engine: str, device: str, context_size: int) -> _Handle:
    if context_size <= 0:
        raise InvalidArgument("context_size must be greater than zero")
    engine = (engine or "auto").strip().lower()
    if engine not in _ENGINES:
        raise InvalidArgument(f"unknown engine {engine!r}; available: {', '.join(_ENGINES)}")
    device = (device or "cpu").strip().lower()
    if device not in ("cpu", "gpu", "cuda"):
        raise InvalidArgument(f"unknown device {device!r}; expected cpu or gpu")
    from ..engine.pipeline import EchoPipeline, InferencePipeline

    if engine == "mock":
        return _Handle(EchoPipeline(), engine)
    dev = "cpu" if (engine == "cpu" or device == "cpu") else "gpu"
    try:
        pipe = InferencePipeline.load(model_path, device=dev, context_size=int(context_size))
    except Exception as e:  # noqa: BLE001
        raise InferenceError(f"failed to load {model_path!r}: {e}") from e
    return _Handle(pipe, engine)


def _parse(input_json: str, params_json: str):
    try:
        inp = json.loads(input_json)
    except json.JSONDecodeError as e:
        raise InvalidInputJson(f"Failed to parse input JSON: {e}") from e
    try:
        params = json.loads(params_json)
    except json.JSONDecodeError as e:
        raise InvalidParamsJson(f"Failed to parse params JSON: {e}") from e
    if not isinstance(inp, dict) or len(inp) != 1:
        raise InvalidInputJson("Failed to parse input JSON: expected one ModelInput variant")
    (kind, body), = inp.items()
    if kind == "Text":
        if not isinstance(body, dict) or not isinstance(body.get("prompt"), str):
            raise InvalidInputJson("Failed to parse input JSON: Text needs a string prompt")
        prompt = body["prompt"]
    elif kind == "Multi" and isinstance(body, dict) and isinstance(body.get("text"), str):
        prompt = body["text"]
    else:
        raise InvalidInputJson(f"Failed to parse input JSON: unsupported input variant {kind!r} for text engines")
    if not isinstance(params, dict):
        raise InvalidParamsJson("Failed to parse params JSON: expected an object")
    from ..engine.engine import SamplingParams

    try:
        sp = SamplingParams(max_tokens=int(params.get("max_tokens", 128)),
                            temperature=float(params.get("temperature", 0.7)),
                            top_p=float(params.get("top_p", 0.9)),
                            seed=None if params.get("seed") is None else int(params["seed"]))
    except (TypeError, ValueError) as e:
        raise InvalidParamsJson(f"Failed to parse params JSON: {e}") from e
    rf = params.get("response_format")
    if isinstance(rf, dict) and rf.get("type") in ("json_object", "json_schema"):
        sp.json_mode = True
    if sp.max_tokens <= 0:
        raise InvalidParamsJson("Failed to parse params JSON: max_tokens must be positive")
    return prompt, sp


def run(handle: _Handle, input_json: str, params_json: str) -> str:
    prompt, sp = _parse(input_json, params_json)
    try:
        text = handle.pipe.run(prompt, sp)
    except Exception as e:  # noqa: BLE001
        raise InferenceError(f"Inference failed: {e}") from e
    return json.dumps({"text": text, "logits": None, "image": None, "audio": None, "video": None})


def stream(handle: _Handle, input_json: str, params_json: str) -> Iterator[str]:
    prompt, sp = _parse(input_json, params_json)
    t0 = time.perf_counter()

    def gen():
        try:
            for delta in handle.pipe.run_stream(prompt, sp):
                yield json.dumps({"TextDelta": delta})
        except Exception as e:  # noqa: BLE001
            raise InferenceError(f"Inference failed: {e}") from e
        yield json.dumps({"Metrics": {"compute_ms": int((time.perf_counter() - t0) * 1000)}})
        yield json.dumps("End")

    return gen()
