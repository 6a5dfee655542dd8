"""Structured output: response_format json_object / json_schema, and the
function-calling envelope, as constrained decoding on the GPU.

Every constrained request carries a `SchemaConstraint`: the C++
`SchemaMatcher` (bloom_b200._runtime) over the compiled schema.  Each step,
while the GPU runs the forward, the engine asks every constrained row's
matcher for its allowed-token bit mask (computed over a byte trie of the
vocabulary and cached per matcher state); the masks are uploaded and
applied to the logits by a kernel before the ordinary argmax / top-p
sampler runs, so the sampled token always keeps the output a valid prefix of
a document the schema accepts, and end-of-sequence is allowed only once the
document is complete.  Nothing is read back to the host for this.

Schema subset and limits follow the reference's validator
(crates/server/src/helpers.rs:2454-2960: keywords $schema, title,
description, type, enum, required, properties, additionalProperties, items;
64 KiB, depth 16, 1,024 nodes, 256 properties, 256 enum values, 1,024
annotation characters), plus one limit of this matcher: at most 64
properties per object.  `validate_json_schema_subset` is the post-hoc check
of a finished document (reference `validate_json_schema_subset`).
"""
from __future__ import annotations

import json
from typing import Any, Dict, List, Optional, Sequence, Tuple

from .._ext import runtime as _rt

MAX_JSON_SCHEMA_BYTES = 64 * 1024
MAX_JSON_SCHEMA_DEPTH = 16
MAX_JSON_SCHEMA_NODES = 1024
MAX_JSON_SCHEMA_PROPERTIES = 256
MAX_JSON_SCHEMA_ENUM_VALUES = 256
MAX_JSON_SCHEMA_ANNOTATION_CHARS = 1024
MAX_MATCHER_PROPERTIES = 64

_KEYWORDS = {"$schema", "title", "description", "type", "enum", "required", "properties", "additionalProperties",
             "items"}
_TYPES = {"object": 1, "array": 2, "string": 4, "number": 8, "integer": 16, "boolean": 32, "null": 64}


class SchemaError(ValueError):
    pass


# ---------------------------------------------------------------- validation
def validate_supported_json_schema(schema: Any) -> None:
    """Raise SchemaError unless `schema` is in the supported subset and limits."""
    enc = json.dumps(schema, separators=(",", ":")).encode()
    if len(enc) > MAX_JSON_SCHEMA_BYTES:
        raise SchemaError(f"response JSON Schema exceeds the {MAX_JSON_SCHEMA_BYTES} byte limit.")
    if not isinstance(schema, dict) or schema.get("type") != "object":
        raise SchemaError("response JSON Schema root type must be object.")
    count = [0]

    def node(s: Any, path: str, depth: int) -> None:
        if depth > MAX_JSON_SCHEMA_DEPTH:
            raise SchemaError(f"response JSON Schema exceeds the maximum depth of {MAX_JSON_SCHEMA_DEPTH}.")
        count[0] += 1
        if count[0] > MAX_JSON_SCHEMA_NODES:
            raise SchemaError(f"response JSON Schema contains more than {MAX_JSON_SCHEMA_NODES} schema nodes.")
        if not isinstance(s, dict):
            raise SchemaError(f"response JSON Schema at {path} must be an object.")
        for k in s:
            if k not in _KEYWORDS:
                raise SchemaError(f"response JSON Schema at {path} uses unsupported keyword {k!r}.")
        for k in ("$schema", "title", "description"):
            if k in s and not (isinstance(s[k], str) and len(s[k]) <= MAX_JSON_SCHEMA_ANNOTATION_CHARS):
                raise SchemaError(f"response JSON Schema {path}.{k} must be a bounded string.")
        ty = s.get("type")
        if ty is not None and ty not in _TYPES:
            raise SchemaError(f"response JSON Schema at {path} has an unsupported type.")
        if "enum" in s:
            ev = s["enum"]
            if not isinstance(ev, list) or not 1 <= len(ev) <= MAX_JSON_SCHEMA_ENUM_VALUES:
                raise SchemaError(f"response JSON Schema at {path}.enum must contain 1 to "
                                  f"{MAX_JSON_SCHEMA_ENUM_VALUES} values.")
        props = s.get("properties")
        if props is not None:
            if not isinstance(props, dict):
                raise SchemaError(f"response JSON Schema at {path}.properties must be an object.")
            if ty != "object":
                raise SchemaError(f"response JSON Schema at {path} can use properties only with type object.")
            if len(props) > MAX_JSON_SCHEMA_PROPERTIES:
                raise SchemaError(f"response JSON Schema at {path} contains more than "
                                  f"{MAX_JSON_SCHEMA_PROPERTIES} properties.")
            if len(props) > MAX_MATCHER_PROPERTIES:
                raise SchemaError(f"response JSON Schema at {path} has {len(props)} properties; constrained "
                                  f"decoding supports at most {MAX_MATCHER_PROPERTIES} per object.")
            for f, ps in props.items():
                if not f or len(f) > 128 or any(ord(c) < 0x20 for c in f):
                    raise SchemaError(f"response JSON Schema at {path} contains an invalid property name.")
                node(ps, f"{path}.{f}", depth + 1)
        if "required" in s:
            if ty != "object":
                raise SchemaError(f"response JSON Schema at {path} can use required only with type object.")
            req = s["required"]
            if not isinstance(req, list) or len(req) > MAX_JSON_SCHEMA_PROPERTIES:
                raise SchemaError(f"response JSON Schema at {path}.required must be an array of field names.")
            seen = set()
            for f in req:
                if not isinstance(f, str):
                    raise SchemaError(f"response JSON Schema at {path}.required must contain strings.")
                if f in seen or props is None or f not in props:
                    raise SchemaError(f"response JSON Schema at {path}.required contains a duplicate or unknown "
                                      f"property {f!r}.")
                seen.add(f)
        if "additionalProperties" in s and (ty != "object" or not isinstance(s["additionalProperties"], bool)):
            raise SchemaError(f"response JSON Schema at {path}.additionalProperties requires type object and a "
                              "boolean value.")
        if "items" in s:
            if ty != "array":
                raise SchemaError(f"response JSON Schema at {path} can use items only with type array.")
            node(s["items"], f"{path}[]", depth + 1)

    node(schema, "$", 0)


def extract_json_schema(wrapper: Any) -> Dict:
    """response_format.json_schema = {name?, description?, strict?, schema}."""
    if not isinstance(wrapper, dict) or not isinstance(wrapper.get("schema"), dict):
        raise SchemaError("response_format=json_schema requires a json_schema.schema object.")
    for k in wrapper:
        if k not in ("name", "description", "strict", "schema"):
            raise SchemaError(f"response_format json_schema contains unsupported field {k!r}.")
    if "strict" in wrapper and not isinstance(wrapper["strict"], bool):
        raise SchemaError("response_format json_schema.strict must be a boolean.")
    return wrapper["schema"]


def response_format_mode(rf: Any) -> Tuple[str, Optional[Dict]]:
    """('text' | 'json_object' | 'json_schema', schema)."""
    if rf is None:
        return "text", None
    if not isinstance(rf, dict):
        raise SchemaError("response_format must be an object.")
    t = rf.get("type")
    if t == "text":
        return "text", None
    if t == "json_object":
        return "json_object", None
    if t == "json_schema":
        schema = extract_json_schema(rf.get("json_schema"))
        validate_supported_json_schema(schema)
        return "json_schema", schema
    raise SchemaError(f"unsupported response_format type {t!r}; expected text, json_object, or json_schema")


def _matches_type(v: Any, t: str) -> bool:
    if t == "object":
        return isinstance(v, dict)
    if t == "array":
        return isinstance(v, list)
    if t == "string":
        return isinstance(v, str)
    if t == "number":
        return isinstance(v, (int, float)) and not isinstance(v, bool)
    if t == "integer":
        return isinstance(v, int) and not isinstance(v, bool)
    if t == "boolean":
        return isinstance(v, bool)
    if t == "null":
        return v is None
    return False


def _json_eq(a: Any, b: Any) -> bool:
    """JSON value equality (true is not 1)."""
    if isinstance(a, bool) or isinstance(b, bool):
        return type(a) is type(b) and a == b
    if isinstance(a, dict) and isinstance(b, dict):
        return a.keys() == b.keys() and all(_json_eq(a[k], b[k]) for k in a)
    if isinstance(a, list) and isinstance(b, list):
        return len(a) == len(b) and all(_json_eq(x, y) for x, y in zip(a, b))
    return a == b


def validate_json_schema_subset(value: Any, schema: Dict, path: str = "$") -> None:
    """Raise SchemaError if a finished document does not satisfy the schema."""
    if "enum" in schema and not any(_json_eq(value, e) for e in schema["enum"]):
        raise SchemaError(f"{path} does not match any allowed enum value")
    t = schema.get("type")
    if t is not None and not _matches_type(value, t):
        raise SchemaError(f"{path} expected type {t}")
    if isinstance(value, dict):
        for f in schema.get("required", []):
            if f not in value:
                raise SchemaError(f"{path} missing required property '{f}'")
        props = schema.get("properties")
        if isinstance(props, dict):
            for f, ps in props.items():
                if f in value:
                    validate_json_schema_subset(value[f], ps, f"{path}.{f}")
            if schema.get("additionalProperties") is False:
                for f in value:
                    if f not in props:
                        raise SchemaError(f"{path} contains unsupported property '{f}'")
    if isinstance(value, list) and isinstance(schema.get("items"), dict):
        for i, item in enumerate(value):
            validate_json_schema_subset(item, schema["items"], f"{path}[{i}]")


# ---------------------------------------------------------------- compilation
def compile_schema(schema: Optional[Dict]) -> Tuple[List[Any], int]:
    """Schema dict -> (SchemaNode list, root id).  None: any JSON object."""
    rt = _rt()
    nodes: List[Any] = []
    if schema is None:
        return nodes, -1

    def build(s: Dict) -> int:
        n = rt.SchemaNode()
        idx = len(nodes)
        nodes.append(n)
        t = s.get("type")
        n.types = _TYPES.get(t, 0) if t else 0
        if "enum" in s:
            n.enum_lits = [json.dumps(e, separators=(",", ":"), ensure_ascii=False) for e in s["enum"]]
        props = s.get("properties") or {}
        keys, kids, req = [], [], []
        required = set(s.get("required", []))
        for f, ps in props.items():
            keys.append(json.dumps(f, ensure_ascii=False)[1:-1])
            kids.append(build(ps) if isinstance(ps, dict) and ps else -1)
            req.append(1 if f in required else 0)
        n.prop_keys, n.prop_nodes, n.prop_required = keys, kids, req
        n.additional = bool(s.get("additionalProperties", True))
        it = s.get("items")
        n.items = build(it) if isinstance(it, dict) and it else -1
        nodes[idx] = n
        return idx

    root = build(schema)
    return nodes, root


# ---------------------------------------------------------------- vocabulary
class TokenVocab:
    """Per tokenizer: the bytes each token decodes to, the ids never allowed
    inside a document (special tokens) and the byte trie of the rest."""

    _cache: Dict[Tuple[int, int], "TokenVocab"] = {}

    def __init__(self, tokenizer, vocab_size: int):
        toks: List[bytes] = []
        special = set()
        inner = getattr(tokenizer, "_t", tokenizer)
        try:
            for tid in getattr(inner, "all_special_ids", []) or []:
                special.add(int(tid))
        except Exception:
            pass
        try:  # tokenizers.Tokenizer: added (special) tokens
            for tid, at in (inner.get_added_tokens_decoder() or {}).items():
                if getattr(at, "special", True):
                    special.add(int(tid))
        except Exception:
            pass
        for i in range(vocab_size):
            try:
                s = tokenizer.decode([i], skip_special_tokens=False)
            except Exception:
                s = ""
            toks.append(s.encode("utf-8", errors="replace"))
        self.vocab_size = vocab_size
        self.token_bytes = toks
        self.excluded = sorted(special)
        self.trie = _rt().VocabTrie(toks, self.excluded)

    @classmethod
    def get(cls, tokenizer, vocab_size: int) -> "TokenVocab":
        key = (id(tokenizer), vocab_size)
        v = cls._cache.get(key)
        if v is None:
            v = cls(tokenizer, vocab_size)
            cls._cache[key] = v
        return v


class SchemaConstraint:
    """One request's constraint: JSON object (schema None) or a JSON Schema."""

    def __init__(self, vocab: TokenVocab, schema: Optional[Dict], eos: Sequence[int]):
        nodes, root = compile_schema(schema)
        self.matcher = _rt().SchemaMatcher(nodes, root)
        self.vocab = vocab
        self.eos = [int(e) for e in eos]
        self.schema = schema

    @property
    def words(self) -> int:
        return (self.vocab.vocab_size + 31) // 32

    def mask_into(self, out_row) -> None:
        """Write the allowed-token mask of the current state into an int32 host row."""
        self.matcher.mask_into(self.vocab.trie, self.eos, out_row)

    def advance(self, token: int) -> bool:
        if token in self.eos or not (0 <= token < self.vocab.vocab_size):
            return True
        return bool(self.matcher.feed(self.vocab.token_bytes[token]))

    def complete(self) -> bool:
        return bool(self.matcher.complete())


def constrain_params(params, response_format: dict, pipeline=None) -> None:
    """Attach the response format to SamplingParams (validated; raises SchemaError)."""
    mode, schema = response_format_mode(response_format)
    if mode == "text":
        return
    params.json_mode = True
    params.json_schema = schema


def repair_json(text: str) -> str:
    """Close an unfinished JSON document; valid documents are returned unchanged."""
    try:
        json.loads(text)
        return text
    except ValueError:
        pass
    stack: List[str] = []
    in_str = esc = False
    start = text.find("{") if "{" in text else text.find("[")
    if start < 0:
        return "{}"
    body = text[start:]
    for c in body:
        if in_str:
            if esc:
                esc = False
            elif c == "\\":
                esc = True
            elif c == '"':
                in_str = False
            continue
        if c == '"':
            in_str = True
        elif c in "{[":
            stack.append("}" if c == "{" else "]")
        elif c in "}]" and stack:
            stack.pop()
    out = body + ('"' if in_str else "")
    out = out.rstrip().rstrip(",").rstrip(":")
    if out.endswith(","):
        out = out[:-1]
    out += "".join(reversed(stack))
    try:
        json.loads(out)
        return out
    except ValueError:
        return "{}"
