"""JSON Schema constrained decoding (C++ matcher + vocabulary masks) and
OpenAI function tools, on CPU.

Intent follows the reference's response-format and tool-calling tests
(crates/server/src/helpers.rs schema validation, tool_calling.rs tests):
schema subset limits, tool definitions and choice modes, envelope parsing,
history validation; plus the properties constrained decoding relies on --
every document a schema accepts is accepted byte by byte, and a token's
mask bit says exactly whether feeding it keeps the prefix valid.
"""
import json
import random

import pytest
import torch

from bloom_b200._ext import runtime
from bloom_b200.engine.structured import (SchemaError, compile_schema, response_format_mode,
                                          validate_json_schema_subset, validate_supported_json_schema)

PERSON = {
    "type": "object",
    "properties": {
        "name": {"type": "string"},
        "age": {"type": "integer"},
        "score": {"type": "number"},
        "color": {"enum": ["red", "green", "blue"]},
        "tags": {"type": "array", "items": {"type": "string"}},
        "ok": {"type": "boolean"},
        "extra": {"type": "null"},
        "nested": {"type": "object", "properties": {"x": {"type": "integer"}}, "required": ["x"],
                   "additionalProperties": False},
    },
    "required": ["name", "age"],
    "additionalProperties": False,
}


def matcher(schema):
    nodes, root = compile_schema(schema)
    return runtime().SchemaMatcher(nodes, root)


def accepts(schema, text):
    m = matcher(schema)
    for ch in text.encode():
        if not m.feed(bytes([ch])):
            return False, False
    return True, m.complete()


# ---------------------------------------------------------------- schema validation
def test_schema_subset_validation():
    validate_supported_json_schema(PERSON)
    bad = [
        ({"type": "array"}, "root type"),
        ({"type": "object", "properties": {"a": {"type": "string", "minLength": 2}}}, "unsupported keyword"),
        ({"type": "object", "required": ["a"]}, "unknown property"),
        ({"type": "object", "properties": {"a": {"type": "date"}}}, "unsupported type"),
        ({"type": "object", "properties": {"a": {"type": "string", "items": {}}}}, "items only"),
        ({"type": "object", "additionalProperties": {"type": "string"}}, "boolean value"),
        ({"type": "object", "properties": {"a": {"enum": []}}}, "enum"),
    ]
    for s, msg in bad:
        with pytest.raises(SchemaError, match=msg):
            validate_supported_json_schema(s)
    deep = {"type": "object"}
    cur = deep
    for _ in range(20):
        cur["properties"] = {"a": {"type": "object"}}
        cur = cur["properties"]["a"]
    with pytest.raises(SchemaError, match="depth"):
        validate_supported_json_schema(deep)
    assert response_format_mode({"type": "json_object"}) == ("json_object", None)
    assert response_format_mode({"type": "json_schema", "json_schema": {"name": "p", "schema": PERSON}})[1] == PERSON
    with pytest.raises(SchemaError):
        response_format_mode({"type": "json_schema", "json_schema": {"name": "p"}})
    with pytest.raises(SchemaError):
        response_format_mode({"type": "xml"})


def test_post_hoc_validation():
    validate_json_schema_subset({"name": "a", "age": 3}, PERSON)
    for doc, msg in [({"name": "a"}, "missing required"), ({"name": "a", "age": 1.5}, "integer"),
                     ({"name": "a", "age": 1, "zz": 1}, "unsupported property"),
                     ({"name": "a", "age": 1, "color": "pink"}, "enum"), ({"name": "a", "age": True}, "integer")]:
        with pytest.raises(SchemaError, match=msg):
            validate_json_schema_subset(doc, PERSON)


# ---------------------------------------------------------------- matcher
def test_matcher_accepts_and_rejects():
    ok = '{"name": "Bo\\"b\\u00e9", "age": -42, "score": 1.5e-3, "color": "green", "tags": ["a", ""],' \
         ' "ok": false, "extra": null, "nested": {"x": 0}}'
    assert accepts(PERSON, ok) == (True, True)
    assert accepts(PERSON, '{"age":1,"name":"x"}') == (True, True)  # any property order
    for bad in ['{"age": 1}', '{"name": "a", "age": 1.5}', '{"name": "a", "age": 01}', '{"name": "a", "age": 1, "age": 2}',
                '{"name": "a", "age": 1, "colour": "red"}', '{"name": "a", "age": 1, "color": "pink"}',
                '{"name": "a", "age": 1, "nested": {}}', '{"name": "a", "age": 1, "ok": nul}',
                '[1]', '{"name": "a\x01"}', '{"name": "a", "age": 1,}', '{"name": "a", "age": 1}}']:
        acc, done = accepts(PERSON, bad)
        assert not (acc and done), bad
    # whitespace runs are bounded
    assert accepts(PERSON, '{' + ' ' * 8 + '"name": "a", "age": 1}') == (True, True)
    assert not accepts(PERSON, '{' + ' ' * 9 + '"name": "a", "age": 1}')[0]
    # json_object mode: any object
    assert accepts(None, '{"a": [1, {"b": null}], "c": "d"}') == (True, True)
    assert not accepts(None, '"str"')[0]


def _gen_value(schema, rng, depth=0):
    if schema is None or not schema:
        return rng.choice([1, "s", None, True, [1, 2], {"k": "v"}])
    if "enum" in schema:
        return rng.choice(schema["enum"])
    t = schema.get("type")
    if t == "object":
        out = {}
        props = schema.get("properties", {})
        for k, ps in props.items():
            if k in schema.get("required", []) or rng.random() < 0.6:
                out[k] = _gen_value(ps, rng, depth + 1)
        return out
    if t == "array":
        return [_gen_value(schema.get("items"), rng, depth + 1) for _ in range(rng.randint(0, 3))]
    if t == "string":
        return "".join(rng.choice("ab \"\\\né中") for _ in range(rng.randint(0, 6)))
    if t == "integer":
        return rng.randint(-10**6, 10**6)
    if t == "number":
        return rng.choice([rng.uniform(-1e3, 1e3), rng.randint(-5, 5), 1e-7])
    if t == "boolean":
        return rng.random() < 0.5
    return None


def _dump(v, rng):
    if rng.random() < 0.5:
        return json.dumps(v, ensure_ascii=rng.random() < 0.5)
    return json.dumps(v, indent=rng.choice([None, 1, 2]), separators=(rng.choice([",", ", "]), rng.choice([":", ": "])),
                      ensure_ascii=False)


def test_generated_documents_are_accepted():
    rng = random.Random(0)
    for _ in range(300):
        doc = _gen_value(PERSON, rng)
        text = _dump(doc, rng)
        validate_json_schema_subset(json.loads(text), PERSON)
        assert accepts(PERSON, text) == (True, True), text


def test_mask_bits_match_feeding_each_token():
    """For states along a document, bit t of the mask <=> feeding token t succeeds."""
    vocab = [b'{', b'}', b'"', b'"name"', b'": ', b'"age":', b'"', b'1', b'12', b'-', b'.', b'e', b'5', b',', b' ',
             b'\n  ', b'"color": "', b'red', b'"re', b'd"', b'green', b'tr', b'ue', b'false', b'null', b'[', b']',
             b'"tags": [', b'x', b'\\', b'n', b'u00', b'}\n', b'", ', b'<eos>', b'']
    eos = [34]
    trie = runtime().VocabTrie(vocab, [34])
    doc = '{"name": "x\\n", "age": 12, "color": "red", "tags": ["x"]}'
    words = (len(vocab) + 31) // 32
    for cut in range(len(doc) + 1):
        m = matcher(PERSON)
        assert m.feed(doc[:cut].encode())
        out = torch.zeros(words, dtype=torch.int32)
        m.mask_into(trie, eos, out)
        for t, tb in enumerate(vocab):
            bit = bool((int(out[t // 32]) >> (t % 32)) & 1)
            if t == 34:
                assert bit == (cut == len(doc)), cut
                continue
            if not tb:
                assert not bit
                continue
            probe = matcher(PERSON)
            probe.feed(doc[:cut].encode())
            assert bit == bool(probe.feed(tb)), (doc[:cut], tb)


def test_mask_cache_hits_inside_strings():
    vocab = [bytes([c]) for c in range(32, 127)] + [b'<eos>']
    trie = runtime().VocabTrie(vocab, [len(vocab) - 1])
    m = matcher(None)
    m.feed(b'{"k": "')
    out = torch.zeros((len(vocab) + 31) // 32, dtype=torch.int32)
    for ch in b"hello world":
        m.mask_into(trie, [len(vocab) - 1], out)
        assert m.feed(bytes([ch]))
    assert m.cache_misses == 1 and m.cache_hits == 10


# ---------------------------------------------------------------- tools
from bloom_b200.server.tool_calling import (ToolError, envelope_schema, normalize_tool_history,  # noqa: E402
                                            parse_tool_output, responses_tool_config, tool_calls_json, tool_config)

WEATHER = [{"type": "function", "function": {
    "name": "get_weather", "description": "Get weather.", "strict": True,
    "parameters": {"type": "object", "properties": {"city": {"type": "string"}}, "required": ["city"],
                   "additionalProperties": False}}}]


def test_tool_config_choice_modes():
    c = tool_config(WEATHER)
    assert c.choice == "auto" and c.parallel
    assert tool_config(WEATHER, "required").choice == "required"
    n = tool_config(WEATHER, {"type": "function", "function": {"name": "get_weather"}})
    assert n.choice == "named" and n.named == "get_weather"
    assert tool_config(WEATHER, "none") is None
    assert tool_config(None) is None
    for tools, choice, msg in [
        (None, "auto", "at least one"),
        ([{"type": "custom", "custom": {"name": "shell"}}], None, "unsupported field|type `function`"),
        ([{"type": "function", "function": {"name": "bad name"}}], None, "ASCII"),
        (WEATHER + WEATHER, None, "duplicate"),
        (WEATHER, {"type": "function", "function": {"name": "other"}}, "undefined"),
        ([{"type": "function", "function": {"name": "f", "strict": True,
                                            "parameters": {"type": "object", "properties": {"a": {"type": "string"}}}}}],
         None, "additionalProperties"),
        ([{"type": "function", "function": {"name": "f", "parameters": {"type": "string"}}}], None, "root type"),
    ]:
        with pytest.raises(ToolError, match=msg):
            tool_config(tools, choice)


def test_envelope_schema_constrains_and_parses():
    cfg = tool_config(WEATHER)
    schema = envelope_schema(cfg)
    validate_supported_json_schema(schema)
    calls = '{"type": "function_calls", "calls": [{"name": "get_weather", "arguments": {"city": "Oslo"}}]}'
    assert accepts(schema, calls) == (True, True)
    assert accepts(schema, '{"type": "message", "content": "hi"}') == (True, True)
    assert not accepts(schema, '{"type": "function_calls", "calls": [{"name": "rm_rf"')[0]
    p = parse_tool_output(calls, cfg)
    assert p.is_calls and p.calls == [("get_weather", '{"city":"Oslo"}')]
    tc = tool_calls_json("chatcmpl-abc", p, with_index=True)
    assert tc[0]["id"] == "call_abc_0" and tc[0]["index"] == 0 and tc[0]["function"]["name"] == "get_weather"
    assert parse_tool_output('{"type": "message", "content": "hi"}', cfg).message == "hi"
    req = tool_config(WEATHER, "required")
    with pytest.raises(ToolError, match="requires a function call"):
        parse_tool_output('{"type": "message", "content": "hi"}', req)
    with pytest.raises(ToolError, match="do not satisfy"):
        parse_tool_output('{"type": "function_calls", "calls": [{"name": "get_weather", "arguments": {}}]}', cfg)
    single = tool_config(WEATHER, parallel_tool_calls=False)
    two = ('{"type": "function_calls", "calls": [{"name": "get_weather", "arguments": {"city": "a"}},'
           ' {"name": "get_weather", "arguments": {"city": "b"}}]}')
    assert len(parse_tool_output(two, cfg).calls) == 2
    with pytest.raises(ToolError, match="between 1 and 1"):
        parse_tool_output(two, single)


def test_responses_flat_tools_bridge():
    cfg, echoed, choice = responses_tool_config([{"type": "function", "name": "get_weather",
                                                  "parameters": WEATHER[0]["function"]["parameters"]}])
    assert cfg.choice == "auto" and echoed[0]["type"] == "function" and choice == "auto"
    assert responses_tool_config(None) == (None, [], "none")
    with pytest.raises(ToolError):
        responses_tool_config([{"type": "web_search"}])


def test_tool_history_validation():
    call = {"id": "call_1", "type": "function", "function": {"name": "get_weather", "arguments": '{"city":"Oslo"}'}}
    msgs = [{"role": "user", "content": "weather?"}, {"role": "assistant", "content": None, "tool_calls": [call]},
            {"role": "tool", "tool_call_id": "call_1", "content": "sunny"}]
    out = normalize_tool_history(msgs)
    assert out[1]["role"] == "assistant" and "get_weather" in out[1]["content"]
    assert out[2]["role"] == "user" and "untrusted" in out[2]["content"] and "sunny" in out[2]["content"]
    for bad, msg in [
        (msgs[:2], "matching tool result"),
        (msgs[:2] + [{"role": "user", "content": "x"}], "before all preceding"),
        (msgs[:2] + [{"role": "tool", "tool_call_id": "call_9", "content": "x"}], "unknown"),
        (msgs[:2] + [{"role": "tool", "tool_call_id": "call_1", "name": "other", "content": "x"}], "does not match"),
        ([msgs[0], {"role": "assistant", "tool_calls": [dict(call, function={"name": "f", "arguments": "[1]"})]}],
         "JSON object"),
    ]:
        with pytest.raises(ToolError, match=msg):
            normalize_tool_history(bad)
