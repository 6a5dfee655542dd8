"""CPU tests: GGUF / safetensors / manifest formats, chat templates, text
utilities, JSON recogniser, engine registry, CPU decoder vs the fp32 oracle."""
import json
import os

import pytest
import torch

from bloom_b200.models.config import preset
from bloom_b200.models.reference import random_weights


# ---------------------------------------------------------------- GGUF
@pytest.fixture(scope="module")
def tiny_gguf(tmp_path_factory):
    from bloom_b200.formats.gguf import GGML_Q8_0, write_decoder_gguf

    cfg = preset("tiny-llama")
    w = random_weights(cfg, seed=0, std=0.08)
    p = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    write_decoder_gguf(p, cfg, w, GGML_Q8_0)
    return cfg, w, p


def test_gguf_roundtrip_and_config(tiny_gguf):
    from bloom_b200.formats.gguf import GGUFFile, config_from_gguf, load_hf_weights

    cfg, w, p = tiny_gguf
    g = GGUFFile(p)
    assert g.version == 3 and g.arch == "llama" and g.primary_dtype() == "Q8_0"
    c2 = config_from_gguf(g)
    for k in ("hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim", "intermediate_size"):
        assert getattr(c2, k) == getattr(cfg, k)
    w2 = load_hf_weights(g)
    for k, v in w.items():
        if v.dim() == 2:
            err = ((w2[k].float() - v.float()).norm() / v.float().norm()).item()
            assert err < 0.01, (k, err)  # Q8_0 rounding only; RoPE permutation undone exactly


def test_gguf_q4_0_blocks():
    from bloom_b200._ext import runtime

    x = torch.randn(4096) * 0.1
    raw = runtime().quantize_q4_0(x)
    assert raw.numel() == 4096 // 32 * 18
    y = runtime().dequant_q4_0(raw, 4096)
    assert ((y - x).norm() / x.norm()).item() < 0.12


def test_q8_0_matmul_matches_float():
    from bloom_b200._ext import runtime

    rt = runtime()
    w = torch.randn(96, 256) * 0.05
    x = torch.randn(3, 256)
    y = rt.q8_0_matmul(x, rt.quantize_q8_0(w), 96, 256)
    ref = x @ w.t()
    assert ((y - ref).norm() / ref.norm()).item() < 0.02


def test_bad_gguf_rejected(tmp_path):
    from bloom_b200.formats.gguf import GGUFFile

    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(Exception):
        GGUFFile(str(p))


# ---------------------------------------------------------------- safetensors + manifest
def test_safetensors_single_and_sharded(tmp_path):
    from bloom_b200.formats.safetensors_io import (SafetensorsError, load_state_dict, resolve_shards, save_file,
                                                    save_sharded)

    t = {"a": torch.randn(4, 8).to(torch.bfloat16), "b": torch.arange(10, dtype=torch.int64)}
    d1 = tmp_path / "single"
    d1.mkdir()
    save_file(t, str(d1 / "model.safetensors"))
    sd = load_state_dict(str(d1))
    assert torch.equal(sd["a"], t["a"]) and torch.equal(sd["b"], t["b"])
    d2 = tmp_path / "sharded"
    d2.mkdir()
    names = save_sharded({f"w{i}": torch.randn(64, 64) for i in range(6)}, str(d2), 40_000)
    assert len(names) > 1 and len(resolve_shards(str(d2))) == len(names)
    os.remove(d2 / names[0])
    with pytest.raises(SafetensorsError):
        resolve_shards(str(d2))


def test_safetensors_header_validation(tmp_path):
    import struct

    from bloom_b200.formats.safetensors_io import SafetensorsError, read_header

    hdr = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 32]}}).encode()
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 16)
    with pytest.raises(SafetensorsError):
        read_header(str(p))


def test_manifest_paths(tiny_gguf, tmp_path):
    from bloom_b200.formats.manifest import ManifestError, estimate_memory, load_manifest, manifest_from_dict
    from bloom_b200.formats.safetensors_io import save_file
    from bloom_b200.models.config import to_hf_config

    cfg, w, p = tiny_gguf
    m = load_manifest(p)
    assert m.family == "Llama" and m.primary_dtype == "Q8" and m.files[0].format == "Gguf"
    hf = tmp_path / "hf"
    hf.mkdir()
    save_file(w, str(hf / "model.safetensors"))
    (hf / "config.json").write_text(json.dumps(to_hf_config(cfg)))
    (hf / "tokenizer.json").write_text("{}")
    m2 = load_manifest(str(hf))
    assert m2.primary_dtype == "BF16" and m2.parameters["num_hidden_layers"] == cfg.num_layers
    (hf / "bloom.json").write_text(m2.to_json())
    m3 = load_manifest(str(hf))
    assert m3.id == m2.id
    with pytest.raises(ManifestError):
        manifest_from_dict({"id": "x"})
    est = estimate_memory(m2, 4096, concurrent_seqs=8, tp=2)
    assert est.kv_bytes_per_token == 2 * cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * 2
    assert est.fits


def test_llama3_8b_memory_estimate_for_b200():
    from bloom_b200.formats.manifest import ModelManifest, estimate_memory

    c = preset("llama3-8b")
    man = ModelManifest(id="l8", family="Llama", version="1", io_schema={"inputs": ["Text"], "outputs": ["Text"]},
                        memory_profile={}, primary_dtype="BF16",
                        parameters={"num_hidden_layers": 32, "hidden_size": 4096, "intermediate_size": 14336,
                                    "vocab_size": 128256, "num_key_value_heads": 8, "head_dim": 128})
    e1 = estimate_memory(man, 2304, concurrent_seqs=256, tp=1)
    e8 = estimate_memory(man, 2304, concurrent_seqs=256, tp=8)
    assert e1.kv_bytes_per_token == 128 * 1024  # 128 KiB per token across layers
    assert e1.fits and e8.per_gpu_bytes < e1.per_gpu_bytes / 4


# ---------------------------------------------------------------- templates / text
def test_chat_templates():
    from bloom_b200.engine.chat_template import classify_template, render, select_template

    msgs = [{"role": "system", "content": "S"}, {"role": "user", "content": "U"}]
    assert render(msgs, "chatml") == "<|im_start|>system\nS<|im_end|>\n<|im_start|>user\nU<|im_end|>\n<|im_start|>assistant\n"
    assert render(msgs, "llama3").startswith("<|begin_of_text|><|start_header_id|>system<|end_header_id|>\n\nS<|eot_id|>")
    assert render(msgs, "llama2") == "<s>[INST] <<SYS>>\nS\n<</SYS>>\n\nU [/INST]"
    assert render([{"role": "user", "content": "U"}], "smollm2").startswith("<|im_start|>system\nYou are a helpful AI")
    assert render(msgs, "qwen3-no-think").endswith("<think>\n\n</think>\n\n")
    assert render(msgs, "gemma").endswith("<start_of_turn>model\n")
    assert classify_template("{{'<|start_header_id|>'}}") == "llama3"
    assert classify_template("<|im_start|>") == "chatml"
    assert select_template("qwen", "qwen3") == "qwen3-no-think"


def test_stop_filter_holds_partial_matches():
    from bloom_b200.engine.text import StopSequenceFilter

    f = StopSequenceFilter(["END"])
    out = []
    for d in ["ab", "cE", "N", "Dxyz"]:
        o, stopped = f.push(d)
        out.append(o)
        if stopped:
            break
    assert "".join(out) == "abc" and stopped
    f2 = StopSequenceFilter(["END"])
    assert f2.push("xE")[0] == "x"
    assert f2.push("y")[0] == "Ey"


def test_detokenizer_incremental_utf8():
    from bloom_b200.engine.text import Detokenizer, Tokenizer

    tok = Tokenizer(None)
    d = Detokenizer(tok)
    s = "héllo ☃ world"
    out = "".join(d.add(t) for t in tok.encode(s))
    assert out == s


def test_json_recogniser_and_repair():
    from bloom_b200._ext import runtime
    from bloom_b200.engine.structured import repair_json

    rt = runtime()
    d = rt.JsonDfa()
    assert d.feed('{"a": [1, 2.5e3, true, null, "x\\u00e9"], ')
    assert not d.can_feed("}")  # a key must follow the comma
    assert d.feed('"b": {}}')
    assert d.complete()
    assert not rt.JsonDfa().feed("{'a': 1}")
    assert not rt.JsonDfa().feed('{"a": 01}')
    assert rt.is_valid_json('[1, {"k": "v"}]')
    d2 = rt.JsonDfa()
    assert d2.pick([5, 6], ['"', "{", "", "", "", "x", "{"], [7]) == 6
    assert json.loads(repair_json('{"a": [1, 2, {"b": "hel')) == {"a": [1, 2, {"b": "hel"}]}
    assert repair_json('{"ok": 1}') == '{"ok": 1}'


def test_registry_routing():
    from bloom_b200.engine.registry import FALLBACK, NATIVE, UNSUPPORTED, default_registry

    r = default_registry()
    assert r.route("Llama", "Safetensors", "BF16", "gpu") == ("b200", NATIVE)
    assert r.route("Llama", "Gguf", "Q8", "gpu") == ("b200", NATIVE)  # block-quantised GPU kernels
    assert r.route("Llama", "Safetensors", "F32", "gpu") == ("b200", FALLBACK)
    assert r.route("Llama", "Gguf", "Q8", "cpu") == ("cpu", NATIVE)
    assert r.route("Whisper", "Gguf", "Q8", "cpu")[1] == UNSUPPORTED
    assert r.route("Gemma", "Safetensors", "BF16", "gpu") == ("b200", NATIVE)
    assert r.route("Wan", "Preset", "BF16", "gpu") == ("wan", NATIVE)
    assert any(e["name"] == "b200" and e["max_tp"] == 8 for e in r.describe())


def test_gemma4_config_from_hf_and_layer_geometry():
    from bloom_b200.models import build_decoder
    from bloom_b200.models.config import from_hf_config

    hf = {"model_type": "gemma4", "eos_token_id": [1, 106],
          "text_config": {"hidden_size": 2560, "num_hidden_layers": 12, "num_attention_heads": 8,
                          "num_key_value_heads": 4, "head_dim": 256, "global_head_dim": 512,
                          "num_global_key_value_heads": 1, "intermediate_size": 10240, "vocab_size": 262144,
                          "sliding_window": 512, "attention_k_eq_v": True, "final_logit_softcapping": 30.0,
                          "rope_parameters": {"full_attention": {"rope_theta": 1e6, "partial_rotary_factor": 0.25},
                                              "sliding_attention": {"rope_theta": 1e4}}}}
    c = from_hf_config(hf)
    assert c.arch == "gemma4" and c.tie_word_embeddings and c.eos_token_ids == [1, 106]
    assert [c.is_sliding(i) for i in range(12)] == [True] * 5 + [False] + [True] * 5 + [False]
    assert c.layer_attn(0) == (256, 4) and c.layer_attn(5) == (512, 1)
    assert c.partial_rotary_factor == 0.25 and c.rope_local_theta == 1e4 and c.sliding_window == 512
    # every layer's KV slot is sized for the widest layer: max(2*4*256, 2*1*512) per token and layer
    assert c.kv_bytes_per_token() == 2 * 12 * 1024 * 2
    with pytest.raises(ValueError):
        from bloom_b200.models.llama import TPInfo

        build_decoder(c, TPInfo(rank=0, size=2), "cpu")


def test_gemma4_oracle_window_and_softcap():
    """The fp32 oracle: a window wider than the sequence is plain causal
    attention, a narrower one changes late positions only; soft-capping
    bounds the logits."""
    import dataclasses

    from bloom_b200.models.config import preset
    from bloom_b200.models.reference import gemma4_forward_logits, gemma4_random_weights

    cfg = preset("tiny-gemma4")
    w = gemma4_random_weights(cfg, seed=1, std=0.08)
    toks = list(range(3, 43))
    wide = gemma4_forward_logits(dataclasses.replace(cfg, sliding_window=1000), w, toks)
    full = gemma4_forward_logits(dataclasses.replace(cfg, sliding_window=len(toks)), w, toks)
    assert torch.allclose(wide, full, atol=1e-4)
    narrow = gemma4_forward_logits(cfg, w, toks)  # window 24
    assert torch.allclose(narrow[:24], full[:24], atol=1e-4)
    assert not torch.allclose(narrow[30:], full[30:], atol=1e-3)
    assert narrow.abs().max().item() <= cfg.final_logit_softcapping + 1e-4


# ---------------------------------------------------------------- CPU engine
def test_cpu_decoder_matches_oracle_on_gguf(tiny_gguf):
    from bloom_b200.engine.cpu_engine import CpuDecoder
    from bloom_b200.formats.gguf import GGUFFile, load_hf_weights
    from bloom_b200.models.reference import forward_logits

    cfg, w, p = tiny_gguf
    dec = CpuDecoder.from_gguf(p)
    prompt = [5, 17, 99, 3, 250]
    toks = list(dec.generate(prompt, 8, temperature=0.0, ignore_eos=True))
    assert len(toks) == 8
    wq = load_hf_weights(GGUFFile(p), dtype=torch.float32)
    logits = forward_logits(cfg, wq, prompt + toks)
    for j, t in enumerate(toks):
        row = logits[len(prompt) - 1 + j]
        assert (row.max() - row[t]).item() <= 0.05 * (row.max() - row.median()).item() + 1e-3


def test_cli_inspect_and_echo_pipeline(tiny_gguf, capsys):
    from bloom_b200.cli.infer import main
    from bloom_b200.engine.engine import SamplingParams
    from bloom_b200.engine.pipeline import InferencePipeline

    cfg, w, p = tiny_gguf
    assert main(["--model", p, "--inspect"]) == 0
    out = json.loads(capsys.readouterr().out)
    for k in ("model_path", "selected_engine", "selected_engine_maturity", "context_size", "manifest",
              "memory_estimate", "engines", "notes"):
        assert k in out
    pipe = InferencePipeline.load("echo")
    assert pipe.run("hello", SamplingParams(max_tokens=10)) == "echo: hello"


def test_cli_cpu_generation(tiny_gguf, capsys):
    from bloom_b200.cli.infer import main

    cfg, w, p = tiny_gguf
    rc = main(["--model", p, "--device", "cpu", "--prompt", "hi", "--max-tokens", "4", "--temperature", "0",
               "--raw", "--quiet"])
    assert rc == 0


def test_inspect_gguf_cli(tiny_gguf, capsys):
    from bloom_b200.cli.inspect_gguf import main

    cfg, w, p = tiny_gguf
    assert main([p, "--json", "--limit", "3"]) == 0
    d = json.loads(capsys.readouterr().out)
    assert d["architecture"] == "llama" and d["version"] == 3 and len(d["tensors"]) == 3
    assert d["tensor_count"] > 3 and d["primary_dtype"] == "Q8_0"
    assert main([p]) == 0 and "GGUF v3" in capsys.readouterr().out
    assert main([p + ".missing"]) == 1


def test_pipeline_layer_ranges():
    from bloom_b200.parallel.pipeline import layer_range

    assert [layer_range(32, s, 2) for s in range(2)] == [(0, 16), (16, 32)]
    assert [layer_range(10, s, 4) for s in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    assert layer_range(80, 7, 8) == (70, 80)
    with pytest.raises(ValueError):
        layer_range(2, 0, 3)


def test_gemma4_checkpoint_loads_through_the_manifest(tmp_path):
    """A Gemma4 safetensors package (HF config with text_config, weights under
    model.language_model.*) routes to the Gemma family and loads into
    Gemma4LM with per-layer geometry (host memory only, no forward)."""
    from bloom_b200.formats.loader import load_manifest, load_weights, model_config
    from bloom_b200.formats.safetensors_io import save_file
    from bloom_b200.models import build_decoder
    from bloom_b200.models.config import preset, to_hf_config
    from bloom_b200.models.reference import gemma4_random_weights

    cfg = preset("tiny-gemma4")
    hf = {"model_type": "gemma4", "eos_token_id": [1, 106], "text_config": {
        "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "global_head_dim": cfg.head_dim_global,
        "num_global_key_value_heads": cfg.num_kv_heads_global, "intermediate_size": cfg.intermediate_size,
        "vocab_size": cfg.vocab_size, "sliding_window": cfg.sliding_window, "attention_k_eq_v": True,
        "final_logit_softcapping": 30.0, "attn_logit_softcapping": 50.0, "max_position_embeddings": 1024,
        "rope_parameters": {"full_attention": {"rope_theta": 1e6, "partial_rotary_factor": 0.25},
                            "sliding_attention": {"rope_theta": 1e4}}}}
    d = tmp_path / "gemma4"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(hf))
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel

    Tokenizer(WordLevel({"<unk>": 0, "<eos>": 1, "a": 2}, unk_token="<unk>")).save(str(d / "tokenizer.json"))
    w = gemma4_random_weights(cfg, seed=0)
    save_file({k: v.contiguous() for k, v in w.items()}, str(d / "model.safetensors"))
    man = load_manifest(str(d))
    assert man.family == "Gemma"
    c2 = model_config(man)
    assert c2.arch == "gemma4" and c2.layer_attn(5) == (512, 1) and c2.attention_k_eq_v
    m = build_decoder(c2, None, "cpu")
    m.shard_full(load_weights(man))
    assert len(m.layers) == cfg.num_layers
    assert m.layers[0]["qkv"].shape == ((4 + 2 * 2) * 256, 256)      # sliding: q + k + v
    assert m.layers[5]["qkv"].shape == ((4 + 1) * 512, 256)          # global, k = v: q + k only
    assert m.kv_elems == 2 * 2 * 16 * 256 and m.cos_sin[(128, 512, False)].shape == (1024, 128)
