"""bloom_quantize: offline weight quantisation of safetensors models.

    python -m bloom_b200.cli.quantize -i model_dir_or_file -o out [-m rtn_int8|rtn_int4|awq_int4] [-g 128]

Every 2-D tensor whose name contains "weight" or "proj" is replaced by
<name>.qweight (u8), <name>.scales and, for int4, <name>.zeros (plus
<name>.col_scale for awq_int4); other tensors pass through.  Flags and output
names follow the reference CLI (crates/engine/src/bin/bloom_quantize.rs); the
quantisers are C++ (csrc/runtime/quantize.cpp).
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import torch


def quantize_state(sd, method: str, group: int, out_dtype=torch.float16):
    from .._ext import runtime

    rt = runtime()
    out = {}
    for name, t in sd.items():
        if t.dim() == 2 and ("weight" in name or "proj" in name) and "norm" not in name:
            if method == "rtn_int4" and t.shape[1] % group == 0:
                q, s, z = rt.quantize_rtn_int4(t, group)
                out.update({f"{name}.qweight": q, f"{name}.scales": s.to(out_dtype), f"{name}.zeros": z.to(out_dtype)})
            elif method == "awq_int4" and t.shape[1] % group == 0:
                q, s, z, c = rt.quantize_awq_int4(t, group)
                out.update({f"{name}.qweight": q, f"{name}.scales": s.to(out_dtype), f"{name}.zeros": z.to(out_dtype),
                            f"{name}.col_scale": c.to(torch.float32)})
            else:  # rtn_int8, and the fallback for shapes the group does not divide
                q, s = rt.quantize_rtn_int8(t)
                out.update({f"{name}.qweight": q, f"{name}.scales": s.to(out_dtype)})
        else:
            out[name] = t
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="bloom_quantize", description="Bloom offline model quantizer")
    ap.add_argument("-i", "--input", required=True)
    ap.add_argument("-o", "--output", required=True)
    ap.add_argument("-m", "--method", default="rtn_int8", choices=["rtn_int8", "rtn_int4", "awq_int4"])
    ap.add_argument("-g", "--group-size", type=int, default=128)
    a = ap.parse_args(argv)
    from ..formats.safetensors_io import load_file, save_file

    t0 = time.perf_counter()
    if os.path.isfile(a.input):
        files = [a.input]
    elif os.path.isdir(a.input):
        files = sorted(os.path.join(a.input, f) for f in os.listdir(a.input) if f.endswith(".safetensors"))
        if not files:
            print(f"error: no .safetensors files in {a.input}", file=sys.stderr)
            return 1
    else:
        print(f"error: input {a.input} does not exist", file=sys.stderr)
        return 1
    out_is_dir = len(files) > 1 or os.path.isdir(a.output) or a.output.endswith(os.sep)
    if out_is_dir:
        os.makedirs(a.output, exist_ok=True)
    for f in files:
        sd = load_file(f)
        q = quantize_state(sd, a.method, a.group_size)
        dst = os.path.join(a.output, os.path.basename(f)) if out_is_dir else a.output
        os.makedirs(os.path.dirname(os.path.abspath(dst)), exist_ok=True)
        save_file(q, dst)
        print(f"{os.path.basename(f)}: {sum(1 for k in q if k.endswith('.qweight'))} tensors quantised -> {dst}")
    print(f"quantization finished in {time.perf_counter() - t0:.2f} s")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
