"""inspect_gguf: print a GGUF file's header, metadata and tensor table.

    python -m bloom_b200.cli.inspect_gguf [--json] [--limit N] model.gguf

Flags follow the reference tool (crates/engine/src/bin/inspect_gguf.rs);
parsing is bloom_b200.formats.gguf (the C++ reader validates the header).
"""
from __future__ import annotations

import argparse
import json
import sys


def summarise(path: str, limit: int = 20) -> dict:
    from ..formats.gguf import GGUFFile

    g = GGUFFile(path)
    md = {}
    for k, v in g.metadata.items():
        if isinstance(v, list) and len(v) > 16:
            md[k] = {"type": "array", "len": len(v), "head": v[:8]}
        else:
            md[k] = v
    tensors = [{"name": n, "type": t.type_name, "shape": list(t.shape), "bytes": t.n_bytes}
               for n, t in list(g.tensors.items())[:limit if limit > 0 else None]]
    return {"path": path, "version": g.version, "architecture": g.arch, "tensor_count": len(g.tensors),
            "metadata_count": len(g.metadata), "primary_dtype": g.primary_dtype(),
            "total_tensor_bytes": sum(t.n_bytes for t in g.tensors.values()), "metadata": md, "tensors": tensors}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="inspect_gguf")
    ap.add_argument("path")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--limit", type=int, default=20, help="tensors to list (0 = all)")
    a = ap.parse_args(argv)
    try:
        s = summarise(a.path, a.limit)
    except Exception as e:  # noqa: BLE001
        print(f"error: {e}", file=sys.stderr)
        return 1
    if a.json:
        print(json.dumps(s, indent=2, default=str))
        return 0
    print(f"GGUF v{s['version']}  arch={s['architecture']}  tensors={s['tensor_count']}  "
          f"metadata={s['metadata_count']}  primary={s['primary_dtype']}  bytes={s['total_tensor_bytes']}")
    for k, v in s["metadata"].items():
        print(f"  {k} = {v if not isinstance(v, dict) else '[array of ' + str(v['len']) + ']'}")
    for t in s["tensors"]:
        print(f"  {t['name']:48s} {t['type']:6s} {t['shape']}")
    if s["tensor_count"] > len(s["tensors"]):
        print(f"  ... {s['tensor_count'] - len(s['tensors'])} more")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
