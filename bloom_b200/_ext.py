"""Loader for the in-tree native extensions.

`cuda()` returns bloom_b200._C (sm_100a kernels), or bloom_b200._C_checked
(the same kernels built with index checks) when BLOOM_KERNEL_CHECKS=1.  On a machine with a GPU a
missing or broken extension is an error, never a silent fallback: the engine
only runs on its own kernels.  `runtime()` returns bloom_b200._runtime (host
C++ runtime), which imports without a GPU.
"""
from __future__ import annotations

import importlib

_cache: dict = {}


class ExtensionMissing(RuntimeError):
    pass


def _load(name: str):
    if name in _cache:
        return _cache[name]
    import torch  # noqa: F401  (loads libc10/libtorch that the extensions link against)

    try:
        mod = importlib.import_module(f"bloom_b200.{name}")
    except ImportError as e:  # pragma: no cover - depends on the build state
        raise ExtensionMissing(
            f"bloom_b200.{name} is not built ({e}); run `python setup.py build_ext --inplace` "
            "or `python -c 'import __graft_entry__ as g; g.build()'`"
        ) from e
    _cache[name] = mod
    return mod


def cuda():
    import os

    return _load("_C_checked" if os.environ.get("BLOOM_KERNEL_CHECKS", "0") == "1" else "_C")


def runtime():
    return _load("_runtime")


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False
