"""Tensor / expert parallel plumbing (communicator, fused NVLink collectives).

The fused collectives never use an NVLink multicast object; the switch that
keeps torch's symmetric memory from creating one is set on import, before
any symmetric buffer exists.
"""
import os as _os

_os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
