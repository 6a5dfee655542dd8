"""Read-only topology probe: devices, SMs, HBM, peer access matrix, NVLink
multicast (NVLS) support, NCCL version, and the measured roofline peaks.

    python -m bloom_b200.utils.probe_gpu [--peaks MEASURED_PEAKS.json]

Only queries attributes; it sets no clock, power, persistence or other
device setting.  Multicast support is read with cuDeviceGetAttribute
(CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED) from the driver library.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
from typing import Dict, List, Optional

import torch

_CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED = 132


def _driver():
    for name in ("libcuda.so.1", "libcuda.so"):
        try:
            return ctypes.CDLL(name)
        except OSError:
            continue
    return None


def multicast_supported(dev: int) -> Optional[bool]:
    lib = _driver()
    if lib is None:
        return None
    try:
        if lib.cuInit(0) != 0:
            return None
        h = ctypes.c_int()
        if lib.cuDeviceGet(ctypes.byref(h), dev) != 0:
            return None
        v = ctypes.c_int()
        if lib.cuDeviceGetAttribute(ctypes.byref(v), _CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, h) != 0:
            return None
        return bool(v.value)
    except (AttributeError, OSError):
        return None


def nvml_info(dev: int) -> Dict[str, object]:
    """Clocks and power as read from NVML (read-only)."""
    try:
        import pynvml

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(dev)
        d = {"sm_clock_mhz": pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
             "sm_clock_max_mhz": pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM),
             "mem_clock_max_mhz": pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_MEM),
             "power_limit_w": pynvml.nvmlDeviceGetEnforcedPowerLimit(h) / 1000.0}
        try:
            links = 0
            for l in range(18):
                try:
                    if pynvml.nvmlDeviceGetNvLinkState(h, l) == pynvml.NVML_FEATURE_ENABLED:
                        links += 1
                except pynvml.NVMLError:
                    break
            d["nvlink_links_up"] = links
        except Exception:  # noqa: BLE001 - NVLink queries are optional
            pass
        return d
    except Exception as e:  # noqa: BLE001
        return {"nvml_error": str(e)}


def probe(peaks_path: Optional[str] = None) -> Dict[str, object]:
    out: Dict[str, object] = {"object": "bloom.gpu_probe", "torch": torch.__version__,
                              "cuda_runtime": torch.version.cuda, "cuda_available": torch.cuda.is_available()}
    try:
        out["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception:  # noqa: BLE001
        out["nccl"] = None
    devices: List[Dict[str, object]] = []
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        d = {"index": i, "name": p.name, "compute_capability": f"{p.major}.{p.minor}",
             "sm_count": p.multi_processor_count, "hbm_bytes": p.total_memory,
             "l2_bytes": getattr(p, "L2_cache_size", None), "is_sm100": (p.major, p.minor) == (10, 0),
             "multicast_supported": multicast_supported(i)}
        d.update(nvml_info(i))
        devices.append(d)
    out["devices"] = devices
    out["peer_access"] = [[(i == j) or torch.cuda.can_device_access_peer(i, j) for j in range(n)] for i in range(n)]
    out["all_pairs_peer"] = all(all(r) for r in out["peer_access"]) if n else False
    out["nvls_candidate"] = n > 1 and all(d.get("multicast_supported") for d in devices)
    path = peaks_path or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                      "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            out["measured_peaks"] = json.load(f)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="probe_gpu")
    ap.add_argument("--peaks")
    args = ap.parse_args(argv)
    print(json.dumps(probe(args.peaks), indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
