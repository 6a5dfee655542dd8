"""Memory telemetry: process RSS, peak RAM, system RAM and per-GPU VRAM.

`MemoryTelemetry.snapshot(devices)` reads /proc/self/status (VmRSS, VmHWM),
/proc/meminfo (MemTotal, MemAvailable) and, for each CUDA device, the driver's
free/total bytes plus the caching allocator's peak; peaks are tracked across
calls for the life of the process.  Used by /metrics, /v1/observability and
the memory-pressure check (either side above 85 %).  Reference:
MemoryTelemetry (crates/engine/src/core/telemetry.rs:13-105).
"""
from __future__ import annotations

import threading
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

HIGH_PRESSURE = 0.85


def _proc_kib(path: str, keys) -> Dict[str, int]:
    out: Dict[str, int] = {}
    try:
        with open(path) as f:
            for line in f:
                name, _, rest = line.partition(":")
                if name in keys:
                    out[name] = int(rest.split()[0]) * 1024
    except OSError:
        pass
    return out


@dataclass
class DeviceMemory:
    index: int
    name: str
    total_bytes: int
    used_bytes: int
    peak_bytes: int
    allocator_peak_bytes: int

    @property
    def utilization(self) -> float:
        return self.used_bytes / self.total_bytes if self.total_bytes else 0.0


@dataclass
class MemorySnapshot:
    rss_bytes: int = 0
    peak_rss_bytes: int = 0
    total_ram_bytes: int = 0
    available_ram_bytes: int = 0
    devices: List[DeviceMemory] = field(default_factory=list)

    @property
    def ram_utilization(self) -> float:
        used = self.total_ram_bytes - self.available_ram_bytes
        return used / self.total_ram_bytes if self.total_ram_bytes else 0.0

    @property
    def high_pressure(self) -> bool:
        return self.ram_utilization > HIGH_PRESSURE or any(d.utilization > HIGH_PRESSURE for d in self.devices)

    def to_dict(self) -> dict:
        d = asdict(self)
        d["ram_utilization"] = round(self.ram_utilization, 4)
        d["high_pressure"] = self.high_pressure
        for dev, src in zip(d["devices"], self.devices):
            dev["utilization"] = round(src.utilization, 4)
        return d

    def summary(self) -> str:
        def gb(x):
            return f"{x / 2**30:.1f} GiB"

        parts = [f"RAM rss {gb(self.rss_bytes)} (peak {gb(self.peak_rss_bytes)}) of {gb(self.total_ram_bytes)}"]
        for dv in self.devices:
            parts.append(f"GPU{dv.index} {dv.name}: {gb(dv.used_bytes)}/{gb(dv.total_bytes)} "
                         f"({100 * dv.utilization:.1f}%, peak {gb(dv.peak_bytes)})")
        return "; ".join(parts)


class MemoryTelemetry:
    _lock = threading.Lock()
    _peak_rss = 0
    _peak_dev: Dict[int, int] = {}

    @classmethod
    def snapshot(cls, devices: Optional[List[int]] = None) -> MemorySnapshot:
        st = _proc_kib("/proc/self/status", ("VmRSS", "VmHWM"))
        mi = _proc_kib("/proc/meminfo", ("MemTotal", "MemAvailable"))
        snap = MemorySnapshot(rss_bytes=st.get("VmRSS", 0), total_ram_bytes=mi.get("MemTotal", 0),
                              available_ram_bytes=mi.get("MemAvailable", 0))
        with cls._lock:
            cls._peak_rss = max(cls._peak_rss, snap.rss_bytes, st.get("VmHWM", 0))
            snap.peak_rss_bytes = cls._peak_rss
        try:
            import torch

            if torch.cuda.is_available():
                idx = devices if devices is not None else list(range(torch.cuda.device_count()))
                for i in idx:
                    free, total = torch.cuda.mem_get_info(i)
                    used = total - free
                    with cls._lock:
                        cls._peak_dev[i] = max(cls._peak_dev.get(i, 0), used)
                        peak = cls._peak_dev[i]
                    snap.devices.append(DeviceMemory(i, torch.cuda.get_device_name(i), int(total), int(used),
                                                     int(peak), int(torch.cuda.max_memory_reserved(i))))
        except Exception:  # pragma: no cover - driver query failures leave the device list empty
            pass
        return snap
