"""Hardware detection and capability levels.

Reads (never changes) the machine: CPU architecture / cores / SIMD flags /
NUMA nodes from /proc and /sys, GPUs through NVML (name, compute capability,
memory, SM count, clocks, power limit, NVLink peers) and classifies the host
into a capability level that picks default serving knobs (tensor-parallel
degree, weight format, batch sizes).

Reference: detect_hardware / HardwareClassifier / InferenceStrategy
(openmini-server/src/hardware/detector.rs, profile.rs:7-82, scheduler.rs).
Only NVML *queries* are issued here: no clock, power or mode is set.
"""
from __future__ import annotations

import os
import platform
from dataclasses import asdict, dataclass, field


@dataclass
class CpuInfo:
    arch: str
    cores_logical: int
    cores_physical: int
    model: str = ""
    flags: list = field(default_factory=list)
    numa_nodes: int = 1


@dataclass
class GpuInfo:
    index: int
    name: str
    compute_capability: tuple
    memory_bytes: int
    sm_count: int = 0
    max_sm_clock_mhz: int = 0
    power_limit_w: float = 0.0
    nvlink_active: int = 0


@dataclass
class HardwareProfile:
    cpu: CpuInfo
    gpus: list
    memory_bytes: int
    level: str
    strategy: dict

    def to_dict(self):
        return asdict(self)


def _cpu() -> CpuInfo:
    arch = platform.machine() or "unknown"
    model, flags, phys = "", [], set()
    try:
        with open("/proc/cpuinfo") as f:
            cur = {}
            for line in f:
                if ":" not in line:
                    if "physical id" in cur and "core id" in cur:
                        phys.add((cur["physical id"], cur["core id"]))
                    cur = {}
                    continue
                k, v = (s.strip() for s in line.split(":", 1))
                cur[k] = v
                if k == "model name" and not model:
                    model = v
                if k in ("flags", "Features") and not flags:
                    flags = v.split()
    except OSError:
        pass
    simd = [f for f in flags if f in ("sse4_2", "avx", "avx2", "avx512f", "avx512bw", "avx512_bf16", "amx_bf16",
                                      "fma", "asimd", "sve", "sve2")]
    numa = 1
    try:
        numa = max(1, len([d for d in os.listdir("/sys/devices/system/node") if d.startswith("node")]))
    except OSError:
        pass
    logical = os.cpu_count() or 1
    return CpuInfo(arch, logical, len(phys) or logical, model, simd, numa)


def _mem() -> int:
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def _gpus(nvml=None) -> list:
    if nvml is None:
        try:
            import pynvml as nvml  # nvidia_ml_py
        except ImportError:
            return []
    try:
        nvml.nvmlInit()
    except Exception:
        return []
    out = []
    try:
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            name = nvml.nvmlDeviceGetName(h)
            name = name.decode() if isinstance(name, bytes) else name
            try:
                cc = tuple(nvml.nvmlDeviceGetCudaComputeCapability(h))
            except Exception:
                cc = (0, 0)
            mem = nvml.nvmlDeviceGetMemoryInfo(h).total
            try:
                sm = nvml.nvmlDeviceGetNumGpuCores(h) // 128
            except Exception:
                sm = 0
            try:
                clk = nvml.nvmlDeviceGetMaxClockInfo(h, nvml.NVML_CLOCK_SM)
            except Exception:
                clk = 0
            try:
                pw = nvml.nvmlDeviceGetEnforcedPowerLimit(h) / 1000.0
            except Exception:
                pw = 0.0
            links = 0
            for l in range(18):
                try:
                    if nvml.nvmlDeviceGetNvLinkState(h, l):
                        links += 1
                except Exception:
                    break
            out.append(GpuInfo(i, name, cc, int(mem), sm, int(clk), pw, links))
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass
    return out


def classify(cpu: CpuInfo, gpus: list, mem: int) -> tuple:
    """Capability level and default serving strategy."""
    bw = [g for g in gpus if tuple(g.compute_capability) >= (10, 0)]
    if len(bw) >= 8 and all(g.nvlink_active >= 1 for g in bw):
        level = "blackwell_nvswitch"
        strat = {"tp": 8, "weight_format": "q4", "max_num_seqs": 256, "tp_transport": "symm"}
    elif bw:
        level = "blackwell"
        strat = {"tp": len(bw), "weight_format": "q4", "max_num_seqs": 32 * len(bw), "tp_transport": "symm"}
    elif gpus:
        level = "gpu_other"
        strat = {"tp": 1, "weight_format": "bf16", "max_num_seqs": 16, "note": "kernels target sm_100a only"}
    else:
        level = "cpu_only"
        strat = {"tp": 1, "weight_format": "bf16", "max_num_seqs": 4, "device": "cpu"}
    return level, strat


def detect_hardware(nvml=None) -> HardwareProfile:
    cpu, mem = _cpu(), _mem()
    gpus = _gpus(nvml)
    level, strat = classify(cpu, gpus, mem)
    return HardwareProfile(cpu, gpus, mem, level, strat)
