"""Runtime tracing: NVTX ranges around engine phases and a per-kernel device-time
table collected with the PyTorch profiler (CUPTI activity records, which also
cover kernels replayed from CUDA graphs).

NVTX ranges cost a host call each, so they are off unless ``OPENMINI_NVTX=1`` is
set (or :func:`enable_nvtx` is called); an external profiler then shows the
engine's schedule / build / decode-graph / commit phases on its timeline.

Reference counterpart: the tracing / metrics spans of
openmini-server/src/monitoring/ (request spans and per-stage latency histograms);
here the spans are device-side ranges and the per-kernel table explains the
decode step's device time.
"""
from __future__ import annotations

import contextlib
import os
from collections import defaultdict

_NVTX = os.environ.get("OPENMINI_NVTX", "0") not in ("", "0", "false", "False")


def enable_nvtx(on: bool = True) -> None:
    global _NVTX
    _NVTX = on


@contextlib.contextmanager
def nvtx_range(name: str):
    """NVTX push / pop around a host-side phase (no-op unless enabled or without CUDA)."""
    if not _NVTX:
        yield
        return
    import torch
    if not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def _device_events(prof):
    import torch
    return [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


def _dur(e) -> float:
    d = getattr(e, "device_time", None)
    return float(d if d is not None else e.cuda_time)


def kernel_table(fn, iters: int = 1, top: int = 25):
    """Run ``fn`` ``iters`` times under the profiler and aggregate the device kernels:
    [(name, launches, total_us, share)] sorted by total device time, plus the sum.

    Times come from the profiler's activity records: use them for shares, not as
    benchmark numbers."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(iters):
            fn()
        torch.cuda.synchronize()
    agg = defaultdict(lambda: [0, 0.0])
    for ev in _device_events(prof):
        key = ev.name or "?"
        if key.startswith(("Memcpy", "Memset")):
            key = key.split(" ")[0]
        agg[key][0] += 1
        agg[key][1] += _dur(ev)
    total = sum(v[1] for v in agg.values()) or 1.0
    rows = sorted(((k, v[0], v[1], v[1] / total) for k, v in agg.items()), key=lambda r: -r[2])
    return rows[:top], total


def kernel_sequence(fn):
    """Device kernels of one call of ``fn`` in launch order: [(name, device_us)]."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    evs = _device_events(prof)
    evs.sort(key=lambda e: e.time_range.start)
    return [(e.name, _dur(e)) for e in evs]


def by_position(seq, prefix: str, period: int):
    """Mean device time of the kernels whose name starts with ``prefix``, grouped by
    their occurrence index modulo ``period`` (e.g. the four GEMMs of a decoder layer)."""
    ds = [d for n, d in seq if n.startswith(prefix)]
    out = []
    for p in range(period):
        xs = ds[p::period]
        out.append((p, len(xs), sum(xs) / len(xs) if xs else 0.0))
    return out


def format_table(rows, total_us: float, per: int = 1, title: str = "") -> str:
    """Markdown table of :func:`kernel_table` rows; ``per`` divides counts and times
    (e.g. per decode step)."""
    out = [title] if title else []
    out.append("| kernel | launches/step | us/step | share |")
    out.append("|---|---|---|---|")
    for name, n, us, share in rows:
        short = name if len(name) <= 90 else name[:87] + "..."
        out.append(f"| `{short}` | {n / per:.1f} | {us / per:.1f} | {share:.3f} |")
    out.append(f"| total | | {total_us / per:.1f} | 1.000 |")
    return "\n".join(out)
