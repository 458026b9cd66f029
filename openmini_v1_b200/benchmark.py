"""Serving benchmark framework: scenarios, latency metrics, exporters, regression check.

Counterpart of the reference's benchmark module (openmini-server/src/benchmark/
scenarios.rs:10-234 scenario catalogue, metrics.rs:19-200 percentiles and
TTFT/TPOT, runner.rs:93-210 runner, ci/regression.rs regression gate). Unlike
the reference runner, which sleeps instead of running inference, this runner
drives a real ``LLMEngine`` step by step: requests arrive on a schedule
(all at once, a steady rate, or bursts), the engine batches them continuously,
and per-request TTFT, TPOT and end-to-end latency are recorded from the
engine's own timestamps.

    python -m openmini_v1_b200.benchmark --scenario short --preset tiny --device cpu
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import math
import statistics
import time
from dataclasses import asdict, dataclass, field

import torch

from .engine.request import RequestStatus, SamplingParams


@dataclass
class Scenario:
    name: str
    num_requests: int
    prompt_len: tuple          # (min, max) tokens, uniform
    output_len: int
    arrival: str = "batch"     # "batch" | "rate" | "burst"
    rate_per_s: float = 0.0    # "rate": Poisson arrivals at this mean rate
    burst_size: int = 0        # "burst": groups of this many arriving together
    burst_gap_s: float = 0.0
    temperature: float = 0.0
    top_p: float = 1.0


SCENARIOS = {
    "short": Scenario("short", 16, (16, 64), 32),
    "medium": Scenario("medium", 16, (256, 512), 128),
    "long": Scenario("long", 8, (1024, 2048), 256),
    "ultra": Scenario("ultra", 4, (8192, 16384), 256),
    "multi_user": Scenario("multi_user", 64, (64, 256), 64, arrival="rate", rate_per_s=50.0,
                           temperature=0.7, top_p=0.9),
    "burst": Scenario("burst", 48, (32, 128), 32, arrival="burst", burst_size=16, burst_gap_s=0.05),
}


def percentile(xs, p: float) -> float:
    """Linear-interpolation percentile (p in [0, 100])."""
    if not xs:
        return float("nan")
    s = sorted(xs)
    k = (len(s) - 1) * p / 100.0
    lo, hi = math.floor(k), math.ceil(k)
    return s[lo] + (s[hi] - s[lo]) * (k - lo)


@dataclass
class LatencyStats:
    count: int = 0
    mean: float = 0.0
    p50: float = 0.0
    p95: float = 0.0
    p99: float = 0.0
    max: float = 0.0

    @staticmethod
    def of(xs) -> "LatencyStats":
        xs = [x for x in xs if x is not None and not math.isnan(x)]
        if not xs:
            return LatencyStats()
        return LatencyStats(len(xs), statistics.fmean(xs), percentile(xs, 50), percentile(xs, 95),
                            percentile(xs, 99), max(xs))


@dataclass
class BenchResult:
    scenario: str
    requests: int
    completed: int
    duration_s: float
    output_tokens: int
    prompt_tokens: int
    throughput_tok_s: float
    requests_per_s: float
    ttft_ms: LatencyStats = field(default_factory=LatencyStats)
    tpot_ms: LatencyStats = field(default_factory=LatencyStats)
    e2e_ms: LatencyStats = field(default_factory=LatencyStats)
    engine_stats: dict = field(default_factory=dict)

    def to_json(self) -> str:
        return json.dumps(asdict(self))

    def to_csv(self) -> str:
        flat = {"scenario": self.scenario, "requests": self.requests, "completed": self.completed,
                "duration_s": self.duration_s, "throughput_tok_s": self.throughput_tok_s,
                "requests_per_s": self.requests_per_s}
        for k in ("ttft_ms", "tpot_ms", "e2e_ms"):
            for m, v in asdict(getattr(self, k)).items():
                flat[f"{k}_{m}"] = v
        buf = io.StringIO()
        w = csv.DictWriter(buf, fieldnames=list(flat))
        w.writeheader()
        w.writerow(flat)
        return buf.getvalue()

    def to_prometheus(self) -> str:
        lines = [f'openmini_bench_throughput_tokens_per_second{{scenario="{self.scenario}"}} {self.throughput_tok_s}']
        for k in ("ttft_ms", "tpot_ms", "e2e_ms"):
            st = getattr(self, k)
            for q in ("p50", "p95", "p99"):
                lines.append(f'openmini_bench_{k}{{scenario="{self.scenario}",quantile="{q}"}} {getattr(st, q)}')
        return "\n".join(lines) + "\n"

    def to_text(self) -> str:
        """Human-readable report (the reference's HumanExporter, export.rs:190-265)."""
        rows = [f"scenario {self.scenario}: {self.completed}/{self.requests} requests in {self.duration_s:.2f} s",
                f"  throughput {self.throughput_tok_s:.1f} tok/s, {self.requests_per_s:.2f} req/s, "
                f"{self.prompt_tokens} prompt + {self.output_tokens} output tokens",
                f"  {'latency (ms)':<14}{'mean':>10}{'p50':>10}{'p95':>10}{'p99':>10}{'max':>10}"]
        for k, label in (("ttft_ms", "TTFT"), ("tpot_ms", "TPOT"), ("e2e_ms", "end to end")):
            st = getattr(self, k)
            rows.append(f"  {label:<14}" + "".join(f"{getattr(st, q):>10.2f}" for q in ("mean", "p50", "p95", "p99",
                                                                                   "max")))
        return "\n".join(rows) + "\n"

    def export_all(self, stem: str) -> list:
        """Write <stem>.json / .csv / .prom / .txt; returns the paths
        (the reference's export_all_formats, export.rs:284)."""
        out = []
        for ext, fn in (("json", self.to_json), ("csv", self.to_csv), ("prom", self.to_prometheus),
                        ("txt", self.to_text)):
            path = f"{stem}.{ext}"
            with open(path, "w") as f:
                f.write(fn())
            out.append(path)
        return out


def _arrivals(sc: Scenario, gen: torch.Generator) -> list:
    n = sc.num_requests
    if sc.arrival == "rate" and sc.rate_per_s > 0:
        gaps = torch.empty(n).exponential_(sc.rate_per_s, generator=gen).tolist()
        t, out = 0.0, []
        for g in gaps:
            out.append(t)
            t += g
        return out
    if sc.arrival == "burst" and sc.burst_size > 0:
        return [(i // sc.burst_size) * sc.burst_gap_s for i in range(n)]
    return [0.0] * n


def run_scenario(engine, sc: Scenario, vocab_size: int, seed: int = 0, max_wall_s: float = 3600.0) -> BenchResult:
    """Drive ``engine`` through ``sc``; arrival times are honoured against the wall clock."""
    gen = torch.Generator().manual_seed(seed)
    lens = torch.randint(sc.prompt_len[0], sc.prompt_len[1] + 1, (sc.num_requests,), generator=gen).tolist()
    prompts = [torch.randint(0, vocab_size, (L,), generator=gen).tolist() for L in lens]
    arrive = _arrivals(sc, gen)
    sp = SamplingParams(temperature=sc.temperature, top_p=sc.top_p, max_tokens=sc.output_len, ignore_eos=True,
                        seed=seed)
    pending = sorted(range(sc.num_requests), key=lambda i: arrive[i])
    reqs = {}
    t0 = time.monotonic()
    while (pending or engine.has_unfinished()) and time.monotonic() - t0 < max_wall_s:
        now = time.monotonic() - t0
        while pending and arrive[pending[0]] <= now:
            i = pending.pop(0)
            r = engine.add_request(f"bench-{sc.name}-{i}", prompts[i], sp)
            r.arrival = t0 + arrive[i]
            reqs[i] = r
        if engine.has_unfinished():
            engine.step()
        elif pending:
            time.sleep(max(0.0, min(0.01, arrive[pending[0]] - now)))
    dur = time.monotonic() - t0
    done = [r for r in reqs.values() if r.status == RequestStatus.FINISHED]
    out_tok = sum(len(r.output_token_ids) for r in done)
    ttft = [(r.first_token_time - r.arrival) * 1e3 for r in done if r.first_token_time]
    tpot = [(r.finish_time - r.first_token_time) * 1e3 / (len(r.output_token_ids) - 1)
            for r in done if r.finish_time and r.first_token_time and len(r.output_token_ids) > 1]
    e2e = [(r.finish_time - r.arrival) * 1e3 for r in done if r.finish_time]
    return BenchResult(sc.name, sc.num_requests, len(done), dur, out_tok, sum(lens), out_tok / max(dur, 1e-9),
                       len(done) / max(dur, 1e-9), LatencyStats.of(ttft), LatencyStats.of(tpot), LatencyStats.of(e2e),
                       dict(getattr(engine, "stats", {})))


# ------------------------------------------------------------------ regression gate
def check_regression(current: BenchResult, baseline: dict, tolerance: float = 0.10) -> list:
    """Compare against a baseline (a previous ``to_json`` dict). Returns human-readable
    failures: throughput below (1 - tol) x baseline, or p50/p99 latencies above (1 + tol) x."""
    fails = []
    bt = baseline.get("throughput_tok_s")
    if bt and current.throughput_tok_s < (1 - tolerance) * bt:
        fails.append(f"throughput {current.throughput_tok_s:.1f} < {(1 - tolerance) * bt:.1f} tok/s")
    for k in ("ttft_ms", "tpot_ms", "e2e_ms"):
        b = baseline.get(k) or {}
        cur = getattr(current, k)
        for q in ("p50", "p99"):
            if b.get(q) and getattr(cur, q) > (1 + tolerance) * b[q]:
                fails.append(f"{k}.{q} {getattr(cur, q):.2f} > {(1 + tolerance) * b[q]:.2f} ms")
    return fails


def main(argv=None):
    from .engine.engine import EngineConfig, LLMEngine
    from .models.config import preset
    from .models.llama import DecoderLM
    ap = argparse.ArgumentParser()
    ap.add_argument("--scenario", default="short", choices=sorted(SCENARIOS))
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--quant", default="bf16")
    ap.add_argument("--format", default="json", choices=["json", "csv", "prometheus", "text"])
    ap.add_argument("--export", default=None, help="also write every format to <stem>.{json,csv,prom,txt}")
    ap.add_argument("--baseline", default=None, help="JSON of a previous run: exit 1 on regression")
    ap.add_argument("--tolerance", type=float, default=0.10)
    a = ap.parse_args(argv)
    cfg = preset(a.preset)
    sc = SCENARIOS[a.scenario]
    m = DecoderLM(cfg, device=a.device, seed=0, weight_format=a.quant if a.device != "cpu" else "bf16")
    eng = LLMEngine(m, EngineConfig(max_num_seqs=max(4, sc.num_requests),
                                    max_model_len=sc.prompt_len[1] + sc.output_len + 16))
    res = run_scenario(eng, sc, cfg.vocab_size)
    print({"json": res.to_json, "csv": res.to_csv, "prometheus": res.to_prometheus, "text": res.to_text}[a.format]())
    if a.export:
        res.export_all(a.export)
    if a.baseline:
        with open(a.baseline) as f:
            fails = check_regression(res, json.load(f), a.tolerance)
        for x in fails:
            print("REGRESSION:", x)
        return 1 if fails else 0
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
