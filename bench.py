"""Headline benchmark: decode tok/s + p50 TTFT / TPOT for the 70B-shape model
served with tensor parallelism over N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Workload (weak scaling, 32 requests per GPU: 256 at N=8 as in the named
config): prompt lengths uniform in [512, 4096] and token ids uniform from a
seed, temperature 0.7 / top-p 0.9, random-init N(0, 0.02) weights quantised to
the 4-bit block format (block 32, one scale per block), bf16 activations and
paged bf16 KV (block 16).

Phases: (1) prefill every request through the engine (TTFT per request);
(2) W warm-up decode steps through ``LLMEngine.step``; (3) end-to-end: K
decode steps through ``LLMEngine.step`` (host scheduling, pinned H2D of the
step's metadata, CUDA-graph forward + sampling, D2H of the sampled tokens),
wall clock between barriers; (4) device: W + K device-driven decode steps
(``begin_multi_decode``: graph replays with the sampled tokens fed back on
the device), K of them timed with CUDA events between barrier + synchronize.
Every number is the max over ranks. The weights streamed per decode step are
far larger than the 126 MB L2, so no flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "decode tok/s + p50 TTFT/TPOT, 70B-shape TP=8, at 1/2/4/8 B200 (device, max/rank)"
BASELINE_VALUE = None  # the reference publishes no number for this model/config


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=32)
    p.add_argument("--warmup", type=int, default=4)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--model", default="llama70b")
    p.add_argument("--quant", default="q4", choices=["q4", "int8", "bf16"])
    p.add_argument("--reqs-per-gpu", type=int, default=32)
    p.add_argument("--prompt-min", type=int, default=512)
    p.add_argument("--prompt-max", type=int, default=4096)
    p.add_argument("--out-tokens", type=int, default=512)
    p.add_argument("--layers", type=int, default=0, help="override layer count (debug only; not the metric)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--trace", type=int, default=0,
                   help="after the timed run, profile this many extra device decode steps and print the "
                        "per-kernel device-time table of every rank to stderr (not part of the metric)")
    p.add_argument("--tp-transport", default="symm", choices=["symm", "symm_push", "nccl"],
                   help="symm: fused reduce/RMSNorm/all-gather over peer memory (partials pulled by the "
                        "reduce kernel); symm_push: the row-parallel GEMM stores its partials into the "
                        "owners' buffers; nccl: all-reduce baseline")
    return p.parse_args()


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout=5.0):
        """Block until nvidia-smi has produced its first sample (it needs ~0.5 s to start)."""
        t = time.monotonic()
        while self.proc is not None and not self.lines and time.monotonic() - t < timeout:
            time.sleep(0.05)

    def mark(self):
        """Samples before this point are warm-up; keep the last one as the clock at the region start."""
        self.start_idx = max(len(self.lines) - 1, 0)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[getattr(self, "start_idx", 0):]:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def reference_arm(a):
    line = {"impl": "reference",
            "unavailable": "reference is a Rust/Cargo workspace with no setup.py/pyproject.toml (pip install "
                           "fails) and no cargo/rustc or vendored crates offline, so it cannot be built here",
            "metric": METRIC, "n_gpus": a.gpus}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)
    return 0


def main():
    a = _args()
    if a.impl == "reference":
        return reference_arm(a)
    import torch
    import torch.distributed as dist

    from openmini_v1_b200 import ops
    from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
    from openmini_v1_b200.engine.request import SamplingParams
    from openmini_v1_b200.models.config import preset
    from openmini_v1_b200.models.llama import DecoderLM
    from openmini_v1_b200.parallel.fused import attach_tp_transport
    from openmini_v1_b200.parallel.state import ParallelState, init_distributed

    rank, world = init_distributed()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    par = ParallelState.build(tp=world)
    cfg = preset(a.model)
    if a.layers:
        cfg.num_layers = a.layers
    B = a.reqs_per_gpu * world
    max_len = a.prompt_max + a.out_tokens
    t_init = time.monotonic()
    model = DecoderLM(cfg, par=par, device=dev, seed=a.seed, weight_format=a.quant)
    # the fused transport covers whole prefill chunks (max_num_batched_tokens), not only decode
    attach_tp_transport(model, par, dev, a.tp_transport, max_rows=16384)
    torch.cuda.synchronize()
    init_s = time.monotonic() - t_init
    eng = LLMEngine(model, EngineConfig(max_num_seqs=B, max_num_batched_tokens=16384, max_model_len=max_len,
                                        enable_prefix_cache=False, use_cuda_graph=True, seed=a.seed))
    g = torch.Generator().manual_seed(a.seed)
    lens = torch.randint(a.prompt_min, a.prompt_max + 1, (B,), generator=g).tolist()
    sp = SamplingParams(temperature=0.7, top_p=0.9, max_tokens=a.out_tokens, ignore_eos=True)
    reqs = [eng.add_request(f"r{i}", torch.randint(0, cfg.vocab_size, (L,), generator=g).tolist(), sp)
            for i, L in enumerate(lens)]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # (1) prefill: TTFT measured from a common start
    barrier()
    t0 = time.monotonic()
    for r in reqs:
        r.arrival = t0
    while any(r.first_token_time is None for r in reqs):
        eng.step()
    barrier()
    prefill_s = max_over_ranks(time.monotonic() - t0)
    ttft_p50 = max_over_ranks(statistics.median(r.ttft for r in reqs))
    # (2) warm-up decode through the public API (also captures the graph)
    for _ in range(a.warmup):
        eng.step()
    ops.check_status(dev)
    # (3) end-to-end decode steps through LLMEngine.step
    barrier()
    t1 = time.monotonic()
    h2d = d2h = 0
    for _ in range(a.steps):
        eng.step()
        h2d += eng.stage.h2d_bytes
        d2h += eng.stage.d2h_bytes
    barrier()
    e2e_s = max_over_ranks(time.monotonic() - t1)
    e2e_tps = B * a.steps / e2e_s
    # (4) device-driven decode steps, CUDA-event timed
    clocks = ClockSampler(local)
    clocks.start()
    h = eng.begin_multi_decode(a.warmup + a.steps)
    for _ in range(a.warmup):
        eng.multi_decode_step(h)
    clocks.wait_first()
    barrier()
    clocks.mark()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(a.steps):
        eng.multi_decode_step(h)
    ev1.record()
    barrier()
    clk = clocks.stop()
    dev_ms = max_over_ranks(ev0.elapsed_time(ev1))
    eng.finish_multi_decode(h)
    ops.check_status(dev)
    ms_per_step = dev_ms / a.steps
    value = B * a.steps / (dev_ms / 1e3)
    launches = (eng.graphs.kernels_per_replay(h["Bp"]) + 1) * a.steps
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None, "dtype": "bf16",
        "data": "synthetic (uniform random token ids from a seed; random-init N(0,0.02) weights)",
        "impl": "native",
        "config": {"model": cfg.name + (f"-L{cfg.num_layers}" if a.layers else ""), "quant": a.quant,
                   "global_batch": B, "seq_len": f"prompt U[{a.prompt_min},{a.prompt_max}] + {a.out_tokens} out",
                   "parallelism": f"tp{world}", "tp_transport": a.tp_transport if world > 1 else None,
                   "temperature": 0.7, "top_p": 0.9,
                   "l2": "inputs larger than L2 (weights streamed per step >> 126 MB); no flush"},
        "ttft_p50_ms": round(ttft_p50 * 1e3, 2), "tpot_p50_ms": round(ms_per_step, 4),
        "tpot_e2e_ms": round(e2e_s / a.steps * 1e3, 4), "prefill_s": round(prefill_s, 3),
        "init_s": round(init_s, 2),
        "e2e": {"value": round(e2e_tps, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d // max(a.steps, 1),
                "d2h_bytes_per_step": d2h // max(a.steps, 1)},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if a.trace > 0:
        from openmini_v1_b200.utils.trace import by_position, format_table, kernel_sequence, kernel_table
        ht = eng.begin_multi_decode(a.trace + 2)  # one warm step, the table, one ordered step
        eng.multi_decode_step(ht)
        barrier()
        rows, total = kernel_table(lambda: eng.multi_decode_step(ht), iters=a.trace)
        seq = kernel_sequence(lambda: eng.multi_decode_step(ht))
        eng.finish_multi_decode(ht)
        gemm = [r for r in rows if "gemm_wq" in r[0] or "gemm_bf16" in r[0]]
        pos = by_position(seq, gemm[0][0], 4) if gemm else []
        table = format_table(rows, total, per=a.trace,
                             title=f"rank {rank}/{world}: {a.trace} profiled decode steps (shares, not timings)")
        for r in range(world):
            if world > 1:
                dist.barrier()
            if r == rank:
                print(table, file=sys.stderr, flush=True)
                if pos:
                    print("top GEMM by position in the layer (qkv, o, gate_up, down): "
                          + ", ".join(f"{p}: {us:.1f} us x{n}" for p, n, us in pos), file=sys.stderr, flush=True)
    if world > 1:
        # Captured decode graphs hold NCCL work; tearing the communicator down
        # under them can block, so ranks leave together after a final barrier.
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)
    return 0


if __name__ == "__main__":
    sys.exit(main())
