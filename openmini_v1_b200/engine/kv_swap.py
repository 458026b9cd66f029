"""KV swap (preemption without recompute) and KV session persistence.

``KVSwapper``: when the scheduler preempts a request, the KV of its computed
positions is copied to (pinned) host memory before its blocks are freed; on
re-admission the blocks are re-allocated and the KV copied back, so the
request resumes where it stopped instead of recomputing its prefix.

``save_session`` / ``restore_session``: a sequence's tokens and KV written to
a safetensors file and loaded into a new request later (possibly by another
engine process with the same model), which then continues decoding without a
prefill.

Reference: KV persistence (bincode save/load), SQLite-backed KV swap and the
CPU<->GPU two-level cache of openmini-server/src/hardware/kv_cache/
(persistence, swap, ess modules; the reference simulates the transfers).
"""
from __future__ import annotations

import torch

from ..train.safetensors import load_file, save_file


class KVSwapper:
    def __init__(self, engine):
        self.eng = engine
        self.pin = engine.device.type == "cuda"
        self.swapped_bytes = 0
        self.swap_outs = 0
        self.swap_ins = 0

    def _gather(self, blocks):
        kv = self.eng.kv
        idx = torch.tensor(blocks, dtype=torch.long, device=self.eng.device)
        out = []
        for layer in range(len(kv.k)):
            parts = [kv.k[layer].index_select(0, idx), kv.v[layer].index_select(0, idx)]
            if kv.idx_k:
                parts.append(kv.idx_k[layer].index_select(0, idx))
            for p in parts:
                h = torch.empty(p.shape, dtype=p.dtype, pin_memory=self.pin)
                h.copy_(p, non_blocking=True)
                out.append(h)
        if self.pin:
            torch.cuda.current_stream(self.eng.device).synchronize()
        return out

    def _scatter(self, blocks, tensors):
        kv = self.eng.kv
        idx = torch.tensor(blocks, dtype=torch.long, device=self.eng.device)
        per = 3 if kv.idx_k else 2
        for layer in range(len(kv.k)):
            dst = [kv.k[layer], kv.v[layer]] + ([kv.idx_k[layer]] if kv.idx_k else [])
            for j, d in enumerate(dst):
                d.index_copy_(0, idx, tensors[layer * per + j].to(self.eng.device, non_blocking=True))

    def swap_out(self, r):
        n = r.num_computed
        if n <= 0:
            return
        nb = (n + 15) // 16
        blocks = self.eng.bm.block_table(r.seq_id)[:nb]
        r.swapped = (n, self._gather(blocks))
        self.swapped_bytes += sum(t.numel() * t.element_size() for t in r.swapped[1])
        self.swap_outs += 1

    def swap_in(self, r) -> int:
        """Restore swapped KV after re-allocation; returns the number of computed positions."""
        sw = getattr(r, "swapped", None)
        if not sw:
            return 0
        n, tensors = sw
        nb = (n + 15) // 16
        self._scatter(self.eng.bm.block_table(r.seq_id)[:nb], tensors)
        r.swapped = None
        self.swapped_bytes -= sum(t.numel() * t.element_size() for t in tensors)
        self.swap_ins += 1
        return n


def save_session(engine, request, path: str):
    """Tokens + KV of the request's computed positions -> safetensors file."""
    n = request.num_computed
    nb = (n + 15) // 16
    blocks = engine.bm.block_table(request.seq_id)[:nb]
    tensors = KVSwapper(engine)._gather(blocks)
    data = {f"kv.{i}": t for i, t in enumerate(tensors)}
    data["tokens"] = torch.tensor(request.all_token_ids[:n], dtype=torch.int64)
    save_file(data, path, {"num_computed": n, "layers": len(engine.kv.k)})


def restore_session(engine, path: str, request_id: str, params, extra_tokens=None):
    """New request continuing a saved session (KV restored, no prefill of the saved prefix).

    ``extra_tokens`` are appended as new prompt tokens (e.g. the user's next turn)."""
    data = load_file(path)
    toks = data.pop("tokens").tolist()
    tensors = [data[f"kv.{i}"] for i in range(len(data))]
    prompt = toks + list(extra_tokens or [])
    r = engine.add_request(request_id, prompt, params)
    r.swapped = (len(toks), tensors)
    return r
