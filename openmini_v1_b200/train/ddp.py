"""Data-parallel gradient reduction overlapped with backward.

Parameters are grouped into buckets (reverse registration order, ~``bucket_mb``
each, so the buckets whose gradients finish first during backward are reduced
first). A post-accumulate-grad hook counts finished gradients per bucket; when
a bucket is complete on the last micro-batch of an accumulation window, its
gradients are flattened into one buffer and an asynchronous all-reduce (NCCL
over NVLink on GPUs, gloo on CPU) is started while backward continues with the
earlier layers. ``finish()`` waits for the outstanding reductions and writes
the averaged gradients back.

Reference: the data-parallel / ZeRO settings of
openmini-server/src/training/distributed_config.rs:399 (configuration only there).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GradReducer:
    def __init__(self, params, group=None, bucket_mb: float = 25.0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.params = [p for p in params if p.requires_grad]
        self.buckets = []
        cur, size = [], 0
        limit = int(bucket_mb * 1024 * 1024)
        for p in reversed(self.params):
            cur.append(p)
            size += p.numel() * 4
            if size >= limit:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self._bucket_of = {id(p): i for i, b in enumerate(self.buckets) for p in b}
        self._ready = [0] * len(self.buckets)
        self._pending = []
        self.sync = True
        self._hooks = []
        if self.world > 1:
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._on_grad))

    def _on_grad(self, p):
        if not self.sync:
            return
        b = self._bucket_of[id(p)]
        self._ready[b] += 1
        if self._ready[b] == len(self.buckets[b]):
            self._launch(b)

    def _launch(self, b):
        grads = [p.grad for p in self.buckets[b]]
        flat = torch.cat([g.reshape(-1) for g in grads])
        work = dist.all_reduce(flat, group=self.group, async_op=True)
        self._pending.append((b, flat, work))

    def begin(self, last_micro_batch: bool):
        """Call before each backward; reductions run only on the window's last micro-batch."""
        self.sync = last_micro_batch
        self._ready = [0] * len(self.buckets)

    def finish(self):
        if self.world == 1:
            return
        launched = {b for b, _, _ in self._pending}
        for b in range(len(self.buckets)):  # buckets with parameters that got no gradient
            if b not in launched and any(p.grad is not None for p in self.buckets[b]):
                for p in self.buckets[b]:
                    if p.grad is None:
                        p.grad = torch.zeros_like(p)
                self._launch(b)
        for b, flat, work in self._pending:
            work.wait()
            flat /= self.world
            o = 0
            for p in self.buckets[b]:
                n = p.numel()
                p.grad.copy_(flat[o:o + n].view_as(p.grad))
                o += n
        self._pending = []

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
