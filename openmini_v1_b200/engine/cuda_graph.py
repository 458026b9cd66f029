"""CUDA-graph capture of the decode step (forward + LM head + sampling).

One graph per batch bucket; all buckets share static input/output buffers
(bucket B uses rows [:B]) and one memory pool. Rows beyond the live batch are
padding: slot -1 (no cache write), one visible key, token 0.

``replay_one`` (multi-step decode) replays a bucket's graph and then runs a
device kernel that feeds each sampled token back as the next input and
advances positions, context lengths, cache slots and RNG offsets, so n decode
steps run with no host round trip (the caller reserves KV blocks first).
"""
from __future__ import annotations

import torch

from .. import _native, ops
from ..models.llama import ForwardBatch


class DecodeGraphs:
    def __init__(self, eng):
        self.eng = eng
        cfg = eng.cfg
        self.sizes = sorted({s for s in cfg.graph_batch_sizes if s <= cfg.max_num_seqs} | {cfg.max_num_seqs})
        self.max_B = self.sizes[-1]
        dev = eng.device
        MB = eng.max_blocks_per_seq
        i32 = dict(dtype=torch.int32, device=dev)
        self.ids = torch.zeros(self.max_B, **i32)
        self.pos = torch.zeros(self.max_B, **i32)
        self.slots = torch.full((self.max_B,), -1, **i32)
        self.rseq = torch.arange(self.max_B, **i32)
        self.rctx = torch.ones(self.max_B, **i32)
        self.bt = torch.zeros(self.max_B, MB, **i32)
        self.lidx = torch.arange(self.max_B, **i32)
        self.temp = torch.zeros(self.max_B, dtype=torch.float32, device=dev)
        self.top_p = torch.ones(self.max_B, dtype=torch.float32, device=dev)
        self.top_k = torch.zeros(self.max_B, **i32)
        self.rng = torch.zeros(self.max_B, 2, dtype=torch.int64, device=dev)
        self.step_ctr = torch.zeros(1, **i32)
        self.hist = None
        self.out_tok, self.out_lp = {}, {}
        self.graphs = {}
        self.launches = {}
        self.pool = None

    def can_run(self, B: int) -> bool:
        return B <= self.max_B

    def bucket(self, B: int) -> int:
        for s in self.sizes:
            if s >= B:
                return s
        raise ValueError(B)

    def _fb(self, B):
        return ForwardBatch(input_ids=self.ids[:B], positions=self.pos[:B], slots=self.slots[:B],
                            block_tables=self.bt[:B], row_seq=self.rseq[:B], row_ctx=self.rctx[:B],
                            max_ctx=self.eng.cfg.max_model_len, logits_idx=self.lidx[:B])

    def _body(self, B):
        m = self.eng.model
        x = m(self._fb(B), self.eng.kv)
        return m.sample(x, self.temp[:B], self.top_p[:B], self.top_k[:B], self.rng[:B], False)[:2]

    def capture(self, B: int):
        eng = self.eng
        c = ops.ctx(eng.device)
        s = torch.cuda.Stream(eng.device)
        s.wait_stream(torch.cuda.current_stream(eng.device))
        with torch.cuda.stream(s):  # eager warm-up: kernel attributes, workspace sizes
            self._body(B)
        torch.cuda.current_stream(eng.device).wait_stream(s)
        torch.cuda.synchronize(eng.device)
        g = torch.cuda.CUDAGraph()
        c.frozen = True
        n0 = _native.C().launch_count()
        try:
            with torch.cuda.graph(g, pool=self.pool):
                tok, lp = self._body(B)
        finally:
            c.frozen = False
        self.launches[B] = _native.C().launch_count() - n0
        if self.pool is None:
            self.pool = g.pool()
        self.graphs[B] = g
        self.out_tok[B], self.out_lp[B] = tok, lp

    def kernels_per_replay(self, B: int) -> int:
        return self.launches.get(B, 0)

    def _load(self, fb: ForwardBatch, samp, B: int, Bp: int):
        self.ids[:B].copy_(fb.input_ids)
        self.pos[:B].copy_(fb.positions)
        self.slots[:B].copy_(fb.slots)
        self.rctx[:B].copy_(fb.row_ctx)
        mb = fb.block_tables.shape[1]
        self.bt[:B, :mb].copy_(fb.block_tables)
        self.temp[:B].copy_(samp["temperature"])
        self.top_p[:B].copy_(samp["top_p"])
        self.top_k[:B].copy_(samp["top_k"])
        self.rng[:B].copy_(samp["rng"])
        if Bp > B:
            self.ids[B:Bp].zero_()
            self.pos[B:Bp].zero_()
            self.slots[B:Bp].fill_(-1)
            self.rctx[B:Bp].fill_(1)
            self.bt[B:Bp].zero_()

    def run(self, fb: ForwardBatch, samp, B: int):
        Bp = self.bucket(B)
        if Bp not in self.graphs:
            self.capture(Bp)
        self._load(fb, samp, B, Bp)
        self.graphs[Bp].replay()
        return self.out_tok[Bp][:B], self.out_lp[Bp][:B], None

    # ------------------------------------------------------------ multi-step
    def prepare_multi(self, fb: ForwardBatch, samp, B: int, n: int) -> int:
        Bp = self.bucket(B)
        if Bp not in self.graphs:
            self.capture(Bp)
        self._load(fb, samp, B, Bp)
        self.hist = torch.zeros(n * Bp, dtype=torch.int32, device=self.eng.device)
        self.step_ctr.zero_()
        return Bp

    def replay_one(self, Bp: int):
        self.graphs[Bp].replay()
        _native.C().decode_advance(self.out_tok[Bp], self.ids[:Bp], self.pos[:Bp], self.rctx[:Bp],
                                   self.slots[:Bp], self.bt[:Bp], self.rng[:Bp], self.hist, self.step_ctr)
