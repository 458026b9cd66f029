"""LLM serving engine: continuous batching over a paged KV cache, CUDA-graph
decode, device-side sampling, and multi-step device decode.

Public API (what servers, the RL rollout and the benchmarks call):

    eng = LLMEngine(model, EngineConfig(...))
    eng.add_request(request_id, prompt_token_ids, SamplingParams(...))
    outs = eng.step()              # one scheduler iteration -> [RequestOutput]
    eng.generate(prompts, params)  # convenience loop

Each ``step()`` stages that step's metadata (token ids, positions, cache slots,
block tables, sampling knobs) in pinned host memory, copies it to the device,
runs the model (a captured CUDA graph for decode batches), samples on the
device and reads the sampled tokens back.

The reference's equivalents are InferenceEngine / StreamGenerator /
generate_streaming (openmini-server/src/model/inference/inference.rs:176-670,
model.rs:4180-4253), which recompute on the CPU per token; here the whole step
is device work.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _native, ops
from ..models.llama import DecoderLM, ForwardBatch
from .request import Request, RequestOutput, RequestStatus, SamplingParams
from .scheduler import Scheduler
from ..utils.trace import nvtx_range


@dataclass
class EngineConfig:
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 8192
    max_model_len: int = 4096
    num_blocks: int | None = None          # None: derive from free device memory
    gpu_memory_utilization: float = 0.90
    enable_prefix_cache: bool = True
    enable_chunked_prefill: bool = True
    use_cuda_graph: bool = True
    graph_batch_sizes: list = field(default_factory=lambda: [1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192,
                                                             224, 256])
    eos_token_id: int | None = None
    seed: int = 0
    speculative_k: int = 0                 # > 0: speculative decoding (greedy and sampled requests)
    speculative_adaptive: bool = True      # per-request draft length follows the acceptance rate
    speculative_k_min: int = 1
    speculative_k_max: int = 0             # 0: speculative_k
    speculative_accept_threshold: float = 0.7
    speculative_acceptance: str = "exact"  # sampled requests: "exact" | "typical" (lossy, accepts more)
    typical_epsilon: float = 0.09          # typical acceptance: p(x) > min(epsilon, delta exp(-H(p)))
    typical_delta: float = 0.3
    draft_engine: object = None            # with speculative_k: an LLMEngine of a draft model proposes instead
    mtp_head: object = None                # with speculative_k: a models.mtp.MTPHead or CALMChunkHead proposes
    preemption_mode: str = "recompute"     # "recompute" | "swap" (KV kept on the host while preempted)


class _Pinned:
    """Reusable pinned staging buffers (one per dtype) for per-step H2D copies."""

    def __init__(self, device):
        self.pin = device.type == "cuda"
        self.i32 = torch.empty(1 << 20, dtype=torch.int32, pin_memory=self.pin)
        self.f32 = torch.empty(1 << 16, dtype=torch.float32, pin_memory=self.pin)
        self.i64 = torch.empty(1 << 16, dtype=torch.int64, pin_memory=self.pin)
        self.out_i32 = torch.empty(1 << 16, dtype=torch.int32, pin_memory=self.pin)
        self.out_f32 = torch.empty(1 << 16, dtype=torch.float32, pin_memory=self.pin)
        self.h2d_bytes = 0
        self.d2h_bytes = 0


class _RestoreOnly:
    """Swap-in only (restored sessions) when preemption recomputes."""

    def __init__(self, eng):
        from .kv_swap import KVSwapper
        self._sw = KVSwapper(eng)

    def swap_out(self, r):
        r.swapped = None
        r.routing = {}

    def swap_in(self, r):
        return self._sw.swap_in(r)


class LLMEngine:
    def __init__(self, model: DecoderLM, config: EngineConfig | None = None):
        self.model = model
        self.cfg = config or EngineConfig()
        self.device = model.device
        self.is_cuda = self.device.type == "cuda"
        self.max_blocks_per_seq = (self.cfg.max_model_len + 15) // 16
        nb = self.cfg.num_blocks or self._auto_blocks()
        self.kv = model.allocate_kv(nb)
        self.bm = _native.rt().BlockManager(nb, 16, self.cfg.enable_prefix_cache)
        self.sched = Scheduler(self.bm, self.cfg.max_num_seqs, self.cfg.max_num_batched_tokens,
                               self.cfg.max_model_len, self.cfg.enable_chunked_prefill)
        self.requests: dict = {}
        self.swapper = None
        from .kv_swap import KVSwapper
        if self.cfg.preemption_mode == "swap":
            self.swapper = KVSwapper(self)
            self.sched.swapper = self.swapper
        else:
            self.sched.swapper = _RestoreOnly(self)
        self.stage = _Pinned(self.device)
        self.graphs = None
        self.spec = None
        if self.cfg.speculative_k > 0:
            from .speculative import DraftModelProposer, NgramProposer
            if self.cfg.mtp_head is not None:
                from ..models.mtp import CALMChunkHead, CALMProposer, MTPProposer
                h = self.cfg.mtp_head
                self.spec = (CALMProposer(h, self.cfg.speculative_k) if isinstance(h, CALMChunkHead)
                             else MTPProposer(h, self.cfg.speculative_k))
            else:
                self.spec = (DraftModelProposer(self.cfg.draft_engine, self.cfg.speculative_k)
                             if self.cfg.draft_engine is not None else NgramProposer(self.cfg.speculative_k))
        self.stats = {"steps": 0, "prefill_tokens": 0, "decode_tokens": 0, "preemptions": 0}
        if self.is_cuda and self.cfg.use_cuda_graph:
            from .cuda_graph import DecodeGraphs
            self.graphs = DecodeGraphs(self)

    def _auto_blocks(self) -> int:
        need = self.cfg.max_num_seqs * self.max_blocks_per_seq + 1
        if not self.is_cuda:
            return max(64, need)
        from ..hardware.memory import kv_block_budget
        free, total = torch.cuda.mem_get_info(self.device)
        budget = kv_block_budget(free, total, self.model.kv_bytes_per_block(), self.cfg.gpu_memory_utilization)
        return int(max(64, min(need, budget)))

    # ---------------------------------------------------------------- API
    def add_request(self, request_id: str, prompt_token_ids, params: SamplingParams | None = None,
                    priority: int = 0, image_embeds: tuple | None = None) -> Request:
        """``image_embeds`` = (first prompt position, features [n, hidden]): the embeddings of
        those n prompt positions are replaced by the features (vision input). The ids at
        those positions should identify the image (see ``models.vision.splice_image``):
        the prefix cache keys on ids."""
        params = params or SamplingParams()
        params.validate()
        req = Request(request_id=request_id, prompt_token_ids=[int(t) for t in prompt_token_ids],
                      params=params, priority=priority)
        if image_embeds is not None:
            p0, emb = image_embeds
            if p0 < 0 or p0 + emb.shape[0] > len(req.prompt_token_ids):
                raise ValueError("image features fall outside the prompt")
            req.image_embeds = (int(p0), emb.to(self.device, self.model.dtype))
        self.sched.add(req)
        self.requests[request_id] = req
        return req

    def abort_request(self, request_id: str):
        r = self.sched.abort(request_id)
        self.requests.pop(request_id, None)
        return r

    def has_unfinished(self) -> bool:
        return self.sched.has_unfinished()

    def take_unfinished(self) -> list:
        """Remove every unfinished request (KV freed) and return the Request objects,
        generated tokens included, for another engine to ``adopt``."""
        out = []
        for r in list(self.sched.running) + list(self.sched.waiting):
            self.sched.abort(r.request_id)
            self.requests.pop(r.request_id, None)
            out.append(r)
        return out

    def adopt(self, req: Request) -> Request:
        """Continue a request taken from another engine: its prompt and generated tokens
        are re-prefilled here (fresh KV) and decoding resumes where it stopped."""
        from .request import _ids
        req.seq_id = next(_ids)
        req.num_computed = 0
        req.routing = {}
        self.sched.add(req)
        self.requests[req.request_id] = req
        return req

    def generate(self, prompts, params=None) -> list:
        """Run prompts (lists of token ids) to completion; returns Requests in input order."""
        reqs = []
        tag = time.monotonic_ns()
        for i, p in enumerate(prompts):
            sp = params[i] if isinstance(params, list) else (params or SamplingParams())
            reqs.append(self.add_request(f"gen-{tag}-{i}", p, sp))
        while any(r.status not in (RequestStatus.FINISHED, RequestStatus.ABORTED) for r in reqs):
            self.step()
        return reqs

    # ---------------------------------------------------------------- step
    def step(self) -> list:
        with nvtx_range("engine.step"):
            return self._step()

    def _step(self) -> list:
        with nvtx_range("schedule"):
            so = self.sched.schedule()
        self.stats["preemptions"] += len(so.preempted)
        if so.kind == "idle":
            return []
        self.stats["steps"] += 1
        if so.kind == "decode":
            for c in so.chunks:
                self._sync_bm_tokens(c.req)
        if so.kind == "decode" and self.spec is not None:
            from .speculative import eligible, spec_decode_step
            if all(eligible(c.req) for c in so.chunks):
                return spec_decode_step(self, so, self.spec)
        with nvtx_range("build"):
            fb, samp, rows_req = self._build(so)
        want_routing = any(c.req.params.return_routing for c in so.chunks)
        if (so.kind == "decode" and fb.embed_override is None and self.graphs is not None
                and self.graphs.can_run(len(so.chunks))
                and not self._needs_eager_sampling(rows_req) and not want_routing):
            with nvtx_range("decode_graph"):
                tok, lp, mask = self.graphs.run(fb, samp, len(so.chunks))
        else:
            if want_routing:
                fb.record_routing = {}
            tok, lp, mask = self._forward_sample(fb, samp, rows_req)
            if want_routing:
                o = 0
                for c in so.chunks:
                    n = c.end - c.start
                    if c.req.params.return_routing:
                        for layer, ids in fb.record_routing.items():
                            c.req.routing.setdefault(layer, []).append(ids[o:o + n].cpu())
                    o += n
        with nvtx_range("commit"):
            return self._commit(so, rows_req, tok, lp, mask)

    def _sync_bm_tokens(self, r: Request):
        n = self.bm.seq_len(r.seq_id)
        if n < r.num_tokens:
            cow = self.bm.append(r.seq_id, r.token_slice(n, r.num_tokens))
            if cow:
                self._apply_cow(cow)

    # ---------------------------------------------------------------- multi-step decode
    def begin_multi_decode(self, n: int):
        """Schedule one decode batch for ``n`` device-driven steps (CUDA graphs only).

        Returns a handle for :meth:`multi_decode_step` / :meth:`finish_multi_decode`;
        KV blocks for the n tokens are reserved up front."""
        if self.graphs is None:
            raise RuntimeError("multi-step decode needs CUDA graphs")
        so = self.sched.schedule()
        if so.kind != "decode":
            raise RuntimeError(f"multi-step decode needs a pure decode batch, scheduler returned {so.kind}")
        for c in so.chunks:
            self._sync_bm_tokens(c.req)
            self.bm.reserve(c.req.seq_id, n)
        fb, samp, rows = self._build(so)
        Bp = self.graphs.prepare_multi(fb, samp, len(rows), n)
        return {"so": so, "rows": rows, "Bp": Bp, "n": n, "done": 0}

    def multi_decode_step(self, h):
        self.graphs.replay_one(h["Bp"])
        h["done"] += 1

    def finish_multi_decode(self, h) -> list:
        B, Bp, k = len(h["rows"]), h["Bp"], h["done"]
        hist = self.graphs.hist[:k * Bp].view(k, Bp)[:, :B].cpu().tolist()
        outs = []
        now = time.monotonic()
        live = list(h["rows"])
        for s in range(k):
            for i, r in enumerate(h["rows"]):
                if r not in live:
                    continue
                t = int(hist[s][i])
                r.num_computed = r.num_tokens
                r.output_token_ids.append(t)
                r.rng_offset += 1
                if r.first_token_time is None:
                    r.first_token_time = now
                self.stats["decode_tokens"] += 1
                reason = self._stop_reason(r, t)
                if reason:
                    r.finish_reason, r.finish_time = reason, now
                    self.sched.finish(r)
                    self.requests.pop(r.request_id, None)
                    live.remove(r)
                outs.append(RequestOutput(request_id=r.request_id, new_token_ids=[t],
                                          output_token_ids=r.output_token_ids, finished=reason is not None,
                                          finish_reason=reason, prompt_tokens=len(r.prompt_token_ids)))
        self.stats["steps"] += k
        return outs

    # ---------------------------------------------------------------- internals
    def _apply_cow(self, cow):
        for src, dst in cow:
            for i in range(len(self.kv.k)):
                self.kv.k[i][dst].copy_(self.kv.k[i][src])
                self.kv.v[i][dst].copy_(self.kv.v[i][src])

    def _needs_eager_sampling(self, rows_req):
        return any(r.params.repetition_penalty != 1.0 or r.params.return_sampling_mask or r.params.return_routing
                   for r in rows_req)

    @staticmethod
    def _prefill_tiles(so, chunks, T):
        """Query tiles for the tensor-core prefill attention: <= 128 consecutive rows of one
        sequence each, as (row_start, rows, seq, keys of the last row), longest first.
        Only prefill batches with enough rows get tiles (decode rows use the split-KV kernel)."""
        if so.kind == "decode" or T < 128:
            return []
        tiles = []
        o = 0
        for si, c in enumerate(chunks):
            n = c.end - c.start
            for t0 in range(0, n, 128):
                rows = min(128, n - t0)
                tiles.append((o + t0, rows, si, c.start + t0 + rows))
            o += n
        tiles.sort(key=lambda x: -x[3])
        return tiles

    def _build(self, so):
        """Stage metadata on pinned host memory and copy it to the device (one H2D per dtype)."""
        chunks = so.chunks
        S = len(chunks)
        T = sum(c.end - c.start for c in chunks)
        mb = self.max_blocks_per_seq
        nL = sum(1 for c in chunks if c.wants_logits)
        tiles = self._prefill_tiles(so, chunks, T)
        n_i32 = 5 * T + S * mb + nL + 4 * len(tiles)
        st = self.stage
        if st.i32.numel() < n_i32:
            st.i32 = torch.empty(2 * n_i32, dtype=torch.int32, pin_memory=st.pin)
        buf = st.i32.numpy()
        ids, pos, slots, rseq, rctx = (buf[k * T:(k + 1) * T] for k in range(5))
        bt = buf[5 * T:5 * T + S * mb].reshape(S, mb)
        o = 0
        logits_rows = []
        rows_req = []
        if so.kind == "decode" and T == S and all(c.wants_logits for c in chunks):
            # one row per sequence: vectorised, the slots in one C++ call
            reqs = [c.req for c in chunks]
            p = np.fromiter((c.start for c in chunks), dtype=np.int32, count=S)
            ids[:] = [c.req.token_slice(c.start, c.end)[0] for c in chunks]
            pos[:] = p
            self.bm.decode_slots([r.seq_id for r in reqs], p, slots)
            rseq[:] = np.arange(S, dtype=np.int32)
            rctx[:] = p + 1
            logits_rows = list(range(S))
            rows_req = reqs
            chunks_loop = ()
        else:
            chunks_loop = chunks
        for si, c in enumerate(chunks_loop):
            r = c.req
            n = c.end - c.start
            ids[o:o + n] = r.token_slice(c.start, c.end)
            pos[o:o + n] = np.arange(c.start, c.end, dtype=np.int32)
            slots[o:o + n] = self.bm.slots(r.seq_id, c.start, c.end)
            rseq[o:o + n] = si
            rctx[o:o + n] = np.arange(c.start + 1, c.end + 1, dtype=np.int32)
            o += n
            if c.wants_logits:
                logits_rows.append(o - 1)
                rows_req.append(r)
        self.bm.fill_block_tables([c.req.seq_id for c in chunks], bt)
        o_t = 5 * T + S * mb + nL
        buf[5 * T + S * mb:o_t] = logits_rows
        if tiles:
            buf[o_t:n_i32] = np.asarray(tiles, dtype=np.int32).reshape(-1)
        d = st.i32[:n_i32].to(self.device, non_blocking=True)
        st.h2d_bytes = n_i32 * 4
        fb = ForwardBatch(
            input_ids=d[0:T], positions=d[T:2 * T], slots=d[2 * T:3 * T], row_seq=d[3 * T:4 * T],
            row_ctx=d[4 * T:5 * T], block_tables=d[5 * T:5 * T + S * mb].view(S, mb),
            max_ctx=(self.cfg.max_model_len if so.kind == "decode" else max(c.end for c in chunks)),
            logits_idx=d[5 * T + S * mb:o_t],
            prefill_tiles=d[o_t:n_i32].view(-1, 4) if tiles else None)
        ov_rows, ov_emb = [], []
        o = 0
        for c in chunks:
            ie = c.req.image_embeds
            n = c.end - c.start
            if ie is not None:
                p0, emb = ie
                a, b = max(c.start, p0), min(c.end, p0 + emb.shape[0])
                if a < b:
                    ov_rows.append(torch.arange(o + a - c.start, o + b - c.start))
                    ov_emb.append(emb[a - p0:b - p0])
            o += n
        if ov_rows:
            fb.embed_override = (torch.cat(ov_rows).to(self.device), torch.cat(ov_emb))
        # sampling knobs
        B = len(rows_req)
        f = st.f32.numpy()
        f[0:B] = [r.params.temperature for r in rows_req]
        f[B:2 * B] = [r.params.top_p for r in rows_req]
        i64 = st.i64.numpy()
        i64[0:B] = [r.params.top_k for r in rows_req]
        i64[B:3 * B:2] = [(r.params.seed if r.params.seed is not None else self.cfg.seed * 7919 + r.seq_id)
                          for r in rows_req]
        i64[B + 1:3 * B:2] = [r.rng_offset for r in rows_req]
        df = st.f32[:2 * B].to(self.device, non_blocking=True)
        di = st.i64[:3 * B].to(self.device, non_blocking=True)
        st.h2d_bytes += 2 * B * 4 + 3 * B * 8
        samp = {"temperature": df[:B], "top_p": df[B:2 * B], "top_k": di[:B].to(torch.int32),
                "rng": di[B:3 * B].view(B, 2)}
        return fb, samp, rows_req

    def _forward_sample(self, fb, samp, rows_req):
        x = self.model(fb, self.kv)
        want_mask = any(r.params.return_sampling_mask for r in rows_req)
        if all(r.params.repetition_penalty == 1.0 for r in rows_req):
            return self.model.sample(x, samp["temperature"], samp["top_p"], samp["top_k"], samp["rng"], want_mask)
        logits = self.model.logits(x)
        if any(r.params.repetition_penalty != 1.0 for r in rows_req):
            L = max(1, max(len(r.all_token_ids) for r in rows_req))
            prev = torch.full((len(rows_req), L), -1, dtype=torch.int32)
            for i, r in enumerate(rows_req):
                t = r.all_token_ids
                prev[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
            pen = torch.tensor([r.params.repetition_penalty for r in rows_req], dtype=torch.float32)
            logits = logits.float()
            ops.repetition_penalty(logits, prev.to(self.device), pen.to(self.device))
        return ops.sample(logits, samp["temperature"], samp["top_p"], samp["top_k"], samp["rng"], want_mask)

    def _commit(self, so, rows_req, tok, lp, mask):
        B = len(rows_req)
        st = self.stage
        toks, lps, masks = [], [], None
        if B:
            if self.is_cuda:
                st.out_i32[:B].copy_(tok, non_blocking=True)
                st.out_f32[:B].copy_(lp, non_blocking=True)
                torch.cuda.current_stream(self.device).synchronize()
                toks = st.out_i32[:B].tolist()
                lps = st.out_f32[:B].tolist()
            else:
                toks, lps = tok.tolist(), lp.tolist()
            st.d2h_bytes = B * 8
            masks = mask.cpu() if mask is not None else None
        now = time.monotonic()
        outs = []
        for c in so.chunks:
            c.req.num_computed = c.end
            if so.kind == "prefill":
                self.stats["prefill_tokens"] += c.end - c.start
        for i, r in enumerate(rows_req):
            t = int(toks[i])
            r.output_token_ids.append(t)
            r.rng_offset += 1
            if r.params.logprobs:
                r.output_logprobs.append(float(lps[i]))
            if r.params.return_sampling_mask and masks is not None:
                r.sampling_masks.append(masks[i].clone())
            if r.first_token_time is None:
                r.first_token_time = now
            self.stats["decode_tokens"] += 1
            reason = self._stop_reason(r, t)
            if reason:
                r.finish_reason = reason
                r.finish_time = now
                self.sched.finish(r)
                self.requests.pop(r.request_id, None)
            outs.append(RequestOutput(request_id=r.request_id, new_token_ids=[t],
                                      output_token_ids=r.output_token_ids, finished=reason is not None,
                                      finish_reason=reason,
                                      logprobs=r.output_logprobs if r.params.logprobs else None,
                                      prompt_tokens=len(r.prompt_token_ids)))
        return outs

    def _stop_reason(self, r: Request, t: int):
        p = r.params
        n = len(r.output_token_ids)
        if n >= p.min_tokens:
            if t in p.stop_token_ids:
                return "stop"
            if not p.ignore_eos and self.cfg.eos_token_id is not None and t == self.cfg.eos_token_id:
                return "stop"
        if n >= p.max_tokens:
            return "length"
        if r.num_tokens >= self.cfg.max_model_len:
            return "length"
        return None
