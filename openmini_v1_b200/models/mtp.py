"""Multi-token prediction (MTP) head and its use as a speculative-decoding proposer.

The head predicts the token after next from the main model's final hidden state h
at position t and the token chosen for position t + 1:

    u  = W_proj [RMSNorm(h); RMSNorm(emb(tok))]          (2D -> D)
    h' = u + W_down SiLU(W_gate RMSNorm(u)) * (W_up RMSNorm(u))
    logits = lm_head(RMSNorm_final(h'))                  (embedding, final norm and head shared)

Fed its own h' and drafted token it chains to k drafts. The main model verifies the
drafts in one forward (``engine.speculative.spec_decode_step``), so the output equals
plain greedy decoding whatever the head predicts; a trained head only raises the
number of tokens accepted per step. ``train_mtp`` distils the head from the main
model's own hidden states and next-next tokens.

The published MTP modules put a full transformer layer where this head has the
SwiGLU block; a layer with attention would need a KV cache of its own per sequence,
which this head avoids.

Reference counterpart: openmini-server/src/model/inference/mtp.rs (MtpDecoder:
candidate generation, verification against the main model, acceptance statistics).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import ops


class MTPHead:
    def __init__(self, model, ffn: int | None = None, seed: int = 0, std: float = 0.02):
        self.model = model
        D = model.cfg.hidden_size
        F_ = ffn or 2 * D
        g = torch.Generator().manual_seed(seed)
        dt, dev = model.dtype, model.device
        r = lambda *s: (torch.randn(*s, generator=g) * std).to(dev, dt)  # noqa: E731
        self.p = {"n_h": torch.ones(D, dtype=dt, device=dev), "n_e": torch.ones(D, dtype=dt, device=dev),
                  "proj": r(D, 2 * D), "n_u": torch.ones(D, dtype=dt, device=dev),
                  "gate_up": r(2 * F_, D), "down": r(D, F_)}
        self.eps = model.cfg.rms_eps

    def parameters(self):
        return list(self.p.values())

    def step(self, h: torch.Tensor, tok: torch.Tensor):
        """h [N, D] final hidden rows, tok [N] int -> (h' [N, D], logits [N, V])."""
        m, p = self.model, self.p
        e = ops.embedding(tok.to(torch.int32), m.embed)
        u = ops.linear(torch.cat([ops.rmsnorm(h.contiguous(), p["n_h"], self.eps),
                                  ops.rmsnorm(e, p["n_e"], self.eps)], dim=-1), p["proj"])
        a = ops.silu_mul(ops.linear(ops.rmsnorm(u, p["n_u"], self.eps), p["gate_up"]))
        h2 = ops.linear(a, p["down"], resid=u)
        return h2, m.logits(ops.rmsnorm(h2, m.norm, self.eps))

    def step_train(self, h, tok):
        """Differentiable fp32 form of :meth:`step` (training on CPU / GPU)."""
        m, p = self.model, self.p
        rms = lambda x, w: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * w  # noqa: E731
        e = m.embed.float()[tok.long()]
        u = torch.cat([rms(h, p["n_h"]), rms(e, p["n_e"])], -1) @ p["proj"].t()
        gu = rms(u, p["n_u"]) @ p["gate_up"].t()
        g_, up = gu.chunk(2, -1)
        h2 = u + (F.silu(g_) * up) @ p["down"].t()
        return h2, rms(h2, m.norm.float()) @ m.lm_head.float().t()


class MTPProposer:
    """Speculative proposer from an MTP head. The engine hands it, after each verified
    step, the final hidden row behind a request's last emitted token (``observe``);
    ``propose`` chains the head from there. Without an observed state it proposes
    nothing (that step is a plain verified decode)."""
    wants_request = True

    def __init__(self, head: MTPHead, k: int = 3):
        self.head, self.k = head, k
        self.state: dict = {}

    def observe(self, req, hidden_row: torch.Tensor, token: int):
        self.state[req.request_id] = (hidden_row.detach(), int(token), req.num_tokens)

    def forget(self, req):
        self.state.pop(req.request_id, None)

    @torch.no_grad()
    def propose(self, toks, k: int | None = None, req=None) -> list:
        k = self.k if k is None else k
        st = self.state.get(req.request_id) if req is not None else None
        if k <= 0 or st is None or st[2] != len(toks):
            return []
        h, t = st[0][None], torch.tensor([st[1]], device=st[0].device)
        out = []
        for _ in range(k):
            h, lg = self.head.step(h, t)
            t = lg.argmax(-1)
            out.append(int(t))
        return out


def train_mtp(head: MTPHead, sequences: list, steps: int = 100, lr: float = 1e-3) -> list:
    """Distil the head: for each position t of each sequence, from the main model's final
    hidden h_t and token x_{t+1}, predict x_{t+2}. Returns the loss per step."""
    from .llama import ForwardBatch
    m = head.model
    dev = m.device
    data = []
    with torch.no_grad():
        for s in sequences:
            T = len(s)
            i32 = dict(dtype=torch.int32, device=dev)
            nb = (T + 15) // 16
            fb = ForwardBatch(torch.tensor(s, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                              torch.arange(nb, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                              torch.arange(T, device=dev))
            h = m(fb, m.allocate_kv(nb)).float()
            data.append((h[:T - 2], torch.tensor(s[1:T - 1], device=dev), torch.tensor(s[2:T], device=dev)))
    h = torch.cat([d[0] for d in data])
    x1 = torch.cat([d[1] for d in data])
    y = torch.cat([d[2] for d in data])
    params = {k: v.detach().float().clone().requires_grad_(True) for k, v in head.p.items()}
    orig = head.p
    head.p = params
    opt = torch.optim.Adam(params.values(), lr=lr)
    losses = []
    for _ in range(steps):
        _, lg = head.step_train(h, x1)
        loss = F.cross_entropy(lg, y.long())
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    head.p = {k: params[k].detach().to(orig[k].dtype) for k in orig}
    return losses


class CALMChunkHead:
    """Chunk-level generation (CALM): from the final hidden state h_t, K parallel heads
    predict the tokens t+1 .. t+K in one step (head i: W_i RMSNorm(h) added to h, then
    the shared LM head). A chunk is cut at the first token whose probability falls below
    ``confidence``; as a proposer the verified speculative step keeps the output equal to
    greedy decoding. Reference counterpart: openmini-server/src/model/inference/calm.rs
    (hidden state -> multi-token chunk with a confidence gate)."""

    def __init__(self, model, k: int = 4, confidence: float = 0.5, seed: int = 0, std: float = 0.02):
        D = model.cfg.hidden_size
        g = torch.Generator().manual_seed(seed)
        self.model, self.k, self.confidence = model, k, confidence
        self.w = [(torch.randn(D, D, generator=g) * std).to(model.device, model.dtype) for _ in range(k)]
        self.eps = model.cfg.rms_eps

    def chunk(self, h: torch.Tensor):
        """h [D] -> (tokens, probabilities) of the confident prefix of the chunk."""
        m = self.model
        toks, probs = [], []
        hn = ops.rmsnorm(h[None].contiguous(), m.norm, self.eps)
        for W in self.w:
            z = ops.linear(hn, W, resid=h[None].contiguous())
            p = torch.softmax(m.logits(ops.rmsnorm(z, m.norm, self.eps)).float(), -1)[0]
            pr, t = p.max(-1)
            if float(pr) < self.confidence:
                break
            toks.append(int(t))
            probs.append(float(pr))
        return toks, probs

    def train(self, sequences: list, steps: int = 100, lr: float = 1e-3) -> list:
        """Fit head i to predict x_{t+1+i} from h_t of the main model (teacher forcing)."""
        from .llama import ForwardBatch
        m = self.model
        dev = m.device
        H, Y = [], []
        with torch.no_grad():
            for s in sequences:
                T = len(s)
                i32 = dict(dtype=torch.int32, device=dev)
                nb = (T + 15) // 16
                fb = ForwardBatch(torch.tensor(s, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                                  torch.arange(nb, **i32)[None], torch.zeros(T, **i32),
                                  torch.arange(1, T + 1, **i32), T, torch.arange(T, device=dev))
                h = m(fb, m.allocate_kv(nb)).float()
                n = T - self.k
                H.append(h[:n])
                Y.append(torch.stack([torch.tensor(s[1 + i:1 + i + n], device=dev) for i in range(self.k)], 1))
        h, y = torch.cat(H), torch.cat(Y)
        ws = [w.detach().float().clone().requires_grad_(True) for w in self.w]
        opt = torch.optim.Adam(ws, lr=lr)
        norm, head = m.norm.float(), m.lm_head.float()
        rms = lambda x: x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * norm  # noqa: E731
        losses = []
        for _ in range(steps):
            loss = sum(F.cross_entropy(rms(h + rms(h) @ W.t()) @ head.t(), y[:, i].long()) for i, W in enumerate(ws))
            opt.zero_grad()
            loss.backward()
            opt.step()
            losses.append(float(loss.detach()) / self.k)
        self.w = [w.detach().to(m.dtype) for w in ws]
        return losses


class CALMProposer(MTPProposer):
    """Speculative proposer from a CALM chunk head (drafts = the confident chunk)."""

    def __init__(self, head: CALMChunkHead, k: int | None = None):
        super().__init__(None, k or head.k)
        self.calm = head

    @torch.no_grad()
    def propose(self, toks, k: int | None = None, req=None) -> list:
        k = self.k if k is None else k
        st = self.state.get(req.request_id) if req is not None else None
        if k <= 0 or st is None or st[2] != len(toks):
            return []
        # the chunk head predicts from h behind the last token; its first draft is the
        # token after the one just emitted, so the chunk is shifted by one
        drafts, _ = self.calm.chunk(st[0])
        return drafts[1:1 + k] if drafts and drafts[0] == st[1] else []
