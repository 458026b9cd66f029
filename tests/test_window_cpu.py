"""Sliding-window attention: the window kernel path equals explicitly masked attention,
windows wider than the context equal dense attention, and incremental decoding matches
a one-shot prefill of the same tokens."""
import math
from types import SimpleNamespace

import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.models.window import window_attention, window_indices


def test_window_indices_and_math():
    sel, n = window_indices(torch.tensor([1, 5, 20], dtype=torch.int32), 8)
    assert n.tolist() == [1, 5, 8] and sel[2].tolist() == list(range(12, 20))
    g = torch.Generator().manual_seed(0)
    Hq, Hkv, D, L, W = 4, 2, 16, 37, 9
    kc = torch.randn(4, Hkv, 16, D, generator=g)
    vc = torch.randn(4, Hkv, 16, D, generator=g)
    bt = torch.tensor([[2, 0, 3, 1]], dtype=torch.int32)
    q = torch.randn(L, Hq * D, generator=g)
    rctx = torch.arange(1, L + 1, dtype=torch.int32)
    fb = SimpleNamespace(max_ctx=L, block_tables=bt, row_seq=torch.zeros(L, dtype=torch.int32), row_ctx=rctx,
                         prefill_tiles=None)
    m = SimpleNamespace(hq=Hq, hd=D, scale=1 / math.sqrt(D))
    out = window_attention(m, q, kc, vc, fb, W)
    K = torch.cat([kc[b] for b in bt[0].tolist()], 1).transpose(0, 1)[:L].repeat_interleave(2, 1)  # [L, Hq, D]
    V = torch.cat([vc[b] for b in bt[0].tolist()], 1).transpose(0, 1)[:L].repeat_interleave(2, 1)
    s = torch.einsum("thd,khd->htk", q.view(L, Hq, D), K) * m.scale
    t = torch.arange(L)
    mask = (t[None, :] > t[:, None]) | (t[None, :] <= t[:, None] - W)
    p = torch.softmax(s.masked_fill(mask[None], float("-inf")), -1)
    want = torch.einsum("htk,khd->thd", p, V).reshape(L, -1)
    assert torch.allclose(out, want, atol=1e-5)


def test_window_model_prefill_equals_decode():
    cfg = tiny()
    cfg.sliding_window, cfg.sliding_window_global_every = 6, 2
    m = DecoderLM(cfg, device="cpu", seed=3)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128, enable_prefix_cache=False))
    prompt = list(range(50, 70))
    r = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True))[0]
    # greedy tokens re-derived by prefilling prompt + generated tokens in one shot
    toks = prompt + r.output_token_ids
    eng2 = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128, enable_prefix_cache=False))
    for j in range(5):
        r2 = eng2.generate([toks[:len(prompt) + j]], SamplingParams(temperature=0.0, max_tokens=1,
                                                                   ignore_eos=True))[0]
        assert r2.output_token_ids[0] == r.output_token_ids[j]
    # a window wider than every context equals the dense model
    dense_cfg = tiny()
    wide = tiny()
    wide.sliding_window = 1000
    a = DecoderLM(dense_cfg, device="cpu", seed=3)
    b = DecoderLM(wide, device="cpu", seed=3)
    sp = SamplingParams(temperature=0.0, max_tokens=4, ignore_eos=True)
    ra = LLMEngine(a, EngineConfig(max_num_seqs=2, max_model_len=128)).generate([prompt], sp)[0]
    rb = LLMEngine(b, EngineConfig(max_num_seqs=2, max_model_len=128)).generate([prompt], sp)[0]
    assert ra.output_token_ids == rb.output_token_ids


def test_attention_sinks_indices():
    sel, n = window_indices(torch.tensor([1, 3, 5, 9, 20], dtype=torch.int32), 4, 2)
    got = [r[:k] for r, k in zip(sel.tolist(), n.tolist())]
    assert got == [[0], [0, 1, 2], [0, 1, 2, 3, 4], [0, 1, 5, 6, 7, 8], [0, 1, 16, 17, 18, 19]]
    cfg = tiny()
    cfg.sliding_window, cfg.attention_sinks = 6, 2
    m = DecoderLM(cfg, device="cpu", seed=5)
    r = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128)).generate(
        [list(range(10, 40))], SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True))[0]
    assert len(r.output_token_ids) == 3
