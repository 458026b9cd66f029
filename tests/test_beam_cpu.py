"""Beam search over the paged KV cache: width 1 equals greedy decoding, wider beams
score at least as well as greedy, hypotheses are re-scored exactly by a full
recompute, and every forked KV block is returned."""
import torch

from openmini_v1_b200.engine.beam import beam_search
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch


def _seq_logprob(m, prompt, out):
    toks = prompt + out
    T = len(toks)
    i32 = dict(dtype=torch.int32)
    nb = (T + 15) // 16 + 1
    fb = ForwardBatch(torch.tensor(toks, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                      torch.arange(nb, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                      torch.arange(len(prompt) - 1, T - 1))
    lp = torch.log_softmax(m.logits(m(fb, m.allocate_kv(nb))).float(), -1)
    return float(lp[torch.arange(len(out)), torch.tensor(out)].sum())


def test_beam_search():
    m = DecoderLM(tiny(), device="cpu", seed=4)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=8, max_model_len=256))
    prompt = list(range(300, 318))
    free0 = eng.bm.num_free()
    greedy = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True))[0]
    assert eng.bm.num_free() == free0
    b1 = beam_search(eng, prompt, beam_width=1, max_tokens=6)
    assert b1[0].token_ids == greedy.output_token_ids
    b4 = beam_search(eng, prompt, beam_width=4, max_tokens=6, length_penalty=0.0)
    assert eng.bm.num_free() == free0
    g_lp = _seq_logprob(m, prompt, greedy.output_token_ids)
    assert b4[0].logprob >= g_lp - 1e-3
    for h in b4:
        assert abs(_seq_logprob(m, prompt, h.token_ids) - h.logprob) < 1e-3
    assert len({tuple(h.token_ids) for h in b4}) == len(b4)
