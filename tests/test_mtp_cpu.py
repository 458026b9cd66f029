"""Multi-token prediction on CPU: a distilled MTP head drafts tokens that the main
model verifies; output equals plain greedy decoding and the trained head gets drafts
accepted (a random one gets none or few)."""
import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM
from openmini_v1_b200.models.mtp import MTPHead, train_mtp


def _greedy(m, prompt, n):
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, use_cuda_graph=False))
    return eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True))[0].output_token_ids


def test_mtp_speculative_equals_greedy_and_accepts():
    cfg = tiny()
    cfg.num_layers = 1
    cfg.vocab_size = 512
    m = DecoderLM(cfg, device="cpu", seed=5)
    prompt = [3, 4, 5, 6]
    ref = _greedy(m, prompt, 40)
    head = MTPHead(m, ffn=256, seed=1)
    losses = train_mtp(head, [prompt + ref], steps=150, lr=3e-3)
    assert losses[-1] < losses[0] * 0.5
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, use_cuda_graph=False, speculative_k=3,
                                    mtp_head=head))
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=40, ignore_eos=True))[0]
    assert out.output_token_ids == ref
    assert eng.stats["spec_accepted"] > 0 and eng.stats["steps"] < 40


def test_calm_chunk_proposer():
    from openmini_v1_b200.models.mtp import CALMChunkHead
    cfg = tiny()
    cfg.num_layers = 1
    cfg.vocab_size = 512
    m = DecoderLM(cfg, device="cpu", seed=6)
    prompt = [7, 8, 9]
    ref = _greedy(m, prompt, 30)
    head = CALMChunkHead(m, k=4, confidence=0.1, seed=2)  # random-init LM head: flat distributions
    losses = head.train([prompt + ref], steps=200, lr=3e-3)
    assert losses[-1] < losses[0] * 0.5
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, use_cuda_graph=False, speculative_k=3,
                                    mtp_head=head))
    out = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=30, ignore_eos=True))[0]
    assert out.output_token_ids == ref
    assert eng.stats["spec_accepted"] > 0
