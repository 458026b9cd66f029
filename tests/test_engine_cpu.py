"""CPU plumbing: tiny Llama through the paged-KV engine,
checked against a no-cache full-recompute oracle; scheduler preemption and
chunked prefill; sampler reference semantics."""
import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
from openmini_v1_b200.ops import reference as ref


def _oracle_greedy(m, prompt, n):
    toks = list(prompt)
    out = []
    for _ in range(n):
        T = len(toks)
        nb = (T + 15) // 16
        kv = m.allocate_kv(nb)
        i32 = dict(dtype=torch.int32)
        fb = ForwardBatch(torch.tensor(toks, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                          torch.arange(nb, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                          torch.tensor([T - 1]))
        t = int(m.logits(m(fb, kv)).argmax())
        out.append(t)
        toks.append(t)
    return out


def test_tiny_greedy_matches_recompute_oracle():
    m = DecoderLM(tiny(), device="cpu", seed=0)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 32000, (16,), generator=g).tolist()
    eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_model_len=256))
    r = eng.generate([prompt], SamplingParams(temperature=0.0, max_tokens=32, ignore_eos=True))[0]
    assert len(r.output_token_ids) == 32
    assert r.output_token_ids == _oracle_greedy(m, prompt, 32)


def test_chunked_prefill_and_batching_equal_single():
    m = DecoderLM(tiny(), device="cpu", seed=1)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (5, 40, 23)]
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    single = []
    for p in prompts:
        e = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=128))
        single.append(e.generate([p], sp)[0].output_token_ids)
    e = LLMEngine(m, EngineConfig(max_num_seqs=3, max_num_batched_tokens=16, max_model_len=128))
    batched = [r.output_token_ids for r in e.generate(prompts, sp)]
    assert batched == single


def test_preemption_under_kv_pressure():
    m = DecoderLM(tiny(), device="cpu", seed=2)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 32000, (30,), generator=g).tolist() for _ in range(3)]
    sp = SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True)
    e = LLMEngine(m, EngineConfig(max_num_seqs=3, max_model_len=128, num_blocks=9, enable_prefix_cache=False))
    outs = e.generate(prompts, sp)
    assert e.stats["preemptions"] > 0
    e2 = LLMEngine(m, EngineConfig(max_num_seqs=3, max_model_len=128, num_blocks=64))
    assert [r.output_token_ids for r in outs] == [r.output_token_ids for r in e2.generate(prompts, sp)]


def test_reference_sampler_semantics():
    V = 50
    lg = torch.randn(1, V)
    t, lp, m = ref.sample(lg, torch.tensor([0.8]), torch.tensor([0.6]), torch.tensor([10]),
                          torch.tensor([[3, 4]]))
    x = lg[0] / 0.8
    top10 = torch.topk(x, 10).indices
    assert set(torch.nonzero(m[0]).flatten().tolist()) <= set(top10.tolist())
    p = torch.softmax(x[m[0]], 0)
    assert float(p.sum()) > 0.99
    assert bool(m[0, int(t[0])])
    words = ref.pack_mask(m)
    assert torch.equal(ref.unpack_mask(words, V), m)


def test_quant_reference_roundtrip():
    w = torch.randn(64, 128) * 0.02
    q, s = ref.quantize_q4(w.bfloat16())
    d = ref.dequant_q4(q, s).float()
    assert (d - w).abs().max() < 0.02 * 4 / 8 + 1e-3
    q8, s8 = ref.quantize_int8(w.bfloat16())
    assert (ref.dequant_int8(q8, s8).float() - w).abs().max() < 1e-3


def test_speculative_ngram_matches_greedy():
    from openmini_v1_b200.engine.speculative import NgramProposer
    p = NgramProposer(3)
    assert p.propose([1, 2, 3, 9, 1, 2]) == [3, 9, 1]
    assert p.propose([5, 6, 7]) == []
    m = DecoderLM(tiny(), device="cpu", seed=4)
    pat = [11, 12, 13, 14, 15, 16, 17, 18] * 4
    sp = SamplingParams(temperature=0.0, max_tokens=24, ignore_eos=True)
    base = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256)).generate([pat, pat[:13]], sp)
    e = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, speculative_k=4))
    spec = e.generate([pat, pat[:13]], sp)
    assert [r.output_token_ids for r in spec] == [r.output_token_ids for r in base]
    assert e.stats["spec_proposed"] > 0
    # draft-model proposer: the model itself as its own draft accepts every proposal
    draft = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=256))
    e2 = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, speculative_k=3, draft_engine=draft))
    spec2 = e2.generate([pat, pat[:13]], sp)
    assert [r.output_token_ids for r in spec2] == [r.output_token_ids for r in base]
    assert e2.stats["spec_accepted"] >= e2.stats["spec_proposed"] - 4  # drafts cut at max_tokens only
    # a different (weaker) draft model still yields exactly the greedy output
    other = LLMEngine(DecoderLM(tiny(), device="cpu", seed=9), EngineConfig(max_num_seqs=1, max_model_len=256))
    e3 = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, speculative_k=3, draft_engine=other))
    assert [r.output_token_ids for r in e3.generate([pat, pat[:13]], sp)] == [r.output_token_ids for r in base]


def test_swap_preemption_and_session_persistence(tmp_path):
    from openmini_v1_b200.engine.kv_swap import restore_session, save_session
    m = DecoderLM(tiny(), device="cpu", seed=2)
    g = torch.Generator().manual_seed(2)
    prompts = [torch.randint(0, 32000, (30,), generator=g).tolist() for _ in range(3)]
    sp = SamplingParams(temperature=0.0, max_tokens=20, ignore_eos=True)
    e = LLMEngine(m, EngineConfig(max_num_seqs=3, max_model_len=128, num_blocks=9, enable_prefix_cache=False,
                                  preemption_mode="swap"))
    outs = e.generate(prompts, sp)
    assert e.stats["preemptions"] > 0 and e.swapper.swap_ins > 0
    e2 = LLMEngine(m, EngineConfig(max_num_seqs=3, max_model_len=128, num_blocks=64))
    assert [r.output_token_ids for r in outs] == [r.output_token_ids for r in e2.generate(prompts, sp)]
    # session: 8 tokens, save, restore in a fresh engine, 8 more == 16 uninterrupted
    full = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=128)).generate(
        [prompts[0]], SamplingParams(temperature=0.0, max_tokens=16, ignore_eos=True))[0].output_token_ids
    a = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=128))
    r = a.add_request("s", prompts[0], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    while r.status.name not in ("FINISHED",):
        a.step()
        if len(r.output_token_ids) == 7:
            save_session(a, r, str(tmp_path / "sess.safetensors"))
    b = LLMEngine(m, EngineConfig(max_num_seqs=1, max_model_len=128))
    r2 = restore_session(b, str(tmp_path / "sess.safetensors"), "s2",
                         SamplingParams(temperature=0.0, max_tokens=9, ignore_eos=True))
    while r2.status.name != "FINISHED":
        b.step()
    assert r.output_token_ids[:7] + r2.output_token_ids == full
