"""Memory network: HNSW recall against brute force and persistence, short-term
window budget, long-term recall into the prompt context, instant KV sessions."""
import numpy as np
import torch

from openmini_v1_b200.memory import HNSWIndex, LongTermMemory, MemoryManager, ShortTermMemory


def test_hnsw_recall_and_state(tmp_path):
    rng = np.random.default_rng(0)
    X = rng.normal(size=(1500, 24)).astype(np.float32)
    ix = HNSWIndex(24, M=12, ef_construction=80, ef=64)
    for v in X:
        ix.add(v)
    Xn = X / np.linalg.norm(X, axis=1, keepdims=True)
    hits = 0
    for q in rng.normal(size=(40, 24)).astype(np.float32):
        truth = set(np.argsort(-(Xn @ (q / np.linalg.norm(q))))[:10].tolist())
        hits += len(truth & {i for _, i in ix.search(q, 10)})
    assert hits / 400 >= 0.9
    ix2 = HNSWIndex.from_state(ix.state())
    assert ix2.search(X[7], 1)[0][1] == 7


def test_short_and_long_term_context(tmp_path):
    st = ShortTermMemory(token_budget=8)
    for i in range(5):
        st.add("s", "user", f"turn number {i}")
    assert [t.text for t in st.window("s")] == ["turn number 3", "turn number 4"]
    vocab = {}

    def emb(text):  # bag of words over a growing vocabulary of 64 hashed slots
        v = np.zeros(64, dtype=np.float32)
        for w in text.lower().split():
            v[hash(w) % 64] += 1
        return v + 1e-3
    p = str(tmp_path / "ltm.pkl")
    lt = LongTermMemory(emb, 64, path=p)
    mm = MemoryManager(ShortTermMemory(8), lt, k=2, min_score=0.5)
    mm.record("a", "user", "my cat is called Tom")
    mm.record("a", "user", "the weather in Paris is rainy")
    for i in range(4):
        mm.record("b", "user", f"unrelated chatter {i}")
    ctx = mm.context("b", "what is my cat called")
    assert ctx[0] == ("memory", "my cat is called Tom")
    lt.save()
    again = LongTermMemory(emb, 64, path=p)
    assert again.search("cat called Tom", 1)[0][1]["text"] == "my cat is called Tom"


def test_instant_memory_roundtrip(tmp_path):
    from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
    from openmini_v1_b200.engine.request import SamplingParams
    from openmini_v1_b200.memory import InstantMemory
    from openmini_v1_b200.models.config import tiny
    from openmini_v1_b200.models.llama import DecoderLM
    m = DecoderLM(tiny(), device="cpu", seed=0)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128))
    sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
    full = eng.generate([[5, 6, 7]], sp)[0].output_token_ids
    r = eng.add_request("x", [5, 6, 7], SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    im = InstantMemory(eng)
    while r.status.name != "FINISHED":
        eng.step()
        if len(r.output_token_ids) == 3:
            im.save("sess", r, str(tmp_path / "s.safetensors"))
    eng2 = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128))  # e.g. after a restart
    im2 = InstantMemory(eng2)
    im2.saved = dict(im.saved)
    r2 = im2.restore("sess", SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True))
    while r2.status.name != "FINISHED":
        eng2.step()
    # the session holds the positions whose KV was computed; generation resumes right after them
    seq = [5, 6, 7] + full
    assert r2.prompt_token_ids == seq[:len(r2.prompt_token_ids)]
    assert r2.prompt_token_ids + r2.output_token_ids == seq[:len(r2.prompt_token_ids) + 3]
