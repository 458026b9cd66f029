"""Multi-head latent attention on CPU: the absorbed form over the paged latent cache
(the path the CUDA kernel runs) against the unabsorbed fp32 statement, a prefill
followed by decode through the engine, and the cache footprint."""
import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import MLAConfig, tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
from openmini_v1_b200.models.mla import mla_attention, mla_reference_layer
from openmini_v1_b200.ops import reference as ref


def _cfg():
    c = tiny()
    c.mla = MLAConfig(enabled=True, qk_nope_dim=32, qk_rope_dim=64, v_head_dim=32)
    return c


def test_absorbed_paged_matches_unabsorbed():
    m = DecoderLM(_cfg(), device="cpu", seed=1)
    T = 21
    i32 = dict(dtype=torch.int32)
    fb = ForwardBatch(torch.arange(T, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                      torch.arange(2, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                      torch.tensor([T - 1]))
    kv = m.allocate_kv(2)
    L = m.layers[0]
    a = torch.randn(T, m.cfg.hidden_size, generator=torch.Generator().manual_seed(0))
    got = mla_attention(m, 0, L, a, fb, kv)
    want = mla_reference_layer(m, L, a, fb.positions)
    assert got.shape == (T, 4 * 32)
    assert (got - want).abs().max().item() < 1e-4 * max(1.0, want.abs().max().item())
    # the cache holds [RMSNorm(c) | RoPE(k_r)] rows at the slots
    assert kv.k[0].shape == (2, 16, 576) and kv.k[0].view(-1, 576)[:T].abs().sum() > 0


def test_mla_engine_prefill_decode_and_footprint():
    m = DecoderLM(_cfg(), device="cpu", seed=2)
    assert m.kv_bytes_per_block() == 2 * 16 * 576 * 4  # two layers of 576-wide fp32 rows
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=64, use_cuda_graph=False))
    reqs = eng.generate([[5, 6, 7, 8, 9], [11, 12, 13]], SamplingParams(temperature=0.0, max_tokens=4,
                                                                       ignore_eos=True))
    assert all(len(r.output_token_ids) == 4 for r in reqs)
    # greedy decode equals recomputing the whole sequence with a fresh cache each step
    toks = [5, 6, 7, 8, 9]
    for _ in range(4):
        T = len(toks)
        i32 = dict(dtype=torch.int32)
        fb = ForwardBatch(torch.tensor(toks, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                          torch.arange(4, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                          torch.tensor([T - 1]))
        toks.append(int(m.logits(m(fb, m.allocate_kv(4))).argmax(-1)))
    assert toks[5:] == reqs[0].output_token_ids


def test_mla_decode_reference_rows():
    g = torch.Generator().manual_seed(3)
    cache = torch.randn(4, 16, 576, generator=g)
    q = torch.randn(3, 2, 576, generator=g)
    bt = torch.tensor([[2, 0, 3, 1]], dtype=torch.int32)
    out = ref.mla_decode(q, cache, bt, torch.zeros(3, dtype=torch.int32), torch.tensor([1, 17, 64], dtype=torch.int32),
                         0.05)
    rows = torch.cat([cache[2], cache[0], cache[3], cache[1]])
    s = (q[1] @ rows[:17].t()) * 0.05
    assert torch.allclose(out[1], torch.softmax(s, -1) @ rows[:17, :512], atol=1e-5)
    assert torch.allclose(out[0], rows[0, :512].expand(2, 512), atol=1e-6)


def _logits(m, T=19):
    i32 = dict(dtype=torch.int32)
    fb = ForwardBatch(torch.arange(3, 3 + T, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                      torch.arange(2, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                      torch.arange(T))
    return m.logits(m(fb, m.allocate_kv(2))).float()


def test_mla_gguf_round_trip(tmp_path):
    """DeepSeek-style GGUF (deepseek2 keys; attn_q or the low-rank attn_q_a / _norm / _b;
    attn_kv_a_mqa, attn_kv_a_norm and attn_kv_b, or the split attn_k_b / attn_v_b in the
    transposed orientation) loads into the same model: identical logits."""
    import numpy as np
    from openmini_v1_b200.gguf.reader import GGUFReader
    from openmini_v1_b200.gguf.writer import GGUFWriter
    from openmini_v1_b200.models.loader import load_gguf_model, save_gguf_model
    for q_lora in (0, 48):
        c = _cfg()
        c.dtype = "float32"
        c.mla.q_lora_rank = q_lora
        m = DecoderLM(c, device="cpu", seed=7)
        p = str(tmp_path / f"mla{q_lora}.gguf")
        save_gguf_model(m, p)
        r = GGUFReader(p)
        assert r.architecture == "deepseek2" and ("blk.0.attn_q_a.weight" in r.tensors) == bool(q_lora)
        got = load_gguf_model(p)
        assert got.cfg.mla.enabled and got.cfg.mla.q_lora_rank == q_lora and got.cfg.mla.qk_nope_dim == 32
        want = _logits(m)
        assert (_logits(got) - want).abs().max().item() < 1e-4 * max(1.0, want.abs().max().item())
        # the split form: attn_k_b stored [H, 512, dn] (transposed), attn_v_b [H, dv, 512]
        p2 = str(tmp_path / f"mla{q_lora}_split.gguf")
        w = GGUFWriter(p2, "deepseek2")
        for k, v in r.metadata.items():
            if k not in ("general.architecture", "general.alignment"):
                w.add_kv(k, v)
        H = c.num_heads
        for name, t in r.tensors.items():
            a = t.to_numpy()
            if name.endswith("attn_kv_b.weight"):
                kvb = a.reshape(H, 32 + 32, 512)
                w.add_tensor(name.replace("kv_b", "k_b"), np.ascontiguousarray(kvb[:, :32].transpose(0, 2, 1)))
                w.add_tensor(name.replace("kv_b", "v_b"), np.ascontiguousarray(kvb[:, 32:]))
            else:
                w.add_tensor(name, a)
        w.write()
        assert (_logits(load_gguf_model(p2)) - want).abs().max().item() < 1e-4 * max(1.0, want.abs().max().item())


def test_mla_low_rank_query_matches_reference():
    c = _cfg()
    c.mla.q_lora_rank = 48
    m = DecoderLM(c, device="cpu", seed=3)
    T = 9
    i32 = dict(dtype=torch.int32)
    fb = ForwardBatch(torch.arange(T, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                      torch.arange(1, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                      torch.tensor([T - 1]))
    L = m.layers[0]
    assert "mla_q_a" in L and "mla_q" not in L
    a = torch.randn(T, c.hidden_size, generator=torch.Generator().manual_seed(1))
    got = mla_attention(m, 0, L, a, fb, m.allocate_kv(1))
    want = mla_reference_layer(m, L, a, fb.positions)
    assert (got - want).abs().max().item() < 1e-4 * max(1.0, want.abs().max().item())
