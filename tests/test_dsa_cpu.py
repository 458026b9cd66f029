"""Dynamic Sparse Attention on CPU: indexer scores / top-k selection against
direct formulas, and a tiny DSA model through the engine. With top_k at least
the context length the sparse path must equal dense attention; with a small
top_k it must still generate deterministically."""
import dataclasses

import torch

from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models import dsa
from openmini_v1_b200.models.config import DSAConfig, tiny
from openmini_v1_b200.models.llama import DecoderLM


def test_topk_ref_ties_and_short_rows():
    s = torch.tensor([[1.0, 3.0, 3.0, 2.0, 3.0, -1.0], [5.0, 4.0, 0, 0, 0, 0]])
    idx, n = dsa.topk_ref(s, torch.tensor([6, 2]), 2)
    assert n.tolist() == [2, 2]
    assert idx[0].tolist() == [1, 2]           # equal scores: lowest positions first
    assert sorted(idx[1].tolist()) == [0, 1]   # context shorter than k keeps everything


def test_index_scores_formula():
    g = torch.Generator().manual_seed(0)
    H, Di, n = 3, 64, 37
    icache = torch.randn(4, 16, Di, generator=g)
    bt = torch.tensor([[2, 0, 3, 1]], dtype=torch.int32)
    qi = torch.randn(1, H * Di, generator=g)
    wi = torch.randn(1, H, generator=g)
    out = dsa.index_scores_ref(qi, wi, icache, bt, torch.tensor([0]), torch.tensor([n]), H, 40)
    keys = torch.stack([icache[int(bt[0, j // 16]), j % 16] for j in range(n)])
    want = (torch.relu(qi.view(H, Di) @ keys.t()) * wi[0][:, None]).sum(0)
    assert torch.allclose(out[0, :n], want, atol=1e-5)
    assert torch.isinf(out[0, n:]).all()


def _dsa_model(top_k, threshold=8, seed=0):
    cfg = dataclasses.replace(tiny(), dsa=DSAConfig(enabled=True, indexer_heads=2, indexer_dim=64, top_k=top_k,
                                                    threshold=threshold))
    return DecoderLM(cfg, device="cpu", seed=seed)


def test_dsa_full_topk_equals_dense():
    m = _dsa_model(top_k=512)
    dense = DecoderLM(tiny(), device="cpu", seed=0, materialize=False)
    dense.layers = [{k: v for k, v in L.items() if k != "indexer"} for L in m.layers]
    for a in ("embed", "norm", "lm_head"):
        if hasattr(m, a):
            setattr(dense, a, getattr(m, a))
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, 32000, (20,), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    a = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128)).generate([prompt], sp)[0]
    b = LLMEngine(dense, EngineConfig(max_num_seqs=2, max_model_len=128)).generate([prompt], sp)[0]
    assert a.output_token_ids == b.output_token_ids


def test_dsa_sparse_generates():
    m = _dsa_model(top_k=8)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, 32000, (24,), generator=g).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    a = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128)).generate([prompt], sp)[0]
    b = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=128)).generate([prompt], sp)[0]
    assert len(a.output_token_ids) == 8 and a.output_token_ids == b.output_token_ids
