"""End-to-end engine on the GPU: native kernels, CUDA-graph decode, multi-step decode."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from openmini_v1_b200 import ops
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.models.config import ModelConfig, tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch


def _small_cfg():
    c = tiny()
    c.dtype = "bfloat16"
    c.num_layers = 3
    c.hidden_size = 512
    c.num_heads = 8
    c.num_kv_heads = 2
    c.head_dim = 64
    c.intermediate_size = 1024
    return c


def _prompts(n, seed=0, lo=5, hi=90):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        L = int(torch.randint(lo, hi, (1,), generator=g))
        out.append(torch.randint(0, 32000, (L,), generator=g).tolist())
    return out


@pytest.mark.parametrize("fmt", ["bf16", "q4", "int8"])
def test_gpu_logits_match_cpu_oracle(fmt):
    cfg = _small_cfg()
    m_gpu = DecoderLM(cfg, device="cuda", seed=3, weight_format=fmt)
    cfg_cpu = ModelConfig.from_dict(cfg.to_dict())
    cfg_cpu.dtype = "float32"
    m_cpu = DecoderLM(cfg_cpu, device="cpu", materialize=False)
    m_cpu.embed = m_gpu.embed.float().cpu()
    m_cpu.lm_head = m_gpu.lm_head.float().cpu()
    m_cpu.norm = m_gpu.norm.float().cpu()
    m_cpu.layers = [{k: (v.dequantize() if hasattr(v, "dequantize") else v).float().cpu() for k, v in L.items()}
                    for L in m_gpu.layers]
    toks = _prompts(1, seed=1, lo=40, hi=41)[0]
    T = len(toks)
    res = []
    for m, dev in ((m_gpu, "cuda"), (m_cpu, "cpu")):
        kv = m.allocate_kv(8)
        i32 = dict(dtype=torch.int32, device=dev)
        fb = ForwardBatch(torch.tensor(toks, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                          torch.arange(8, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                          torch.tensor([T - 1], device=dev))
        res.append(m.logits(m(fb, kv)).float().cpu())
    torch.cuda.synchronize()
    ops.check_status()
    cos = torch.nn.functional.cosine_similarity(res[0], res[1]).item()
    assert cos > 0.995, cos


def test_engine_graph_equals_eager():
    cfg = _small_cfg()
    prompts = _prompts(5, seed=2)
    sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
    outs = []
    for graphs in (False, True):
        m = DecoderLM(cfg, device="cuda", seed=5)
        eng = LLMEngine(m, EngineConfig(max_num_seqs=8, max_model_len=256, use_cuda_graph=graphs,
                                        graph_batch_sizes=[1, 2, 4, 8]))
        outs.append([r.output_token_ids for r in eng.generate(prompts, sp)])
    assert outs[0] == outs[1]
    ops.check_status()


def test_engine_sampling_and_prefix_cache():
    cfg = _small_cfg()
    m = DecoderLM(cfg, device="cuda", seed=6)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=8, max_model_len=512, graph_batch_sizes=[1, 2, 4, 8]))
    base = _prompts(1, seed=3, lo=64, hi=65)[0]
    sp = SamplingParams(temperature=0.7, top_p=0.9, top_k=50, max_tokens=8, ignore_eos=True, seed=123)
    r1 = eng.generate([base], sp)[0]
    r2 = eng.generate([base], sp)[0]  # prefix-cache hit on the first 48 tokens
    assert r1.output_token_ids == r2.output_token_ids
    assert eng.bm.prefix_hit_rate() > 0


def test_multi_step_decode_matches_single_step():
    cfg = _small_cfg()
    prompts = _prompts(3, seed=4)
    sp = SamplingParams(temperature=0.0, max_tokens=10, ignore_eos=True)
    m = DecoderLM(cfg, device="cuda", seed=7)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_model_len=256, enable_prefix_cache=False,
                                    graph_batch_sizes=[1, 2, 4]))
    ref_out = [r.output_token_ids for r in eng.generate(prompts, sp)]
    reqs = [eng.add_request(f"m{i}", p, sp) for i, p in enumerate(prompts)]
    eng.step()  # prefill -> first token
    h = eng.begin_multi_decode(9)
    for _ in range(9):
        eng.multi_decode_step(h)
    eng.finish_multi_decode(h)
    assert [r.output_token_ids for r in reqs] == ref_out
