"""Benchmark framework on CPU: scenarios run through the real engine, percentiles,
exporters and the regression gate."""
import json

from openmini_v1_b200.benchmark import SCENARIOS, Scenario, check_regression, percentile, run_scenario
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM


def test_percentile():
    assert percentile([1, 2, 3, 4], 50) == 2.5
    assert percentile([5], 99) == 5
    assert percentile(list(range(101)), 95) == 95


def test_run_scenarios_and_regression():
    cfg = tiny()
    eng = LLMEngine(DecoderLM(cfg, device="cpu", seed=0), EngineConfig(max_num_seqs=8, max_model_len=256))
    res = run_scenario(eng, Scenario("t", 6, (8, 24), 5), cfg.vocab_size)
    assert res.completed == 6 and res.output_tokens == 30
    assert res.ttft_ms.count == 6 and res.tpot_ms.count == 6 and res.e2e_ms.p99 >= res.e2e_ms.p50 > 0
    burst = run_scenario(eng, Scenario("b", 6, (8, 16), 3, arrival="burst", burst_size=3, burst_gap_s=0.02),
                         cfg.vocab_size)
    assert burst.completed == 6
    rate = run_scenario(eng, Scenario("r", 4, (8, 16), 3, arrival="rate", rate_per_s=200.0), cfg.vocab_size)
    assert rate.completed == 4
    j = json.loads(res.to_json())
    assert check_regression(res, j) == []
    worse = dict(j, throughput_tok_s=j["throughput_tok_s"] * 2)
    assert any("throughput" in f for f in check_regression(res, worse))
    assert "ttft_ms_p99" in res.to_csv() and 'quantile="p50"' in res.to_prometheus()
    txt = res.to_text()
    assert "scenario t: 6/6 requests" in txt and "TTFT" in txt and "p99" in txt
    import tempfile, os
    with tempfile.TemporaryDirectory() as d:
        paths = res.export_all(os.path.join(d, "run"))
        assert [p.rsplit(".", 1)[1] for p in paths] == ["json", "csv", "prom", "txt"]
        assert json.load(open(paths[0]))["completed"] == 6
    assert {"short", "medium", "long", "ultra", "multi_user", "burst"} <= set(SCENARIOS)
