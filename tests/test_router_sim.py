"""Routing-policy simulation on CPU (reference: evaluation/benchmark_agent_load_scheduler.py)."""
import json

import pytest

from nanovllm_self_b200.pd.multiprocess import router_sim
from nanovllm_self_b200.pd.multiprocess.agent_scheduler import RouterConfig


def _rows(lengths):
    return [{"id": f"r{i}", "prompt_ids": [0] * n_in, "input_tokens": n_in, "max_tokens": n_out,
             "session_id": f"s{i % 3}", "task_type": "mixed_agent"} for i, (n_in, n_out) in enumerate(lengths)]


def test_quantile_interpolates():
    assert router_sim.quantile([1, 2, 3, 4], 0.5) == 2.5
    assert router_sim.quantile([5], 0.99) == 5
    assert router_sim.quantile([0, 10], 0.9) == pytest.approx(9.0)


def test_burst_on_one_worker_serialises_the_service_times():
    rows = _rows([(400, 14), (800, 28), (4000, 14)])
    s = router_sim.simulate(rows, 1, "round_robin", "burst")["summary"]
    cfg = RouterConfig()
    svc = [cfg.base_request_overhead_s + i / cfg.prefill_tokens_per_s + o / cfg.decode_tokens_per_s
           + cfg.step_overhead_s * ((i >= cfg.long_input_threshold) + (o >= cfg.long_output_threshold))
           for i, o in [(400, 14), (800, 28), (4000, 14)]]
    assert s["makespan_s"] == pytest.approx(sum(svc))
    assert s["queue_wait_s"]["max"] == pytest.approx(svc[0] + svc[1])
    assert s["worker_load_imbalance"] == pytest.approx(1.0)


def test_load_aware_balances_a_skewed_trace_better_than_round_robin():
    # every other request is long: round robin puts all long ones on worker 0
    rows = _rows([(4000, 256) if i % 2 == 0 else (64, 8) for i in range(40)])
    out = router_sim.compare(rows, 2, "burst")
    rr, la = out["policies"]["round_robin"], out["policies"]["load_aware"]
    assert la["makespan_s"] < rr["makespan_s"]
    assert la["worker_load_imbalance"] < rr["worker_load_imbalance"]
    assert out["vs_round_robin"]["load_aware"]["tok_s_over_round_robin"] > 1.0


def test_affinity_keeps_sessions_on_their_worker():
    rows = _rows([(100, 16)] * 30)
    s = router_sim.simulate(rows, 3, "affinity_load_aware", "rate", rate=1.0)["summary"]
    assert s["affinity_hit_rate"] == pytest.approx(1.0)


def test_cli_prints_every_policy(capsys):
    router_sim.main(["--workers", "2", "--trace", "agent", "--requests", "24", "--arrival", "rate", "--rate", "2"])
    out = json.loads(capsys.readouterr().out)
    assert set(out["policies"]) == {"round_robin", "load_aware", "affinity_load_aware"}
    assert out["requests"] == 24
