"""TokenSpeed cost measurement on the host: the round-robin shapes of a measurement run, and timings a host reports
turned into cost tables the round policy accepts."""

import os

import pytest

from eagle4_b200.core.calibration import AttentionShape
from eagle4_b200.core.cost_table import cost_model_problem, load_cost_tables
from eagle4_b200.core.limits import ComputeIntensity
from eagle4_b200.plugins.tokenspeed.measurement import CostMeasurement, MeasurePolicy


def test_measure_policy_cycles_the_sweep_at_the_measured_batch_only():
    p = MeasurePolicy(4, ComputeIntensity.HIGH, node_top_k=4)
    shapes = [p.next_round(4) for _ in range(len(p.drafts) * len(p.verifies))]
    assert {s[0] for s in shapes} == set(p.drafts) and {s[1] for s in shapes} == set(p.verifies)
    assert p.next_round(3) is None
    p.restart()
    assert p.next_round(4) == shapes[0]


def test_host_timings_fit_into_cost_tables(tmp_path):
    m = CostMeasurement(str(tmp_path), batch_size=2, intensity=ComputeIntensity.HIGH, node_top_k=4, verify_num=16,
                        context_step=512, context_stop=2048, draft=AttentionShape(1), target=AttentionShape(16),
                        samples=2)
    policy = MeasurePolicy(2, ComputeIntensity.HIGH, node_top_k=4)
    assert not m.record("llm", 3, 8, 100, 1.0)  # another batch size does not count
    context = 100
    while not m.complete:
        dw, vw = policy.next_round(2)
        # a plausible host: the draft step ~1/25 of the target forward, both growing with width and context
        assert m.record("slm", 2, dw, context, 380.0 + 15.0 * dw + 0.01 * context)
        assert m.record("llm", 2, vw, context, 10000.0 + 90.0 * vw + 0.2 * context)
        context += 7
        if context > 2048:
            context = 100
    path = m.write()
    tables = load_cost_tables(path)
    assert list(tables) == [2] and cost_model_problem(tables[2], target_is_moe=False) is None
    assert os.path.isdir(os.path.join(str(tmp_path), "cost", "bs_2"))
    with pytest.raises(ValueError):
        CostMeasurement(str(tmp_path / "x"), batch_size=1, intensity=ComputeIntensity.HIGH, node_top_k=4,
                        verify_num=16, context_step=512, context_stop=1024, draft=AttentionShape(1),
                        target=AttentionShape(16)).write()


def test_tokenspeed_algorithm_config():
    import pytest

    from eagle4_b200.core.config import Mode
    from eagle4_b200.plugins.tokenspeed.adapter import HarnessDrafter
    from eagle4_b200.plugins.tokenspeed.config import parse_algorithm_config

    static = parse_algorithm_config({"mode": "static"})
    assert static.harness.mode is Mode.STATIC and not static.sampled_proposals
    chain = parse_algorithm_config({"intensity": "chain_intensity", "chain_width_table": [[1, 6], [16, 4], [64, 2]]})
    assert chain.fully_scheduled and chain.chain_width(1) == 6 and chain.chain_width(20) == 4
    assert chain.chain_width(512) == 2
    part = parse_algorithm_config({"intensity": "chain_intensity", "data_path": "/cal",
                                   "chain_width_table": [[8, 4]]})
    assert not part.fully_scheduled and part.chain_width(4) is None
    assert parse_algorithm_config({"data_path": "/cal", "sampled_proposals": True}).sampled_proposals
    bad = [
        {},                                                          # serve mode without data or a full table
        {"mode": "static", "sampled_proposals": True},               # sampling is a serve-mode option
        {"mode": "calibrate"},                                       # calibrate writes under data_path
        {"data_path": "/cal", "chain_width_table": [[1, 4]]},        # a table needs chain intensity
        {"intensity": "chain_intensity", "chain_width_table": [[4, 4], [2, 3]]},  # not increasing
        {"intensity": "chain_intensity", "chain_width_table": [[1, 1]]},           # width below 2
        {"mode": "static", "sampled_proposals": "yes"},
        {"mode": "static", "unknown_key": 1},
    ]
    for cfg in bad:
        with pytest.raises(ValueError):
            parse_algorithm_config(cfg)
    drafter = HarnessDrafter()
    assert drafter.configure_algorithm({"mode": "static"}).harness.mode is Mode.STATIC
