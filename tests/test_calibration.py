"""Calibration fits, chain widths and the small core helpers. (Byte-identity of the fitted files with the reference's,
the outlier filter, sweep plans and chain-width schedules are checked against the reference's golden traces in
``test_core_oracle.py``.)"""

import json
import os
import random

import pytest

from eagle4_b200.core import calibration as cal
from eagle4_b200.core import chain_width as cw


def test_sweep_plan_and_attention_shape():
    with pytest.raises(ValueError):
        cal.CacheSweepPlan.from_params(cal.MeasureParams(100, 4096, 1, 16, 4, 16, 8))

    class C:
        num_hidden_layers = 8
        layer_types = ["linear_attention"] * 6 + ["full_attention", "sliding_attention"]
        sliding_window = 512

    assert cal.attention_shape(C()) == cal.AttentionShape(2, 1, 512)


def _random_table(rng, bs, widths):
    from eagle4_b200.core.cost_table import BatchCostTable, CostCurve, IntervalCost
    ivs = []
    for _ in range(3):
        base = rng.uniform(8000, 12000) * (1 + 0.01 * bs)
        tv = [base * (1 + 0.004 * bs * (w - 1) + rng.uniform(0, 0.01)) for w in widths]
        dv = [base / rng.uniform(8, 20)]
        ivs.append(IntervalCost(CostCurve.from_values(tv, [w - 1 for w in widths]), CostCurve.from_values(dv, [0])))
    return BatchCostTable(batch_size=bs, intervals=tuple(ivs), cache_length_start=256, cache_length_step=256,
                          target_max_qo_len_query=16, target_max_qo_len_cache=16, draft_max_qo_len=1,
                          model_ratio=(10.0,) * 3)


def test_chain_width_from_tables_and_files(tmp_path):
    rng = random.Random(1)
    widths = [1, 2, 4, 8, 16]
    table = _random_table(rng, 1, widths)
    prof = cw.AcceptProfile.from_counts(100, [90, 80, 70, 60, 50, 40, 30, 20, 10, 5, 2, 1, 0, 0, 0])
    w = cw.chain_width(table, prof, 16)
    assert w in widths
    cw.save_accept_profile(str(tmp_path), 100, [90, 80, 70])
    cw.save_round_times(str(tmp_path), [{"batch_size": 1, "width": 1, "round_us": 1000.0, "count": 5},
                                        {"batch_size": 1, "width": 4, "round_us": 1500.0, "count": 5}])
    sched = cw.chain_widths(str(tmp_path), 16, 8)
    assert sched == [(1, 8, 4)] and cw.width_at(sched, 3) == 4
    cw.merge_tree_rounds(str(tmp_path), [{"batch_size": 8, "width": 16, "round_us": 100.0, "accept": 3.0,
                                          "count": 9}])
    cw.merge_tree_rounds(str(tmp_path), [{"batch_size": 8, "width": 4, "round_us": 50.0, "accept": 2.0,
                                          "count": 9}])
    assert set(cw.load_tree_rounds(str(tmp_path))[8]) == {4, 16}
    with pytest.raises(ValueError):
        cw.AcceptProfile.from_counts(10, [5, 6])


def test_small_helpers(tmp_path):
    from eagle4_b200.core.candidate_calibration import load_candidate_crossover, save_candidate_crossover
    from eagle4_b200.core.models import target_is_moe
    from eagle4_b200.models.eagle4_structure import base_layer_overrides, latent_moe_config

    assert target_is_moe({"num_experts": 8}) and not target_is_moe({"num_experts": 0})
    assert base_layer_overrides({"enable_moe": True, "moe_architecture": "nemotron_latent_relu2", "use_rope": False}) \
        == {"hidden_act": "silu", "max_position_embeddings": 1}
    assert latent_moe_config({"hidden_act": "relu2"})["topk_group"] == 1
    ident = {"device": "NVIDIA B200", "candidates": 128}
    save_candidate_crossover(str(tmp_path), ident, 4096)
    assert load_candidate_crossover(str(tmp_path), ident) == 4096
    assert load_candidate_crossover(str(tmp_path), {"device": "other"}) is None
    (tmp_path / "candidate_topk.json").write_text(json.dumps({"identity": ident, "max_single_pass_elements": -1}))
    with pytest.raises(ValueError):
        load_candidate_crossover(str(tmp_path), ident)


def test_packaged_profile_selection(tmp_path, monkeypatch):
    from eagle4_b200.core import cost_profiles as cp
    from eagle4_b200.models import configs

    target = configs.qwen38_27b().to_hf()
    draft = configs.qwen38_draft(configs.qwen38_27b()).to_hf()
    monkeypatch.setattr(cp, "PROFILES", tmp_path)
    cp.write_profile(str(tmp_path / "b200"), devices=["NVIDIA B200"], tp_size=1, target_config=target,
                     draft_config=draft)
    setup = dict(device_name="NVIDIA B200", tp_size=1, dtype="bfloat16", quantization=None, target_config=target,
                 draft_config=draft)
    assert cp.packaged_cost_profile(**setup) == str(tmp_path / "b200")
    assert cp.packaged_cost_profile(**dict(setup, tp_size=2)) is None
    assert cp.packaged_cost_profile(**dict(setup, target_config=dict(target, hidden_size=4096))) is None


def test_shipped_b200_profile_matches_the_named_shapes_and_passes_the_cost_model():
    from eagle4_b200.core import cost_profiles as cp
    from eagle4_b200.core.cost_table import cost_model_problem, load_cost_tables
    from eagle4_b200.models import configs

    target = configs.qwen38_27b()
    setup = dict(device_name="NVIDIA B200", tp_size=1, dtype="bfloat16", quantization=None,
                 target_config=target.to_hf(), draft_config=configs.qwen38_draft(target).to_hf())
    path = cp.packaged_cost_profile(**setup)
    assert path is not None and path.endswith("qwen3.8-27b-b200-tp1")
    assert cp.packaged_cost_profile(**dict(setup, device_name="NVIDIA H100 80GB HBM3")) is None
    tables = load_cost_tables(os.path.join(path, "cost"))
    assert sorted(tables) == [1, 2, 4, 8]
    assert all(cost_model_problem(t, target_is_moe=False) is None for t in tables.values())
