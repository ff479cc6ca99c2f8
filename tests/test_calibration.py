"""Calibration fits, chain widths and the small core helpers, against the reference's pure-Python core as an oracle.

The oracle is the unmodified ``eagle-harness`` installed under ``baseline/_ref`` (skipped when absent). The fitted
files must be byte-identical for the same raw timings, since both sides read each other's calibration directories.
"""

import json
import os
import random
import sys

import numpy as np
import pytest

from eagle4_b200.core import calibration as cal
from eagle4_b200.core import chain_width as cw
from eagle4_b200.core.cost_table import load_cost_tables
from eagle4_b200.core.limits import ComputeIntensity, draft_query_lens, verify_buckets

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def oracle():
    if not os.path.isdir(os.path.join(REF, "eagle_harness")):
        pytest.skip("reference package not installed under baseline/_ref")
    sys.path.insert(0, REF)
    try:
        import eagle_harness.core.calibration as rcal
        import eagle_harness.core.chain_width as rcw
        import eagle_harness.core.limits as rlim
    finally:
        sys.path.remove(REF)
    return rcal, rcw, rlim


def _raw(root, bs, intensity, rng, *, step=256, stop=4096, top_k=4, verify=16, loop_top_m=16, layers=16):
    paths = cal.CalibrationPaths(root)
    params = cal.MeasureParams(context_step=step, context_stop=stop, batch_size=bs, verify_num=verify,
                               node_top_k=top_k, loop_top_m=loop_top_m, repeat_cnt=8)
    paths.write_measure_params(params)
    lens = {"slm": [q for q in draft_query_lens(bs, intensity) if q <= top_k],
            "llm": [q for q in verify_buckets(bs, intensity) if q <= max(verify, loop_top_m)]}
    for model, qs in lens.items():
        for q in qs:
            recs_c, recs_m = [], []
            for kv in range(step // 2, stop + 1, step // 32):
                for _ in range(3):
                    attn = (2.0 + 0.001 * kv * (1 + 0.05 * q)) * rng.uniform(0.9, 1.1)
                    if rng.random() < 0.05:
                        attn *= 5  # an outlier
                    recs_c.append(cal.MeasureRecord(int(attn * 8), 8, q, kv, f"cache_{model}", bs))
                    model_us = (9000 + 30 * q) * rng.uniform(0.97, 1.03) + attn * layers
                    recs_m.append(cal.MeasureRecord(int(model_us * 4), 4, q, kv, f"model_{model}", bs))
            cal.save_jsonl(os.path.join(paths.raw(bs, "cache", model), f"cache_qo_len_{q}.jsonl"), recs_c)
            cal.save_jsonl(os.path.join(paths.raw(bs, "model", model), f"model_qo_len_{q}.jsonl"), recs_m)
    return paths, params


def _tree(root):
    out = {}
    for d, _, names in os.walk(root):
        for n in names:
            with open(os.path.join(d, n), encoding="utf-8") as f:
                out[os.path.relpath(os.path.join(d, n), root)] = f.read()
    return out


@pytest.mark.parametrize("intensity", [ComputeIntensity.HIGH, ComputeIntensity.CHAIN])
def test_fits_byte_identical(oracle, tmp_path, intensity):
    rcal, _, rlim = oracle
    rint = rlim.ComputeIntensity(intensity.value)
    for bs in (1, 8, 32):
        rng = random.Random(bs)
        mine, params = _raw(str(tmp_path / "mine"), bs, intensity, rng)
        theirs = str(tmp_path / "theirs")
        os.makedirs(theirs, exist_ok=True)
        import shutil
        shutil.copytree(os.path.join(mine.data_path, "test"), os.path.join(theirs, "test"), dirs_exist_ok=True)
        cal.fit_batch(mine, params, intensity, cal.AttentionShape(1), cal.AttentionShape(16, 4, 1024))
        rparams = rcal.MeasureParams(**{k: getattr(params, k) for k in params.__dataclass_fields__})
        rcal.fit_batch(rcal.CalibrationPaths(theirs), rparams, rint, rcal.AttentionShape(1),
                       rcal.AttentionShape(16, 4, 1024))
    a, b = _tree(os.path.join(mine.data_path, "cost")), _tree(os.path.join(theirs, "cost"))
    assert sorted(a) == sorted(b) and a == b
    assert sorted(load_cost_tables(mine.cost)) == [1, 8, 32]


def test_step_timing_fits_identical(oracle, tmp_path):
    rcal, _, rlim = oracle
    rng = random.Random(3)
    intensity = ComputeIntensity.HIGH
    params = cal.MeasureParams(256, 4096, 4, 16, 4, 16, 8)
    d = [cal.StepTiming(q, kv, 300 + q + kv * 0.01 * rng.uniform(0.99, 1.01))
         for q in draft_query_lens(4, intensity) if q <= 4 for kv in range(128, 4097, 128)]
    t = [cal.StepTiming(q, kv, 9000 + 20 * q + kv * 0.2 * rng.uniform(0.99, 1.01))
         for q in verify_buckets(4, intensity) if q <= 16 for kv in range(128, 4097, 128)]
    cal.fit_step_timings(cal.CalibrationPaths(str(tmp_path / "a")), params, intensity, (cal.AttentionShape(1), d),
                         (cal.AttentionShape(16), t))
    conv = lambda xs: [rcal.StepTiming(x.query_length, x.cache_length, x.time_us) for x in xs]
    rcal.fit_step_timings(rcal.CalibrationPaths(str(tmp_path / "b")), rcal.MeasureParams(256, 4096, 4, 16, 4, 16, 8),
                          rlim.ComputeIntensity.HIGH, (rcal.AttentionShape(1), conv(d)),
                          (rcal.AttentionShape(16), conv(t)))
    assert _tree(str(tmp_path / "a")) == _tree(str(tmp_path / "b"))


def test_remove_outliers_identical(oracle):
    rcal = oracle[0]
    rng = np.random.default_rng(0)
    for n in (1, 2, 5, 40, 200):
        for spread in (0.0, 0.05, 0.5):
            data = list(100 * (1 + spread * rng.standard_normal(n)))
            if n > 5:
                data[0] *= 8
            for conv in (0.2, 0.35):
                a = cal.remove_outliers(data, convergence_threshold=conv)
                b = rcal.remove_outliers(data, convergence_threshold=conv)
                assert (a[0], list(a[1]), a[2]) == (b[0], [float(x) for x in b[1]], b[2])


def test_sweep_plan_and_attention_shape(oracle):
    rcal = oracle[0]
    for step, stop, fast in ((256, 4096, False), (1024, 65536, True), (512, 16384, True), (64, 2048, False)):
        p = cal.MeasureParams(step, stop, 1, 16, 4, 16, 8, enable_fast_measurement=fast)
        rp = rcal.MeasureParams(step, stop, 1, 16, 4, 16, 8, enable_fast_measurement=fast)
        assert cal.CacheSweepPlan.from_params(p).__dict__ == rcal.CacheSweepPlan.from_params(rp).__dict__
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


def test_chain_widths_identical(oracle):
    _, rcw, _ = oracle
    rng = random.Random(5)
    for trial in range(30):
        n = rng.randint(3, 15)
        drafts = 1000
        counts = sorted((rng.randint(0, drafts) for _ in range(n)), reverse=True)
        prof, rprof = cw.AcceptProfile.from_counts(drafts, counts), rcw.AcceptProfile.from_counts(drafts, counts)
        rounds = {b: {w: rng.uniform(5000, 30000) * (1 + 0.02 * w * b / 8) for w in range(0, 17)}
                  for b in (1, 4, 16, 64, 256)}
        for allow in (False, True):
            assert cw.served_width_schedule(rounds, prof, 16, 512, allow_no_spec=allow) == \
                rcw.served_width_schedule(rounds, rprof, 16, 512, allow_no_spec=allow)
        tree = {b: {w: (rng.uniform(5000, 30000) * (1 + 0.05 * w * b / 8), rng.uniform(1, 1 + w / 4),
                        rng.randint(1, 200)) for w in (1, 4, 8, 16)} for b in (1, 8, 32, 64, 128, 256)}
        assert cw.served_tree_schedule(tree, 16, 512) == rcw.served_tree_schedule(tree, 16, 512)


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
