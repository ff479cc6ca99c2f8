"""The core algorithm against the reference's own pure-Python core run as an oracle (identical decisions).

The reference package is the unmodified ``eagle-harness`` installed under ``baseline/_ref``; these tests are skipped
when it is absent.
"""

import os
import random
import sys

import pytest
import torch

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def oracle():
    if not os.path.isdir(os.path.join(REF, "eagle_harness")):
        pytest.skip("reference package not installed under baseline/_ref")
    sys.path.insert(0, REF)
    try:
        import eagle_harness.core.cost_model as cm
        import eagle_harness.core.cost_table as ct
        import eagle_harness.core.draft_tree as dt
        import eagle_harness.core.limits as lim
        import eagle_harness.core.live_costs as lc
    finally:
        sys.path.remove(REF)
    return {"cm": cm, "ct": ct, "lim": lim, "lc": lc, "dt": dt}


def _curves(rng, widths, draft_ratio):
    base = rng.uniform(8000, 12000)
    tv = [base * (1 + 0.02 * (w - 1) ** 0.8 + rng.uniform(-0.01, 0.01)) for w in widths]
    tv[0] = base
    dv = [base / draft_ratio]
    return tv, dv


def _tables(mod_ct, rng, bss=(1, 4, 8, 32, 128, 512), widths=(1, 8, 16, 32), ratio=20.0, intervals=3):
    tables = {}
    for bs in bss:
        ivs, ratios = [], []
        for _ in range(intervals):
            scale = 1 + bs / 64
            tv, dv = _curves(rng, widths, ratio)
            tv = [v * scale ** (0.3 * (w > 1)) for v, w in zip(tv, widths)]
            tgt = mod_ct.CostCurve(tuple(tv), tuple(round(v / tv[0], 4) for v in tv), tuple(w - 1 for w in widths),
                                   (), ())
            dr = mod_ct.CostCurve(tuple(dv), (1.0,), (0,), (), ())
            ivs.append(mod_ct.IntervalCost(tgt, dr))
            ratios.append(round(tv[0] / dv[0], 4))
        tables[bs] = mod_ct.BatchCostTable(bs, 1024, 1024, widths[-1], widths[-1], 1, tuple(ivs), tuple(ratios))
    return tables


def _mirror(tables, ct_mod):
    out = {}
    for bs, t in tables.items():
        ivs = tuple(ct_mod.IntervalCost(ct_mod.CostCurve(iv.target.value, iv.target.ratio, iv.target.index),
                                        ct_mod.CostCurve(iv.draft.value, iv.draft.ratio, iv.draft.index))
                    for iv in t.intervals)
        out[bs] = ct_mod.BatchCostTable(t.batch_size, t.cache_length_start, t.cache_length_step,
                                        t.target_max_qo_len_query, t.target_max_qo_len_cache, t.draft_max_qo_len, ivs,
                                        t.model_ratio)
    return out


def test_limits_match(oracle):
    from eagle4_b200.core import limits as ours

    lim = oracle["lim"]
    for bs in (1, 2, 3, 7, 8, 9, 33, 64, 65, 512):
        for it in ours.ComputeIntensity:
            assert ours.verify_buckets(bs, it) == lim.verify_buckets(bs, lim.ComputeIntensity(it.value))
            assert ours.draft_query_lens(bs, it) == lim.draft_query_lens(bs, lim.ComputeIntensity(it.value))
    for bs in range(1, 600, 7):
        assert ours.nearest_cost_batch_size(bs, ours.COST_BATCH_SIZES) == lim.nearest_cost_batch_size(
            bs, lim.COST_BATCH_SIZES)
    for args in [(4, 12, 16, 1), (1, 15, 16, 1), (8, 31, 64, 4), (1, 6, 16, 16)]:
        assert ours.req_to_token_span(*args) == lim.req_to_token_span(*args)


@pytest.mark.parametrize("seed", range(6))
def test_cost_model_decisions_match(oracle, seed):
    from eagle4_b200.core import cost_model as ocm
    from eagle4_b200.core import cost_table as oct_

    rcm, rct, lim = oracle["cm"], oracle["ct"], oracle["lim"]
    rng = random.Random(seed)
    ratio = rng.choice([7.0, 15.0, 25.0, 40.0])
    ref_tables = _tables(rct, rng, ratio=ratio)
    our_tables = _mirror(ref_tables, oct_)
    it = rng.choice(["high_intensity", "low_intensity"])
    ref = rcm.CostModel(ref_tables, rcm.CostModelParams(), lim.ComputeIntensity(it), 4, 12, 16)
    ours = ocm.CostModel(our_tables, ocm.CostModelParams(), ocm.ComputeIntensity(it), 4, 12, 16)
    for _ in range(60):
        bs = rng.choice([1, 2, 5, 8, 16, 40, 200, 512])
        ctx = rng.randint(0, 5000)
        rv, ov = ref.verify_cost(bs, ctx), ours.verify_cost(bs, ctx)
        assert (rv.value, rv.index, rv.threshold) == (ov.value, ov.index, ov.threshold)
        rrow, orow = ref.draft_cost_row(bs, ctx), ours.draft_cost_row(bs, ctx)
        assert rrow.batch_size_ratio == orow.batch_size_ratio and rrow.adjust_cost_ratio == orow.adjust_cost_ratio
        for depth in range(12):
            deltas = sorted(rng.uniform(0, 3) for _ in range(5))
            past = ref.history_verify_num(bs)
            assert past == ours.history_verify_num(bs)
            a = ref.tree_width(depth, bs, past, rrow, deltas)
            b = ours.tree_width(depth, bs, past, orow, deltas)
            assert (a.width, a.verify_num, a.stop) == (b.width, b.verify_num, b.stop)
        scores = [1.001]
        for _ in range(40):
            scores.append(scores[-1] + rng.uniform(0, 0.9) * (0.97 ** len(scores)))
        req = rng.choice([16, 32, 8])
        lag = rng.random() < 0.5
        assert ref.verify_num_paged(scores, req, bs, ctx, lagged=lag) == ours.verify_num_paged(scores, req, bs, ctx,
                                                                                                 lagged=lag)
        vn = rng.choice([1, 4, 8, 16])
        ref.record_verify_num(bs, vn)
        ours.record_verify_num(bs, vn)
        assert ref.verify_count(bs, 40) == ours.verify_count(bs, 40)


def test_tree_policy_export_matches(oracle):
    from eagle4_b200.core import cost_model as ocm
    from eagle4_b200.core import cost_table as oct_

    rcm, rct, lim = oracle["cm"], oracle["ct"], oracle["lim"]
    rng = random.Random(11)
    ref_tables = _tables(rct, rng, ratio=18.0)
    ref = rcm.CostModel(ref_tables, rcm.CostModelParams(), lim.ComputeIntensity.HIGH, 4, 12, 16)
    ours = ocm.CostModel(_mirror(ref_tables, oct_), ocm.CostModelParams(), ocm.ComputeIntensity.HIGH, 4, 12, 16)
    a, b = ref.tree_policy_costs(), ours.tree_policy_costs()
    assert a.history_floors == b.history_floors and a.initial_widths == b.initial_widths
    for x, y in zip(a.batches, b.batches):
        assert x.cost_batch_size == y.cost_batch_size
        for ix, iy in zip(x.intervals, y.intervals):
            assert ix.depth_thresholds == iy.depth_thresholds
            assert ix.verify_cost_deltas == iy.verify_cost_deltas and ix.verify_tier == iy.verify_tier


def test_chain_stop_matches(oracle):
    from eagle4_b200.core import cost_model as ocm
    from eagle4_b200.core import cost_table as oct_

    rcm, rct, lim = oracle["cm"], oracle["ct"], oracle["lim"]
    rng = random.Random(5)
    widths = (1, 2, 4, 6, 8, 10, 12, 14, 16)
    ref_tables = _tables(rct, rng, widths=widths, ratio=30.0)
    ref = rcm.CostModel(ref_tables, rcm.CostModelParams(), lim.ComputeIntensity.CHAIN, 1, 15, 16)
    ours = ocm.CostModel(_mirror(ref_tables, oct_), ocm.CostModelParams(), ocm.ComputeIntensity.CHAIN, 1, 15, 16)
    assert ref.chain_rounds and ours.chain_rounds
    for bs in (1, 3, 16, 100, 512):
        for depth in range(15):
            d = [0.0, rng.uniform(0, 2)]
            assert ref.chain_stop(depth, bs, d) == ours.chain_stop(depth, bs, d)
    a, b = ref.chain_policy_costs(), ours.chain_policy_costs()
    for x, y in zip(a.batches, b.batches):
        for ix, iy in zip(x.intervals, y.intervals):
            assert [tuple(vars(t).values()) for t in ix] == [tuple(vars(t).values()) for t in iy]


def test_draft_tree_matches(oracle):
    from eagle4_b200.core.draft_tree import DraftTree, TreeShape

    rdt = oracle["dt"]
    k, depth, bs, H = 4, 6, 3, 8
    ref = rdt.DraftTree(rdt.TreeShape(k, depth), bs, H, torch.float32, torch.device("cpu"), max_verify=16)
    ours = DraftTree(TreeShape(k, depth), bs, H, torch.float32, "cpu", max_verify=16)
    g = torch.Generator().manual_seed(0)
    p0, t0, h0 = torch.rand(bs, k, generator=g), torch.randint(0, 100, (bs, k), generator=g), torch.rand(bs, H)
    for t in (ref, ours):
        t.stage_root(bs, p0, t0, h0)
        t.begin(bs)
    for step in range(1, depth):
        p = torch.rand(bs * k, k, generator=g)
        tk = torch.randint(0, 100, (bs * k, k), generator=g)
        hh = torch.rand(bs * k, H, generator=g)
        for t in (ref, ours):
            t.step(bs, step, p, tk, hh)
        assert torch.equal(ref.deltas, ours.deltas)
    for name in ("scores", "tokens", "parents", "front_scores", "best"):
        assert torch.equal(getattr(ref, name), getattr(ours, name))
    for count in (7, 15):
        a = ref.verify_rows_reference(bs, depth, count)
        b = ours.verify_rows_reference(bs, depth, count)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        ra, rb = ref.rank_reference(bs, depth, count), ours.rank_reference(bs, depth, count)
        assert torch.equal(ra[0], rb[0]) and torch.equal(ra[1], rb[1])


def test_live_costs_match(oracle, tmp_path):
    from eagle4_b200.core import live_costs as olc

    rlc, lim = oracle["lc"], oracle["lim"]
    widths = lambda b: lim.verify_buckets(b, lim.ComputeIntensity.HIGH)  # noqa: E731
    key_args = dict(gpu="NVIDIA B200", gpu_count=1, model="m:1", draft="d:2", engine="e", dtype="bf16")
    ref = rlc.LiveCosts(widths, key=rlc.CostKey(**key_args))
    ours = olc.LiveCosts(widths, key=olc.CostKey(**key_args))
    assert ref.key.digest == ours.key.digest
    rng = random.Random(3)
    for _ in range(400):
        b = rng.choice([1, 8, 32])
        w = ref.seed_width(b)
        assert w == ours.seed_width(b)
        width = w if w is not None else rng.choice(widths(b) + [0])
        ctx = rng.randint(0, 9000)
        us = rng.uniform(100, 20000) * (5 if rng.random() < 0.02 else 1)
        ref.record(b, width, ctx, us)
        ours.record(b, width, ctx, us)
        if rng.random() < 0.2:
            ref.record(b, 0, ctx, us / 20)
            ours.record(b, 0, ctx, us / 20)
    assert ref.to_dict() == ours.to_dict()
    for b in (1, 4, 8, 16, 32):
        assert ref.priced(b) == ours.priced(b)
    ta, tb = ref.tables(also=(4, 16)), ours.tables(also=(4, 16))
    assert sorted(ta) == sorted(tb)
    for b in ta:
        assert ta[b].model_ratio == tb[b].model_ratio
        assert [iv.target.value for iv in ta[b].intervals] == [iv.target.value for iv in tb[b].intervals]
    path = str(tmp_path / "c.json")
    ours.save(path)
    again = rlc.LiveCosts(widths, key=rlc.CostKey(**key_args))
    assert again.load(path) and again.to_dict() == ours.to_dict()
