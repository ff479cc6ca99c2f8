"""RoundPlan (runtime/round_plan.py): a tree round's stop rule fixed at the round's start restates the cost model's
per-depth decisions exactly; the engine's draft loop runs from it, and its check mode counts no disagreement."""

import random

import pytest
import torch

from eagle4_b200.core.config import harness_config_from_dict
from eagle4_b200.runtime.engine import Engine
from eagle4_b200.runtime.round_plan import DECIDE, KIND, LAST, RoundCheck, round_plan

from test_engine_cpu import _models
from test_serve_policy import _write_tables


def _engine(tmp_path, steps=6, ratio=20.0):
    _write_tables(str(tmp_path), bss=(1, 2), widths=(1, 8, 16), ratio=ratio)
    cfg = harness_config_from_dict({"data_path": str(tmp_path)})
    tgt, drf = _models()
    return Engine(tgt, drf, max_reqs=2, max_len=160, steps=steps, top_k=2, verify_tokens=16, config=cfg)


@pytest.mark.parametrize("ratio", [6.0, 20.0, 80.0])
def test_plan_restates_the_cost_model(tmp_path, ratio):
    eng = _engine(tmp_path, ratio=ratio)
    model = eng.policy.cost
    rnd = random.Random(1)
    checked = 0
    for bs in (1, 2):
        for context in (64, 1500, 3000):
            tiny = model.state.tiny
            row = model.draft_cost_row(bs, context)
            past = model.history_verify_num(bs)
            check = RoundCheck()
            check.begin(model)
            plan = round_plan(model, bs, context, eng.steps - 1)
            after = model.state.tiny
            # the per-depth calls in the engine's order: a DECIDE sets the one-request flag that later depths read
            model.state.tiny = tiny
            kinds = []
            for d in range(eng.steps - 1):
                kinds.append(KIND[model.width_step(d)])
                if kinds[-1] == DECIDE:
                    model.state.tiny = bs == 1
            assert plan.kind == kinds and model.state.tiny == after
            assert plan.budget == model.deltas_budget(past) - 1
            for d, kind in enumerate(plan.kind):
                if kind != DECIDE:
                    continue
                first = check._first
                for _ in range(50):
                    deltas = sorted(rnd.uniform(0.0, 3.0) for _ in range(model.node_top_k + 1))
                    check._first = first
                    check.compare(model, plan, d, bs, past, row, deltas)
                    checked += 1
            assert check.disagreed == 0, check.notes
            if LAST in plan.kind:
                assert plan.min_depth <= plan.kind.index(LAST) + 1
    assert checked > 0
    t = plan.tensors("cpu")
    assert t["kind"].dtype == torch.int32 and t["bar"].dtype == torch.float64 and t["terms"].shape == (3,)


def test_engine_rounds_follow_the_plan(tmp_path):
    eng = _engine(tmp_path)
    eng.round_check = RoundCheck()
    g = torch.Generator().manual_seed(3)
    prompts = torch.randint(0, eng.target.cfg.vocab_size, (2, 40), generator=g).tolist()
    out = eng.generate(prompts, 24, speculative=True)
    tgt, drf = _models()
    plain = Engine(tgt, drf, max_reqs=2, max_len=160, steps=6, top_k=2, verify_tokens=16).generate(
        prompts, 24, speculative=False)
    assert out == plain
    assert eng.round_check.decided > 0
    assert eng.round_check.disagreed == 0, eng.round_check.notes
