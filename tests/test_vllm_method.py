"""vLLM method pieces on the host: the method_config reader, the per-batch policy hooks, and the served-round
recording of the speculator (with a fake draft round)."""

import json
import os

import numpy as np
import pytest

from eagle4_b200.plugins.vllm.batch_policy import BatchPolicy
from eagle4_b200.plugins.vllm.config import parse_method_config


def test_method_config_defaults_and_refusals(tmp_path):
    m = parse_method_config({"mode": "serve"})
    assert (m.max_verify_width, m.node_top_k, m.tree_depth, m.depth_stop_gain) == (32, 4, 12, "derived")
    assert m.num_speculative_tokens == 31 and m.lookahead >= 48
    c = parse_method_config({"intensity": "chain_intensity"})
    assert (c.node_top_k, c.max_verify_width) == (1, 16)
    for bad in ({"node_top_k": 2.5}, {"max_verify_width": 65}, {"record_rounds": "yes"}, {"depth_stop_gain": -1},
                {"record_rounds": True}, {"not_a_key": 1}):
        with pytest.raises((ValueError, NotImplementedError)):
            parse_method_config(bad)
    with pytest.raises(NotImplementedError):  # a fixed gain needs the device depth stop
        parse_method_config({"depth_stop_gain": 0.5})
    assert parse_method_config({"depth_stop_gain": None}).depth_stop_gain is None
    r = parse_method_config({"record_rounds": True, "data_path": str(tmp_path)})
    assert r.record_rounds


def test_batch_policy_native_ranges_limit_and_budget():
    p = BatchPolicy(verify_batch_limit=32, schedule=[(1, 4, 8), (5, 8, 0), (9, 64, 4)], max_num_reqs=64)
    assert not p.suspend_drafting(3, None) and p.suspend_drafting(6, None) and p.suspend_drafting(40, None)
    drafts = np.array([7, 7, 3])
    assert p.verify_budget(["a", "b", "c"], drafts) is drafts  # width 8 at bs 3: nothing to cut
    ten = np.full(10, 7)
    assert np.array_equal(p.verify_budget(list(range(10)), ten), np.full(10, 3))  # width 4 at bs 10
    assert p.summary() == {"batches": 2, "trimmed": 1, "suspended": 2}
    assert not BatchPolicy().suspend_drafting(500, None)


def test_speculator_records_served_rounds(tmp_path):
    import torch

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.core.chain_width import load_tree_rounds
    from eagle4_b200.plugins.vllm.adapter import HarnessSpeculator

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=2, max_len=256)
    method = parse_method_config({"mode": "static", "data_path": str(tmp_path), "record_rounds": True,
                                  "max_verify_width": 8, "node_top_k": 2, "tree_depth": 4})
    spec = HarnessSpeculator.__new__(HarnessSpeculator)
    spec.load_model(llm.draft, max_reqs=2, max_len=256, method=method)
    assert spec.batch_policy.limit is None and not spec.suspend_drafting(2, [0, 1])
    host = llm.engine
    prompts = [torch.arange(5, 30), torch.arange(40, 52)]
    for b, p in enumerate(prompts):
        first, aux = host.prefill(b, p)
        spec.prefill_request(b, p, aux, int(first[0]))
    for _ in range(3):
        tokens, prow = spec.propose_tree([0, 1])
        w = tokens.shape[1]
        holder = {}

        def accept(out, t):
            acc, cnt, bonus, emitted = spec.accept_round([0, 1], t, prow, host.target.logits(out), None, round_us=900.0)
            holder["e"] = emitted
            return acc, cnt, bonus

        tk, acc, cnt, bonus, aux = host._verify_forward(2, w, tokens[:, 1:] if w > 1 else None, prow, None,
                                                        accept=accept)
        host.L[:2] += cnt.long()
        host.root[:2] = bonus
    spec.close()
    cells = load_tree_rounds(str(tmp_path))
    assert cells and 2 in cells and all(v[0] == 900.0 and v[1] >= 1 for v in cells[2].values())
    assert os.path.exists(os.path.join(str(tmp_path), "rounds", "tree.json"))
