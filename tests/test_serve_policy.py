"""Serve mode: the measured cost model sizes every round (offline tables or live costs) and the output still equals
plain greedy decoding."""

import json
import os

import torch

from eagle4_b200.core.config import harness_config_from_dict
from eagle4_b200.core.cost_table import CostCurve, write_interval
from eagle4_b200.runtime.engine import Engine
from eagle4_b200.runtime.policy import fit_width

from test_engine_cpu import _models


def _write_tables(root, bss=(1, 2), widths=(1, 8), ratio=20.0):
    for bs in bss:
        for i in range(2):
            tv = [1000.0 * (1 + 0.01 * (w - 1)) for w in widths]
            tgt = CostCurve.from_values(tv, [w - 1 for w in widths])
            dft = CostCurve.from_values([tv[0] / ratio], [0])
            kw = dict(batch_size=bs, cache_length_start=1024, cache_length_step=1024, max_query_length_query=widths[-1],
                      max_query_length_cache=widths[-1])
            write_interval(os.path.join(root, "cost", f"bs_{bs}", "model_llm", f"model_interval_{i}.json"), tgt, **kw)
            write_interval(os.path.join(root, "cost", f"bs_{bs}", "model_slm", f"model_interval_{i}.json"), dft,
                           **dict(kw, max_query_length_query=1))


def test_fit_width():
    assert fit_width(5, [16, 8, 1], 20) == 8
    assert fit_width(9, [16, 8, 1], 12) == 8
    assert fit_width(1, [16, 8, 1], 3) == 1


def test_offline_cost_model_rounds_equal_plain(tmp_path):
    _write_tables(str(tmp_path))
    cfg = harness_config_from_dict({"data_path": str(tmp_path)})
    tgt, drf = _models()
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, tgt.cfg.vocab_size, (2, 40), generator=g).tolist()
    eng = Engine(tgt, drf, max_reqs=2, max_len=128, steps=4, top_k=2, verify_tokens=8, config=cfg)
    assert eng.policy.cost is not None and eng.policy.live is None
    out = eng.generate(prompts, 20, speculative=True)
    plain = Engine(tgt, drf, max_reqs=2, max_len=128, steps=4, top_k=2, verify_tokens=8).generate(
        prompts, 20, speculative=False)
    assert out == plain
    assert eng.last_width in (1, 8)


def test_live_costs_seed_then_price(tmp_path):
    cfg = harness_config_from_dict({"cost_cache": str(tmp_path)})
    tgt, drf = _models()
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, tgt.cfg.vocab_size, (1, 24), generator=g).tolist()
    eng = Engine(tgt, drf, max_reqs=1, max_len=160, steps=4, top_k=2, verify_tokens=8, config=cfg)
    eng.tree_choice = None  # every round speculates: this test times the seed sweep
    live = eng.policy.live
    out = eng.generate(prompts, 40, speculative=True)
    plain = Engine(tgt, drf, max_reqs=1, max_len=160, steps=4, top_k=2, verify_tokens=8).generate(
        prompts, 40, speculative=False)
    assert out == plain
    # the seed sweep timed every captured width and the draft step of bucket 1
    assert live.seed_width(1) is None and live.ready(1)


def test_served_chain_policy_probes_then_serves_best():
    from eagle4_b200.runtime.policy import ServedChainPolicy

    p = ServedChainPolicy([2, 4, 8], block=2, explore=2, refresh=0)
    seen = []
    for _ in range(6):  # exploration: every width in blocks of two rounds
        w = p.width(1)
        seen.append(w)
        # width 4 gains 3 tokens in 1.2 units, width 8 gains 4 in 2.0, width 2 gains 1.5 in 1.0
        p.record(1, w, {2: 1.0, 4: 1.2, 8: 2.0}[w], {2: 1.5, 4: 3.0, 8: 4.0}[w])
    assert sorted(seen) == [2, 2, 4, 4, 8, 8]
    assert p.width(1) == 4  # 2.5 tokens per unit beats 1.5 and 2.0
    assert p.width(3) == 2  # bucket 4 starts exploring from the first width


def _serve(c, rounds, spec_us, native_us, spec_tokens=1.0, settled=lambda i: True, start=0):
    """Drive a ServedTreeChoice with a fake clock: each round's period comes from the action's price."""
    for i in range(start, start + rounds):
        ch = c.choice(1)
        us = spec_us(i) if ch == c.SPECULATE else native_us(i)
        c.record(1, ch, us, spec_tokens if ch == c.SPECULATE else 1.0, settled=settled(i))


def test_served_tree_choice_switches_to_native_when_faster():
    from eagle4_b200.runtime.policy import ServedTreeChoice

    c = ServedTreeChoice(block=2, explore=2, refresh=0)
    _serve(c, 4, lambda i: 1.6, lambda i: 1.0)  # speculation: 1 token in 1.6 units; native: 1 token in 1.0
    assert c.choice(1) == ServedTreeChoice.NATIVE
    c2 = ServedTreeChoice(block=1, explore=2, refresh=0)
    _serve(c2, 4, lambda i: 1.5, lambda i: 1.0, spec_tokens=3.0)  # speculation: 3 tokens in 1.5
    assert c2.choice(1) == ServedTreeChoice.SPECULATE


def test_served_tree_choice_ignores_capture_rounds():
    """The first round of each action captures its graphs (a period 40x a served round): those periods are not
    priced, so an inflated native probe cannot lock in speculation."""
    from eagle4_b200.runtime.policy import ServedTreeChoice

    c = ServedTreeChoice(block=4, explore=8, refresh=256)
    seen = set()
    for i in range(64):
        ch = c.choice(1)
        cap = ch not in seen
        seen.add(ch)
        us = (400.0 if cap else 16.0) if ch == c.SPECULATE else (400.0 if cap else 10.0)
        c.record(1, ch, us, 1.0, settled=not cap)
    assert c.choice(1) == ServedTreeChoice.NATIVE
    assert c.share(ServedTreeChoice.NATIVE) > 0.6


def test_served_tree_choice_drops_stalls_and_follows_rate_changes():
    """A single stalled native period (settled, but 50x its median) is filtered; after the decision's interval the
    bucket explores again from fresh samples, so a change in measured rates moves the choice."""
    from eagle4_b200.runtime.policy import ServedTreeChoice

    c = ServedTreeChoice(block=4, explore=8, refresh=64, max_interval=64)
    _serve(c, 40, lambda i: 16.0, lambda i: 500.0 if i == 5 else 10.0)
    assert c.choice(1) == ServedTreeChoice.NATIVE
    # acceptance rises: speculation now yields 4 tokens per 16-unit round
    _serve(c, 400, lambda i: 16.0, lambda i: 10.0, spec_tokens=4.0, start=40)
    assert c.choice(1) == ServedTreeChoice.SPECULATE
    # and falls again
    _serve(c, 400, lambda i: 16.0, lambda i: 10.0, spec_tokens=1.0, start=440)
    assert c.choice(1) == ServedTreeChoice.NATIVE


def test_served_tree_choice_backs_off_while_the_choice_holds():
    from eagle4_b200.runtime.policy import ServedTreeChoice

    c = ServedTreeChoice(block=4, explore=8, refresh=32, max_interval=1024)
    _serve(c, 3000, lambda i: 16.0, lambda i: 10.0)
    # exploration rounds (speculative probes) become rarer as the same decision repeats
    assert c.share(ServedTreeChoice.NATIVE) > 0.95
    assert c._interval[1] == 1024


def test_served_tree_choice_ties_serve_native():
    from eagle4_b200.runtime.policy import ServedTreeChoice

    c = ServedTreeChoice(block=4, explore=8, refresh=0)
    # noisy, equal rates: speculation must win by two standard errors, so it does not
    _serve(c, 32, lambda i: 10.0 + (i % 3), lambda i: 10.0 + ((i + 1) % 3))
    assert c.choice(1) == ServedTreeChoice.NATIVE


def test_chain_rounds_equal_plain_on_cpu():
    import torch

    from eagle4_b200.api import LLM, TreeSpec

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 1, 5), max_len=256,
                        max_batch=2, config='{"mode": "serve"}')
    assert llm.engine.chain_policy is not None
    p = torch.randint(0, 4096, (2, 20), generator=torch.Generator().manual_seed(0))
    a = llm.generate(p, 14)
    b = llm.generate(p, 14, speculative=False)
    assert torch.equal(a, b)
    assert sum(llm.engine.chain_policy.rounds.values()) > 0


def test_serve_mode_mixes_native_and_speculative_rounds_exactly():
    import torch

    from eagle4_b200.api import LLM, TreeSpec

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256,
                        config='{"mode": "serve"}')
    llm.engine.tree_choice.block = 2  # alternate quickly: 2 speculative, 2 native, ...
    p = torch.randint(0, 4096, (1, 24), generator=torch.Generator().manual_seed(0))
    a = llm.generate(p, 20)
    b = llm.generate(p, 20, speculative=False)
    assert torch.equal(a, b)
    assert sum(llm.engine.tree_choice.rounds.values()) >= 4


def test_round_recorder_writes_jsonl(tmp_path):
    import json

    import torch

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.runtime.recorder import RoundRecorder

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256)
    llm.engine.recorder = RoundRecorder(str(tmp_path / "rounds.jsonl"), flush_every=1)
    p = torch.randint(0, 4096, (1, 16), generator=torch.Generator().manual_seed(0))
    llm.generate(p, 8)
    recs = [json.loads(l) for l in open(tmp_path / "rounds.jsonl")]
    assert recs and recs[0]["kind"] == "tree" and recs[0]["width"] >= 1
    assert llm.engine.recorder.summary()["rounds"] == len(recs)
