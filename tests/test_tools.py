"""The checking tools (eagle4_b200/tools): parity statuses and the fp32 arbitration rule, an in-process parity run
of speculative against plain decoding, and the mixed-stop batch check (including a broken engine it must catch)."""

import json

import torch

from eagle4_b200.tools import parity, stop_check


def test_bf16_spacing_and_judge_rule():
    assert parity.bf16_spacing(16.0) == 0.125 and parity.bf16_spacing(31.9) == 0.125
    assert parity.bf16_spacing(1.0) == 2 ** -7 and parity.bf16_spacing(-3.0) == 2 ** -6
    logits = {1: 20.0, 2: 19.8, 3: 18.0, 4: 21.0}
    best = (4, 21.0)
    assert parity.judge(1, 2, logits.__getitem__, best).status == "fp32_pass"  # 0.2 <= 2 x 0.125
    assert parity.judge(1, 3, logits.__getitem__, best).status == "fail"
    assert parity.judge(1, 4, logits.__getitem__, best).status == "fp32_argmax"
    assert parity.first_divergence([1, 2, 3], [1, 2, 4]) == 2 and parity.first_divergence([1, 2], [1, 2, 3]) is None


def test_classify_with_model_scorer_and_rejudge():
    scorer = parity.ModelScorer("tiny", device="cpu", max_len=256)
    prompt = list(range(5, 30))
    ref = scorer.bf16.generate([torch.tensor(prompt)], 6, speculative=False)[0].tolist()
    assert parity.classify(prompt, ref, ref, scorer)["status"] == "identical"
    assert parity.classify(prompt, ref, ref[:4], scorer)["status"] == "length"
    prefix = prompt + ref[:3]
    lg = scorer._last_logits(scorer.fp32, prefix)
    worst = int(lg.argmin())
    bad = ref[:3] + [worst] + ref[4:]
    row = parity.classify(prompt, ref, bad, scorer)
    assert row["status"] == "fail" and row["index"] == 3 and row["bf16_gap"] > parity.TIE_GAP
    # the same divergence judged again from the saved logits, under a tolerance wide enough to pass it
    wide = parity.rejudge_row({**row, "tolerance_ulps": 1e9})
    assert wide["status"] == "fp32_pass"
    assert parity.rejudge_row(row)["status"] == "fail"


def test_parity_run_and_compare_in_process(tmp_path):
    spec, plain, rep = tmp_path / "spec.json", tmp_path / "plain.json", tmp_path / "rep.json"
    common = ["--model", "tiny", "--synthetic", "3", "--min-len", "8", "--max-len", "40", "--vocab", "4096",
              "--max-new-tokens", "10"]
    assert parity.main(["run", *common, "--out", str(spec)]) == 0
    assert parity.main(["run", *common, "--no-spec", "--out", str(plain)]) == 0
    assert parity.main(["compare", str(plain), str(spec), "--out", str(rep)]) == 0
    doc = json.loads(rep.read_text())
    assert doc["passes"] and doc["counts"] == {"identical": 3}
    # a corrupted candidate is reported (unjudged without a model) and fails the run
    bad = json.loads(spec.read_text())
    bad["results"][0]["output_ids"][2] += 1
    spec.write_text(json.dumps(bad))
    assert parity.main(["compare", str(plain), str(spec)]) == 1


def test_violation_rules():
    v = stop_check.violations
    assert v("plain", [1, 2, 3], "length", 3, 9, 8) == []
    assert v("plain", [1, 2], "stop", 3, 9, 8)
    assert v("stop_token", [1, 9], "stop", 3, 9, 8) == []
    assert v("stop_token", [9, 1, 2], "length", 3, 9, 8)  # went on past its stop token
    assert v("stop_token", [1, 2], "eos", 3, 9, 8)  # ended early for another request's reason
    assert v("eos", [1, 8], "eos", 3, 9, 8) == []
    assert v("ignore_eos", [8, 8, 8], "length", 3, 9, 8) == []
    assert v("ignore_eos", [1, 8], "eos", 3, 9, 8)


def _scheduler_post(llm, broken=False):
    from eagle4_b200.runtime.scheduler import RequestParams, Scheduler

    sched = Scheduler(llm.engine)
    if broken:  # checks only the last token of each round: tokens past a stop leak out
        def take(req, tokens):
            req.output.extend(tokens)
            p = req.params
            if tokens and tokens[-1] in p.stop_token_ids:
                req.finish_reason = "stop"
            elif len(req.output) >= p.max_new_tokens:
                del req.output[p.max_new_tokens:]
                req.finish_reason = "length"
            return req.finished

        sched._take = take
    return sched


def test_stop_check_mixed_batch_in_process_and_a_broken_engine():
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.runtime.scheduler import RequestParams
    from eagle4_b200.tools import prompts

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=8, max_len=256)
    ps = prompts.synthetic(8, lo=8, hi=40, vocab=4096, seed=1)

    def batch_post(broken):
        # all requests of a call are submitted before the first round, so they share rounds
        def run(bodies):
            sched = _scheduler_post(llm, broken)
            reqs = [sched.submit(b["prompt_ids"], RequestParams(
                max_new_tokens=b["max_new_tokens"], stop_token_ids=tuple(b.get("stop_token_ids", ())),
                eos_token_id=b.get("eos_token_id"), ignore_eos=b.get("ignore_eos", False))) for b in bodies]
            sched.run()
            return [{"output_ids": r.output, "finish_reason": r.finish_reason} for r in reqs]
        return run

    def check(broken):
        run = batch_post(broken)
        outs = run([{"prompt_ids": p, "max_new_tokens": 12} for _, p in ps])
        stop, eos = stop_check.pick_enders([o["output_ids"] for o in outs])
        kinds = [stop_check.KINDS[i % 4] for i in range(len(ps))]
        replies = run([stop_check.request_for(k, p, 12, stop, eos) for k, (_, p) in zip(kinds, ps)])
        return sum(bool(stop_check.violations(k, r["output_ids"], r["finish_reason"], 12, stop, eos))
                   for k, r in zip(kinds, replies))

    assert check(False) == 0
    assert check(True) > 0


def test_stop_check_main_in_process(tmp_path):
    out = tmp_path / "stop.json"
    rc = stop_check.main(["--model", "tiny", "--synthetic", "8", "--min-len", "8", "--max-len", "40",
                          "--vocab", "4096", "--concurrency", "4", "--max-new-tokens", "12", "--out", str(out)])
    rep = json.loads(out.read_text())
    assert rc == 0 and rep["violations"] == 0 and rep["requests"] == 8


def test_sampling_check_passes_speculation_and_rejects_a_wrong_sampler(capsys):
    """Speculative and plain sampling draw from one distribution (tiny model, temperature 0.05, draws of one call
    sharing speculative rounds); a sampler at another temperature is rejected."""
    from eagle4_b200.tools import sampling_check as sc

    prompts = sc.synthetic_prompts(1, 12, 4096, seed=0)
    kw = dict(samples=256, tokens=3, batch=64)
    meta = {"tokens": 3}
    plain = {"meta": meta, "prompts": [{"prompt_ids": prompts[0], "samples": s} for s in
                                       sc.sample_in_process("tiny", prompts, temperature=0.05, speculative=False,
                                                            seed=1, **kw)]}
    spec = {"meta": meta, "prompts": [{"prompt_ids": prompts[0], "samples": s} for s in
                                      sc.sample_in_process("tiny", prompts, temperature=0.05, speculative=True,
                                                           seed=2, **kw)]}
    colder = {"meta": meta, "prompts": [{"prompt_ids": prompts[0], "samples": s} for s in
                                        sc.sample_in_process("tiny", prompts, temperature=0.02, speculative=False,
                                                             seed=3, **kw)]}
    assert sc.compare(plain, spec, log=lambda s: None)
    assert not sc.compare(plain, colder, log=lambda s: None)


def test_homogeneity_pools_rare_cells():
    from collections import Counter

    from eagle4_b200.tools.sampling_check import homogeneity

    a = Counter({1: 50, 2: 50, 3: 2, 4: 1})
    b = Counter({1: 48, 2: 52, 5: 3})
    stat, dof, p, tvd = homogeneity(a, b)
    assert dof == 2 and p > 0.5 and 0 < tvd < 0.1  # cells 1, 2 and the pooled rest
    assert homogeneity(Counter({1: 5}), Counter({1: 5})) is None
