"""Continuous batching (runtime/scheduler.py): admission between rounds, retirement on per-request stop conditions,
page-budget waits, padded graph buckets. Greedy outputs must not depend on the batch a request shares rounds with,
so every request's tokens equal its tokens generated alone."""

import pytest
import torch

from eagle4_b200.api import LLM, TreeSpec
from eagle4_b200.runtime.pages import OutOfPages
from eagle4_b200.runtime.scheduler import RequestParams, Scheduler


def _llm(max_batch=2, **kw):
    return LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=max_batch,
                         max_len=256, **kw)


def _prompts(n, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(1, 4096, (int(torch.randint(5, 40, (1,), generator=g)),), generator=g) for _ in range(n)]


def _alone(llm, prompt, n, speculative):
    return llm.generate([prompt], n, speculative=speculative)[0].tolist()


@pytest.mark.parametrize("speculative", [True, False])
def test_continuous_batching_matches_each_request_alone(speculative):
    llm = _llm(max_batch=2)
    prompts = _prompts(5)
    lens = [7, 3, 11, 5, 9]
    alone = [_alone(llm, p, n, False) for p, n in zip(prompts, lens)]
    sched = Scheduler(llm.engine, speculative=speculative)
    reqs = [sched.submit(p, RequestParams(max_new_tokens=n)) for p, n in zip(prompts, lens)]
    seen_batches = set()
    while not sched.idle:
        sched.step()
        seen_batches.add(len(sched.running))
        assert len(sched.running) <= 2
    for r, want, n in zip(reqs, alone, lens):
        assert r.finish_reason == "length" and r.output == want, (r.rid, r.output, want)
    assert sorted(sched.free_slots) == [0, 1] and llm.engine.pages.free_pages == llm.engine.pages.num_pages - 1


def test_stop_conditions_per_request():
    llm = _llm(max_batch=4)
    prompts = _prompts(4, seed=1)
    free = [_alone(llm, p, 12, False) for p in prompts]
    sched = Scheduler(llm.engine)
    stop_tok = free[0][4]
    eos = free[1][3]
    reqs = [
        sched.submit(prompts[0], RequestParams(max_new_tokens=12, stop_token_ids=(stop_tok,))),
        sched.submit(prompts[1], RequestParams(max_new_tokens=12, eos_token_id=eos)),
        sched.submit(prompts[2], RequestParams(max_new_tokens=12, eos_token_id=eos, ignore_eos=True)),
        sched.submit(prompts[3], RequestParams(max_new_tokens=12)),
    ]
    sched.run()
    assert reqs[0].finish_reason == "stop" and reqs[0].output == free[0][:free[0].index(stop_tok) + 1]
    assert reqs[1].finish_reason == "eos" and reqs[1].output == free[1][:free[1].index(eos) + 1]
    # one request's stop set never ends another: ignore_eos runs to its length, the plain one too
    assert reqs[2].finish_reason == "length" and reqs[2].output == free[2]
    assert reqs[3].finish_reason == "length" and reqs[3].output == free[3]


def test_stop_strings_need_a_detokenizer_and_end_on_the_string():
    llm = _llm(max_batch=1)
    p = _prompts(1, seed=2)[0]
    free = _alone(llm, p, 10, False)
    with pytest.raises(ValueError):
        Scheduler(llm.engine).submit(p, RequestParams(max_new_tokens=10, stop=("x",)))
    detok = lambda ids: " ".join(str(t) for t in ids)  # noqa: E731
    sched = Scheduler(llm.engine, detokenize=detok)
    r = sched.submit(p, RequestParams(max_new_tokens=10, stop=(str(free[5]),)))
    sched.run()
    assert r.finish_reason == "stop" and str(free[5]) in detok(r.output) and len(r.output) <= 6


def test_admission_waits_for_pages_and_refuses_what_never_fits():
    # room for one request at a time: the second waits for the first to release its pages
    prompts = _prompts(2, seed=3)
    span = 9  # one round's tree rows: max(verify tokens, steps * top-k) + 1
    pages = [-(-(int(p.numel()) + 8 + span) // 16) for p in prompts]
    llm = _llm(max_batch=2, kv_tokens=16 * max(pages))
    assert llm.engine.span == span and llm.engine.pages.free_pages < sum(pages)
    alone = [_alone(llm, p, 8, False) for p in prompts]
    sched = Scheduler(llm.engine)
    reqs = [sched.submit(p, RequestParams(max_new_tokens=8)) for p in prompts]
    sched.step()
    assert len(sched.running) == 1 and len(sched.waiting) == 1
    sched.run()
    assert [r.output for r in reqs] == alone
    small = _llm(max_batch=1, kv_tokens=16)  # two pages besides the trash page
    s2 = Scheduler(small.engine)
    s2.submit(prompts[0], RequestParams(max_new_tokens=64))
    with pytest.raises(OutOfPages):
        s2.step()


def test_padded_bucket_rounds_match():
    # 9 running requests replay the graph bucket of 10 (the calibration grid has no 9): the padding row must not
    # disturb the real rows
    llm = _llm(max_batch=10)
    assert llm.engine.bucket(9) == 10 and llm.engine.bucket(8) == 8
    prompts = _prompts(9, seed=4)
    alone = [_alone(llm, p, 4, False) for p in prompts]
    sched = Scheduler(llm.engine)
    reqs = [sched.submit(p, RequestParams(max_new_tokens=4)) for p in prompts]
    sched.run()
    assert [r.output for r in reqs] == alone


def test_llm_complete_texts_with_stops():
    from tests.helpers import word_tokenizer

    llm = _llm(max_batch=2)
    tok = word_tokenizer(4096)
    prompts = _prompts(3)
    alone = [_alone(llm, p, 6, False) for p in prompts]
    texts = [" ".join(f"<{i}>" for i in p.tolist()) for p in prompts]
    out = llm.complete(texts, tok, max_new_tokens=6, ignore_eos=True)
    assert [o["token_ids"] for o in out] == alone and all(o["finish_reason"] == "length" for o in out)
    stop = f"<{alone[1][2]}>"
    out = llm.complete([texts[1]], tok, max_new_tokens=6, stop=stop, ignore_eos=True)[0]
    assert out["finish_reason"] == "stop" and stop not in out["text"]
    assert out["token_ids"] == alone[1][:alone[1].index(alone[1][2]) + 1]
    ids = llm.complete([p.tolist() for p in prompts], max_new_tokens=4)
    assert [o["token_ids"] for o in ids] == [a[:4] for a in alone] and "text" not in ids[0]
    with pytest.raises(ValueError):
        llm.complete(["text"], max_new_tokens=2)


@pytest.mark.parametrize("temperature", [0.0, 0.05])
def test_batched_prefill_gives_each_request_its_own_result(temperature):
    """Admitted requests prefilled together (in groups bounded by a token budget) emit exactly what one-by-one
    prefills emit: greedy, and sampled with the same seed."""
    prompts = _prompts(5, seed=4)
    lens = [6, 4, 7, 3, 5]

    def serve(batch_prefill, budget=8192):
        llm = _llm(max_batch=3, temperature=temperature, sample_seed=2)
        sched = Scheduler(llm.engine, batch_prefill=batch_prefill, prefill_tokens=budget)
        reqs = [sched.submit(p, RequestParams(max_new_tokens=n)) for p, n in zip(prompts, lens)]
        sched.run()
        return [r.output for r in reqs]

    want = serve(False)
    assert serve(True) == want
    assert serve(True, budget=40) == want  # several groups per admission step


def test_batched_prefill_engine_matches_single_prefills():
    llm = _llm(max_batch=3)
    eng = llm.engine
    prompts = _prompts(3, seed=6)
    one = []
    for b, p in enumerate(prompts):
        eng.slot[b] = b
        one.append(int(eng.prefill(b, p)[0][0]))
    state = [t.clone() for t in eng.tcache.ssm]
    firsts = eng.prefill_many([0, 1, 2], prompts)
    assert [int(f[0]) for f in firsts] == one
    for a, b in zip(state, eng.tcache.ssm):
        assert torch.allclose(a[:3], b[:3], atol=1e-6)


@pytest.mark.parametrize("model", ["tiny", "tiny-mamba"])
def test_chunked_prefill_matches_one_forward(model):
    """A prompt longer than the prefill chunk goes through the target in pieces (the recurrent and conv states and the
    KV carry over between pieces): the first token, the aux rows, the states and the speculative output equal one
    forward's."""
    def run(chunk):
        llm = LLM.synthetic(model, device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=1,
                            max_len=256)
        eng = llm.engine
        eng.prefill_chunk = chunk
        prompt = _prompts(1, seed=9)[0].repeat(3)[:70]
        eng.slot[0] = 0
        first, aux = eng.prefill(0, prompt)
        state = [t[:1].clone() for t in eng.tcache.ssm] + [t[:1].clone() for t in eng.tcache.conv]
        return int(first[0]), aux, state, llm.generate([prompt], 12, speculative=True)[0].tolist()

    f1, a1, s1, g1 = run(8192)
    f2, a2, s2, g2 = run(16)
    assert f1 == f2 and g1 == g2
    assert torch.allclose(a1, a2, atol=1e-5)
    for a, b in zip(s1, s2):
        assert torch.allclose(a, b, atol=1e-5)


def test_prompt_leading_rows_get_only_draft_kv():
    """The draft's share of a prefill writes the leading rows' KV without their attention or MLP: the KV equals a
    full draft forward's over the same rows."""
    llm = _llm(max_batch=1)
    eng = llm.engine
    prompt = _prompts(1, seed=3)[0].repeat(4)[:60]
    eng.slot[0] = 0
    first, aux = eng.prefill(0, prompt)
    lead = prompt.shape[0] - min(prompt.shape[0], eng.verify_tokens)
    slots = eng._slots(torch.tensor(0), torch.arange(lead))
    k_kv, v_kv = eng.dcache.k.view(-1, *eng.dcache.k.shape[-2:])[slots], eng.dcache.v.view(-1, *eng.dcache.v.shape[-2:])[slots]
    eng.dcache.k.zero_()
    eng.dcache.v.zero_()
    pos = torch.arange(lead)
    nxt = prompt[1:lead + 1]
    eng.draft.forward(nxt, eng.draft.project(aux[:lead]), pos, torch.zeros(lead, dtype=torch.int32), slots,
                      torch.zeros(lead, dtype=torch.int32), (pos + 1).int(), torch.zeros(lead, 1, dtype=torch.int32),
                      torch.zeros(lead, dtype=torch.int32), eng.dcache, max_keys=lead)
    assert torch.equal(eng.dcache.k.view(-1, *eng.dcache.k.shape[-2:])[slots], k_kv)
    assert torch.equal(eng.dcache.v.view(-1, *eng.dcache.v.shape[-2:])[slots], v_kv)


def test_native_rounds_count_positions_left_without_draft_kv():
    """Above the verify batch limit every round is native; a request's pending ring holds N rows, so each native
    token after the ring is full leaves one position without draft KV, and the count follows rows that move."""
    llm = _llm(max_batch=2)
    eng = llm.engine
    n = eng.verify_tokens
    eng.verify_batch_limit = 1
    prompts = [p[:8] if p.shape[0] >= 8 else p.repeat(8)[:8] for p in _prompts(2, seed=5)]
    sched = Scheduler(eng)
    reqs = [sched.submit(p, RequestParams(max_new_tokens=n + 6)) for p in prompts]
    sched.run()
    assert all(len(r.output) == n + 6 for r in reqs)
    # ring full after the prefill (N of the 8 prompt rows pending); the first emitted token is the prefill's, so
    # n + 5 native rounds per request, each one a hole
    assert eng.stats.draft_kv_holes == 2 * (n + 5)
