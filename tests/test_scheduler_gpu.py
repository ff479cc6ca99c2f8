"""Continuous batching on the GPU: requests join and leave CUDA-graph rounds replayed at padded batch buckets; every
request's greedy tokens equal its tokens generated alone."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("speculative", [True, False])
def test_continuous_batching_on_gpu_matches_alone(speculative):
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native
    from eagle4_b200.runtime.scheduler import RequestParams, Scheduler

    llm = LLM.synthetic("tiny", device="cuda", tree=TreeSpec(4, 2, 8), max_batch=10, max_len=512)
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(1, 4096, (int(torch.randint(8, 120, (1,), generator=g)),), generator=g)
               for _ in range(13)]
    lens = [int(torch.randint(3, 24, (1,), generator=g)) for _ in prompts]
    alone = [llm.generate([p], n, speculative=False)[0].tolist() for p, n in zip(prompts, lens)]
    sched = Scheduler(llm.engine, speculative=speculative)
    reqs = [sched.submit(p, RequestParams(max_new_tokens=n)) for p, n in zip(prompts, lens)]
    batches = set()
    while not sched.idle:
        sched.step()
        batches.add(len(sched.running))
    assert [r.output for r in reqs] == alone
    assert 9 in batches or any(b not in llm.engine.buckets for b in batches)  # a padded bucket was replayed
    native.check_errors(torch.device("cuda"))


def test_batched_prefill_on_gpu_matches_single_prefills():
    """Several prompts in one prefill forward: each request's recurrent state and attention cache end as its own
    prefill leaves them (within bf16 rounding: a longer forward may take another GEMM partition)."""
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    llm = LLM.synthetic("tiny", device="cuda", tree=TreeSpec(4, 2, 8), max_batch=4, max_len=512)
    eng = llm.engine
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(1, 4096, (n,), generator=g) for n in (37, 120, 9, 64)]
    for b in range(4):
        eng.slot[b] = b
    def keys():  # every request's K rows in position order (the pages may move between the two prefills)
        return [[t[eng._slots(torch.tensor(b, device="cuda"), torch.arange(p.numel(), device="cuda"))].float()
                 for b, p in enumerate(prompts)] for t in eng.tcache.k]

    single = [int(eng.prefill(b, p)[0][0]) for b, p in enumerate(prompts)]
    ssm = [t[:4].float().clone() for t in eng.tcache.ssm]
    k = keys()
    firsts = [int(f[0]) for f in eng.prefill_many([0, 1, 2, 3], prompts)]
    torch.cuda.synchronize()
    native.check_errors(torch.device("cuda"))
    assert sum(a == b for a, b in zip(firsts, single)) >= 3  # a near tie may flip one first token
    for a, b in zip(ssm, eng.tcache.ssm):
        assert (a - b[:4].float()).abs().max() <= 2e-2 * (a.abs().max() + 1e-6)
    for layer_a, layer_b in zip(k, keys()):
        for a, b in zip(layer_a, layer_b):
            assert (a - b).abs().max() <= 2e-2 * (a.abs().max() + 1e-6)


def test_chunked_prefill_on_gpu_matches_one_forward():
    """A prompt longer than the prefill chunk goes through in pieces: the recurrent states and the attention keys
    end as one forward leaves them (within bf16 rounding: pieces may take another GEMM partition)."""
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    llm = LLM.synthetic("tiny", device="cuda", tree=TreeSpec(4, 2, 8), max_batch=1, max_len=512)
    eng = llm.engine
    prompt = torch.randint(1, 4096, (200,), generator=torch.Generator().manual_seed(13))
    eng.slot[0] = 0
    rows = eng._slots(torch.tensor(0, device="cuda"), torch.arange(200, device="cuda"))
    results = []
    for chunk in (8192, 48):
        eng.prefill_chunk = chunk
        eng.prefill(0, prompt)
        torch.cuda.synchronize()
        native.check_errors(torch.device("cuda"))
        results.append(([t[:1].float().clone() for t in eng.tcache.ssm],
                        [t[rows].float().clone() for t in eng.tcache.k]))
    for a, b in zip(results[0][0] + results[0][1], results[1][0] + results[1][1]):
        assert (a - b).abs().max() <= 2e-2 * (a.abs().max() + 1e-6)
