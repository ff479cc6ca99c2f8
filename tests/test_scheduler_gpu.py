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
