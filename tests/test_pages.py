"""The KV page pool: pages mapped into block-table rows on admission, returned on release, unmapped entries on the
trash page, refusal when the pool runs out; an engine with a pool smaller than max_reqs * max_len serves requests of
different lengths with the same output as plain decoding."""

import pytest
import torch

from eagle4_b200.runtime.pages import OutOfPages, PagePool


def test_reserve_release_and_trash():
    bt = torch.full((3, 4), 7, dtype=torch.int32)
    pool = PagePool(bt, num_pages=6, page=16)
    assert bt.eq(0).all() and pool.free_pages == 5
    pool.reserve(0, 20)  # 2 pages
    pool.reserve(1, 16)  # 1 page
    assert bt[0, :2].tolist() == [1, 2] and bt[1, 0].item() == 3 and bt[0, 2:].eq(0).all()
    pool.reserve(0, 33)  # grows to 3 pages
    assert bt[0, :3].tolist() == [1, 2, 4] and pool.free_pages == 1
    with pytest.raises(OutOfPages):
        pool.reserve(2, 40)
    pool.release(0)
    assert bt[0].eq(0).all() and pool.free_pages == 4
    pool.reserve(2, 40)
    assert sorted(bt[2, :3].tolist()) == [1, 2, 4]
    with pytest.raises(ValueError):
        pool.reserve(1, 16 * 5)  # more than a row maps


def test_engine_with_a_small_pool_equals_plain():
    from eagle4_b200.api import LLM, TreeSpec

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=3, max_len=256)
    eng = llm.engine
    from eagle4_b200.runtime.engine import Engine

    small = Engine(llm.target, llm.draft, max_reqs=3, max_len=256, steps=4, top_k=2, verify_tokens=8,
                   kv_tokens=3 * 96)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 4096, (n,), generator=g) for n in (20, 45, 33)]
    out = small.generate(prompts, 16, speculative=True)
    ref = eng.generate(prompts, 16, speculative=False)
    assert out == ref
    assert small.pages.num_pages == 3 * 96 // 16 + 2
