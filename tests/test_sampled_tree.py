"""Recursive rejection without replacement keeps the target distribution (the sampled-tree oracle)."""

import os
import sys

import torch

from eagle4_b200.core.sampled_tree import draw_children, filter_proposal_logits, reject_children

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def test_output_law_equals_target():
    torch.manual_seed(0)
    vocab, cand, draws, n = 12, 8, 3, 200_000
    p = torch.softmax(torch.randn(vocab) * 1.5, dim=-1)
    ids = torch.randperm(vocab)[:cand]
    logits = p[ids].log() + 0.3 * torch.randn(cand)  # a draft close to the target
    g = torch.Generator().manual_seed(1)
    prop = draw_children(logits.expand(n, cand).contiguous(), ids.expand(n, cand).contiguous(), draws, generator=g)
    res = reject_children(p.expand(n, vocab), prop, torch.rand(n, draws, generator=g), torch.rand(n, generator=g))
    freq = torch.bincount(res.tokens, minlength=vocab).double() / n
    # chi-square statistic against the target law (11 dof; 40 is far beyond the 0.9999 quantile)
    chi2 = (((freq - p.double()) ** 2) / p.double()).sum() * n
    assert chi2 < 40, chi2
    assert (res.accepted_position >= 0).float().mean() > 0.2  # the draft actually gets accepted


def test_filter_keeps_topk_topp_minp():
    lg = torch.tensor([[2.0, 1.0, 0.5, -1.0, -3.0]])
    one = lambda v: torch.tensor([v])  # noqa: E731
    out = filter_proposal_logits(lg, one(1.0), one(2), one(1.0), one(0.0))
    assert torch.isinf(out[0, 2:]).all() and torch.isfinite(out[0, :2]).all()
    out = filter_proposal_logits(lg, one(1.0), one(5), one(0.5), one(0.0))
    assert torch.isfinite(out[0, 0]) and torch.isinf(out[0, 1:]).all()


def test_matches_reference_oracle():
    if not os.path.isdir(os.path.join(REF, "eagle_harness")):
        return
    sys.path.insert(0, REF)
    try:
        from eagle_harness.core import sampled_tree as rst
    finally:
        sys.path.remove(REF)
    torch.manual_seed(3)
    rows, vocab, cand, draws = 64, 50, 16, 4
    logits = torch.randn(rows, cand)
    ids = torch.stack([torch.randperm(vocab)[:cand] for _ in range(rows)])
    u = torch.rand(rows, cand)
    a = draw_children(logits, ids, draws, uniforms=u)
    b = rst.draw_children(logits, ids, draws, uniforms=u)
    assert torch.equal(a.positions, b.positions) and torch.equal(a.tokens, b.tokens)
    p = torch.softmax(torch.randn(rows, vocab), dim=-1)
    cu, fu = torch.rand(rows, draws), torch.rand(rows)
    ra, rb = reject_children(p, a, cu, fu), rst.reject_children(p, b, cu, fu)
    assert torch.equal(ra.tokens, rb.tokens) and torch.equal(ra.accepted_position, rb.accepted_position)


def _shard_protocol(logits, temperature, parent, nodes, q_store, q_ids, node_slot, k, seed, rnd, stream, bounds):
    """The vocabulary-parallel accept simulated in one process over vocabulary shards ``bounds``: global row
    statistics, candidate probabilities, the sparse walk, per-shard residual masses, the owner's draw."""
    from eagle4_b200.core import sampled_tree as st

    bs, n = parent.shape
    S, C = q_store.shape[1], q_store.shape[2]
    lg = logits.double() / temperature
    mx = lg.amax(-1)
    z = torch.exp(lg - mx[:, None]).sum(-1)
    node = nodes.reshape(-1)
    qrow = torch.arange(bs).repeat_interleave(n) * S + torch.where(node < 0, torch.zeros_like(node), node + 1)
    ids = q_ids.reshape(bs * S, C)[qrow].long()
    p = torch.exp(lg.gather(1, ids) - mx[:, None]) / z[:, None]
    acc, cnt, final, r_final = st.sampled_walk_sparse_reference(p, parent, nodes, q_store, q_ids, node_slot, k, seed,
                                                                rnd, stream)
    resid = [st.shard_residual(logits[:, lo:hi], lo, temperature, mx, z, final, nodes, q_ids, r_final, n)
             for lo, hi in bounds]
    masses = torch.stack([r.sum(1) for r in resid])
    toks = torch.stack([st.shard_draw_reference(r, lo, masses, i, seed, rnd, stream)
                        for i, (r, (lo, _)) in enumerate(zip(resid, bounds))])
    return acc, cnt, toks.amax(0)


def test_vocab_parallel_walk_and_draw_equal_the_full_walk():
    """The sharded protocol's accepted paths and final tokens equal the full-vocabulary walk's (float64, 3 shards)."""
    from eagle4_b200.core import sampled_tree as st
    from eagle4_b200.core.draft_tree import TreeShape

    g = torch.Generator().manual_seed(7)
    bs, k, c, v = 5, 3, 12, 300
    shape = TreeShape(k, 3)
    n = 1 + k + 2
    parent = torch.zeros(bs, n, dtype=torch.int32)
    parent[:, 0] = -1
    parent[:, 1 + k:] = 1
    nodes = torch.full((bs, n), -1, dtype=torch.int64)
    nodes[:, 1:1 + k] = torch.arange(k)
    nodes[:, 1 + k:] = shape.layer_start(2) + torch.arange(2)
    cap = shape.capacity
    q_store = torch.softmax(torch.randn(bs, 1 + cap, c, generator=g) * 1.5, -1).float()
    q_ids = torch.stack([torch.stack([torch.randperm(v, generator=g)[:c] for _ in range(1 + cap)])
                         for _ in range(bs)]).int()
    node_slot = torch.stack([torch.randperm(c, generator=g)[:cap] for _ in range(bs)]).int()
    bounds = [(0, 128), (128, 256), (256, 300)]
    for rnd in range(25):
        logits = torch.randn(bs * n, v, generator=g) * 2
        acc, cnt, bonus = _shard_protocol(logits, 0.8, parent, nodes, q_store, q_ids, node_slot, k, 9, rnd, 0x10000,
                                          bounds)
        racc, rcnt, rbonus = st.sampled_walk_reference(logits, 0.8, parent, nodes, q_store, q_ids, node_slot, k, 9,
                                                       rnd, 0x10000)
        assert torch.equal(cnt, rcnt) and torch.equal(bonus, rbonus)
        for b in range(bs):
            assert torch.equal(acc[b, :int(cnt[b])], racc[b, :int(rcnt[b])])
