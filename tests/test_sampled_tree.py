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
