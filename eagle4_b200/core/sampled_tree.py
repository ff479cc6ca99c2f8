"""Sampled trees (temperature > 0): ordered proposals and recursive rejection without replacement.

Children of a node are drawn without replacement from the draft's candidate distribution ``q`` (Gumbel-top-k: the
order of ``log q + Gumbel`` keys is a sample of successive draws without replacement). At verify time the children
are tried in draw order; child ``i`` is accepted with probability ``min(1, p'(y) / (m * q_i(y)))`` where ``q_i`` is
``q`` conditioned on the earlier draws and ``p'`` the residual target mass after the earlier rejections; after a
rejection the *whole* conditional ``q_i`` (scaled by the residual mass) is subtracted from the residual. If every
child is rejected the token is drawn from the normalised residual. This is the recursion of Recursive Speculative
Decoding (Jeon et al., arXiv:2402.14160); it leaves the output distribution equal to the target's.

The functions here run in float64 and serve as the numerical oracle of the GPU sampler and of the distribution tests
(the same contract as ``eagle_harness/core/sampled_tree.py:38-128``).
"""

from __future__ import annotations

from typing import NamedTuple, Optional

import torch


class ChildProposals(NamedTuple):
    probs: torch.Tensor  # [rows, C] proposal distribution over the candidate slots
    token_ids: torch.Tensor  # [rows, C] vocabulary id of every candidate slot
    positions: torch.Tensor  # [rows, n] drawn candidate slots, in draw order
    tokens: torch.Tensor  # [rows, n] drawn vocabulary ids
    scores: torch.Tensor  # [rows, n] the n largest q values (sample-independent ranking scores)


class RejectionResult(NamedTuple):
    tokens: torch.Tensor  # [rows] accepted child token or residual draw
    accepted_position: torch.Tensor  # [rows] draw index of the accepted child, -1 for a residual draw


def filter_proposal_logits(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                           min_p: torch.Tensor) -> torch.Tensor:
    """Per-row temperature, then top-k / top-p on the unfiltered probabilities and min-p relative to the mode;
    removed candidates get -inf. Ties rank by candidate index."""
    scaled = logits.float() / temperature.float()[:, None]
    p = torch.softmax(scaled, dim=-1)
    order = torch.sort(-p, dim=-1, stable=True).indices
    sorted_p = p.gather(1, order)
    mass_before_sorted = sorted_p.cumsum(dim=-1) - sorted_p
    rank = torch.empty_like(order)
    rank.scatter_(1, order, torch.arange(p.shape[1], device=p.device).expand_as(order).contiguous())
    mass_before = mass_before_sorted.gather(1, rank)
    keep = (rank < top_k[:, None]) & (mass_before < top_p[:, None])
    keep &= p >= min_p[:, None] * p.amax(dim=-1, keepdim=True)
    return scaled.masked_fill(~keep, float("-inf"))


def draw_children(logits: torch.Tensor, token_ids: torch.Tensor, count: int, *,
                  generator: Optional[torch.Generator] = None, uniforms: Optional[torch.Tensor] = None
                  ) -> ChildProposals:
    """``count`` ordered draws without replacement from ``softmax(logits)`` (Gumbel-top-k)."""
    if logits.ndim != 2 or token_ids.shape != logits.shape or not 1 <= count <= logits.shape[1]:
        raise ValueError("expected matching [rows, candidates] logits/ids and count within the candidate width")
    q = torch.softmax(logits.float(), dim=-1)
    if uniforms is None:
        uniforms = torch.rand(q.shape, dtype=q.dtype, device=q.device, generator=generator)
    tiny = torch.finfo(q.dtype).tiny
    gumbel = -torch.log(-torch.log(uniforms.clamp_min(tiny)))
    keys = torch.log(q) + gumbel
    pos = keys.topk(count, dim=-1).indices
    return ChildProposals(q, token_ids, pos, token_ids.gather(1, pos), q.topk(count, dim=-1).values)


def reject_children(target_probs: torch.Tensor, proposals: ChildProposals, uniforms: torch.Tensor,
                    final_uniforms: torch.Tensor) -> RejectionResult:
    """Recursive rejection over each row's drawn children (float64), then a residual draw if all are rejected."""
    rows, vocab = target_probs.shape
    n = proposals.positions.shape[1]
    if uniforms.shape != (rows, n) or final_uniforms.shape != (rows,):
        raise ValueError("one accept coin per draw and one final coin per row are required")
    dev = target_probs.device
    resid = target_probs.double().clone()
    q = proposals.probs.double().clone()
    chosen = torch.full((rows,), -1, dtype=torch.int64, device=dev)
    out = torch.zeros(rows, dtype=torch.int64, device=dev)
    tiny = torch.finfo(torch.float64).tiny
    for i in range(n):
        slot = proposals.positions[:, i: i + 1]
        tok = proposals.tokens[:, i: i + 1]
        m = resid.sum(dim=-1, keepdim=True)
        cond = q / q.sum(dim=-1, keepdim=True).clamp_min(tiny)
        qy = cond.gather(1, slot).flatten()
        py = resid.gather(1, tok).flatten()
        take = (chosen < 0) & (qy > 0) & (uniforms[:, i] * m.flatten() * qy < py)
        chosen = torch.where(take, torch.full_like(chosen, i), chosen)
        out = torch.where(take, tok.flatten(), out)
        dense = torch.zeros(rows, vocab, dtype=torch.float64, device=dev)
        dense.scatter_(1, proposals.token_ids, cond)
        resid = torch.where((chosen < 0)[:, None], (resid - m * dense).clamp_min(0), resid)
        q.scatter_(1, slot, 0)
    cdf = resid.cumsum(dim=-1)
    draw = torch.searchsorted(cdf.contiguous(), (final_uniforms.double() * cdf[:, -1])[:, None].contiguous(),
                              right=True).flatten().clamp_max(vocab - 1)
    return RejectionResult(torch.where(chosen < 0, draw, out), chosen)
