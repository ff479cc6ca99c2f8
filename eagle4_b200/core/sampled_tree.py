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
        raise ValueError("logits and ids must share one [rows, candidates] shape, and the draw count fit in it")
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


# ------------------------------------------------------------------------------------------------------------------
# The GPU sampler's definitions in float64: the same random streams (SplitMix64 keyed by seed, round, stream, index),
# Gumbel-top-k children and the tree walk over verify rows (``eagle4_b200/csrc/sampled.cu``).

_M64 = (1 << 64) - 1


def _mix64(z):
    import numpy as np

    z = (z + np.uint64(0x9E3779B97F4A7C15)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & np.uint64(_M64)
    return z ^ (z >> np.uint64(31))


def stream_uniforms(seed: int, round_: int, stream: int, index) -> torch.Tensor:
    """Uniforms in (0, 1) of the GPU sampler's streams: 24 high bits of the mixed key, centred (float64)."""
    import numpy as np

    with np.errstate(over="ignore"):
        idx = np.asarray(index, dtype=np.uint64)
        h = _mix64(np.uint64(seed & _M64) ^ np.uint64(((round_ & 0xFFFFFFFF) << 32) | (stream & 0xFFFFFFFF)))
        h = _mix64(h ^ idx)
        u = ((h >> np.uint64(40)).astype(np.float64) + 0.5) / 16777216.0
    return torch.from_numpy(np.asarray(u, dtype=np.float64))


def sample_children_reference(logits: torch.Tensor, cand_ids: torch.Tensor, k: int, temperature: float, seed: int,
                              round_: int, stream: int):
    """``(q [R, C], child probs [R, k], child ids [R, k], child slots [R, k])``: Gumbel-top-k of ``log q`` with the
    GPU sampler's uniforms (row ``r``, candidate ``c`` uses index ``r * C + c``)."""
    r, c = logits.shape
    q = torch.softmax(logits.double() / temperature, dim=-1)
    u = stream_uniforms(seed, round_, stream, range(r * c)).view(r, c).to(q.device)
    keys = torch.where(q > 0, torch.log(q) - torch.log(-torch.log(u)), torch.full_like(q, float("-inf")))
    slots = torch.sort(-keys, dim=-1, stable=True).indices[:, :k]
    return q, q.gather(1, slots), cand_ids.gather(1, slots), slots


def sampled_walk_reference(logits: torch.Tensor, temperature: float, row_parent: torch.Tensor,
                           row_node: torch.Tensor, q_store: torch.Tensor, q_ids: torch.Tensor,
                           node_slot: torch.Tensor, top_k: int, seed: int, round_: int, stream: int):
    """The tree rejection walk of the GPU sampler in float64: ``(accepted rows [bs, n], counts [bs], final token
    [bs])``. Children of a row are tried in node order (= draw order) while they are the first draws; the final token
    is drawn from the normalised residual in vocabulary order."""
    bs, n = row_parent.shape
    v = logits.shape[1]
    acc = torch.zeros(bs, n, dtype=torch.int64)
    cnt = torch.zeros(bs, dtype=torch.int32)
    bonus = torch.zeros(bs, dtype=torch.int64)
    for b in range(bs):
        row, path = 0, [0]
        while True:
            p = torch.softmax(logits[b * n + row].double() / temperature, dim=-1)
            nd = int(row_node[b, row])
            slot = 0 if nd < 0 else 1 + nd
            ids = q_ids[b, slot].long()
            q = q_store[b, slot].double().clone()
            resid = p.clone()
            moved = False
            expect = 0
            for j in range(row + 1, n):
                if int(row_parent[b, j]) != row:
                    continue
                cn = int(row_node[b, j])
                draw = cn if cn < top_k else (cn - top_k) % top_k
                if draw != expect:
                    break
                expect += 1
                s = int(node_slot[b, cn])
                qsum = float(q.sum())
                m = float(resid.sum())
                qy = float(q[s]) / qsum if qsum > 0 else 0.0
                u = float(stream_uniforms(seed, round_, stream, [b * n + j])[0])
                if q[s] > 0 and u * m * qy < float(resid[ids[s]]):
                    path.append(j)
                    row = j
                    moved = True
                    break
                scale = m / qsum if qsum > 0 else 0.0
                resid[ids] = (resid[ids] - scale * q).clamp_min(0)
                q[s] = 0
            if moved:
                continue
            cdf = resid.cumsum(0)
            target = float(stream_uniforms(seed, round_, stream + 1, [b])[0]) * float(cdf[-1])
            tok = int(torch.searchsorted(cdf, torch.tensor([target], dtype=cdf.dtype), right=True)[0].clamp_max(v - 1))
            acc[b, : len(path)] = torch.tensor(path)
            cnt[b] = len(path)
            bonus[b] = tok
            break
    return acc, cnt, bonus


# ------------------------------------------------------------------------------------------------------------------
# Vocabulary-parallel definitions (tensor parallelism): the walk from the target probabilities at the candidates, then
# the final draw by the rank whose shard holds the target mass (``eagle4_b200/csrc/sampled.cu`` sparse mode,
# ``shard_mass_kernel``, ``shard_draw_kernel``).

def sampled_walk_sparse_reference(p_cand: torch.Tensor, row_parent: torch.Tensor, row_node: torch.Tensor,
                                  q_store: torch.Tensor, q_ids: torch.Tensor, node_slot: torch.Tensor, top_k: int,
                                  seed: int, round_: int, stream: int):
    """The tree walk from ``p_cand [bs * n, C]`` (target probabilities at each verify row's candidate ids): (accepted
    rows [bs, n], counts [bs], final row [bs], residual at the final row's candidates [bs, C]). The residual mass is
    the mass outside the candidates (1 - their sum, at least 0) plus the candidates' residual."""
    bs, n = row_parent.shape
    C = q_store.shape[2]
    acc = torch.zeros(bs, n, dtype=torch.int64)
    cnt = torch.zeros(bs, dtype=torch.int32)
    final = torch.zeros(bs, dtype=torch.int32)
    r_final = torch.zeros(bs, C, dtype=torch.float64)
    for b in range(bs):
        row, path = 0, [0]
        while True:
            r = p_cand[b * n + row].double().clone()
            outside = max(1.0 - float(r.sum()), 0.0)
            nd = int(row_node[b, row])
            q = q_store[b, 0 if nd < 0 else 1 + nd].double().clone()
            moved, expect = False, 0
            for j in range(row + 1, n):
                if int(row_parent[b, j]) != row:
                    continue
                cn = int(row_node[b, j])
                draw = cn if cn < top_k else (cn - top_k) % top_k
                if draw != expect:
                    break
                expect += 1
                s = int(node_slot[b, cn])
                qsum = float(q.sum())
                m = outside + float(r.sum())
                qy = float(q[s]) / qsum if qsum > 0 else 0.0
                u = float(stream_uniforms(seed, round_, stream, [b * n + j])[0])
                if q[s] > 0 and u * m * qy < float(r[s]):
                    path.append(j)
                    row, moved = j, True
                    break
                scale = m / qsum if qsum > 0 else 0.0
                r = (r - scale * q).clamp_min(0)
                q[s] = 0
            if moved:
                continue
            acc[b, :len(path)] = torch.tensor(path)
            cnt[b], final[b], r_final[b] = len(path), row, r
            break
    return acc, cnt, final, r_final


def shard_residual(logits: torch.Tensor, lo: int, temperature: float, mx: torch.Tensor, z: torch.Tensor,
                   final_row: torch.Tensor, row_node: torch.Tensor, q_ids: torch.Tensor, r_final: torch.Tensor,
                   n: int) -> torch.Tensor:
    """The final rows' residual over this rank's shard ``[lo, lo + Vl)`` ([bs, Vl], float64): target probabilities,
    replaced at candidate ids (first occurrence) by the walk's residual."""
    bs = final_row.shape[0]
    vl = logits.shape[1]
    S = q_ids.shape[1]
    out = torch.zeros(bs, vl, dtype=torch.float64)
    for b in range(bs):
        g = b * n + int(final_row[b])
        out[b] = torch.exp(logits[g].double() / temperature - float(mx[g])) / float(z[g])
        nd = int(row_node[b, int(final_row[b])])
        ids = q_ids.view(-1, q_ids.shape[-1])[b * S + (0 if nd < 0 else 1 + nd)].tolist()
        seen = set()
        for c, i in enumerate(ids):
            if i in seen:
                continue
            seen.add(i)
            if lo <= i < lo + vl:
                out[b, i - lo] = float(r_final[b, c])
    return out


def shard_draw_reference(resid: torch.Tensor, lo: int, masses: torch.Tensor, rank: int, seed: int, round_: int,
                         stream: int) -> torch.Tensor:
    """Final tokens: target = u * (sum of the ranks' masses), the owning rank searches its shard in vocabulary
    order; -1 on the other ranks. ``masses`` [world, bs]."""
    bs = resid.shape[0]
    tok = torch.full((bs,), -1, dtype=torch.int64)
    for b in range(bs):
        col = masses[:, b].double()
        target = float(stream_uniforms(seed, round_, stream + 1, [b])[0]) * float(col.sum())
        run, owner = 0.0, -1
        for r in range(col.shape[0]):
            if col[r] > 0:
                owner = r
            if run + float(col[r]) > target and col[r] > 0:
                owner = r
                break
            run += float(col[r])
        if owner != rank:
            continue
        cdf = resid[b].cumsum(0)
        i = int(torch.searchsorted(cdf, torch.tensor([target - run], dtype=cdf.dtype), right=True)[0])
        tok[b] = lo + min(i, resid.shape[1] - 1)
    return tok
