"""The draft tree of one decode round: node scores, frontier, work deltas, verify selection.

All buffers are fixed-shape tensors so each per-depth update can live inside a CUDA graph. The semantics follow the
reference (``eagle_harness/core/draft_tree.py:1-372``) because the cost model's inputs and the verify layout depend
on them:

* the root (last accepted token) scores ``ROOT_SCORE``; depth 1 is the draft extend's top-``K``;
* a step expands the ``K`` frontier nodes of depth ``d`` into ``K*K`` children scored ``parent * prob``; all join the
  tree and the best ``K`` become the next frontier (ties to the lower node);
* node numbering: depth 1 at ``[0, K)``, depth ``d >= 2`` at ``K + (d-2)*K*K``; ``parents`` starts ``arange(-1, K)``;
* work deltas ``deltas[slot, v-1, j]``: batch mean of the ``v``-th prefix sum of ``sort(best_prev ++ layer_top[:j])``;
* the verify set is the best ``count`` nodes by depth-decayed score (``DEPTH_DECAY**d`` for ``d >= 2``), emitted in
  node order so any prefix is a tree.

On CUDA every update is one launch of this package's ``tree_*`` kernels (``eagle4_b200/csrc/tree.cu``); the
``*_reference`` methods are the torch definitions the kernels are tested against.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable, NamedTuple, Optional, Tuple

import torch

ROOT_SCORE = 1.001
DEPTH_DECAY = 0.9999


def _pow2_at_least(n: int) -> int:
    return 1 << max(n - 1, 0).bit_length()


@dataclass(frozen=True)
class TreeShape:
    top_k: int
    max_depth: int
    work_cap: int = 64

    def __post_init__(self) -> None:
        if self.top_k < 1 or self.max_depth < 2:
            raise ValueError(f"{self}: a draft tree has at least one child per node and two levels")

    def layer_start(self, depth: int) -> int:
        return 0 if depth == 1 else self.top_k + (depth - 2) * self.top_k * self.top_k

    def num_nodes(self, depth: int) -> int:
        return self.layer_start(depth + 1)

    def num_parents(self, depth: int) -> int:
        return 0 if depth < 2 else (self.top_k + 1) + (depth - 2) * self.top_k

    def count_before_step(self, step: int) -> int:
        return 1 + self.top_k + (step - 1) * self.top_k * self.top_k

    @property
    def capacity(self) -> int:
        return self.num_nodes(self.max_depth)

    @property
    def parent_capacity(self) -> int:
        return (self.top_k + 1) + (self.max_depth - 1) * self.top_k

    def node_depths(self) -> torch.Tensor:
        """Depth (1-based) of every node slot, ``[capacity]`` int64."""
        out = torch.empty(self.capacity, dtype=torch.int64)
        for d in range(1, self.max_depth + 1):
            out[self.layer_start(d): self.layer_start(d + 1)] = d
        return out

    def decay(self, device) -> torch.Tensor:
        out = torch.ones(self.capacity, dtype=torch.float32)
        for d in range(2, self.max_depth + 1):
            out[self.layer_start(d): self.layer_start(d + 1)] = DEPTH_DECAY ** d
        return out.to(device)


class VerifySelection(NamedTuple):
    parent_list: torch.Tensor
    top_scores_index: torch.Tensor
    draft_tokens: torch.Tensor


class DraftTree:
    """Per-round tree state for up to ``max_bs`` requests (static buffers)."""

    def __init__(self, shape: TreeShape, max_bs: int, hidden_size: int, dtype: torch.dtype, device,
                 *, max_verify: int, delta_slots: Optional[Iterable[int]] = None):
        k = shape.top_k
        if not 1 <= max_verify <= shape.work_cap:
            raise ValueError(f"max_verify {max_verify} is outside 1..{shape.work_cap} (the tree's best-set size)")
        slots = frozenset(range(shape.max_depth) if delta_slots is None else delta_slots)
        if not slots <= set(range(shape.max_depth)):
            raise ValueError(f"delta_slots {sorted(slots)} outside 0..{shape.max_depth - 1}")
        self.delta_slots = slots
        self.shape, self.max_bs, self.max_verify = shape, max_bs, max_verify
        self.keep_draw_order = False  # sampled trees keep the root's children in draw order
        self.last_nodes: Optional[torch.Tensor] = None  # node of every row of the last verify selection (-1: root)
        f32, i64 = torch.float32, torch.int64
        dev = torch.device(device)
        self.device = dev
        self.root_probs = torch.zeros(max_bs, k, dtype=f32, device=dev)
        self.root_tokens = torch.zeros(max_bs, k, dtype=i64, device=dev)
        self.root_hidden = torch.zeros(max_bs, hidden_size, dtype=dtype, device=dev)
        self.scores = torch.zeros(max_bs, shape.capacity, dtype=f32, device=dev)
        self.tokens = torch.zeros(max_bs, shape.capacity, dtype=i64, device=dev)
        self.parents = torch.zeros(max_bs, shape.parent_capacity, dtype=i64, device=dev)
        self.parents[:, : k + 1] = torch.arange(-1, k, dtype=i64, device=dev)
        self.front_scores = torch.zeros(max_bs, k, dtype=f32, device=dev)
        self.front_tokens = torch.zeros(max_bs * k, dtype=i64, device=dev)
        self.front_hidden = torch.zeros(max_bs * k, hidden_size, dtype=dtype, device=dev)
        # Frontier node index per lane (global numbering); the row attention uses it to find ancestors.
        self.front_nodes = torch.zeros(max_bs, k, dtype=i64, device=dev)
        self.ancestors = torch.zeros(max_bs, k, shape.max_depth, dtype=torch.int32, device=dev)
        self.best = torch.zeros(max_bs, shape.work_cap, dtype=f32, device=dev)
        self.best_prev = torch.zeros_like(self.best)
        self.layer_top = torch.zeros(max_bs, k, dtype=f32, device=dev)
        self.decay = shape.decay(dev)
        self.deltas = torch.zeros(shape.max_depth, max_verify, k + 1, dtype=f32, device=dev)
        self._extra_mask = (torch.arange(k).view(1, -1) < torch.arange(k + 1).view(-1, 1)).float().to(dev)
        depths = range(1, shape.max_depth + 1)
        self._layer_bounds = torch.tensor([shape.layer_start(d + 1) for d in depths], dtype=i64, device=dev)
        self._layer_starts = torch.tensor([shape.layer_start(d) for d in depths], dtype=i64, device=dev)
        self._frontier_base = torch.tensor([shape.num_parents(d) if d > 1 else 1 for d in depths],
                                           dtype=i64, device=dev)

    # ------------------------------------------------------------------ round
    def stage_root(self, bs: int, probs: torch.Tensor, tokens: torch.Tensor, hidden: torch.Tensor) -> None:
        for dst, src in ((self.root_probs, probs), (self.root_tokens, tokens), (self.root_hidden, hidden)):
            if src.data_ptr() != dst.data_ptr():
                dst[:bs].copy_(src)

    def begin(self, bs: int) -> None:
        if self.scores.is_cuda:
            from eagle4_b200.ops import tree_ops

            tree_ops.tree_begin(self, bs, ROOT_SCORE, deltas=0 in self.delta_slots)
        else:
            self.begin_reference(bs)
            if 0 in self.delta_slots:
                self._store_deltas_reference(bs, 0)

    def begin_reference(self, bs: int) -> None:
        k = self.shape.top_k
        if self.keep_draw_order:  # sampled trees: node order must stay the draw order
            probs, toks = self.root_probs[:bs].clone(), self.root_tokens[:bs].clone()
        else:
            probs, order = torch.sort(self.root_probs[:bs], dim=-1, descending=True, stable=True)
            toks = torch.gather(self.root_tokens[:bs], 1, order)
        self.scores[:bs, :k] = probs
        self.tokens[:bs, :k] = toks
        self.front_scores[:bs] = probs
        self.front_tokens[: bs * k] = toks.reshape(-1)
        self.front_hidden[: bs * k] = self.root_hidden[:bs].repeat_interleave(k, dim=0)
        self.front_nodes[:bs] = torch.arange(k, device=self.scores.device)
        self.best_prev[:bs].zero_()
        self.best_prev[:bs, 0] = ROOT_SCORE
        self.best[:bs].zero_()
        self.best[:bs, 0] = ROOT_SCORE
        ranked = torch.sort(probs, dim=-1, descending=True).values if self.keep_draw_order else probs
        self.best[:bs, 1: 1 + k] = ranked
        self.layer_top[:bs] = ranked

    def set_step_slots(self, bs: int, step: int, slots: torch.Tensor) -> None:
        self.ancestors[:bs, :, step - 1] = slots.to(torch.int32)

    def keep_rows(self, rows: torch.Tensor) -> None:
        n, k = rows.numel(), self.shape.top_k
        for buf in (self.root_probs, self.root_tokens, self.root_hidden, self.scores, self.tokens, self.parents,
                    self.front_scores, self.front_nodes, self.ancestors, self.best, self.best_prev, self.layer_top,
                    self.front_tokens.view(self.max_bs, k), self.front_hidden.view(self.max_bs, k, -1)):
            buf[:n] = buf.index_select(0, rows)

    def step(self, bs: int, step: int, probs: torch.Tensor, tokens: torch.Tensor, hidden: torch.Tensor) -> None:
        if not 1 <= step < self.shape.max_depth:
            raise ValueError(f"step {step} outside 1..{self.shape.max_depth - 1}")
        if probs.is_cuda:
            from eagle4_b200.ops import tree_ops

            tree_ops.tree_step(self, bs, step, probs, tokens, hidden, deltas=step in self.delta_slots)
        else:
            self.step_reference(bs, step, probs, tokens, hidden)
            if step in self.delta_slots:
                self._store_deltas_reference(bs, step)

    def step_reference(self, bs: int, step: int, probs: torch.Tensor, tokens: torch.Tensor,
                       hidden: torch.Tensor) -> None:
        s, k = self.shape, self.shape.top_k
        layer = (self.front_scores[:bs, :, None] * probs.float().view(bs, k, k)).reshape(bs, k * k)
        start = s.layer_start(step + 1)
        self.scores[:bs, start: start + k * k] = layer
        ltoks = tokens.long().view(bs, k * k)
        self.tokens[:bs, start: start + k * k] = ltoks
        top, pick = torch.topk(layer, k, dim=-1)
        p0 = s.num_parents(step + 1)
        self.parents[:bs, p0: p0 + k] = pick + start
        lane = torch.div(pick, k, rounding_mode="floor")
        rows = (lane + torch.arange(bs, device=lane.device)[:, None] * k).reshape(-1)
        self.front_scores[:bs] = top
        self.front_tokens[: bs * k] = torch.gather(ltoks, 1, pick).reshape(-1)
        self.front_hidden[: bs * k] = hidden.view(bs * k, -1).index_select(0, rows)
        self.front_nodes[:bs] = pick + start
        self.ancestors[:bs] = self.ancestors[:bs].reshape(bs * k, -1).index_select(0, rows).view(bs, k, -1)
        self.best_prev[:bs] = self.best[:bs]
        self.best[:bs] = torch.topk(torch.cat([self.best[:bs], layer], dim=-1), s.work_cap, dim=-1).values
        self.layer_top[:bs] = top

    def _store_deltas_reference(self, bs: int, slot: int) -> None:
        k = self.shape.top_k
        extra = self.layer_top[:bs, None, :] * self._extra_mask.view(1, k + 1, k)
        best = self.best_prev[:bs, None, :].expand(bs, k + 1, self.shape.work_cap)
        merged = torch.sort(torch.cat([best, extra], dim=-1), dim=-1, descending=True).values
        sums = merged[..., : self.max_verify].cumsum(dim=-1)
        self.deltas[slot] = sums.mean(dim=0).transpose(0, 1)

    # --------------------------------------------------------------- verify
    def rank(self, bs: int, depth: int, count: int) -> Tuple[torch.Tensor, torch.Tensor]:
        count = min(count, self.shape.num_nodes(depth))
        return self.rank_reference(bs, depth, count)

    def rank_reference(self, bs: int, depth: int, count: int) -> Tuple[torch.Tensor, torch.Tensor]:
        n = self.shape.num_nodes(depth)
        decayed = self.scores[:bs, :n] * self.decay[:n]
        top, ranked = torch.sort(decayed, dim=-1, descending=True, stable=True)
        root = top.new_full((bs, 1), ROOT_SCORE)
        return ranked[:, :count], torch.cumsum(torch.cat([root, top[:, :count]], dim=-1), dim=-1)

    def select(self, bs: int, depth: int, ranked: torch.Tensor, verify_tokens: int) -> VerifySelection:
        index = torch.sort(ranked[:, : verify_tokens - 1], dim=-1).values
        toks = torch.gather(self.tokens[:bs], 1, index)
        return VerifySelection(self.parents[:bs, : self.shape.num_parents(depth)].contiguous(), index, toks)

    def verify_rows(self, bs: int, depth: int, count: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """The best ``count`` nodes of a ``depth``-level tree as verify rows: tokens ``[bs, count]`` and parent rows
        ``[bs, count + 1]`` int32 (row 0 the root with -1; row r's parent row, 0 meaning the root)."""
        if self.scores.is_cuda:
            from eagle4_b200.ops import tree_ops

            return tree_ops.select_rows(self, bs, depth, count)
        return self.verify_rows_reference(bs, depth, count)

    def node_parent(self, bs: int, index: torch.Tensor) -> torch.Tensor:
        """Global parent node of each node in ``index`` (``-1`` for depth-1 nodes)."""
        layer = torch.bucketize(index, self._layer_bounds, right=True)
        local = index - self._layer_starts[layer]
        col = self._frontier_base[(layer - 1).clamp(min=0)] + torch.div(local, self.shape.top_k,
                                                                          rounding_mode="floor")
        return torch.where(layer == 0, torch.full_like(index, -1), self.parents[:bs].gather(1, col))

    def verify_rows_reference(self, bs: int, depth: int, count: int) -> Tuple[torch.Tensor, torch.Tensor]:
        ranked, _ = self.rank_reference(bs, depth, count)
        index = torch.sort(ranked, dim=-1).values
        toks = torch.gather(self.tokens[:bs], 1, index)
        pnode = self.node_parent(bs, index)
        hit = index[:, None, :] == pnode[:, :, None]
        prow = torch.where(hit.any(-1), hit.int().argmax(-1) + 1, torch.zeros_like(pnode))
        root = prow.new_full((bs, 1), -1)
        self.last_nodes = torch.cat([index.new_full((bs, 1), -1), index], dim=1)
        return toks, torch.cat([root, prow], dim=1).int()


def rows_meta(parent_rows: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Depth (root 0) and 64-bit ancestor-or-self mask of every verify row from ``parent_rows [bs, n]``.

    Row ``r`` sees row ``j`` iff bit ``j`` of ``mask[r]`` is set. Rows follow node order (parents first), so one
    pass in row order suffices. Returned as ``(depth int32 [bs, n], mask int64 [bs, n])``.
    """
    bs, n = parent_rows.shape
    if n > 64:
        raise ValueError("verify rows are limited to 64 (one mask word per row)")
    pr = parent_rows.long().cpu()
    depth = torch.zeros(bs, n, dtype=torch.int64)
    mask = torch.zeros(bs, n, dtype=torch.int64)
    for r in range(n):
        p = pr[:, r]
        has = p >= 0
        pc = p.clamp(min=0)
        bit = torch.tensor(1, dtype=torch.int64) << r if r < 63 else torch.tensor(-(1 << 63), dtype=torch.int64)
        pm = mask.gather(1, pc[:, None]).squeeze(1)
        pd = depth.gather(1, pc[:, None]).squeeze(1)
        mask[:, r] = torch.where(has, pm, torch.zeros_like(pm)) | bit
        depth[:, r] = torch.where(has, pd + 1, torch.zeros_like(pd))
    return depth.int().to(parent_rows.device), mask.to(parent_rows.device)
