"""Draft-tree updates on CUDA tensors: one sm_100a kernel launch per update (``eagle4_b200/csrc/tree.cu``).

The round's first level, each depth's step and the verify-row selection are single kernels; a level whose work
deltas the cost model reads computes them in the same launch (per-request merges, then the batch mean in the last
CTA to finish).
"""

from __future__ import annotations

import torch


def _C():
    from eagle4_b200.ops.native import _C

    return _C


def _delta_args(tree, slot: int, deltas: bool):
    """The per-request rows, the output slot and the arrival counter of an in-kernel work-delta update."""
    if not deltas:
        return torch.Tensor(), torch.Tensor(), torch.Tensor()
    if getattr(tree, "_delta_rows", None) is None:
        k = tree.shape.top_k
        tree._delta_rows = torch.zeros(tree.max_bs, tree.max_verify, k + 1, dtype=torch.float32, device=tree.device)
        tree._delta_counter = torch.zeros(1, dtype=torch.int32, device=tree.device)
    return tree._delta_rows, tree.deltas[slot], tree._delta_counter


def tree_begin(tree, bs: int, root_score: float, *, deltas: bool) -> None:
    rows, out, counter = _delta_args(tree, 0, deltas)
    _C().tree_begin(tree.root_probs[:bs].float().contiguous(), tree.root_tokens[:bs].long().contiguous(),
                    tree.root_hidden[:bs].contiguous(), bs, tree.shape.top_k, bool(tree.keep_draw_order),
                    float(root_score), tree.scores, tree.tokens, tree.front_scores, tree.front_tokens,
                    tree.front_hidden, tree.front_nodes, tree.best, tree.best_prev, tree.layer_top, rows, out, counter)


def tree_step(tree, bs: int, step: int, probs, tokens, hidden, *, deltas: bool) -> None:
    s = tree.shape
    rows, out, counter = _delta_args(tree, step, deltas)
    _C().tree_step(probs, tokens, hidden, bs, s.top_k, step, s.layer_start(step + 1), s.num_parents(step + 1),
                   tree.scores, tree.tokens, tree.parents, tree.front_scores, tree.front_tokens, tree.front_hidden,
                   tree.front_nodes, tree.ancestors, tree.best, tree.best_prev, tree.layer_top, rows, out, counter)


def select_rows(tree, bs: int, depth: int, count: int):
    n = tree.shape.num_nodes(depth)
    count = min(count, n)
    toks, prow, nodes = _C().select_rows(tree.scores, tree.decay, tree.tokens, tree.parents, bs, n, tree.shape.top_k,
                                         count)
    tree.last_nodes = nodes
    return toks, prow
