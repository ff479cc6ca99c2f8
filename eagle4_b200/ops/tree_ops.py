"""Draft-tree updates on CUDA tensors: one sm_100a kernel launch per update (``eagle4_b200/csrc/tree.cu``).

``DraftTree.begin`` stays a handful of tensor copies (once per round); the per-depth step and the verify-row
selection are single kernels. The work deltas read by the cost model's decisions use the tensor definition.
"""

from __future__ import annotations

import torch


def _C():
    from eagle4_b200.ops.native import _C

    return _C


def tree_begin(tree, bs: int, root_score: float, *, deltas: bool) -> None:
    tree.begin_reference(bs)
    if deltas:
        tree._store_deltas_reference(bs, 0)


def tree_step(tree, bs: int, step: int, probs, tokens, hidden, *, deltas: bool) -> None:
    s = tree.shape
    _C().tree_step(probs, tokens, hidden, bs, s.top_k, step, s.layer_start(step + 1), s.num_parents(step + 1),
                   tree.scores, tree.tokens, tree.parents, tree.front_scores, tree.front_tokens, tree.front_hidden,
                   tree.front_nodes, tree.ancestors, tree.best, tree.best_prev, tree.layer_top)
    if deltas:
        tree._store_deltas_reference(bs, step)


def select_rows(tree, bs: int, depth: int, count: int):
    n = tree.shape.num_nodes(depth)
    count = min(count, n)
    toks, prow, nodes = _C().select_rows(tree.scores, tree.decay, tree.tokens, tree.parents, bs, n, tree.shape.top_k,
                                         count)
    tree.last_nodes = nodes
    return toks, prow
