"""The EAGLE_HARNESS drafter inside TokenSpeed: the tree policy the ``Eagle`` drafter delegates to (seed the first
lanes, expand the next ones, choose the verify window) with the draft tree and round policy of this package.

Both TokenSpeed lines are served: the public policy names (``capabilities`` contract) and the release engine's
private names alias the same methods. Reference counterpart: ``eagle_harness/tokenspeed/drafter.py``.
"""

from __future__ import annotations

from typing import Optional

import torch

from eagle4_b200.core.draft_tree import DraftTree, TreeShape
from eagle4_b200.plugins.common import host_base

ALGORITHM = "EAGLE_HARNESS"
_Eagle = host_base("tokenspeed.runtime.execution.drafter.eagle:Eagle")


class HarnessDrafter(_Eagle):
    """Tree policy over a fixed-shape draft tree (graph-capturable buffers, one per batch bucket)."""

    tree: Optional[DraftTree] = None
    options = None  # TokenSpeedOptions of the launch

    def configure_algorithm(self, algorithm_config):
        """TokenSpeed hands over the launch's ``--speculative-algorithm-config`` (``plugins.tokenspeed.config``)."""
        from eagle4_b200.plugins.tokenspeed.config import parse_algorithm_config

        self.options = parse_algorithm_config(algorithm_config)
        return self.options

    def bind_tree_shape(self, top_k: int, depth: int, max_bs: int, hidden: int, device, verify: int) -> None:
        self.tree = DraftTree(TreeShape(top_k, depth), max_bs, hidden, torch.bfloat16, device, max_verify=verify)

    def seed_tree(self, bs, logits_output, frontier):
        """Depth 1: the root's top-K candidates (``logits_output``: probs, tokens, hidden of the root rows)."""
        probs, tokens, hidden = logits_output
        self.tree.stage_root(bs, probs, tokens, hidden)
        self.tree.begin(bs)
        return self.tree.front_tokens[: bs * self.tree.shape.top_k]

    def expand_tree(self, bs, step, logits_output):
        """Depth ``step + 1``: the frontier's K x K children scored, the best K kept."""
        probs, tokens, hidden = logits_output
        self.tree.step(bs, step, probs, tokens, hidden)
        return self.tree.front_tokens[: bs * self.tree.shape.top_k]

    def verify_window(self, bs, next_tokens):
        """The best ``next_tokens - 1`` nodes (plus the root) as verify rows: tokens and parent rows."""
        depth = self.tree.shape.max_depth
        return self.tree.verify_rows(bs, depth, int(next_tokens) - 1)

    # whole rounds: TokenSpeed may hand the draft round to this package (``plugins.host_round.HostDrafter``)
    drafter = None

    def attach(self, drafter) -> None:
        self.drafter = drafter

    def prefill_request(self, rid, prompt_ids, aux_hidden_states, first_token) -> None:
        self.drafter.admit(rid, prompt_ids, aux_hidden_states, first_token)

    def draft_round(self, rids):
        """Extend, steps under the round policy and the verify selection: (tokens [bs, w], parent rows [bs, w])."""
        return self.drafter.propose(rids)

    def accept_round(self, rids, tokens, target_ids, parent_rows, aux_hidden_states):
        """Greedy accept of the verified rows (target ids per row), then the accepted path to the drafter; returns
        (accepted rows, counts, bonus, emitted tokens per request)."""
        from eagle4_b200.plugins.common import accept_greedy_rows

        acc, cnt, bonus = accept_greedy_rows(target_ids, tokens, parent_rows)
        return acc, cnt, bonus, self.drafter.accept(rids, tokens, acc, cnt, bonus, aux_hidden_states)

    # the release engine's names for the same policy
    _seed_tree_lanes = seed_tree
    _expand_tree_lanes = expand_tree
    _draft_window = verify_window
