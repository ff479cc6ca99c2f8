"""The ``eagle_harness`` speculative method inside vLLM (Model Runner V2 builds carrying the speculative-method
registry): method spec, speculator, tree accept and accepted-path KV compaction on this package's kernels.

Reference counterparts: ``eagle_harness/vllm/{plugin,speculator,tree_accept,round_commit,verify_layout}.py``. vLLM
keeps scheduling, KV allocation and the target forward; the speculator drafts the tree (round policy + draft tree),
lays out the verify rows (depth positions and 64-bit ancestor words), accepts with the fused kernels and compacts the
accepted rows' KV. Classes subclass vLLM's when it is installed, ``object`` otherwise.
"""

from __future__ import annotations

from typing import Optional

import torch

from eagle4_b200 import ops
from eagle4_b200.core.config import HarnessConfig, parse_harness_config
from eagle4_b200.core.draft_tree import rows_meta
from eagle4_b200.core.limits import req_to_token_span
from eagle4_b200.plugins.common import accept_greedy_rows, host_base

METHOD = "eagle_harness"

_MethodSpec = host_base("vllm.v1.spec_decode.registry:SpeculativeMethodSpec")
_Speculator = host_base("vllm.v1.worker.gpu.spec_decode.speculator:DraftModelSpeculator")


class HarnessMethodSpec(_MethodSpec):
    """How vLLM sizes the method: the tree budget from the opaque method config, KV headroom per request."""

    config: Optional[HarnessConfig] = None

    TREE_KEYS = {"node_top_k": 4, "tree_depth": 12, "max_verify_width": 16}  # the vLLM tree's own keys

    def configure(self, speculative_config):
        raw = dict(getattr(speculative_config, "method_config", None) or {})
        tree = {k: int(raw.pop(k, v)) for k, v in self.TREE_KEYS.items()}
        self.config = parse_harness_config(raw)
        self.top_k, self.depth, self.width = tree["node_top_k"], tree["tree_depth"], tree["max_verify_width"]
        return {"num_speculative_tokens": self.width - 1, "max_verify_width": self.width}

    def num_lookahead_tokens(self, page_size: int = 1) -> int:
        return req_to_token_span(self.top_k, self.depth, self.width, page_size)


class TreeAccept:
    """The rejection sampler vLLM calls on the verify logits: fused greedy accept (temperature 0) or the sampled
    tree walk (temperature > 0; q store and node slots from the speculator's sampled draft)."""

    def __init__(self, sampled_state=None):
        self.sampled_state = sampled_state

    def __call__(self, target_ids: torch.Tensor, draft_tokens: torch.Tensor, parent_rows: torch.Tensor):
        return accept_greedy_rows(target_ids, draft_tokens, parent_rows)


class HarnessSpeculator(_Speculator):
    """Tree speculator: verify layout, accept and KV compaction (the draft forward is the host's draft model)."""

    @staticmethod
    def verify_layout(parent_rows: torch.Tensor, base_positions: torch.Tensor):
        """Positions of the verify rows (``base + depth``) and their 64-bit ancestor-or-self words."""
        depth, mask = rows_meta(parent_rows)
        return base_positions[:, None] + depth.long(), mask

    def prepare_verify_inputs(self, parent_rows: torch.Tensor, base_positions: torch.Tensor):
        return self.verify_layout(parent_rows, base_positions)

    def make_rejection_sampler(self, *args, **kwargs):
        return TreeAccept()

    def post_accept(self, k_caches, v_caches, src_slots: torch.Tensor, dst_slots: torch.Tensor) -> None:
        """Move the accepted rows' K/V from their verify slots to the committed positions (all layers, one launch)."""
        ops.kv_commit(k_caches, v_caches, src_slots, dst_slots)
