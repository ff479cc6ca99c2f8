"""The ``eagle_harness`` speculative method inside vLLM (Model Runner V2 builds carrying the speculative-method
registry): method spec, speculator (draft rounds through ``plugins.host_round.HostDrafter``), tree accept (greedy and
sampled) and accepted-path KV compaction on this package's kernels.

Reference counterparts: ``eagle_harness/vllm/{plugin,speculator,tree_accept,round_commit,verify_layout}.py``. vLLM
keeps scheduling, KV allocation and the target forward; the speculator drafts the tree (round policy + draft tree),
lays out the verify rows (depth positions and 64-bit ancestor words), accepts with the fused kernels and compacts the
accepted rows' KV. Classes subclass vLLM's when it is installed, ``object`` otherwise.
"""

from __future__ import annotations

from typing import Optional

import torch

from eagle4_b200 import ops
from eagle4_b200.core.config import HarnessConfig, Mode
from eagle4_b200.core.draft_tree import rows_meta
from eagle4_b200.core.limits import req_to_token_span
from eagle4_b200.plugins.common import accept_greedy_rows, host_base
from eagle4_b200.plugins.vllm.config import MethodConfig

METHOD = "eagle_harness"

_MethodSpec = host_base("vllm.v1.spec_decode.registry:SpeculativeMethodSpec")
_Speculator = host_base("vllm.v1.worker.gpu.spec_decode.speculator:DraftModelSpeculator")


class HarnessMethodSpec(_MethodSpec):
    """How vLLM sizes the method: the tree budget from the opaque method config (``plugins.vllm.config``), KV headroom
    per request."""

    config: Optional[HarnessConfig] = None
    method: Optional[MethodConfig] = None

    def configure(self, speculative_config):
        """Fill vLLM's speculative config (draft-token schedule per batch size, ``num_speculative_tokens``, the
        draft's aux layers: ``plugins.vllm.schedule``) and keep the parsed method."""
        from eagle4_b200.plugins.vllm.schedule import configure_speculative_config

        self.method = configure_speculative_config(speculative_config)
        self.config = self.method.harness
        self.top_k, self.depth, self.width = self.method.node_top_k, self.method.tree_depth, self.method.max_verify_width
        return {"num_speculative_tokens": getattr(speculative_config, "num_speculative_tokens", None)
                or self.method.num_speculative_tokens, "max_verify_width": self.width}

    def num_lookahead_tokens(self, page_size: int = 1) -> int:
        return req_to_token_span(self.top_k, self.depth, self.width, page_size)

    def linear_attn_verify_extension(self, vllm_config):
        """GDN / Mamba2 layers under tree verify (``plugins.vllm.tree_verify``); None for chains (vLLM's kernels)."""
        from eagle4_b200.plugins.vllm.tree_verify import create_extension

        return create_extension(vllm_config)


class TreeAccept:
    """The rejection sampler vLLM calls on the verify rows: the fused greedy accept (temperature 0, on target ids or
    logits), or with a sampling drafter the recursive tree rejection over the drafter's draw-order children and q
    store (the target's logits at the engine's temperature; ``eagle_harness/vllm/tree_accept.py``)."""

    def __init__(self, drafter=None):
        self.drafter = drafter  # a HostDrafter (its engine keeps the round's q store and round counter)

    def __call__(self, target: torch.Tensor, draft_tokens: torch.Tensor, parent_rows: torch.Tensor):
        """``target``: ``[bs * w]`` target ids or ``[bs * w, V]`` logits. Returns (accepted rows [bs, w] (-1 pad),
        counts [bs], bonus tokens [bs])."""
        bs = draft_tokens.shape[0]
        eng = self.drafter.engine if self.drafter is not None else None
        if eng is not None and eng.sampled:
            if target.dim() != 2:
                raise ValueError("a sampled tree accept needs the target's logits")
            from eagle4_b200.runtime.engine import SAMPLED_STREAM

            acc, cnt, bonus = ops.sampled_accept(target.float(), eng.temperature, parent_rows, draft_tokens,
                                                 self.drafter.tree_nodes(bs), eng.q_store, eng.q_ids, eng.node_slot,
                                                 eng.top_k, eng.seed, eng.round_ctr, SAMPLED_STREAM)
            ops.advance_round(eng.round_ctr)
            return acc, cnt, bonus
        if target.dim() == 2:
            target = target.argmax(-1)
        return accept_greedy_rows(target, draft_tokens, parent_rows)


class HarnessSpeculator(_Speculator):
    """Tree speculator: the draft rounds (``HostDrafter``: extend, steps under the round policy, verify selection),
    the verify layout, the accept and the KV compaction; vLLM keeps scheduling, KV allocation and the target forward.

    The draft side is reached through ``load_model`` (vLLM hands the speculator its models; here the draft model and
    the tree budget), ``prefill_request`` after a request's target prefill, ``propose_tree`` before each verify and
    ``accept_round`` after it (``eagle_harness/vllm/speculator.py:96,247``)."""

    drafter = None
    batch_policy = None
    served_rounds = None

    def load_model(self, draft_model, *, max_reqs: int, max_len: int, tree=(12, 4, 16), config=None,
                   temperature: float = 0.0, seed: int = 0, method: Optional[MethodConfig] = None,
                   linear_layers=None, key=None) -> None:
        """``draft_model``: a ``DraftModel`` or the vLLM draft model class holding one. ``method`` (a parsed
        ``method_config``) sets the tree, the harness config, the batch policy and the
        served-round recording; without it ``tree`` = (depth, top-k, verify width) and ``config`` do.
        ``linear_layers``: the target's GDN / Mamba2 layers, checked to hand their rows to the tree verify (a tree
        only); ``key``: this worker's setup, checked against the calibration data's before serving."""
        import dataclasses

        from eagle4_b200.core.chain_width import chain_widths
        from eagle4_b200.plugins.host_round import HostDrafter, ServedTreeRounds
        from eagle4_b200.plugins.vllm.batch_policy import BatchPolicy

        from eagle4_b200.models.draft import DraftModel

        if not isinstance(draft_model, DraftModel):  # vLLM's model class (plugins.vllm.models) after load_weights
            draft_model = draft_model.draft
            if draft_model is None:
                raise RuntimeError("the draft model's weights are not loaded")
        if method is not None:
            if key is not None:
                from eagle4_b200.plugins.vllm.schedule import verify_widths

                verify_widths(method, key=key)  # refuses data measured on another setup
            tree = (method.tree_depth, method.node_top_k, method.max_verify_width)
            config = method.harness
            if method.depth_stop_gain is None:  # no depth stop: full-depth trees (the static policy)
                config = dataclasses.replace(config, mode=Mode.STATIC)
        steps, top_k, width = tree
        if linear_layers is not None and top_k > 1:
            from eagle4_b200.plugins.vllm.tree_verify import check_tree_verifiable

            check_tree_verifiable(linear_layers)
        self.drafter = HostDrafter(draft_model, max_reqs=max_reqs, max_len=max_len, steps=steps, top_k=top_k,
                                   verify_tokens=width, config=config, temperature=temperature, seed=seed)
        schedule = None
        if config is not None and config.data_path:
            schedule = chain_widths(config.data_path, width, max_reqs, allow_no_spec=True)
        self.batch_policy = BatchPolicy(verify_batch_limit=self.drafter.engine.verify_batch_limit, schedule=schedule,
                                        max_num_reqs=max_reqs)
        if method is not None and method.record_rounds:
            self.served_rounds = ServedTreeRounds(config.data_path)

    def suspend_drafting(self, num_reqs, req_ids):
        """vLLM's per-batch hook: True decodes this batch natively."""
        return self.batch_policy.suspend_drafting(num_reqs, req_ids)

    def verify_budget(self, req_ids, num_draft_tokens):
        """vLLM's per-batch hook: each request's drafts to verify (a prefix of its tree rows)."""
        return self.batch_policy.verify_budget(req_ids, num_draft_tokens)

    def prefill_request(self, req_id, prompt_ids: torch.Tensor, aux_hidden_states: torch.Tensor, first_token) -> None:
        self.drafter.admit(req_id, prompt_ids, aux_hidden_states, first_token)

    def propose_tree(self, req_ids):
        """The round's verify rows per request: (tokens [bs, w], parent rows [bs, w], positions offsets and ancestor
        words from ``verify_layout`` once the host adds its base positions)."""
        return self.drafter.propose(req_ids)

    def accept_round(self, req_ids, draft_tokens: torch.Tensor, parent_rows: torch.Tensor, target: torch.Tensor,
                     aux_hidden_states: Optional[torch.Tensor], round_us: Optional[float] = None):
        """Accept the verified rows (``target``: ids or logits of the rows) and hand the accepted path to the drafter.
        ``round_us``: the host's measured period of this round (recorded when ``record_rounds`` is on). Returns
        (accepted rows, counts, bonus, emitted tokens per request)."""
        from eagle4_b200.plugins.vllm.tree_verify import commit_accepted

        acc, cnt, bonus = self.make_rejection_sampler()(target, draft_tokens, parent_rows)
        commit_accepted(acc, cnt)  # the target's GDN / Mamba2 states resume after the accepted path
        emitted = self.drafter.accept(req_ids, draft_tokens, acc, cnt, bonus, aux_hidden_states)
        if self.served_rounds is not None and round_us:
            self.served_rounds.record(len(req_ids), draft_tokens.shape[1], round_us,
                                      sum(len(e) for e in emitted) / max(1, len(emitted)))
        return acc, cnt, bonus, emitted

    def close(self) -> None:
        """The method ends: recorded served rounds are written."""
        if self.served_rounds is not None:
            self.served_rounds.flush()

    def finish_request(self, req_id) -> None:
        self.drafter.release(req_id)

    @staticmethod
    def verify_layout(parent_rows: torch.Tensor, base_positions: torch.Tensor):
        """Positions of the verify rows (``base + depth``) and their 64-bit ancestor-or-self words."""
        depth, mask = rows_meta(parent_rows)
        return base_positions[:, None] + depth.long(), mask

    def prepare_verify_inputs(self, parent_rows: torch.Tensor, base_positions: torch.Tensor):
        """The verify layout; also stages the tree for the target's GDN / Mamba2 layers."""
        from eagle4_b200.plugins.vllm.tree_verify import stage_tree

        stage_tree(parent_rows)
        return self.verify_layout(parent_rows, base_positions)

    def make_rejection_sampler(self, *args, **kwargs):
        return TreeAccept(self.drafter)

    def post_accept(self, k_caches, v_caches, src_slots: torch.Tensor, dst_slots: torch.Tensor) -> None:
        """Move the accepted rows' K/V from their verify slots to the committed positions (all layers, one launch)."""
        ops.kv_commit(k_caches, v_caches, src_slots, dst_slots)
