"""``LlamaForCausalLMEagle4`` for TokenSpeed: a draft forward that exits with candidate rows instead of logits.

TokenSpeed's drafter asks its draft model's exit for the sampled rows of a forward and then for the top-``k`` next
tokens of each. The EAGLE-4 head never needs the full-vocabulary logits for that: ``exit_logits`` selects the sampled
rows (``ctx.gather_ids``, unless the forward already ran one row per request) and returns them as
:class:`CandidateRows` with an empty ``[rows, 0]`` logits tensor; ``candidate_topk(normed, k)`` then runs the low-rank
shortlist, the exact re-scoring of the ``C`` candidates and the top-``k`` of their softmax (this package's candidate
kernels). Under a vocabulary-sharded head, ``candidate_head`` merges the ranks' candidates before the softmax
(``plugins.candidate_logits``), which equals the softmax of the full row with ``-inf`` outside the candidates.
Prompt log-probabilities and query shards are refused: the head computes no full-vocabulary rows.

Reference counterpart: ``eagle_harness/tokenspeed/models.py:39,50,126,144`` (``CandidateRows``, the model, its
candidate head and the candidate all-gather); the exit's field names are TokenSpeed's.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Iterable, Optional, Set, Tuple

import torch

from eagle4_b200 import ops
from eagle4_b200.models import weights as wmod
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.eagle4_config import check_supported, draft_config_from_hf
from eagle4_b200.plugins.candidate_logits import (AllGather, Candidates, merge_candidates, scatter_to_vocab,
                                                  shard_candidates)


@dataclass
class CandidateRows:
    """A draft forward's exit. ``normed``: the sampled rows' final-norm output (the candidate head's input);
    ``hidden_states``: what the next draft forward takes; ``next_token_logits``: empty ``[rows, 0]``."""

    next_token_logits: torch.Tensor
    hidden_states: torch.Tensor
    normed: torch.Tensor
    candidate_ids: Optional[torch.Tensor] = None


class LlamaForCausalLMEagle4(torch.nn.Module):
    def __init__(self, config: Any, mapping: Any = None, quant_config: Any = None, prefix: str = ""):
        """``mapping``: TokenSpeed's parallel mapping (``mapping.lm_head`` with ``tp_rank`` / ``tp_size``); the head is
        sharded over it when ``tp_size > 1`` and an ``all_gather`` is given to ``load_weights``."""
        super().__init__()
        if quant_config is not None:
            raise NotImplementedError("eagle4_b200 drafts are served in bf16 (no quantization)")
        hf = config.to_dict() if hasattr(config, "to_dict") else dict(config)
        check_supported(hf)
        self.cfg = draft_config_from_hf(hf)
        if not self.cfg.low_rank:
            raise NotImplementedError("the TokenSpeed exit needs the EAGLE-4 low-rank candidate head")
        if self.cfg.draft_vocab_size not in (None, self.cfg.vocab_size):
            raise NotImplementedError("EAGLE-4 drafts with a reduced vocabulary (d2t) are not served on TokenSpeed")
        head = getattr(mapping, "lm_head", None)
        self.tp_rank = int(getattr(head, "tp_rank", 0))
        self.tp_size = int(getattr(head, "tp_size", 1))
        self.num_candidates = int(self.cfg.low_rank["num_candidates"])
        self.draft: Optional[DraftModel] = None
        self.all_gather: Optional[AllGather] = None
        self.vocab_start, self.vocab_rows = 0, self.cfg.vocab_size

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]], embed: Optional[torch.Tensor] = None,
                     all_gather: Optional[AllGather] = None) -> Set[str]:
        """The checkpoint (full vocabulary). With ``tp_size > 1`` and ``all_gather``, this rank keeps its vocabulary
        shard of ``lm_head`` and the low-rank scores (``ceil(V / tp)`` rows) and merges candidates over the group."""
        sd = {name: t for name, t in weights}
        self.draft = DraftModel(self.cfg, wmod.draft_from_state_dict(self.cfg, sd, embed=embed))
        if self.tp_size > 1 and all_gather is not None:
            w = self.draft.w
            per = -(-self.cfg.vocab_size // self.tp_size)
            self.vocab_start = self.tp_rank * per
            self.vocab_rows = max(0, min(per, self.cfg.vocab_size - self.vocab_start))
            self.shard = {n: w[n][self.vocab_start:self.vocab_start + self.vocab_rows].contiguous()
                          for n in ("lm_head", "lr_scores")}
            self.all_gather = all_gather
        return set(sd)

    def _model(self) -> DraftModel:
        if self.draft is None:
            raise RuntimeError("load_weights first")
        return self.draft

    # ---- the exit: sampled rows, no logits
    def exit_logits(self, input_ids: torch.Tensor, hidden_states: torch.Tensor, aux_hidden_states: Any,
                    ctx: Any) -> CandidateRows:
        """``hidden_states``: the forward's normed rows; ``aux_hidden_states``: one tensor, the next forward's
        input rows; ``ctx``: TokenSpeed's logits context (``gather_ids``, ``logits_rows_selected``)."""
        if getattr(ctx, "input_logprob_rows", None) is not None or getattr(ctx, "query_shard", None) is not None:
            raise NotImplementedError("the EAGLE-4 draft computes no prompt log-probabilities and runs no query shards")
        (nxt,) = aux_hidden_states
        gather = getattr(ctx, "gather_ids", None)
        if gather is not None and not getattr(ctx, "logits_rows_selected", False) \
                and gather.shape[0] != hidden_states.shape[0]:
            hidden_states, nxt = hidden_states[gather], nxt[gather]
        return CandidateRows(next_token_logits=hidden_states.new_empty(hidden_states.shape[0], 0),
                             hidden_states=nxt, normed=hidden_states)

    # ---- candidate head
    def candidates(self, normed: torch.Tensor) -> Candidates:
        """The top ``C`` candidates of each row (exact fp32 logits, global ids), merged over the ranks."""
        w = self._model().w
        if self.all_gather is None:
            ids, logits = ops.candidate_logits(normed, w["lr_down"], w["lr_scores"], w["lm_head"], self.num_candidates)
            return Candidates(logits.float(), ids.long())
        shard = shard_candidates(normed, w["lr_down"], self.shard["lr_scores"], self.shard["lm_head"],
                                 num_candidates=min(self.num_candidates, self.vocab_rows),
                                 vocab_start=self.vocab_start, vocab_rows=self.vocab_rows)
        return merge_candidates(shard, self.num_candidates, self.all_gather)

    def candidate_head(self, normed: torch.Tensor, k: int):
        """``(candidates, (probabilities [rows, k], ids [rows, k]))``: the softmax over the ``C`` candidates and its
        top ``k`` (largest first)."""
        c = self.candidates(normed)
        probs = torch.softmax(c.logits, dim=-1)
        p, pick = torch.topk(probs, k, dim=-1)
        return c, (p, torch.gather(c.token_ids, -1, pick))

    def candidate_topk(self, normed: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-``k`` next tokens of each row: (fp32 probabilities, int64 ids)."""
        if self.all_gather is None:
            return self._model().candidates(normed, k)
        return self.candidate_head(normed, k)[1]

    def full_logits(self, normed: torch.Tensor) -> torch.Tensor:
        """``[rows, vocab]`` fp32, ``-inf`` outside the candidates (for a host sampler that reads whole rows)."""
        return scatter_to_vocab(self.candidates(normed), self.cfg.vocab_size)


EntryClass = [LlamaForCausalLMEagle4]
