"""Full-vocabulary logits from the EAGLE-4 candidate head, for hosts whose samplers read a whole-vocabulary row.

The candidate head scores every token with the low-rank estimate ``(h @ down^T) @ scores^T``, keeps the top ``C``
ids and re-scores those exactly (``lm_head[id] . h``, fp32). A host that shards the vocabulary over tensor-parallel
ranks runs that per shard (``shard_candidates``: the shard's real rows only, ids offset to global) and merges the
ranks' ``C`` candidates into the top ``C`` overall (``merge_candidates``, one all-gather of ``2C`` values per row). The
host's sampler and its top-k read ``scatter_to_vocab``'s ``[rows, vocab]`` fp32 row, ``-inf`` outside the candidates:
its softmax equals the softmax over the candidates, so the host draws exactly what the engine's own candidate head
draws. ``candidate_logits_processor`` wraps it as SGLang's ``LogitsProcessor`` for the draft's prefill path.

Reference counterpart: ``eagle_harness/sglang/candidate_logits.py:38,55`` (``shard_candidates``,
``merge_candidates``); the host-facing names are kept so a host integration reads the same. The shortlist and the
exact re-scoring run this package's candidate kernels (``ops.candidate_logits``).
"""

from __future__ import annotations

from typing import Callable, NamedTuple, Optional

import torch

from eagle4_b200 import ops

AllGather = Callable[[torch.Tensor], torch.Tensor]  # [rows, n] -> [rows, ranks * n], rank-major along the last dim


class Candidates(NamedTuple):
    logits: torch.Tensor     # [rows, C] fp32, exact
    token_ids: torch.Tensor  # [rows, C] int64, global vocabulary ids


def shard_candidates(hidden: torch.Tensor, down_proj: torch.Tensor, score_head: torch.Tensor, lm_head: torch.Tensor,
                     *, num_candidates: int, vocab_start: int = 0, vocab_rows: Optional[int] = None) -> Candidates:
    """This rank's ``C`` candidates over its vocabulary shard. ``score_head [V_shard, r]`` and ``lm_head
    [V_shard, H]`` may carry padding rows past ``vocab_rows`` (the shard's real rows); those are never chosen."""
    rows = score_head.shape[0] if vocab_rows is None else int(vocab_rows)
    if not 0 < num_candidates <= rows:
        raise ValueError(f"num_candidates={num_candidates} must be in [1, {rows}] (the shard's real vocabulary rows)")
    ids, logits = ops.candidate_logits(hidden, down_proj, score_head[:rows], lm_head[:rows], num_candidates)
    return Candidates(logits.float(), ids.long() + int(vocab_start))


def merge_candidates(shard: Candidates, num_candidates: int, all_gather: Optional[AllGather] = None) -> Candidates:
    """The top ``num_candidates`` over every rank's candidates (``all_gather`` None: one rank, returned as is)."""
    if all_gather is None:
        return Candidates(shard.logits.float(), shard.token_ids)
    logits = all_gather(shard.logits.float())
    ids = all_gather(shard.token_ids)
    top, pick = torch.topk(logits, num_candidates, dim=-1, sorted=False)
    return Candidates(top, torch.gather(ids, -1, pick))


def group_all_gather(group=None) -> AllGather:
    """An ``AllGather`` over a ``torch.distributed`` process group (NCCL on GPUs, gloo on CPU)."""
    import torch.distributed as dist

    def gather(x: torch.Tensor) -> torch.Tensor:
        parts = [torch.empty_like(x) for _ in range(dist.get_world_size(group))]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=-1)

    return gather


def scatter_to_vocab(candidates: Candidates, vocab_size: int) -> torch.Tensor:
    """``[rows, vocab_size]`` fp32 logits: the candidates' exact logits, ``-inf`` everywhere else."""
    full = torch.full((candidates.logits.shape[0], vocab_size), float("-inf"), dtype=torch.float32,
                      device=candidates.logits.device)
    return full.scatter_(1, candidates.token_ids, candidates.logits.float())


def candidate_logits_processor(config, candidate_fn: Callable[[torch.Tensor], Candidates]):
    """SGLang's ``LogitsProcessor`` with the candidate head as its LM head; ``candidate_fn(hidden) -> Candidates`` runs
    the shard and merge steps (it owns the weights). SGLang is imported here, so this module imports without it."""
    from sglang.srt.layers.logits_processor import LogitsProcessor

    class CandidateLogitsProcessor(LogitsProcessor):
        def __init__(self):
            super().__init__(config)
            if getattr(self, "do_tensor_parallel_all_gather_dp_attn", False) or getattr(self, "use_attn_tp_group",
                                                                                        False):
                raise NotImplementedError("the EAGLE-4 candidate head runs under plain tensor parallelism only")
            if getattr(self, "logit_scale", None) is not None or getattr(self, "final_logit_softcapping", None):
                raise NotImplementedError("the EAGLE-4 candidate head has no logit scale or soft-capping")

        def _get_logits(self, hidden_states, lm_head, logits_metadata, embedding_bias=None, use_logits_buffer=True):
            if embedding_bias is not None:
                raise NotImplementedError("the EAGLE-4 candidate head takes no embedding bias")
            logits = scatter_to_vocab(candidate_fn(hidden_states), self.vocab_size)
            return self._copy_logits_to_buffer(logits, logits_metadata, use_buffer=use_logits_buffer)

    return CandidateLogitsProcessor()
