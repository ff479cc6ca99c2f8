"""The stop rule of one speculative tree round, fixed once per round: ``RoundPlan``.

A tree round drafts depth by depth; at DECIDE depths the cost model compares the work the next level would gain
(the batch-mean work deltas the step kernel copies to the host) with a bar that depends on the depth and the
batch's cost row. Everything except the deltas is known when the round starts, so the plan holds it per depth: the
step kind, the bar, the cost terms, the deltas row the host reads and the width column compared with column 0. The
engine's draft loop runs from the plan (``Engine._draft_round``); ``RoundPlan.stop`` evaluates the cost model's
DECIDE rule in the same order and precision (Python floats), so a round stops where ``CostModel.tree_width`` would.
``tensors`` packs the plan into device arrays, the input a device-side stop would read.

Chain rounds, sampled trees and the fixed tree shape without a cost model take no plan (``round_plan`` returns
None); they keep the cost model's per-depth calls.

Reference counterpart: ``RoundPlan`` / ``round_plan`` / ``GraphRound`` and the ``EAGLE_DRAFT_ROUND_CHECK``
comparison in ``eagle_harness/sglang/draft_round.py:54-160,472-620`` (the closed draft-round megakernel it checks
is not built here).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import torch

from eagle4_b200.core.cost_model import CostModel, WidthStep

KEEP, LAUNCH, DECIDE, LAST = 0, 1, 2, 3
KIND = {WidthStep.KEEP: KEEP, WidthStep.LAUNCH: LAUNCH, WidthStep.DECIDE: DECIDE, WidthStep.LAST: LAST}


@dataclass
class RoundPlan:
    """Per depth ``d`` (0 is the round's first level): ``kind[d]`` and, at DECIDE depths, ``bar[d]``. A DECIDE
    depth stops the round when ``(deltas[lane] - deltas[0]) / cost * ratio * async_ratio < bar[d]``, with
    ``deltas`` the host row ``budget`` copied at the last LAUNCH depth."""

    kind: List[int]
    bar: List[float]
    cost: float
    ratio: float
    async_ratio: float
    budget: int
    lane: int

    @property
    def fixed_depth(self) -> Optional[int]:
        """Depth levels of a round that decides nothing (the first LAST depth + 1), else None."""
        if DECIDE in self.kind:
            return None
        return next((d + 1 for d, k in enumerate(self.kind) if k == LAST), len(self.kind))

    @property
    def min_depth(self) -> int:
        """The fewest depth levels the round can stop at."""
        return next((d + 1 for d, k in enumerate(self.kind) if k in (DECIDE, LAST)), len(self.kind))

    def stop(self, depth: int, deltas: Sequence[float]) -> bool:
        return (deltas[self.lane] - deltas[0]) / self.cost * self.ratio * self.async_ratio < self.bar[depth]

    def tensors(self, device) -> Dict[str, torch.Tensor]:
        """The plan as device arrays: ``kind`` int32 and ``bar`` float64 per depth, ``terms`` float64
        ``[cost, ratio, async_ratio]``, ``index`` int32 ``[budget, lane]``."""
        return {"kind": torch.tensor(self.kind, dtype=torch.int32, device=device),
                "bar": torch.tensor(self.bar, dtype=torch.float64, device=device),
                "terms": torch.tensor([self.cost, self.ratio, self.async_ratio], dtype=torch.float64, device=device),
                "index": torch.tensor([self.budget, self.lane], dtype=torch.int32, device=device)}


def round_plan(policy: CostModel, bs: int, context: int, max_depth: int) -> Optional[RoundPlan]:
    """The plan the cost model's per-depth calls give this round (with their side effect: a DECIDE sets the size
    tier's one-request flag before the width cap is read), or None for chain rounds."""
    if policy.chain_rounds:
        return None
    row = policy.draft_cost_row(bs, context)
    # the deltas row, like the cost row, is read before the round's first DECIDE (which can change the size tier
    # both depend on), as the per-depth loop reads them
    budget = policy.deltas_budget(policy.history_verify_num(bs)) - 1
    kinds: List[int] = []
    bars: List[float] = []
    lane = 0
    for depth in range(max_depth):
        step = policy.width_step(depth)
        kinds.append(KIND[step])
        bar = 0.0
        if step is WidthStep.DECIDE:
            policy.state.tiny = bs == 1
            lane = policy._capped_width()
            bar = policy.tree_depth_threshold(depth, row)
        bars.append(bar)
    return RoundPlan(kinds, bars, row.cost_values[-1], row.model_cost_ratio, policy.params.async_layer_ratio, budget,
                     lane)


class RoundCheck:
    """Counts the DECIDE depths where a plan's stop and the cost model's own ``tree_width`` disagree (a check mode
    of the engine's draft loop; the count stays 0 when the plan restates the rule)."""

    def __init__(self) -> None:
        self.decided = 0
        self.disagreed = 0
        self.notes: List[str] = []
        self._tiny = False
        self._first = True

    def begin(self, policy: CostModel) -> None:
        """Before ``round_plan``: the size tier's one-request flag as the round's first DECIDE would see it (the
        plan sets it for the rest of the round, as that DECIDE does)."""
        self._tiny = policy.state.tiny
        self._first = True

    def compare(self, policy: CostModel, plan: RoundPlan, depth: int, bs: int, past: int, row, deltas) -> None:
        ours = plan.stop(depth, deltas)
        after = policy.state.tiny
        policy.state.tiny = self._tiny if self._first else after
        theirs = policy.tree_width(depth, bs, past, row, deltas).stop
        policy.state.tiny = after
        self._first = False
        self.decided += 1
        if ours != theirs:
            self.disagreed += 1
            if len(self.notes) < 16:
                self.notes.append(f"bs {bs} depth {depth}: plan {ours}, cost model {theirs}, deltas {list(deltas)}")

    def summary(self) -> str:
        return f"{self.disagreed} of {self.decided} decided depths disagree"
