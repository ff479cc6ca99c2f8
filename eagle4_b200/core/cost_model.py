"""The measured cost model that sizes every draft round (host side).

From calibrated or live-measured costs it decides:

* the **tree width / stop** at every second depth: the work one more draft level adds per unit of draft cost, scaled
  by the target/draft cost ratio, against a threshold that grows with depth (reference
  ``eagle_harness/core/cost_model.py:549-617``);
* the **verify budget**: pairwise pruning of verify widths whose score gain per measured verify-cost increase falls
  under a stability threshold (``:764-804``);
* the **chain stop** of top-1 chains, by tier, with a lookahead over a verify-cost cliff (``:620-683``);
* the batch **size class** from the verify cost at 8 tokens (``:341-368``);
* immutable per-batch **policy tables** a device-side policy can read (``:370-424``, ``:685-719``).

The constants, the formulas (including the order of their floating-point operations, so exported thresholds are
bit-identical) and the order in which decisions update the model's state are the behaviour users calibrate against,
and equal the reference's. The structure is this package's: the per-size-class constants live in one rule table, the
round state (size class, tiny flag, interval) in one small record, decisions are functions of a cost *view* of one
batch size, and the policy exports replay the decisions on a fresh model of the same tables.
"""

from __future__ import annotations

import copy
import enum
import math
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, NamedTuple, Optional, Sequence, Tuple

from eagle4_b200.core.cost_table import BatchCostTable
from eagle4_b200.core.limits import (
    MAX_BATCH_SIZE_CHAIN,
    MAX_BATCH_SIZE_TREE,
    MAX_CHAIN_DEPTH,
    MAX_CHAIN_VERIFY_NUM,
    MAX_NODE_TOP_K,
    MAX_VERIFY_NUM,
    ComputeIntensity,
    check_shape,
    max_batch_size,
    nearest_cost_batch_size,
)


class SizeClass(enum.IntEnum):
    SMALL = 0
    MEDIUM = 1
    LARGE = 2
    HUGE = 3


class ChainTier(enum.IntEnum):
    TINY = 0
    SMALL = 1
    MEDIUM = 2
    LARGE = 3


@dataclass(frozen=True)
class ChainCoef:
    threshold: float
    depth_loss: float
    cost_power: float


@dataclass(frozen=True)
class CostModelParams:
    threshold: float = 2.5
    async_layer_ratio: float = 0.9
    depth_loss_ratio: float = 0.04
    chain_coef: Tuple[ChainCoef, ChainCoef, ChainCoef, ChainCoef] = (
        ChainCoef(2.60, 0.24, 0.00),
        ChainCoef(2.85, 0.24, 0.00),
        ChainCoef(2.54, 0.24, 0.70),
        ChainCoef(1.55, 0.24, 0.00),
    )
    chain_ref_cost: float = 2.43
    chain_cliff_min_cost: float = 0.15
    chain_cliff_ratio: float = 1.5
    chain_scale_tiny: float = 1.25
    chain_tiny_max_bs: int = 2
    chain_scale_small: float = 1.45
    chain_scale_medium: float = 2.00


def depth_loss_ratio(draft_family: str, *, target_is_moe: bool, intensity: ComputeIntensity) -> float:
    """Acceptance lost per draft depth: 0.04 (EAGLE-4), 0.08 (EAGLE-3), 0.64 (EAGLE), else 0.16; twice that for an
    MoE target; a chain's is the family value itself (doubled, then halved)."""
    base = {"eagle4": 0.04, "eagle3": 0.08, "eagle": 0.64}.get(draft_family, 0.16)
    factor = 2.0 if (target_is_moe or intensity is ComputeIntensity.CHAIN) else 1.0
    r = base * factor
    return r * 0.5 if intensity is ComputeIntensity.CHAIN else r


@dataclass(frozen=True)
class DraftCostRow:
    cost_values: Tuple[float, ...]
    cost_index: Tuple[int, ...]
    cost_state: float
    adjust_cost_ratio: float
    model_cost_ratio: float
    batch_size_ratio: float


@dataclass(frozen=True)
class VerifyCost:
    value: Tuple[float, ...]
    index: Tuple[int, ...]
    threshold: float


@dataclass(frozen=True)
class ChainStopTerms:
    """One chain decision: ``gain = raw*2/gain_scale``; stop when ``gain/cost < threshold``; with a cliff, the
    two-step gain ``gain + raw*2/cliff_gain_scale`` over ``cliff_cost`` gets a second chance."""

    gain_scale: float
    cost: float
    threshold: float
    cliff_gain_scale: float
    cliff_cost: float


@dataclass(frozen=True)
class ChainPolicyBatch:
    cache_length_step: int
    intervals: Tuple[Tuple[ChainStopTerms, ...], ...]


@dataclass(frozen=True)
class ChainPolicyCosts:
    batches: Tuple[ChainPolicyBatch, ...]


@dataclass(frozen=True)
class TreePolicyInterval:
    verify_widths: Tuple[int, ...]
    verify_cost_deltas: Tuple[Tuple[float, ...], ...]
    draft_cost: float
    model_cost_ratio: float
    depth_thresholds: Tuple[Tuple[float, ...], ...]  # rows: SMALL..HUGE, then tiny
    verify_tier: int
    verify_thresholds: Tuple[float, float]


@dataclass(frozen=True)
class TreePolicyBatch:
    cost_batch_size: int
    cache_length_step: int
    intervals: Tuple[TreePolicyInterval, ...]


@dataclass(frozen=True)
class TreePolicyCosts:
    batches: Tuple[TreePolicyBatch, ...]
    history_floors: Tuple[int, ...]
    initial_widths: Tuple[int, ...]
    async_layer_ratio: float


@dataclass(frozen=True)
class WidthDecision:
    width: int
    verify_num: int
    stop: bool


class WidthStep(enum.Enum):
    KEEP = "keep"  # grow at the full top-k, no decision
    LAST = "last"  # the deepest level: stop
    LAUNCH = "launch"  # grow at the capped width; the host copies this depth's deltas for the next decision
    DECIDE = "decide"  # read the deltas copied one depth earlier and decide


# ---------------------------------------------------------------------------------------------------- small rules
def find_majority(nums: Sequence[int]) -> int:
    """The first value to reach a strict majority of ``nums`` while scanning them in order; -1 when none does."""
    need = len(nums) // 2 + 1
    tally: Dict[int, int] = {}
    for x in nums:
        tally[x] = tally.get(x, 0) + 1
        if tally[x] == need:
            return x
    return -1


def verify_cost_delta(previous: float, current: float) -> float:
    """Verify cost increase from ``previous`` to ``current``; a rise of 0.04 (relative) or less is free."""
    rise = current - previous
    return rise if rise > 0.04 else 0.0


def stable_verify_thresholds(threshold: float) -> Tuple[float, float]:
    """Pruning bars ``(when the recent majority budget is within the candidate, when it is beyond it)``."""
    return threshold * 0.95, threshold * 1.05


def adjust_cost_ratio(model_cost_ratio: float) -> float:
    """Threshold multiplier for a target/draft cost ratio. A ratio outside 5..100 cannot drive speculation."""
    if model_cost_ratio < 5:
        raise ValueError(f"model_cost_ratio {model_cost_ratio:.2f} is below 5: the draft costs too much against the "
                         "target for speculation to pay")
    if model_cost_ratio > 100:
        raise ValueError(f"model_cost_ratio {model_cost_ratio:.2f} is above 100: the draft's timing looks wrong")
    steps = (8, 1.30), (12, 1.10), (17, 1.30), (23, 1.50), (32, 1.80), (64, 2.20)
    return next((f for bound, f in steps if model_cost_ratio < bound), 2.70)


class _ClassRule(NamedTuple):
    """What a batch's size class sets."""

    verify_threshold_high: float  # pruning threshold at high compute intensity
    verify_threshold_other: float  # ... at the other intensities
    batch_size_ratio: float  # draft-threshold scale
    history_floor: int  # smallest verify budget remembered for the batch
    chain_slack: int  # extra chain verify tokens above the recent budget
    width_cap: int  # widest tree level


_RULES = {
    SizeClass.SMALL: _ClassRule(2.40, 2.00, 1.25, 16, 4, 8),
    SizeClass.MEDIUM: _ClassRule(2.10, 1.80, 1.50, 8, 2, 8),
    SizeClass.LARGE: _ClassRule(1.80, 1.60, 1.75, 4, 2, 4),
    SizeClass.HUGE: _ClassRule(1.50, 1.40, 2.00, 2, 0, 4),
}
_TINY_FLOOR, _TINY_SLACK, _TINY_BS_RATIO = 32, 4, 1.00  # a batch of one request
CHAIN_COST_INDEX = (0, 1, 3, 5, 7, 9, 11, 13, 15)


def classify_verify(cost_at8: float, batch_size: int, target_is_moe: bool) -> SizeClass:
    """Size class from the verify cost at 8 tokens relative to 1 token (values outside the plausible range are
    refused: below 0.85, or 0.70 for an MoE target, and above 4)."""
    floor = 0.70 if target_is_moe else 0.85
    if cost_at8 <= 1.25 or batch_size == 1:
        if cost_at8 < floor:
            raise ValueError(f"verify cost at 8 tokens is {cost_at8} of one token's: implausibly low")
        return SizeClass.SMALL
    if cost_at8 > 4.0:
        raise ValueError(f"verify cost at 8 tokens is {cost_at8} of one token's: implausibly high")
    bounds = ((1.60, SizeClass.MEDIUM), (2.20, SizeClass.LARGE))
    return next((c for b, c in bounds if cost_at8 < b), SizeClass.HUGE)


@dataclass
class _RoundState:
    """The mutable part of the model between calls: the last classified size, whether the batch is one request,
    and the context interval of the last priced round."""

    size: SizeClass = SizeClass.SMALL
    tiny: bool = False
    interval: int = 0

    @property
    def rule(self) -> _ClassRule:
        return _RULES[self.size]


def _cost_at8(target) -> float:
    """The target's relative cost at the first measured width of 8 tokens or more (the widest if none is)."""
    return next((r for r, i in zip(target.ratio, target.index) if i >= 7), target.ratio[-1])


# ---------------------------------------------------------------------------------------------------- the model
@dataclass
class CostModel:
    """Per-worker stateful cost model (not thread safe)."""

    tables: Dict[int, BatchCostTable]
    params: CostModelParams
    intensity: ComputeIntensity
    node_top_k: int
    tree_depth: int
    verify_num: int
    target_is_moe: bool = False
    state: _RoundState = field(default_factory=_RoundState)
    # the requested budgets of the last five verify-width decisions (seeded with five distinct sentinels)
    recent_verify_nums: List[int] = field(default_factory=lambda: [-5, -4, -3, -2, -1])

    def __post_init__(self) -> None:
        self.max_batch_size = max_batch_size(self.intensity)
        self.set_tables(self.tables)
        # the last 16 verify budgets per batch size
        self._budgets = [[self.verify_num] * 16 for _ in range(self.max_batch_size)]

    # ---------------------------------------------------------------- tables
    def set_tables(self, tables: Dict[int, BatchCostTable], refused: Iterable[int] = ()) -> None:
        """Swap in new tables (live refresh); the round state and the budget history stay. Batch sizes in
        ``refused`` are never used."""
        self.tables = tables
        usable = sorted(set(tables) - set(refused))
        self._nearest = {b: nearest_cost_batch_size(b, usable) for b in range(1, self.max_batch_size + 1)} \
            if usable else {}

    def table(self, batch_size: int) -> Optional[BatchCostTable]:
        """The cost table that prices ``batch_size`` (the nearest measured size), None without tables."""
        if not self._nearest:
            return None
        if batch_size not in self._nearest:
            raise ValueError(f"batch size {batch_size} is not in 1..{self.max_batch_size}")
        return self.tables[self._nearest[batch_size]]

    def _priced(self, batch_size: int) -> BatchCostTable:
        t = self.table(batch_size)
        if t is None:
            raise ValueError(f"no cost table prices batch size {batch_size}")
        return t

    @property
    def interval_index(self) -> int:
        return self.state.interval

    def update_interval(self, batch_size: int, average_cache_len: int) -> BatchCostTable:
        t = self._priced(batch_size)
        self.state.interval = t.interval_index(average_cache_len)
        return t

    def draft_cost_row(self, batch_size: int, average_cache_len: int) -> DraftCostRow:
        """Draft-side inputs of a round at this context (also selects the interval)."""
        t = self.update_interval(batch_size, average_cache_len)
        ratio = t.model_ratio[self.state.interval]
        draft = t.intervals[self.state.interval].draft
        scale = _TINY_BS_RATIO if self.state.tiny else self.state.rule.batch_size_ratio
        scale = max(1.0, scale / ((20 / ratio + 1) / 2))
        return DraftCostRow(draft.ratio, draft.index, draft.ratio[-1], adjust_cost_ratio(ratio), ratio, scale)

    def verify_cost(self, batch_size: int, average_cache_len: int) -> Optional[VerifyCost]:
        """The target's verify cost curve at this context (also classifies the batch's size)."""
        t = self.table(batch_size)
        if t is None:
            return None
        target = t.intervals[t.interval_index(average_cache_len)].target
        self.state.size = classify_verify(_cost_at8(target), batch_size, self.target_is_moe)
        rule = self.state.rule
        bar = rule.verify_threshold_high if self.intensity is ComputeIntensity.HIGH else rule.verify_threshold_other
        return VerifyCost(target.ratio, target.index, bar)

    # ---------------------------------------------------------------- verify budget history
    def _floor(self) -> int:
        return _TINY_FLOOR if self.state.tiny else self.state.rule.history_floor

    def history_verify_num(self, batch_size: int) -> int:
        """The verify budget a round of ``batch_size`` starts from: the largest recent budget, floored by size class
        (for chains: plus a slack, capped at the configured width)."""
        recent = max(self._budgets[batch_size - 1])
        if self.intensity is ComputeIntensity.CHAIN:
            slack = _TINY_SLACK if self.state.tiny else self.state.rule.chain_slack
            return min(recent + slack, self.verify_num)
        return max(recent, self._floor())

    @property
    def max_history_verify_num(self) -> int:
        if self.intensity is ComputeIntensity.CHAIN:
            return self.verify_num
        return max(self.verify_num, _TINY_FLOOR, max(r.history_floor for r in _RULES.values()))

    def record_verify_num(self, batch_size: int, verify_num: int) -> None:
        self._budgets[batch_size - 1] = self._budgets[batch_size - 1][1:] + [verify_num]

    def verify_count(self, batch_size: int, draft_count: int) -> int:
        """How many drafted nodes a round ranks for verification."""
        if self.intensity is ComputeIntensity.CHAIN:
            return draft_count
        recent = max(max(self._budgets[batch_size - 1]), self._floor())
        return min(self.verify_num, draft_count, max(2 * recent, 16))

    # ---------------------------------------------------------------- round shape
    @property
    def chain_rounds(self) -> bool:
        """Top-1 chains verified up to the full calibrated chain width."""
        return (self.intensity is ComputeIntensity.CHAIN and self.node_top_k == 1
                and self.verify_num == CHAIN_COST_INDEX[-1] + 1)

    @property
    def verifies_whole_draft(self) -> bool:
        return self.chain_rounds

    def deltas_budget(self, past_verify_num: int) -> int:
        return self.verify_num if self.chain_rounds else past_verify_num

    @property
    def launch_depths(self) -> Tuple[int, ...]:
        first = 1 if self.chain_rounds else 0
        return tuple(range(first, self.tree_depth - 1, 2))

    def width_step(self, depth: int) -> WidthStep:
        """What the drafter does at ``depth``: chains decide at even depths >= 2; trees (after two full-width levels
        for one request) decide at odd depths."""
        if self.chain_rounds:
            if depth == self.tree_depth - 1:
                return WidthStep.LAST
            if depth == 0:
                return WidthStep.KEEP
            return (WidthStep.DECIDE, WidthStep.LAUNCH)[depth % 2]
        if self.state.tiny and depth < 2:
            return WidthStep.KEEP
        if depth == self.tree_depth - 1:
            return WidthStep.LAST
        return (WidthStep.LAUNCH, WidthStep.DECIDE)[depth % 2]

    def _capped_width(self) -> int:
        return min(self.node_top_k, self.state.rule.width_cap)

    def tree_depth_threshold(self, depth: int, row: DraftCostRow) -> float:
        """Gain per draft cost that one more level must reach at ``depth``."""
        scale = row.batch_size_ratio
        if depth <= 1:
            scale = (scale + 1.00) / 2
        elif depth > 5 and scale > 1.3:
            scale = scale * 1.1
        p = self.params
        return p.threshold * (depth * p.depth_loss_ratio + 1.0) * row.adjust_cost_ratio * scale

    def tree_width(self, depth: int, batch_size: int, past_verify_num: int, row: Optional[DraftCostRow],
                   deltas: Optional[Sequence[float]] = None) -> WidthDecision:
        """The width of the next level at ``depth``, or stop. ``deltas``: the batch-mean work gained by widths
        0..K at the depth whose deltas the host copied (DECIDE steps need them)."""
        step = self.width_step(depth)
        if self.chain_rounds and step is not WidthStep.LAST:
            return WidthDecision(1, past_verify_num, step is WidthStep.DECIDE
                                 and self.chain_stop(depth, batch_size, _need(deltas, depth)))
        if step is WidthStep.LAST:
            return WidthDecision(-1, -1, True)
        if step is WidthStep.KEEP:
            return WidthDecision(self.node_top_k, past_verify_num, False)
        if step is WidthStep.LAUNCH:
            return WidthDecision(self._capped_width(), past_verify_num, False)
        deltas = _need(deltas, depth)
        self.state.tiny = batch_size == 1
        width = self._capped_width()
        per_cost = (deltas[width] - deltas[0]) / row.cost_values[-1] * row.model_cost_ratio \
            * self.params.async_layer_ratio
        if per_cost < self.tree_depth_threshold(depth, row):
            return WidthDecision(width, past_verify_num, True)
        if self.state.size in (SizeClass.MEDIUM, SizeClass.LARGE):  # next power of two
            width = 1 << (width - 1).bit_length()
        return WidthDecision(width, past_verify_num, False)

    # ---------------------------------------------------------------- chains
    def classify_chain(self, batch_size: int, cost_ratio: Optional[Sequence[float]] = None
                       ) -> Tuple[ChainTier, float]:
        """Chain tier from the mean relative cost of verifying 2, 4 and 8 tokens."""
        if cost_ratio is None:
            cost_ratio = self._priced(batch_size).intervals[self.state.interval].target.ratio
        scale = (cost_ratio[1] + cost_ratio[3] + cost_ratio[7]) / (3.0 * cost_ratio[0])
        p = self.params
        if scale <= p.chain_scale_tiny or batch_size <= p.chain_tiny_max_bs:
            return ChainTier.TINY, scale
        bounds = ((p.chain_scale_small, ChainTier.SMALL), (p.chain_scale_medium, ChainTier.MEDIUM))
        return next((t for b, t in bounds if scale < b), ChainTier.LARGE), scale

    def _chain_decides(self, depth: int) -> bool:
        return depth != 0 and depth != self.tree_depth - 1 and depth % 2 == 0

    def chain_stop(self, depth: int, batch_size: int, deltas: Optional[Sequence[float]] = None) -> bool:
        if not self._chain_decides(depth):
            return False
        deltas = _need(deltas, depth)
        t = self.chain_stop_terms(depth, batch_size)
        raw = deltas[1] - deltas[0]
        gain = raw * 2.0 / t.gain_scale
        stop = gain / t.cost < t.threshold
        if stop and t.cliff_cost > 0.0:  # a cliff ahead: the two-step extension gets a second chance
            stop = (gain + raw * 2.0 / t.cliff_gain_scale) / t.cliff_cost < t.threshold
        return stop

    def chain_stop_terms(self, depth: int, batch_size: int) -> ChainStopTerms:
        if not self._chain_decides(depth):
            return ChainStopTerms(0.0, 0.0, 0.0, 0.0, 0.0)
        t = self._priced(batch_size)
        target = t.intervals[self.state.interval].target
        if tuple(target.index) != CHAIN_COST_INDEX or any(type(i) is not int for i in target.index):
            raise ValueError(f"chain costs must be measured at widths {[i + 1 for i in CHAIN_COST_INDEX]}, "
                             f"found indices {list(target.index)}")
        per_step = target.ratio[1:]  # verify cost after 1, 2, 4, ... drafted steps
        coef = self.params.chain_coef[self.classify_chain(batch_size, target.ratio)[0]]
        p = self.params
        here = depth // 2
        ahead = min(here + 1, len(per_step) - 1)
        draft_step = 1.0 / t.model_ratio[self.state.interval]
        cost = draft_step * 2 + max(0, per_step[ahead] - per_step[here])
        mean_iter = sum(c + draft_step * (2 * i + 1) for i, c in enumerate(per_step)) / len(per_step)
        threshold = coef.threshold * (p.chain_ref_cost / mean_iter) ** coef.cost_power
        cliff_scale = cliff_cost = 0.0
        if ahead + 1 < len(per_step):
            rise_next = per_step[ahead] - per_step[here]
            rise_after = per_step[ahead + 1] - per_step[ahead]
            if rise_next > p.chain_cliff_min_cost and rise_next > p.chain_cliff_ratio * max(rise_after, 0.0):
                cliff_scale = 1.0 + (depth + 2) * coef.depth_loss
                cliff_cost = draft_step * 4 + max(0, per_step[ahead + 1] - per_step[here])
        return ChainStopTerms(1.0 + depth * coef.depth_loss, cost, threshold, cliff_scale, cliff_cost)

    # ---------------------------------------------------------------- verify budget
    def verify_num_paged(self, scores: Sequence[float], requested: int, batch_size: int, average_cache_len: int,
                         *, lagged: bool) -> Tuple[int, bool]:
        """Verify tokens per request, from cumulative node scores (this round's, or last round's when ``lagged``).

        Every measured width up to the request is a candidate; a wider candidate whose score gain over a narrower
        one does not pay for its verify-cost increase falls back to the narrowest drafted width. The bar is lower
        while the recent majority budget is within the candidate (a stable budget stays stable)."""
        majority = find_majority(self.recent_verify_nums)
        limit = min(len(scores) if lagged else requested, requested)
        self.recent_verify_nums = self.recent_verify_nums[1:] + [requested]
        cost = self.verify_cost(batch_size, average_cache_len)
        if cost is None:
            raise ValueError(f"no verify cost for batch size {batch_size}")
        widths = [i for i in cost.index if i < limit]
        if max(widths) == 0:
            self.recent_verify_nums[-1] = 1
            return 1, False
        fallback = widths[1]
        alive = [True] * len(widths)
        low, high = stable_verify_thresholds(cost.threshold)
        for a in range(len(widths) - 1):
            for b in range(a + 1, len(widths)):
                held = widths[b] if alive[b] else fallback
                rise = verify_cost_delta(cost.value[a], cost.value[b])
                if rise > 0.0 and (scores[widths[b]] - scores[widths[a]]) / rise < (low if majority <= held + 1
                                                                                    else high):
                    alive[b] = False
        chosen = max(w if ok else fallback for w, ok in zip(widths, alive)) + 1
        self.recent_verify_nums[-1] = chosen
        if chosen == 1 or requested < chosen:
            chosen = min(widths[1:]) + 1
        return chosen, False

    # ---------------------------------------------------------------- policy export
    def _fresh(self, **changes) -> "CostModel":
        """A new model of the same configuration and tables (every table usable, a fresh budget history and round
        state): the exports replay decisions on it, leaving this model untouched."""
        kw = dict(tables=self.tables, params=self.params, intensity=self.intensity, node_top_k=self.node_top_k,
                  tree_depth=self.tree_depth, verify_num=self.verify_num, target_is_moe=self.target_is_moe)
        kw.update(changes)
        return CostModel(**kw)

    def tree_policy_costs(self) -> TreePolicyCosts:
        """Immutable per-batch inputs of the tree policy (for a device-side policy)."""
        _check_tree_export(self)
        twin = self._fresh()
        variants = [(False, s) for s in SizeClass] + [(True, SizeClass.SMALL)]  # every size class, then tiny
        batches = []
        for bs in range(1, MAX_BATCH_SIZE_TREE + 1):
            t = twin._priced(bs)
            intervals = []
            for iid in range(len(t.intervals)):
                ctx = (iid + 1) * t.cache_length_step
                vc = twin.verify_cost(bs, ctx)
                tier = int(twin.state.size)
                thresholds = []
                for tiny, size in variants:
                    twin.state.tiny, twin.state.size = tiny, size
                    row = twin.draft_cost_row(bs, ctx)
                    thresholds.append(tuple(twin.tree_depth_threshold(d, row) for d in range(self.tree_depth)))
                if not all(math.isfinite(x) for r in thresholds for x in r):
                    raise ValueError(f"depth thresholds are not finite at batch size {bs}, interval {iid}")
                intervals.append(TreePolicyInterval(
                    verify_widths=tuple(vc.index),
                    verify_cost_deltas=tuple(tuple(verify_cost_delta(a, b) for b in vc.value) for a in vc.value),
                    draft_cost=row.cost_values[-1], model_cost_ratio=row.model_cost_ratio,
                    depth_thresholds=tuple(thresholds), verify_tier=tier,
                    verify_thresholds=stable_verify_thresholds(vc.threshold)))
            batches.append(TreePolicyBatch(t.batch_size, t.cache_length_step, tuple(intervals)))
        twin = twin._fresh(verify_num=1)
        floors, widths = [], []
        for tiny, size in variants:
            twin.state.tiny, twin.state.size = tiny, size
            floors.append(twin.history_verify_num(1))
            if not tiny:
                widths.append(twin.tree_width(0, 1, 1, twin.draft_cost_row(1, 0)).width)
        return TreePolicyCosts(tuple(batches), tuple(floors), tuple(widths), self.params.async_layer_ratio)

    def chain_policy_costs(self) -> ChainPolicyCosts:
        """Immutable per-batch chain stop terms (for a device-side chain policy)."""
        _check_chain_export(self)
        twin = self._fresh()
        twin.state = copy.copy(self.state)
        batches = []
        for bs in range(1, MAX_BATCH_SIZE_CHAIN + 1):
            t = twin._priced(bs)
            intervals = []
            for iid in range(len(t.intervals)):
                twin.state.interval = iid
                try:
                    terms = tuple(twin.chain_stop_terms(d, bs) for d in range(self.tree_depth))
                except (OverflowError, ZeroDivisionError) as e:
                    raise ValueError(f"chain stop terms overflow at batch size {bs}, interval {iid}") from e
                for d, term in enumerate(terms):
                    if not _terms_ok(term, self._chain_decides(d)):
                        raise ValueError(f"chain stop terms are invalid at batch size {bs}, interval {iid}, "
                                         f"depth {d}: {term}")
                intervals.append(terms)
            batches.append(ChainPolicyBatch(t.cache_length_step, tuple(intervals)))
        return ChainPolicyCosts(tuple(batches))


def _need(deltas: Optional[Sequence[float]], depth: int) -> Sequence[float]:
    if deltas is None:
        raise ValueError(f"the decision at depth {depth} needs the work deltas copied from the device")
    return deltas


def _terms_ok(t: ChainStopTerms, decides: bool) -> bool:
    vals = (t.gain_scale, t.cost, t.threshold, t.cliff_gain_scale, t.cliff_cost)
    if any(not math.isfinite(v) or v < 0 for v in vals):
        return False
    if decides and min(t.gain_scale, t.cost, t.threshold) <= 0:
        return False
    return (t.cliff_gain_scale > 0) == (t.cliff_cost > 0)


# ---------------------------------------------------------------------------------------------------- export checks
def _int_in(name: str, v, lo: int, hi: Optional[int] = None) -> Optional[str]:
    if type(v) is not int or v < lo or (hi is not None and v > hi):
        return f"{name}={v!r} is not an integer in {lo}..{hi if hi is not None else 'inf'}"
    return None


def _raise_first(problems: Sequence[Optional[str]], what: str) -> None:
    found = [p for p in problems if p]
    if found:
        raise ValueError(f"{what}: {found[0]}")


def _check_tree_export(m: CostModel) -> None:
    _raise_first([_int_in("tree_depth", m.tree_depth, 2), _int_in("node_top_k", m.node_top_k, 1),
                  _int_in("verify_num", m.verify_num, 2)], "tree policy export")
    check_shape(m.intensity, m.node_top_k, m.tree_depth, m.verify_num, MAX_BATCH_SIZE_TREE)
    p = m.params
    _raise_first([f"{n}={getattr(p, n)!r} must be finite and positive" for n in ("threshold", "async_layer_ratio")
                  if not (math.isfinite(getattr(p, n)) and getattr(p, n) > 0)]
                 + [f"depth_loss_ratio={p.depth_loss_ratio!r} must be finite and non-negative"
                    if not (math.isfinite(p.depth_loss_ratio) and p.depth_loss_ratio >= 0) else None],
                 "tree policy export")
    _check_tables(m, chain=False)


def _check_chain_export(m: CostModel) -> None:
    if m.intensity is not ComputeIntensity.CHAIN:
        raise ValueError("chain policy export: the model must run at chain intensity")
    _raise_first([_int_in("node_top_k", m.node_top_k, 1, 1), _int_in("tree_depth", m.tree_depth, 2, MAX_CHAIN_DEPTH),
                  _int_in("verify_num", m.verify_num, 2, MAX_CHAIN_VERIFY_NUM)], "chain policy export")
    p = m.params
    if len(p.chain_coef) != len(ChainTier):
        raise ValueError("chain policy export: one chain coefficient per tier (four) is needed")
    for c in p.chain_coef:
        good = isinstance(c, ChainCoef) and all(math.isfinite(v) for v in (c.threshold, c.depth_loss, c.cost_power))
        if not good or c.threshold <= 0 or c.depth_loss < 0 or c.cost_power < 0:
            raise ValueError(f"chain policy export: chain coefficient {c!r} is out of range")
    for name in ("chain_ref_cost", "chain_cliff_min_cost", "chain_cliff_ratio", "chain_scale_tiny",
                 "chain_scale_small", "chain_scale_medium"):
        v = getattr(p, name)
        if not math.isfinite(v) or v < 0 or (v == 0 and name != "chain_cliff_min_cost"):
            raise ValueError(f"chain policy export: {name}={v!r} is out of range")
    if not p.chain_scale_tiny < p.chain_scale_small < p.chain_scale_medium:
        raise ValueError("chain policy export: the tier scales must increase from tiny to medium")
    _raise_first([_int_in("chain_tiny_max_bs", p.chain_tiny_max_bs, 0, MAX_BATCH_SIZE_CHAIN)], "chain policy export")
    _check_tables(m, chain=True)


def _curve_problem(name: str, curve, bound: int, chain: bool) -> Optional[str]:
    n = len(curve.index)
    if n == 0 or (name == "target" and not 2 <= n <= 32):
        return f"{name} curve has {n} widths"
    if len(curve.value) != n or len(curve.ratio) != n:
        return f"{name} curve lengths differ"
    idx = curve.index
    if idx[0] != 0 or any(type(i) is not int or not 0 <= i < bound for i in idx) \
            or any(b <= a for a, b in zip(idx, idx[1:])):
        return f"{name} curve indices {idx!r} are not increasing from 0 below {bound}"
    if chain and name == "target" and tuple(idx) != CHAIN_COST_INDEX:
        return f"chain target indices {idx!r} differ from {CHAIN_COST_INDEX}"
    if any(not math.isfinite(v) or v <= 0 for v in (*curve.value, *curve.ratio)):
        return f"{name} costs are not finite and positive"
    return None


def _check_tables(m: CostModel, *, chain: bool) -> None:
    what = f"{'chain' if chain else 'tree'} policy export"
    if not m.tables:
        raise ValueError(f"{what}: no cost tables")
    for bs, t in m.tables.items():
        if type(bs) is not int or bs < 1 or (chain and bs > MAX_BATCH_SIZE_CHAIN) \
                or type(t.batch_size) is not int or t.batch_size != bs:
            raise ValueError(f"{what}: table key {bs!r} holds batch size {t.batch_size!r}")
        if type(t.cache_length_step) is not int or t.cache_length_step <= 0:
            raise ValueError(f"{what}: batch size {bs} has context step {t.cache_length_step!r}")
        if not t.intervals or len(t.intervals) != len(t.model_ratio):
            raise ValueError(f"{what}: batch size {bs} lacks intervals or model ratios")
        for iid, (iv, ratio) in enumerate(zip(t.intervals, t.model_ratio)):
            if not math.isfinite(ratio) or ratio <= 0:
                raise ValueError(f"{what}: batch size {bs}, interval {iid}: model ratio {ratio!r}")
            if not chain:
                adjust_cost_ratio(ratio)
            for name, curve, bound in (("target", iv.target, MAX_VERIFY_NUM), ("draft", iv.draft, MAX_NODE_TOP_K)):
                problem = _curve_problem(name, curve, bound, chain)
                if problem:
                    raise ValueError(f"{what}: batch size {bs}, interval {iid}: {problem}")


# ---------------------------------------------------------------------------------------------------- fixed shape
@dataclass
class FixedShapePolicy:
    """Policy without cost tables: full depth every round, ``verify_num`` tokens verified (or ``force_width`` while
    the live costs seed a width)."""

    intensity: ComputeIntensity
    node_top_k: int
    tree_depth: int
    verify_num: int
    force_width: Optional[int] = None
    launch_depths: Tuple[int, ...] = ()
    verifies_whole_draft: bool = False

    @property
    def max_history_verify_num(self) -> int:
        return self.verify_num

    def deltas_budget(self, past_verify_num: int) -> int:
        return past_verify_num

    def width_step(self, depth: int) -> WidthStep:
        return WidthStep.LAST if depth >= self.tree_depth - 1 else WidthStep.KEEP

    def draft_cost_row(self, batch_size: int, average_cache_len: int) -> None:
        return None

    def history_verify_num(self, batch_size: int) -> int:
        return self.verify_num

    def verify_count(self, batch_size: int, draft_count: int) -> int:
        return min(self.verify_num, draft_count)

    def tree_width(self, depth: int, batch_size: int, past_verify_num: int, row=None, deltas=None) -> WidthDecision:
        if depth >= self.tree_depth - 1:
            return WidthDecision(-1, -1, True)
        return WidthDecision(self.node_top_k, past_verify_num, False)

    def verify_num_paged(self, scores, requested: int, batch_size: int, average_cache_len: int, *, lagged: bool):
        return min(self.verify_num if self.force_width is None else self.force_width, requested), False

    def record_verify_num(self, batch_size: int, verify_num: int) -> None:
        return None
