"""The measured cost model that sizes every draft round (host side).

It decides, from calibrated or live-measured costs:

* the **tree width / stop** after every second depth: the work gained by one more draft level per unit of draft
  cost, scaled by the target/draft cost ratio, against a depth-dependent threshold
  (``eagle_harness/core/cost_model.py:549-617``);
* the **verify budget**: pairwise pruning of verify widths whose score gain per measured verify-cost increase
  falls under a stability threshold (``:764-804``);
* the **chain stop** for top-1 chains with tiers and a cliff lookahead (``:620-683``);
* the batch **size class** from the verify cost at 8 tokens (``:341-368``);
* immutable per-batch **policy tables** for a device-side policy (``:370-424``, ``:685-719``).

Constants, thresholds and evaluation order are part of the behaviour users calibrate against, so they equal the
reference's; the code around them is this package's own.
"""

from __future__ import annotations

import enum
import math
from collections import Counter
from dataclasses import dataclass, field, replace
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

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


_FAMILY_DEPTH_LOSS = {"eagle4": 0.04, "eagle3": 0.08, "eagle": 0.64}


def depth_loss_ratio(draft_family: str, *, target_is_moe: bool, intensity: ComputeIntensity) -> float:
    """Per-depth acceptance loss of a draft family: doubled for MoE targets; chains double then halve."""
    r = _FAMILY_DEPTH_LOSS.get(draft_family, 0.16)
    chain = intensity is ComputeIntensity.CHAIN
    if target_is_moe or chain:
        r *= 2.0
    if chain:
        r *= 0.5
    return r


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
    """One chain decision: ``gain = raw*2/gain_scale``; stop when ``gain/cost < threshold``; with a cliff the
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
    KEEP = "keep"
    LAST = "last"
    LAUNCH = "launch"
    DECIDE = "decide"


def find_majority(nums: Sequence[int]) -> int:
    """First element to pass a strict majority while scanning in order, -1 if none does."""
    seen: Counter = Counter()
    half = len(nums) // 2
    for x in nums:
        seen[x] += 1
        if seen[x] > half:
            return x
    return -1


def verify_cost_delta(previous: float, current: float) -> float:
    """Verify cost increase; increases of 0.04 (relative) or less count as free."""
    d = current - previous
    return d if d > 0.04 else 0.0


def stable_verify_thresholds(threshold: float) -> Tuple[float, float]:
    """(threshold when the majority budget is <= the candidate, when it is >)."""
    return threshold * 0.95, threshold * 1.05


# (upper bound on the model cost ratio, adjust factor); ratios of 64 and above get 2.70.
_ADJUST_STEPS = ((8, 1.30), (12, 1.10), (17, 1.30), (23, 1.50), (32, 1.80), (64, 2.20))


def adjust_cost_ratio(model_cost_ratio: float) -> float:
    """Threshold multiplier for a target/draft cost ratio; ratios outside 5..100 are refused."""
    if model_cost_ratio < 5:
        raise ValueError(
            f"Invalid model_cost_ratio: {model_cost_ratio:.2f}. The ratio is too low "
            "(below 5), which is not suitable for speculative sampling."
        )
    if model_cost_ratio > 100:
        raise ValueError(
            f"Invalid model_cost_ratio: {model_cost_ratio:.2f}. The ratio is too high "
            "(above 100), which may indicate poor draft model performance."
        )
    for bound, factor in _ADJUST_STEPS:
        if model_cost_ratio < bound:
            return factor
    return 2.70


_VERIFY_THRESHOLD = {  # size class -> (high intensity, other intensities)
    SizeClass.SMALL: (2.40, 2.00),
    SizeClass.MEDIUM: (2.10, 1.80),
    SizeClass.LARGE: (1.80, 1.60),
    SizeClass.HUGE: (1.50, 1.40),
}
_BS_RATIO = {SizeClass.SMALL: 1.25, SizeClass.MEDIUM: 1.50, SizeClass.LARGE: 1.75, SizeClass.HUGE: 2.00}
_HISTORY_FLOOR = {SizeClass.SMALL: 16, SizeClass.MEDIUM: 8, SizeClass.LARGE: 4, SizeClass.HUGE: 2}
_CHAIN_SLACK = {SizeClass.SMALL: 4, SizeClass.MEDIUM: 2, SizeClass.LARGE: 2, SizeClass.HUGE: 0}
CHAIN_COST_INDEX = (0, 1, 3, 5, 7, 9, 11, 13, 15)


def classify_verify(cost_at8: float, batch_size: int, target_is_moe: bool) -> SizeClass:
    """Batch size class from the relative verify cost at 8 tokens (with the reference's sanity bounds)."""
    if cost_at8 <= 1.25 or batch_size == 1:
        if cost_at8 < 0.85 and (cost_at8 < 0.70 or not target_is_moe):
            raise ValueError(f"EAGLE-Harness: cost_state={cost_at8} is too low, which is not expected.")
        return SizeClass.SMALL
    if cost_at8 < 1.60:
        return SizeClass.MEDIUM
    if cost_at8 < 2.20:
        return SizeClass.LARGE
    if cost_at8 > 4.0:
        raise ValueError(f"EAGLE-Harness: cost_state={cost_at8} is too high, which is not expected.")
    return SizeClass.HUGE


@dataclass
class _Tier:
    tiny: bool = False
    size: SizeClass = SizeClass.SMALL


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

    tier: _Tier = field(default_factory=_Tier)
    interval_index: int = 0
    recent_verify_nums: List[int] = field(default_factory=lambda: [-5, -4, -3, -2, -1])

    def __post_init__(self) -> None:
        self.max_batch_size = max_batch_size(self.intensity)
        self.set_tables(self.tables)
        self._history = [[self.verify_num] * 16 for _ in range(self.max_batch_size)]

    # ---------------------------------------------------------------- tables
    def set_tables(self, tables: Dict[int, BatchCostTable], refused: Iterable[int] = ()) -> None:
        """Swap in new tables (live refresh); state and history stay. ``refused`` sizes are never used."""
        self.tables = tables
        usable = sorted(set(tables) - set(refused))
        self._nearest = [0] + [nearest_cost_batch_size(b, usable) for b in range(1, self.max_batch_size + 1)] \
            if usable else []

    def table(self, batch_size: int) -> Optional[BatchCostTable]:
        if not self._nearest:
            return None
        if not 1 <= batch_size <= self.max_batch_size:
            raise ValueError(f"batch_size={batch_size} is outside 1..{self.max_batch_size}.")
        return self.tables[self._nearest[batch_size]]

    def _table_or_raise(self, batch_size: int) -> BatchCostTable:
        t = self.table(batch_size)
        if t is None:
            raise ValueError(f"No cost data found for batch_size={batch_size}.")
        return t

    def update_interval(self, batch_size: int, average_cache_len: int) -> BatchCostTable:
        t = self._table_or_raise(batch_size)
        self.interval_index = t.interval_index(average_cache_len)
        return t

    def draft_cost_row(self, batch_size: int, average_cache_len: int) -> DraftCostRow:
        t = self.update_interval(batch_size, average_cache_len)
        ratio = t.model_ratio[self.interval_index]
        adjust = adjust_cost_ratio(ratio)
        draft = t.intervals[self.interval_index].draft
        bs_ratio = 1.00 if self.tier.tiny else _BS_RATIO[self.tier.size]
        bs_ratio = max(1.0, bs_ratio / ((20 / ratio + 1) / 2))
        return DraftCostRow(draft.ratio, draft.index, draft.ratio[-1], adjust, ratio, bs_ratio)

    def verify_cost(self, batch_size: int, average_cache_len: int) -> Optional[VerifyCost]:
        t = self.table(batch_size)
        if t is None:
            return None
        target = t.intervals[t.interval_index(average_cache_len)].target
        at8 = target.ratio[-1]
        for r, idx in zip(target.ratio, target.index):
            if idx >= 7:
                at8 = r
                break
        self.tier.size = classify_verify(at8, batch_size, self.target_is_moe)
        high, other = _VERIFY_THRESHOLD[self.tier.size]
        return VerifyCost(target.ratio, target.index, high if self.intensity is ComputeIntensity.HIGH else other)

    def _verify_cost_or_raise(self, batch_size: int, average_cache_len: int) -> VerifyCost:
        c = self.verify_cost(batch_size, average_cache_len)
        if c is None:
            raise ValueError(f"Cost data for batch size {batch_size} not found.")
        return c

    # ---------------------------------------------------------------- history
    def _floored_history(self, batch_size: int) -> int:
        floor = 32 if self.tier.tiny else _HISTORY_FLOOR[self.tier.size]
        return max(max(self._history[batch_size - 1]), floor)

    def history_verify_num(self, batch_size: int) -> int:
        if self.intensity is ComputeIntensity.CHAIN:
            slack = 4 if self.tier.tiny else _CHAIN_SLACK[self.tier.size]
            return min(max(self._history[batch_size - 1]) + slack, self.verify_num)
        return self._floored_history(batch_size)

    @property
    def max_history_verify_num(self) -> int:
        if self.intensity is ComputeIntensity.CHAIN:
            return self.verify_num
        return max(self.verify_num, 32, *_HISTORY_FLOOR.values())

    @property
    def chain_rounds(self) -> bool:
        return (
            self.intensity is ComputeIntensity.CHAIN
            and self.node_top_k == 1
            and self.verify_num == CHAIN_COST_INDEX[-1] + 1
        )

    @property
    def verifies_whole_draft(self) -> bool:
        return self.chain_rounds

    def deltas_budget(self, past_verify_num: int) -> int:
        return self.verify_num if self.chain_rounds else past_verify_num

    @property
    def launch_depths(self) -> Tuple[int, ...]:
        return tuple(range(1 if self.chain_rounds else 0, self.tree_depth - 1, 2))

    def record_verify_num(self, batch_size: int, verify_num: int) -> None:
        h = self._history[batch_size - 1]
        h.pop(0)
        h.append(verify_num)

    def verify_count(self, batch_size: int, draft_count: int) -> int:
        if self.intensity is ComputeIntensity.CHAIN:
            return draft_count
        return min(self.verify_num, draft_count, max(self._floored_history(batch_size) * 2, 16))

    # ------------------------------------------------------------ tree width
    def _width_cap(self) -> int:
        cap = 8 if self.tier.size in (SizeClass.SMALL, SizeClass.MEDIUM) else 4
        return min(self.node_top_k, cap)

    def width_step(self, depth: int) -> WidthStep:
        last = depth == self.tree_depth - 1
        if self.chain_rounds:
            if last:
                return WidthStep.LAST
            if depth == 0:
                return WidthStep.KEEP
            return WidthStep.LAUNCH if depth % 2 else WidthStep.DECIDE
        if self.tier.tiny and depth < 2:
            return WidthStep.KEEP
        if last:
            return WidthStep.LAST
        return WidthStep.LAUNCH if depth % 2 == 0 else WidthStep.DECIDE

    def tree_depth_threshold(self, depth: int, row: DraftCostRow) -> float:
        r = row.batch_size_ratio
        if depth <= 1:
            r = (r + 1.00) / 2
        elif depth > 5 and r > 1.3:
            r = r * 1.1
        p = self.params
        return p.threshold * (depth * p.depth_loss_ratio + 1.0) * row.adjust_cost_ratio * r

    def tree_width(self, depth: int, batch_size: int, past_verify_num: int, row: Optional[DraftCostRow],
                   deltas: Optional[Sequence[float]] = None) -> WidthDecision:
        step = self.width_step(depth)
        if self.chain_rounds and step is not WidthStep.LAST:
            if step is WidthStep.DECIDE and deltas is None:
                raise ValueError(f"tree_width at depth {depth} needs the host score deltas.")
            stop = step is WidthStep.DECIDE and self.chain_stop(depth, batch_size, deltas)
            return WidthDecision(1, past_verify_num, stop)
        if step is WidthStep.KEEP:
            return WidthDecision(self.node_top_k, past_verify_num, False)
        if step is WidthStep.LAST:
            return WidthDecision(-1, -1, True)
        if step is WidthStep.LAUNCH:
            return WidthDecision(self._width_cap(), past_verify_num, False)
        if deltas is None:
            raise ValueError(f"tree_width at depth {depth} needs the host score deltas.")
        self.tier.tiny = batch_size == 1
        width = self._width_cap()
        gain = deltas[width] - deltas[0]
        p = self.params
        per_cost = gain / row.cost_values[-1] * row.model_cost_ratio * p.async_layer_ratio
        if per_cost < self.tree_depth_threshold(depth, row):
            return WidthDecision(width, past_verify_num, True)
        if self.tier.size in (SizeClass.MEDIUM, SizeClass.LARGE):
            width = 1 << (width - 1).bit_length()
        return WidthDecision(width, past_verify_num, False)

    # ------------------------------------------------------------ chain depth
    def classify_chain(self, batch_size: int, cost_ratio: Optional[Sequence[float]] = None) -> Tuple[ChainTier, float]:
        if cost_ratio is None:
            cost_ratio = self._table_or_raise(batch_size).intervals[self.interval_index].target.ratio
        scale = (cost_ratio[1] + cost_ratio[3] + cost_ratio[7]) / (3.0 * cost_ratio[0])
        p = self.params
        if scale <= p.chain_scale_tiny or batch_size <= p.chain_tiny_max_bs:
            return ChainTier.TINY, scale
        if scale < p.chain_scale_small:
            return ChainTier.SMALL, scale
        if scale < p.chain_scale_medium:
            return ChainTier.MEDIUM, scale
        return ChainTier.LARGE, scale

    def _chain_decides(self, depth: int) -> bool:
        return not (depth == 0 or depth == self.tree_depth - 1 or depth % 2 == 1)

    def chain_stop(self, depth: int, batch_size: int, deltas: Optional[Sequence[float]] = None) -> bool:
        if not self._chain_decides(depth):
            return False
        if deltas is None:
            raise ValueError(f"chain_stop at depth {depth} needs the host score deltas.")
        t = self.chain_stop_terms(depth, batch_size)
        raw = deltas[1] - deltas[0]
        gain = raw * 2.0 / t.gain_scale
        stop = gain / t.cost < t.threshold
        if stop and t.cliff_cost > 0.0:
            stop = (gain + raw * 2.0 / t.cliff_gain_scale) / t.cliff_cost < t.threshold
        return stop

    def chain_stop_terms(self, depth: int, batch_size: int) -> ChainStopTerms:
        if not self._chain_decides(depth):
            return ChainStopTerms(0.0, 0.0, 0.0, 0.0, 0.0)
        t = self._table_or_raise(batch_size)
        target = t.intervals[self.interval_index].target
        if tuple(target.index) != CHAIN_COST_INDEX or any(type(i) is not int for i in target.index):
            raise ValueError(f"Invalid chain cost index: {list(target.index)}")
        llm = target.ratio[1:]
        tier, _ = self.classify_chain(batch_size, target.ratio)
        p = self.params
        coef = p.chain_coef[tier]
        cur = depth // 2
        nxt = min(cur + 1, len(llm) - 1)
        step_cost = 1.0 / t.model_ratio[self.interval_index]
        cost = step_cost * 2 + max(0, llm[nxt] - llm[cur])
        gain_scale = 1.0 + depth * coef.depth_loss
        ref_iter = sum(c + step_cost * (2 * i + 1) for i, c in enumerate(llm)) / len(llm)
        threshold = coef.threshold * (p.chain_ref_cost / ref_iter) ** coef.cost_power
        cliff_scale = cliff_cost = 0.0
        if nxt + 1 < len(llm):
            up_next = llm[nxt] - llm[cur]
            up_after = llm[nxt + 1] - llm[nxt]
            if up_next > p.chain_cliff_min_cost and up_next > p.chain_cliff_ratio * max(up_after, 0.0):
                cliff_scale = 1.0 + (depth + 2) * coef.depth_loss
                cliff_cost = step_cost * 4 + max(0, llm[nxt + 1] - llm[cur])
        return ChainStopTerms(gain_scale, cost, threshold, cliff_scale, cliff_cost)

    # ------------------------------------------------------------ verify budget
    def verify_num_paged(self, scores: Sequence[float], requested: int, batch_size: int, average_cache_len: int,
                         *, lagged: bool) -> Tuple[int, bool]:
        """Verify tokens per request from cumulative node scores (this round's, or last round's when lagged)."""
        majority = find_majority(self.recent_verify_nums)
        cap = len(scores) if lagged else requested
        self.recent_verify_nums = self.recent_verify_nums[1:] + [requested]
        cost = self._verify_cost_or_raise(batch_size, average_cache_len)
        index = [i for i in cost.index if i < min(cap, requested)]
        if max(index) == 0:
            self.recent_verify_nums[-1] = 1
            return 1, False
        values = cost.value[: len(index)]
        gains = [scores[i] for i in index]
        kept = list(index)
        reset = kept[1]
        low, high = stable_verify_thresholds(cost.threshold)
        for i in range(len(index) - 1):
            for j in range(i + 1, len(index)):
                bar = low if majority <= kept[j] + 1 else high
                d = verify_cost_delta(values[i], values[j])
                if d > 0.0 and (gains[j] - gains[i]) / d < bar:
                    kept[j] = reset
        verify_num = max(kept) + 1
        self.recent_verify_nums[-1] = verify_num
        if verify_num == 1 or requested < verify_num:
            verify_num = min(index[1:]) + 1
        return verify_num, False

    # ------------------------------------------------------------ policy export
    def tree_policy_costs(self) -> TreePolicyCosts:
        """Per-batch immutable tree policy inputs (for a device-side policy); this model's state is untouched."""
        self._validate_tree_export()
        m = replace(self, tier=_Tier(), interval_index=0, recent_verify_nums=list(self.recent_verify_nums))
        batches = []
        for bs in range(1, MAX_BATCH_SIZE_TREE + 1):
            t = m._table_or_raise(bs)
            ivs = []
            for iid in range(len(t.intervals)):
                ctx = (iid + 1) * t.cache_length_step
                vc = m._verify_cost_or_raise(bs, ctx)
                vtier = int(m.tier.size)
                rows_thr = []
                row = None
                for variant in range(5):
                    m.tier = _Tier(tiny=variant == 4, size=SizeClass(variant % 4))
                    row = m.draft_cost_row(bs, ctx)
                    rows_thr.append(tuple(m.tree_depth_threshold(d, row) for d in range(self.tree_depth)))
                if not all(math.isfinite(x) for r in rows_thr for x in r):
                    raise ValueError(f"Nonfinite depth thresholds for batch_size={bs}, interval={iid}.")
                ivs.append(TreePolicyInterval(
                    verify_widths=tuple(vc.index),
                    verify_cost_deltas=tuple(tuple(verify_cost_delta(a, b) for b in vc.value) for a in vc.value),
                    draft_cost=row.cost_values[-1],
                    model_cost_ratio=row.model_cost_ratio,
                    depth_thresholds=tuple(rows_thr),
                    verify_tier=vtier,
                    verify_thresholds=stable_verify_thresholds(vc.threshold),
                ))
            batches.append(TreePolicyBatch(t.batch_size, t.cache_length_step, tuple(ivs)))
        floors, widths = [], []
        m = replace(m, verify_num=1)
        for variant in range(5):
            m.tier = _Tier(tiny=variant == 4, size=SizeClass(variant % 4))
            floors.append(m.history_verify_num(1))
            if variant < 4:
                widths.append(m.tree_width(0, 1, 1, m.draft_cost_row(1, 0)).width)
        return TreePolicyCosts(tuple(batches), tuple(floors), tuple(widths), self.params.async_layer_ratio)

    def chain_policy_costs(self) -> ChainPolicyCosts:
        self._validate_chain_export()
        m = replace(self)
        out = []
        for bs in range(1, MAX_BATCH_SIZE_CHAIN + 1):
            t = m._table_or_raise(bs)
            ivs = []
            for iid in range(len(t.intervals)):
                m.interval_index = iid
                try:
                    terms = tuple(m.chain_stop_terms(d, bs) for d in range(self.tree_depth))
                except (OverflowError, ZeroDivisionError) as e:
                    raise ValueError(f"Invalid chain stop terms for batch_size={bs}, interval={iid}.") from e
                for d, term in enumerate(terms):
                    vals = (term.gain_scale, term.cost, term.threshold, term.cliff_gain_scale, term.cliff_cost)
                    if (any(not math.isfinite(v) or v < 0 for v in vals)
                            or (self._chain_decides(d) and min(term.gain_scale, term.cost, term.threshold) <= 0)
                            or ((term.cliff_gain_scale > 0) != (term.cliff_cost > 0))):
                        raise ValueError(f"Invalid chain stop terms for batch_size={bs}, interval={iid}, depth={d}.")
                ivs.append(terms)
            out.append(ChainPolicyBatch(t.cache_length_step, tuple(ivs)))
        return ChainPolicyCosts(tuple(out))

    def _validate_tree_export(self) -> None:
        for name, lo in (("tree_depth", 2), ("node_top_k", 1), ("verify_num", 2)):
            v = getattr(self, name)
            if type(v) is not int or v < lo:
                raise ValueError(f"{name}={v!r} must be an integer >= {lo} for tree policy export.")
        check_shape(self.intensity, self.node_top_k, self.tree_depth, self.verify_num, MAX_BATCH_SIZE_TREE)
        for name in ("threshold", "async_layer_ratio", "depth_loss_ratio"):
            v = getattr(self.params, name)
            if not math.isfinite(v) or v < 0 or (name != "depth_loss_ratio" and v == 0):
                raise ValueError(f"Invalid tree policy parameter {name}={v!r}.")
        self._validate_tables(chain=False)

    def _validate_chain_export(self) -> None:
        if self.intensity is not ComputeIntensity.CHAIN:
            raise ValueError("Chain policy export requires chain intensity.")
        for name, lo, hi in (("node_top_k", 1, 1), ("tree_depth", 2, MAX_CHAIN_DEPTH),
                             ("verify_num", 2, MAX_CHAIN_VERIFY_NUM)):
            v = getattr(self, name)
            if type(v) is not int or not lo <= v <= hi:
                raise ValueError(f"{name}={v!r} must be an integer in {lo}..{hi} for chain policy export.")
        p = self.params
        if len(p.chain_coef) != len(ChainTier):
            raise ValueError("Chain policy requires four chain_coef entries.")
        for c in p.chain_coef:
            ok = (isinstance(c, ChainCoef) and math.isfinite(c.threshold) and c.threshold > 0
                  and math.isfinite(c.depth_loss) and c.depth_loss >= 0
                  and math.isfinite(c.cost_power) and c.cost_power >= 0)
            if not ok:
                raise ValueError(f"Invalid chain coefficient {c!r}.")
        for name in ("chain_ref_cost", "chain_cliff_min_cost", "chain_cliff_ratio", "chain_scale_tiny",
                     "chain_scale_small", "chain_scale_medium"):
            v = getattr(p, name)
            if not math.isfinite(v) or v < 0 or (name != "chain_cliff_min_cost" and v == 0):
                raise ValueError(f"Invalid chain policy parameter {name}={v!r}.")
        if not p.chain_scale_tiny < p.chain_scale_small < p.chain_scale_medium:
            raise ValueError("Chain tier scale thresholds must be strictly increasing.")
        if type(p.chain_tiny_max_bs) is not int or not 0 <= p.chain_tiny_max_bs <= MAX_BATCH_SIZE_CHAIN:
            raise ValueError(f"Invalid chain_tiny_max_bs={p.chain_tiny_max_bs!r}.")
        self._validate_tables(chain=True)

    def _validate_tables(self, *, chain: bool) -> None:
        if not self.tables:
            raise ValueError(f"No cost data found for {'chain' if chain else 'tree'} policy export.")
        for bs, t in self.tables.items():
            if (type(bs) is not int or bs < 1 or (chain and bs > MAX_BATCH_SIZE_CHAIN)
                    or type(t.batch_size) is not int or t.batch_size != bs):
                raise ValueError(f"Invalid measured batch_size={bs!r}; table reports {t.batch_size!r}.")
            if type(t.cache_length_step) is not int or t.cache_length_step <= 0:
                raise ValueError(f"Invalid cache_length_step={t.cache_length_step!r} for batch_size={bs}.")
            if not t.intervals or len(t.intervals) != len(t.model_ratio):
                raise ValueError(f"Missing cost intervals or model ratios for batch_size={bs}.")
            for iid, (iv, ratio) in enumerate(zip(t.intervals, t.model_ratio)):
                where = f"batch_size={bs}, interval={iid}"
                if not math.isfinite(ratio) or ratio <= 0:
                    raise ValueError(f"Model cost ratio must be finite and positive for {where}.")
                if not chain:
                    adjust_cost_ratio(ratio)
                for name, curve, bound in (("target", iv.target, MAX_VERIFY_NUM), ("draft", iv.draft, MAX_NODE_TOP_K)):
                    n = len(curve.index)
                    if n == 0 or (name == "target" and not 2 <= n <= 32):
                        raise ValueError(f"Invalid {name} width count {n} for {where}.")
                    if len(curve.value) != n or len(curve.ratio) != n:
                        raise ValueError(f"Mismatched {name} cost lengths for {where}.")
                    if (curve.index[0] != 0 or any(type(i) is not int or not 0 <= i < bound for i in curve.index)
                            or any(a >= b for a, b in zip(curve.index, curve.index[1:]))):
                        raise ValueError(f"Invalid {name} cost indices {curve.index!r} for {where}.")
                    if chain and name == "target" and tuple(curve.index) != CHAIN_COST_INDEX:
                        raise ValueError(f"Invalid chain cost indices {curve.index!r} for {where}.")
                    if any(not math.isfinite(v) or v <= 0 for v in (*curve.value, *curve.ratio)):
                        raise ValueError(f"{name} costs must be finite and positive for {where}.")


@dataclass
class FixedShapePolicy:
    """Policy without cost tables: full depth every round, ``verify_num`` tokens verified (or ``force_width``)."""

    intensity: ComputeIntensity
    node_top_k: int
    tree_depth: int
    verify_num: int
    force_width: Optional[int] = None
    launch_depths: Tuple[int, ...] = ()

    @property
    def verifies_whole_draft(self) -> bool:
        return False

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
        w = self.verify_num if self.force_width is None else self.force_width
        return min(w, requested), False

    def record_verify_num(self, batch_size: int, verify_num: int) -> None:
        return None
