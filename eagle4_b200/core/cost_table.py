"""Calibrated cost tables: the on-disk format the cost model reads.

Layout (kept identical to the reference so existing calibration directories load unchanged,
``eagle_harness/core/cost_table.py:1-13``)::

    <data_path>/cost/bs_<N>/model_llm/model_interval_<i>.json   target verify curve
    <data_path>/cost/bs_<N>/model_slm/model_interval_<i>.json   draft step curve

Each interval file holds ``value`` (microseconds per measured query length), ``ratio`` (``value / value[0]``),
``index`` (query length minus one), ``array_query`` / ``array_cache`` and the grid fields
``cache_length_start``, ``cache_length_step``, ``max_query_length_query``, ``max_query_length_cache``.
"""

from __future__ import annotations

import json
import logging
import math
import os
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Dict, List, Optional, Tuple

if TYPE_CHECKING:  # pragma: no cover
    from eagle4_b200.core.live_costs import CostKey

log = logging.getLogger(__name__)

# Ranges the cost model accepts (it raises mid-round otherwise): target/draft cost ratio, and the target's cost at
# 8 verify tokens relative to 1 token (0.85 lower bound for dense targets, 0.70 for MoE).
MODEL_RATIO_RANGE = (5.0, 100.0)
VERIFY8_RATIO_RANGE = (0.70, 4.0)


@dataclass(frozen=True)
class CostCurve:
    """Cost of one model at one context interval per measured query length (``index[i] + 1`` tokens)."""

    value: Tuple[float, ...]
    ratio: Tuple[float, ...]
    index: Tuple[int, ...]
    array_query: Tuple[float, ...] = ()
    array_cache: Tuple[float, ...] = ()

    @classmethod
    def from_json(cls, data: dict) -> "CostCurve":
        return cls(
            value=tuple(data["value"]),
            ratio=tuple(data["ratio"]),
            index=tuple(data["index"]),
            array_query=tuple(data.get("array_query", ())),
            array_cache=tuple(data.get("array_cache", ())),
        )

    @classmethod
    def from_values(cls, values, index) -> "CostCurve":
        """A curve whose ratios are derived from ``values`` (rounded to 4 places as the files store them)."""
        base = values[0]
        return cls(tuple(values), tuple(round(v / base, 4) for v in values), tuple(index))


@dataclass(frozen=True)
class IntervalCost:
    """Target ("llm" on disk) and draft ("slm") curves of one context interval."""

    target: CostCurve
    draft: CostCurve


@dataclass(frozen=True)
class BatchCostTable:
    """All context intervals of one calibrated batch size."""

    batch_size: int
    cache_length_start: int
    cache_length_step: int
    target_max_qo_len_query: int
    target_max_qo_len_cache: int
    draft_max_qo_len: int
    intervals: Tuple[IntervalCost, ...]
    model_ratio: Tuple[float, ...]  # target.value[0] / draft.value[0] per interval, -1 when the draft cost is 0
    _clamp_warned: bool = field(default=False, init=False, repr=False, compare=False)

    @property
    def max_interval_id(self) -> int:
        return len(self.intervals) - 1

    def interval_index(self, average_cache_len: int) -> int:
        """Interval of an average committed length: ``(len - step) // step`` clamped into the table."""
        step = self.cache_length_step
        idx = (average_cache_len - step) // step
        if idx > self.max_interval_id and not self._clamp_warned:
            log.warning(
                "Cost table for batch size %d clamps context %d at its last interval (calibrated to %d); "
                "recalibrate for longer contexts.",
                self.batch_size, average_cache_len, (len(self.intervals) + 1) * step,
            )
            object.__setattr__(self, "_clamp_warned", True)
        return max(0, min(idx, self.max_interval_id))


def _interval_files(path: str) -> Dict[int, dict]:
    found: Dict[int, dict] = {}
    if not os.path.isdir(path):
        return found
    for name in os.listdir(path):
        if not (name.startswith("model_interval_") and name.endswith(".json")):
            continue
        try:
            idx = int(name[len("model_interval_"):-len(".json")])
            with open(os.path.join(path, name), encoding="utf-8") as f:
                found[idx] = json.load(f)
        except (ValueError, json.JSONDecodeError):
            log.warning("%s is not a readable cost interval; ignored", name)
    return found


def load_batch_table(batch_dir: str, batch_size: int) -> BatchCostTable:
    """Read one ``bs_<N>`` directory; every interval needs both curves."""
    llm = _interval_files(os.path.join(batch_dir, "model_llm"))
    slm = _interval_files(os.path.join(batch_dir, "model_slm"))
    if not llm and not slm:
        raise RuntimeError(f"{batch_dir} holds no cost interval for batch size {batch_size}")
    last = max(list(llm) + list(slm))
    intervals: List[IntervalCost] = []
    ratios: List[float] = []
    for i in range(last + 1):
        t, d = llm.get(i), slm.get(i)
        if not t or not d:
            raise RuntimeError(
                f"Missing interval {i} for batch size {batch_size}: target={t is not None}, draft={d is not None}."
            )
        intervals.append(IntervalCost(CostCurve.from_json(t), CostCurve.from_json(d)))
        t0 = t["value"][0] if t["value"] else 0
        d0 = d["value"][0] if d["value"] else 0
        ratios.append(round(t0 / d0, 4) if d0 > 0 else -1.0)
    first_t = next(iter(llm.values()))
    first_d = next(iter(slm.values()))
    return BatchCostTable(
        batch_size=batch_size,
        cache_length_start=first_t["cache_length_start"],
        cache_length_step=first_t["cache_length_step"],
        target_max_qo_len_query=first_t["max_query_length_query"],
        target_max_qo_len_cache=first_t["max_query_length_cache"],
        draft_max_qo_len=first_d["max_query_length_query"],
        intervals=tuple(intervals),
        model_ratio=tuple(ratios),
    )


def table_problem(table: BatchCostTable) -> Optional[str]:
    """Why ``table`` is malformed (None if fine): finite positive costs, matching lengths, index rising from 0."""
    for i, iv in enumerate(table.intervals):
        for name, c in (("target", iv.target), ("draft", iv.draft)):
            n = len(c.index)
            if not c.value or len(c.value) != n or len(c.ratio) != n:
                return f"interval {i}: the {name} curve's value, ratio and index lists differ in length"
            if not all(math.isfinite(v) and v > 0 for v in c.value):
                return f"interval {i}: {name} costs {c.value} include a non-positive or non-finite value"
            if c.index[0] != 0 or any(b <= a for a, b in zip(c.index, c.index[1:])):
                return f"interval {i}: {name} query lengths {c.index} do not start at 0 and increase"
    return None


def verify_cost_at8(curve: CostCurve) -> float:
    """Relative target cost at the first measured query length of 8 or more tokens (else the widest)."""
    for r, idx in zip(curve.ratio, curve.index):
        if idx >= 7:
            return r
    return curve.ratio[-1]


def cost_model_problem(table: BatchCostTable, *, target_is_moe: bool = False) -> Optional[str]:
    """Why the cost model could not decide from ``table`` (None if it can)."""
    problem = table_problem(table)
    if problem is not None:
        return problem
    for i, iv in enumerate(table.intervals):
        ratio = table.model_ratio[i]
        if not MODEL_RATIO_RANGE[0] <= ratio <= MODEL_RATIO_RANGE[1]:
            return f"interval {i}: the target costs {ratio} draft steps, outside {MODEL_RATIO_RANGE}"
        at8 = verify_cost_at8(iv.target)
        lo = VERIFY8_RATIO_RANGE[0] if target_is_moe else 0.85
        if not lo <= at8 <= VERIFY8_RATIO_RANGE[1]:
            return f"interval {i}: verifying 8 tokens costs {at8} of one token, outside {(lo, VERIFY8_RATIO_RANGE[1])}"
    return None


def load_cost_tables(cost_dir: str, key: Optional["CostKey"] = None) -> Dict[int, BatchCostTable]:
    """Every ``bs_<N>`` table under ``cost_dir`` (empty when the directory is absent).

    With ``key`` the directory's ``key.json`` (in the parent of ``cost_dir``) must name the same setup.
    """
    if not os.path.isdir(cost_dir):
        log.error("no cost tables at %s", cost_dir)
        return {}
    if key is not None:
        from eagle4_b200.core.live_costs import check_key

        check_key(os.path.dirname(os.path.normpath(cost_dir)), key)
    tables: Dict[int, BatchCostTable] = {}
    for entry in sorted(os.listdir(cost_dir)):
        bdir = os.path.join(cost_dir, entry)
        if not (entry.startswith("bs_") and os.path.isdir(bdir)):
            continue
        try:
            bs = int(entry[3:])
        except ValueError as e:
            raise RuntimeError(f"{entry}: a cost directory entry that is not bs_<batch size>") from e
        if not (os.path.isdir(os.path.join(bdir, "model_llm")) and os.path.isdir(os.path.join(bdir, "model_slm"))):
            log.warning("batch size %d has no model cost directory; it is left out", bs)
            continue
        table = load_batch_table(bdir, bs)
        problem = table_problem(table)
        if problem is not None:
            raise RuntimeError(f"the cost model refuses the tables under {bdir}: {problem}")
        tables[bs] = table
    return tables


def write_interval(path: str, curve: CostCurve, *, batch_size: int, cache_length_start: int,
                   cache_length_step: int, max_query_length_query: int, max_query_length_cache: int,
                   extra: Optional[dict] = None) -> None:
    """Write one ``model_interval_<i>.json`` in the on-disk format."""
    data = {
        "value": list(curve.value),
        "index": list(curve.index),
        "ratio": list(curve.ratio),
        "array_query": list(curve.array_query),
        "array_cache": list(curve.array_cache),
        "batch_size": batch_size,
        "max_query_length_query": max_query_length_query,
        "max_query_length_cache": max_query_length_cache,
        "cache_length_start": cache_length_start,
        "cache_length_step": cache_length_step,
    }
    if extra:
        data.update(extra)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        json.dump(data, f, indent=2)
    os.replace(tmp, path)
