"""Chain verify width per batch size, and the tree's verify width under load, from measured costs.

A chain round of width ``w`` drafts ``w - 1`` tokens and verifies them with the root. It gains
``1 + a_1 + ... + a_{w-1}`` tokens per request (``a_d``: share of rounds whose first ``d`` drafts are all accepted)
and costs ``V(B, w) + (w - 1) * D(B)`` from the cost tables, or the served round period ``R(B, w)`` when that was
measured (width 1 = root-only verify, width 0 = native decode in the same engine). Each batch size takes the width
with the most tokens per microsecond; batch sizes between calibrated ones take the nearest calibrated one's width
(ties to the larger). Same decision rules and file formats as reference ``eagle_harness/core/chain_width.py:1-368``:

* ``<data_path>/accept/chain.json``: ``{"drafts": n, "accepted_per_position": [...]}``;
* ``<data_path>/rounds/chain.json``: ``{"rounds": [{"batch_size", "width", "round_us", "count"}, ...]}``;
* ``<data_path>/rounds/tree.json``: ``{"rounds": [{"batch_size", "width", "round_us", "accept", "count"}, ...]}``.

For a tree whose verify width the engine fixes per batch size, :func:`served_tree_schedule` keeps the configured
width below a switch batch size and narrows from there; the switch maximises the round-weighted log gain summed
over every compared batch size at or above it.
"""

from __future__ import annotations

import json
import math
import os
import statistics
from dataclasses import dataclass
from typing import Dict, Iterable, List, Mapping, Optional, Sequence, Tuple

from eagle4_b200.core.cost_table import BatchCostTable, CostCurve, load_cost_tables
from eagle4_b200.core.limits import nearest_cost_batch_size
from eagle4_b200.core.live_costs import CostKey, check_key

PROFILE_FILE = os.path.join("accept", "chain.json")
ROUNDS_FILE = os.path.join("rounds", "chain.json")
TREE_ROUNDS_FILE = os.path.join("rounds", "tree.json")

Schedule = List[Tuple[int, int, int]]  # (first batch size, last batch size, width)


@dataclass(frozen=True)
class AcceptProfile:
    """``rates[d]``: share of rounds that accept drafted token ``d + 1`` (and every one before it)."""

    rates: Tuple[float, ...]

    @classmethod
    def from_counts(cls, drafts: int, accepted_per_position: Sequence[int]) -> "AcceptProfile":
        if drafts <= 0:
            raise ValueError(f"{drafts} drafted rounds: an acceptance profile is measured over one round or more")
        c = list(accepted_per_position)
        if any(not 0 <= x <= drafts for x in c) or any(later > earlier for earlier, later in zip(c, c[1:])):
            raise ValueError(f"accepted counts per position {c} are not a non-increasing sequence within the drafted rounds")
        return cls(tuple(x / drafts for x in c))

    @property
    def max_width(self) -> int:
        return len(self.rates) + 1

    def expected_tokens(self, width: int) -> float:
        if not 1 <= width <= self.max_width:
            raise ValueError(f"width {width} is beyond the profile's widths 1..{self.max_width}")
        return 1.0 + sum(self.rates[:width - 1])


def _read_json(path: str) -> Optional[dict]:
    try:
        with open(path, encoding="utf-8") as f:
            return json.load(f)
    except FileNotFoundError:
        return None


def _write_json(path: str, data: dict, **kw) -> str:
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        json.dump(data, f, **kw)
    return path


def load_accept_profile(data_path: str) -> Optional[AcceptProfile]:
    data = _read_json(os.path.join(data_path, PROFILE_FILE))
    return None if data is None else AcceptProfile.from_counts(data["drafts"], data["accepted_per_position"])


def save_accept_profile(data_path: str, drafts: int, accepted_per_position: Sequence[int]) -> str:
    AcceptProfile.from_counts(drafts, accepted_per_position)  # validate before writing
    return _write_json(os.path.join(data_path, PROFILE_FILE),
                       {"drafts": drafts, "accepted_per_position": list(accepted_per_position)})


def median_cost(curves: Sequence[CostCurve], query_length: int) -> Optional[float]:
    """Median over the context intervals of the cost at ``query_length`` tokens (None if an interval lacks it)."""
    i = query_length - 1
    if not curves or any(i not in c.index for c in curves):
        return None
    return statistics.median(c.value[c.index.index(i)] for c in curves)


def _best_width(price: Mapping[int, float], profile: AcceptProfile, max_width: int,
                start: Tuple[int, float]) -> int:
    """The width with the most tokens per microsecond among ``price`` (widths >= 2 the profile covers), starting
    from ``start`` = (width, rate); strict improvement is needed to move."""
    best, best_rate = start
    cap = min(max_width, profile.max_width)
    for w in sorted(price):
        us = price[w]
        if 2 <= w <= cap and us > 0:
            rate = profile.expected_tokens(w) / us
            if rate > best_rate:
                best, best_rate = w, rate
    return best


def chain_width(table: BatchCostTable, profile: AcceptProfile, max_width: int) -> Optional[int]:
    """Best width at the table's batch size, pricing rounds from the cost tables (None without root-only verify or
    draft-step costs)."""
    targets = [iv.target for iv in table.intervals]
    plain = median_cost(targets, 1)
    step = median_cost([iv.draft for iv in table.intervals], 1)
    if not plain or not step or plain <= 0 or step <= 0:
        return None
    price = {}
    for w in range(2, min(max_width, profile.max_width) + 1):
        v = median_cost(targets, w)
        if v is not None:
            price[w] = v + (w - 1) * step
    return _best_width(price, profile, max_width, (1, 1.0 / plain))


def served_chain_width(round_us: Mapping[int, float], profile: AcceptProfile, max_width: int, *,
                       allow_no_spec: bool = False) -> Optional[int]:
    """Best width from served round periods at one batch size (None when root-only verify was not timed)."""
    plain = round_us.get(1)
    if plain is None or plain <= 0:
        return None
    start = (1, 1.0 / plain)
    native = round_us.get(0) if allow_no_spec else None
    if native is not None and 0 < native <= plain:
        start = (0, 1.0 / native)
    return _best_width(round_us, profile, max_width, start)


def merge_ranges(rows: Iterable[Tuple[int, int, int]]) -> Schedule:
    """Rows in batch-size order with consecutive equal values merged."""
    out: Schedule = []
    for first, last, value in rows:
        if out and out[-1][2] == value:
            out[-1] = (out[-1][0], last, value)
        else:
            out.append((first, last, value))
    return out


def _ranges(widths: Mapping[int, int], max_batch_size: int) -> Schedule:
    return merge_ranges((b, b, widths[nearest_cost_batch_size(b, widths)]) for b in range(1, max_batch_size + 1))


def _schedule(per_batch: Mapping[int, Optional[int]], max_batch_size: int) -> Optional[Schedule]:
    if not per_batch or any(w is None for w in per_batch.values()):
        return None
    return _ranges(per_batch, max_batch_size)


def chain_width_schedule(tables: Mapping[int, BatchCostTable], profile: AcceptProfile, max_width: int,
                         max_batch_size: int) -> Optional[Schedule]:
    return _schedule({b: chain_width(t, profile, max_width) for b, t in tables.items()}, max_batch_size)


def served_width_schedule(rounds: Mapping[int, Mapping[int, float]], profile: AcceptProfile, max_width: int,
                          max_batch_size: int, *, allow_no_spec: bool = False) -> Optional[Schedule]:
    return _schedule({b: served_chain_width(r, profile, max_width, allow_no_spec=allow_no_spec)
                      for b, r in rounds.items()}, max_batch_size)


def load_round_times(data_path: str) -> Optional[Dict[int, Dict[int, float]]]:
    data = _read_json(os.path.join(data_path, ROUNDS_FILE))
    if data is None:
        return None
    out: Dict[int, Dict[int, float]] = {}
    for row in data["rounds"]:
        out.setdefault(int(row["batch_size"]), {})[int(row["width"])] = float(row["round_us"])
    return out


def save_round_times(data_path: str, rows: Sequence[Mapping[str, float]]) -> str:
    for row in rows:
        if row["batch_size"] < 1 or row["width"] < 0 or row["round_us"] <= 0:
            raise ValueError(f"served round time {dict(row)} has a batch size below 1, a negative width or a non-positive period")
    return _write_json(os.path.join(data_path, ROUNDS_FILE), {"rounds": [dict(r) for r in rows]}, indent=1)


def chain_widths(data_path: str, max_width: int, max_batch_size: int, *, allow_no_spec: bool = False,
                 key: Optional[CostKey] = None) -> Optional[Schedule]:
    """The chain-width schedule a calibration directory gives (None when it lacks the acceptance profile, or both
    the served round times and the cost tables). Measured round periods take precedence over cost tables, which
    only estimate them. A directory keyed to another setup than ``key`` is refused."""
    profile = load_accept_profile(data_path)
    if profile is not None and key is not None:
        check_key(data_path, key)
    if profile is None:
        return None
    periods = load_round_times(data_path)
    if periods is None:
        tables = load_cost_tables(os.path.join(data_path, "cost"))
        return chain_width_schedule(tables, profile, max_width, max_batch_size) if tables else None
    return served_width_schedule(periods, profile, max_width, max_batch_size, allow_no_spec=allow_no_spec)


def width_at(schedule: Sequence[Tuple[int, int, int]], batch_size: int) -> int:
    for first, last, w in schedule:
        if first <= batch_size <= last:
            return w
    raise ValueError(f"no chain width is scheduled for batch size {batch_size} (schedule {list(schedule)})")


# --------------------------------------------------------------------------------------------- tree under load
def _check_tree_row(row: Mapping[str, float]) -> None:
    if row["batch_size"] < 1 or row["width"] < 1 or row["round_us"] <= 0 or row["accept"] < 1 or row["count"] < 1:
        raise ValueError(f"served tree round {dict(row)} needs a batch size, width, accept length and round count "
                         "of at least 1 and a positive period")


TreeCells = Dict[int, Dict[int, Tuple[float, float, int]]]  # batch size -> width -> (round us, accept, rounds)


def load_tree_rounds(data_path: str, key: Optional[CostKey] = None) -> Optional[TreeCells]:
    data = _read_json(os.path.join(data_path, TREE_ROUNDS_FILE))
    if data is None:
        return None
    if key is not None:
        check_key(data_path, key)
    out: TreeCells = {}
    for row in data["rounds"]:
        _check_tree_row(row)
        out.setdefault(int(row["batch_size"]), {})[int(row["width"])] = (
            float(row["round_us"]), float(row["accept"]), int(row["count"]))
    return out


def merge_tree_rounds(data_path: str, rows: Sequence[Mapping[str, float]]) -> str:
    """Replace the (batch size, width) cells ``rows`` measured in ``rounds/tree.json``, keep the others."""
    for row in rows:
        _check_tree_row(row)
    path = os.path.join(data_path, TREE_ROUNDS_FILE)
    old = _read_json(path)
    cells = {(int(r["batch_size"]), int(r["width"])): dict(r) for r in (old or {"rounds": []})["rounds"]}
    cells.update({(int(r["batch_size"]), int(r["width"])): dict(r) for r in rows})
    os.makedirs(os.path.dirname(path), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        json.dump({"rounds": [cells[k] for k in sorted(cells)]}, f, indent=1)
    os.replace(tmp, path)
    return path


def served_tree_schedule(rounds: Mapping[int, Mapping[int, Tuple[float, float, int]]], width: int,
                         max_batch_size: int) -> Optional[Schedule]:
    """Verify-width ranges for a tree configured ``width`` wide (None when narrowing never gains)."""
    compared: Dict[int, Tuple[int, float]] = {}
    for b, cells in rounds.items():
        if width not in cells:
            continue
        narrower = [(acc / us, w, n) for w, (us, acc, n) in cells.items() if w < width]
        if not narrower:
            continue
        us, acc, n = cells[width]
        rate, w_best, n_best = max(narrower)  # ties on rate keep the wider width
        compared[b] = (w_best, min(n, n_best) * math.log(rate * us / acc))
    switch, run, best = None, 0.0, 0.0
    for b in sorted(compared, reverse=True):
        run += compared[b][1]
        if run > best:
            switch, best = b, run
    if switch is None:
        return None
    later = _ranges({b: w for b, (w, _) in compared.items() if b >= switch}, max_batch_size)
    rows: Schedule = [(1, switch - 1, width)] if switch > 1 else []
    narrowed: Schedule = []
    for first, last, w in later:
        if last < switch:
            continue
        narrowed.append((max(first, switch), last, min(w, narrowed[-1][2]) if narrowed else w))
    return merge_ranges(rows + narrowed)
