"""Live costs: cost tables measured on the served rounds themselves, keyed to the serving setup.

A *track* is one (batch bucket, verify width) pair, width ``DRAFT_WIDTH`` (0) holding one draft step; it has one cell
per 1024-token context interval. A cell's value is the fastest of its first ``seed_samples`` timings, then an EMA
(``alpha``) whose samples are clamped at ``OUTLIER_RATIO`` times the cell, so one stalled round moves a cell by a few
percent at most while a lasting change still converges. A bucket is *ready* once every captured width and the draft
step have ``seed_samples`` timings; until then the round policy forces the width :meth:`LiveCosts.seed_width` names
(width 1 first, then widest first). A bucket between two ready buckets is priced by linear interpolation in the batch
size. The tables come out as the same ``BatchCostTable`` objects the cost model reads.

The cache file (``version`` 2, ``cells`` as ``[bucket, width, interval, us, samples]`` rows in sorted order), the
``CostKey`` fields and their digest are shared with the reference (``eagle_harness/core/live_costs.py:39-356``) so
caches interoperate; the prices follow the same rules (nearest seeded interval, ties to the lower one; interpolation
across widths and buckets), so the tables are the same.
"""

from __future__ import annotations

import hashlib
import json
import logging
import math
import os
from dataclasses import asdict, dataclass
from typing import Callable, Dict, Optional, Sequence, Tuple

from eagle4_b200.core.cost_table import BatchCostTable, CostCurve, IntervalCost

log = logging.getLogger(__name__)

KEY_FILE = "key.json"
CACHE_VERSION = 2
OUTLIER_RATIO = 2.0
DRAFT_WIDTH = 0  # the cell width that holds one draft step


@dataclass(frozen=True)
class CostKey:
    """The setup a set of costs belongs to."""

    gpu: str
    gpu_count: int
    model: str
    draft: str
    engine: str
    dtype: str

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "CostKey":
        return cls(**{name: data[name] for name in cls.__dataclass_fields__})

    @property
    def digest(self) -> str:
        return hashlib.sha256(json.dumps(self.to_dict(), sort_keys=True).encode()).hexdigest()[:16]


def config_digest(model_path: str) -> str:
    """``<last path component>:<12 hex of sha256(name + config.json bytes)>``."""
    name = os.path.basename(os.path.normpath(model_path))
    h = hashlib.sha256(name.encode())
    cfg = os.path.join(model_path, "config.json")
    if os.path.isfile(cfg):
        with open(cfg, "rb") as f:
            h.update(f.read())
    else:
        h.update(model_path.encode())
    return f"{name}:{h.hexdigest()[:12]}"


def write_key(data_path: str, key: CostKey) -> None:
    os.makedirs(data_path, exist_ok=True)
    with open(os.path.join(data_path, KEY_FILE), "w", encoding="utf-8") as f:
        json.dump(key.to_dict(), f, indent=2)


def read_key(data_path: str) -> Optional[CostKey]:
    try:
        with open(os.path.join(data_path, KEY_FILE), encoding="utf-8") as f:
            return CostKey.from_dict(json.load(f))
    except FileNotFoundError:
        return None


def check_key(data_path: str, key: CostKey) -> None:
    """Refuse tables measured on another setup; accept unkeyed ones with a warning."""
    stored = read_key(data_path)
    if stored is None:
        log.warning("the cost tables under %s have no %s; they are used as if measured on %s (calibrate again to record the setup)",
                    data_path, KEY_FILE, key)
        return
    if stored != key:
        diff = {f: (getattr(stored, f), getattr(key, f)) for f in key.__dataclass_fields__
                if getattr(stored, f) != getattr(key, f)}
        raise ValueError(
            f"the cost tables under {data_path} belong to another setup (field: (theirs, this server's)) {diff}; "
            "calibrate on this setup, or leave data_path unset so the served rounds price themselves"
        )


@dataclass
class Cell:
    us: float = 0.0
    samples: int = 0


class LiveCosts:
    """Live cost cells of one serving setup (``key``) and draft shape.

    ``widths(bucket)`` lists the captured verify widths of a batch bucket (the seed sweep's targets)."""

    def __init__(self, widths: Callable[[int], Sequence[int]], key: Optional[CostKey] = None,
                 draft_shape: Tuple[int, int] = (1, 1), context_step: int = 1024, context_intervals: int = 16,
                 seed_samples: int = 3, alpha: float = 0.05):
        self.widths, self.key, self.draft_shape = widths, key, tuple(draft_shape)
        self.context_step, self.context_intervals = context_step, context_intervals
        self.seed_samples, self.alpha = seed_samples, alpha
        self._tracks: Dict[Tuple[int, int], Dict[int, Cell]] = {}  # (bucket, width) -> interval -> cell
        self._samples: Dict[Tuple[int, int], int] = {}  # (bucket, width) -> timings over all intervals
        self._ready_memo: Optional[frozenset] = None

    # ----------------------------------------------------------------- cells
    @property
    def cells(self) -> Dict[Tuple[int, int, int], Cell]:
        """Every cell by ``(bucket, width, interval)`` (a fresh dict; edit through :meth:`record`)."""
        return {(b, w, i): c for (b, w), track in self._tracks.items() for i, c in track.items()}

    def interval(self, context: int) -> int:
        """The context interval of a round whose mean committed length is ``context``."""
        i = (context - self.context_step) // self.context_step
        return min(max(i, 0), self.context_intervals - 1)

    def record(self, bucket: int, width: int, context: int, us: float) -> None:
        """One timing of a served round (non-finite or non-positive timings are ignored)."""
        if not math.isfinite(us) or us <= 0:
            return
        cell = self._tracks.setdefault((bucket, width), {}).setdefault(self.interval(context), Cell())
        if cell.samples >= self.seed_samples:
            cell.us += self.alpha * (min(us, OUTLIER_RATIO * cell.us) - cell.us)
        else:
            cell.us = us if cell.samples == 0 else min(cell.us, us)
        cell.samples += 1
        self._samples[(bucket, width)] = self._samples.get((bucket, width), 0) + 1
        self._ready_memo = None

    # ----------------------------------------------------------------- seeding
    def _timed(self, bucket: int, width: int) -> int:
        return self._samples.get((bucket, width), 0)

    def seed_width(self, bucket: int) -> Optional[int]:
        """The verify width the next round at ``bucket`` must use to seed its cells (width 1 first, then the widest
        first); None once every captured width has ``seed_samples`` timings."""
        pending = [w for w in self.widths(bucket) if self._timed(bucket, w) < self.seed_samples]
        if not pending:
            return None
        return 1 if 1 in pending else max(pending)

    def _ready_set(self) -> frozenset:
        if self._ready_memo is None:
            buckets = {b for b, _ in self._tracks}
            self._ready_memo = frozenset(
                b for b in buckets
                if self.seed_width(b) is None and self._timed(b, DRAFT_WIDTH) >= self.seed_samples)
        return self._ready_memo

    def ready(self, bucket: int) -> bool:
        """Whether ``bucket``'s own cells price it (every width and the draft step seeded)."""
        return bucket in self._ready_set()

    def _bracket(self, bucket: int) -> Optional[Tuple[int, int]]:
        """The nearest ready buckets below and above an unready ``bucket`` (None if it is ready or lacks one)."""
        ready = self._ready_set()
        if bucket in ready:
            return None
        below = max((b for b in ready if b < bucket), default=None)
        above = min((b for b in ready if b > bucket), default=None)
        return None if below is None or above is None else (below, above)

    def priced(self, bucket: int) -> bool:
        return self.ready(bucket) or self._bracket(bucket) is not None

    # ----------------------------------------------------------------- prices
    def _own(self, bucket: int, width: int, interval: int) -> Optional[float]:
        """The track's price at ``interval``: its nearest seeded cell (ties to the lower interval), else its fastest
        cell with any timing, else None."""
        track = self._tracks.get((bucket, width), {})
        seeded = [i for i, c in track.items() if c.samples >= self.seed_samples]
        if seeded:
            return track[min(seeded, key=lambda i: (abs(i - interval), i))].us
        timed = [c.us for c in track.values() if c.samples]
        return min(timed) if timed else None

    def _across_widths(self, bucket: int, width: int, interval: int) -> float:
        """A ready bucket's price at any width: its own track, or the line between the captured widths around it."""
        if width == DRAFT_WIDTH or width in self.widths(bucket):
            return self._own(bucket, width, interval) or 0.0
        captured = sorted(self.widths(bucket))
        lo = max((w for w in captured if w < width), default=captured[0])
        hi = min((w for w in captured if w > width), default=captured[-1])
        a = self._own(bucket, lo, interval) or 0.0
        if hi == lo:
            return a
        b = self._own(bucket, hi, interval) or 0.0
        return a + (width - lo) / (hi - lo) * (b - a)

    def _across_buckets(self, bucket: int, width: int, interval: int) -> float:
        """An unready bucket's price: its own seeded cell, else the line between the ready buckets around it."""
        cell = self._tracks.get((bucket, width), {}).get(interval)
        if cell is not None and cell.samples >= self.seed_samples:
            return cell.us
        bracket = self._bracket(bucket)
        if bracket is None:
            raise ValueError(f"batch bucket {bucket} is not between two priced buckets")
        lo, hi = bracket
        a, b = self._across_widths(lo, width, interval), self._across_widths(hi, width, interval)
        return a + (bucket - lo) / (hi - lo) * (b - a)

    def verify_us(self, bucket: int, width: int) -> Optional[float]:
        """Microseconds of one verify of ``width`` at ``bucket`` (first interval), None when unpriced."""
        v = self._own(bucket, width, 0)
        if v is None and self._bracket(bucket) is not None:
            v = self._across_buckets(bucket, width, 0)
        return v

    def tables(self, also: Sequence[int] = ()) -> Dict[int, BatchCostTable]:
        """Cost tables of every priced bucket that has cells, and of the priced buckets in ``also``."""
        out: Dict[int, BatchCostTable] = {}
        for bucket in sorted({b for b, _ in self._tracks} | set(also)):
            if self.ready(bucket):
                price = lambda b, w, i: self._own(b, w, i) or 0.0  # noqa: E731
            elif self._bracket(bucket) is not None:
                price = self._across_buckets
            else:
                continue
            widths = sorted(self.widths(bucket))
            intervals, ratios = [], []
            for i in range(self.context_intervals):
                verify = [price(bucket, w, i) or 0.0 for w in widths]
                step = price(bucket, DRAFT_WIDTH, i) or 0.0
                intervals.append(IntervalCost(CostCurve.from_values(verify, [w - 1 for w in widths]),
                                              CostCurve.from_values([step], [0])))
                ratios.append(round(verify[0] / step, 4))
            out[bucket] = BatchCostTable(batch_size=bucket, cache_length_start=self.context_step,
                                         cache_length_step=self.context_step, target_max_qo_len_query=widths[-1],
                                         target_max_qo_len_cache=widths[-1], draft_max_qo_len=1,
                                         intervals=tuple(intervals), model_ratio=tuple(ratios))
        return out

    # ----------------------------------------------------------------- cache file
    def to_dict(self) -> dict:
        rows = sorted((b, w, i, c.us, c.samples) for (b, w), t in self._tracks.items() for i, c in t.items())
        return {"version": CACHE_VERSION, "key": None if self.key is None else self.key.to_dict(),
                "draft_shape": list(self.draft_shape), "context_step": self.context_step,
                "context_intervals": self.context_intervals, "cells": [list(r) for r in rows]}

    def save(self, path: str) -> None:
        """Write the cache atomically (a temporary file renamed over ``path``)."""
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        tmp = f"{path}.tmp"
        with open(tmp, "w", encoding="utf-8") as f:
            json.dump(self.to_dict(), f)
        os.replace(tmp, path)

    def _parse(self, data) -> Dict[Tuple[int, int], Dict[int, Cell]]:
        """The tracks of a cache file written for this setup; ValueError names what does not fit."""
        if not isinstance(data, dict):
            raise ValueError("the cache is not a JSON object")
        if data.get("version") != CACHE_VERSION:
            raise ValueError(f"cache version {data.get('version')!r}, this build reads {CACHE_VERSION}")
        key = None if data.get("key") is None else CostKey.from_dict(data["key"])
        if key != self.key:
            raise ValueError("the cache was measured on another setup")
        grid = (data.get("draft_shape"), data["context_step"], data["context_intervals"])
        if grid != (list(self.draft_shape), self.context_step, self.context_intervals):
            raise ValueError("the cache has another draft shape or context grid")
        tracks: Dict[Tuple[int, int], Dict[int, Cell]] = {}
        for row in data["cells"]:
            b, w, i, us, n = row
            ints_ok = all(type(v) is int for v in (b, w, i, n))
            if not ints_ok or b <= 0 or n <= 0 or not 0 <= i < self.context_intervals:
                raise ValueError(f"cell {row!r} is out of range")
            if w not in (DRAFT_WIDTH, *self.widths(b)):
                raise ValueError(f"cell {row!r} has a width this server does not capture")
            if isinstance(us, bool) or not isinstance(us, (int, float)) or not math.isfinite(us) or us <= 0:
                raise ValueError(f"cell {row!r} has no valid time")
            track = tracks.setdefault((b, w), {})
            if i in track:
                raise ValueError(f"cell {row!r} appears twice")
            track[i] = Cell(us, n)
        return tracks

    def load(self, path: str) -> bool:
        """Adopt the cache at ``path`` if it was written for this setup and grid; False (nothing adopted)
        otherwise, after logging why."""
        try:
            with open(path, encoding="utf-8") as f:
                tracks = self._parse(json.load(f))
        except (OSError, ValueError, TypeError, KeyError) as e:
            log.info("live cost cache %s not used (%s): costs are measured again", path, e)
            return False
        self._tracks = tracks
        self._samples = {bw: sum(c.samples for c in t.values()) for bw, t in tracks.items()}
        self._ready_memo = None
        return True

    def cache_path(self, cache_dir: str) -> str:
        if self.key is None:
            raise ValueError("live costs without a setup key have no cache file")
        return os.path.join(cache_dir, f"{self.key.digest}.json")
