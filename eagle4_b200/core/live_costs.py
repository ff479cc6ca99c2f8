"""Live costs: cost tables measured on the served rounds themselves, keyed to the serving setup.

A cell is one (batch bucket, verify width, 1024-token context interval). Its value is the fastest of its first
``seed_samples`` timings, then an EMA (``alpha``) whose samples are clamped at ``OUTLIER_RATIO`` times the cell.
A seed sweep forces each captured verify width (width 1 first, then widest first). Buckets between two ready
buckets are priced by linear interpolation in the batch size. Cells become the same ``BatchCostTable`` objects the
cost model reads. The cache file format (``version`` 2, ``cells`` as ``[bucket, width, interval, us, samples]``)
and key fields are shared with the reference (``eagle_harness/core/live_costs.py:39-356``) so caches interoperate.
"""

from __future__ import annotations

import hashlib
import json
import logging
import math
import os
from dataclasses import asdict, dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

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
        log.warning("Cost tables under %s carry no %s: they are assumed to be for %s. Calibrate again to key them.",
                    data_path, KEY_FILE, key)
        return
    if stored != key:
        diff = {f: (getattr(stored, f), getattr(key, f)) for f in key.__dataclass_fields__
                if getattr(stored, f) != getattr(key, f)}
        raise ValueError(
            f"Cost tables under {data_path} were measured on another setup (stored vs this server): {diff}. "
            "Calibrate for this setup, or drop data_path to measure costs on the served rounds."
        )


@dataclass
class Cell:
    us: float = 0.0
    samples: int = 0


@dataclass
class LiveCosts:
    widths: Callable[[int], Sequence[int]]
    key: Optional[CostKey] = None
    draft_shape: Tuple[int, int] = (1, 1)
    context_step: int = 1024
    context_intervals: int = 16
    seed_samples: int = 3
    alpha: float = 0.05
    cells: Dict[Tuple[int, int, int], Cell] = field(default_factory=dict)
    _counts: Dict[Tuple[int, int], int] = field(default_factory=dict, init=False, repr=False, compare=False)
    _ready: set = field(default_factory=set, init=False, repr=False, compare=False)
    _indexed_cells: Optional[dict] = field(default=None, init=False, repr=False, compare=False)

    def interval(self, context: int) -> int:
        return max(0, min((context - self.context_step) // self.context_step, self.context_intervals - 1))

    def _reindex(self) -> None:
        if self._indexed_cells is self.cells:
            return
        self._indexed_cells = self.cells
        counts: Dict[Tuple[int, int], int] = {}
        for (b, w, _), c in self.cells.items():
            counts[b, w] = counts.get((b, w), 0) + c.samples
        self._counts = counts
        self._ready = {b for b, _ in counts if self._seeded(b)}

    def _n(self, bucket: int, width: int) -> int:
        self._reindex()
        return self._counts.get((bucket, width), 0)

    def seed_width(self, bucket: int) -> Optional[int]:
        """The width the next round at ``bucket`` must force (width 1 first, then widest first), None once seeded."""
        order = sorted(self.widths(bucket), key=lambda w: (w != 1, -w))
        for w in order:
            if self._n(bucket, w) < self.seed_samples:
                return w
        return None

    def _seeded(self, bucket: int) -> bool:
        return self.seed_width(bucket) is None and self._n(bucket, DRAFT_WIDTH) >= self.seed_samples

    def ready(self, bucket: int) -> bool:
        self._reindex()
        return bucket in self._ready

    def _neighbours(self, bucket: int) -> Optional[Tuple[int, int]]:
        if self.ready(bucket):
            return None
        lower = [b for b in self._ready if b < bucket]
        upper = [b for b in self._ready if b > bucket]
        if not lower or not upper:
            return None
        return max(lower), min(upper)

    def priced(self, bucket: int) -> bool:
        return self.ready(bucket) or self._neighbours(bucket) is not None

    def record(self, bucket: int, width: int, context: int, us: float) -> None:
        if not math.isfinite(us) or us <= 0:
            return
        self._reindex()
        cell = self.cells.setdefault((bucket, width, self.interval(context)), Cell())
        if cell.samples < self.seed_samples:
            cell.us = us if cell.samples == 0 else min(cell.us, us)
        else:
            cell.us += self.alpha * (min(us, OUTLIER_RATIO * cell.us) - cell.us)
        cell.samples += 1
        self._counts[bucket, width] = self._counts.get((bucket, width), 0) + 1
        if bucket not in self._ready and self._seeded(bucket):
            self._ready.add(bucket)

    # ----------------------------------------------------------------- tables
    def _value(self, bucket: int, width: int, interval: int) -> Optional[float]:
        for d in range(self.context_intervals):
            for i in (interval - d, interval + d):
                c = self.cells.get((bucket, width, i))
                if c is not None and c.samples >= self.seed_samples:
                    return c.us
        pool = [c.us for (b, w, _), c in self.cells.items() if b == bucket and w == width and c.samples]
        return min(pool) if pool else None

    def verify_us(self, bucket: int, width: int) -> Optional[float]:
        v = self._value(bucket, width, 0)
        if v is None and self._neighbours(bucket) is not None:
            v = self._interpolated(bucket, width, 0)
        return v

    def _at_width(self, bucket: int, width: int, interval: int) -> float:
        if width == DRAFT_WIDTH or width in self.widths(bucket):
            return self._value(bucket, width, interval) or 0.0
        ws = sorted(self.widths(bucket))
        lo = max((w for w in ws if w < width), default=ws[0])
        hi = min((w for w in ws if w > width), default=ws[-1])
        a = self._value(bucket, lo, interval) or 0.0
        b = self._value(bucket, hi, interval) or 0.0
        return a if hi == lo else a + (width - lo) / (hi - lo) * (b - a)

    def _interpolated(self, bucket: int, width: int, interval: int) -> float:
        own = self.cells.get((bucket, width, interval))
        if own is not None and own.samples >= self.seed_samples:
            return own.us
        nb = self._neighbours(bucket)
        if nb is None:
            raise ValueError(f"batch bucket {bucket} has no ready buckets on both sides")
        lo, hi = nb
        a, b = self._at_width(lo, width, interval), self._at_width(hi, width, interval)
        return a + (bucket - lo) / (hi - lo) * (b - a)

    def tables(self, also: Sequence[int] = ()) -> Dict[int, BatchCostTable]:
        out: Dict[int, BatchCostTable] = {}
        for bucket in sorted({b for b, _, _ in self.cells} | set(also)):
            if self.ready(bucket):
                val = self._value
            elif self._neighbours(bucket) is not None:
                val = self._interpolated
            else:
                continue
            ws = sorted(self.widths(bucket))
            ivs: List[IntervalCost] = []
            ratios: List[float] = []
            for i in range(self.context_intervals):
                tgt = [val(bucket, w, i) or 0.0 for w in ws]
                dft = val(bucket, DRAFT_WIDTH, i) or 0.0
                ivs.append(IntervalCost(CostCurve.from_values(tgt, [w - 1 for w in ws]),
                                        CostCurve.from_values([dft], [0])))
                ratios.append(round(tgt[0] / dft, 4))
            out[bucket] = BatchCostTable(
                batch_size=bucket, cache_length_start=self.context_step, cache_length_step=self.context_step,
                target_max_qo_len_query=ws[-1], target_max_qo_len_cache=ws[-1], draft_max_qo_len=1,
                intervals=tuple(ivs), model_ratio=tuple(ratios),
            )
        return out

    # ----------------------------------------------------------------- cache
    def to_dict(self) -> dict:
        return {
            "version": CACHE_VERSION,
            "key": None if self.key is None else self.key.to_dict(),
            "draft_shape": list(self.draft_shape),
            "context_step": self.context_step,
            "context_intervals": self.context_intervals,
            "cells": [[b, w, i, c.us, c.samples] for (b, w, i), c in sorted(self.cells.items())],
        }

    def save(self, path: str) -> None:
        """Atomic write (temp file + rename)."""
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        tmp = f"{path}.tmp"
        with open(tmp, "w", encoding="utf-8") as f:
            json.dump(self.to_dict(), f)
        os.replace(tmp, path)

    def load(self, path: str) -> bool:
        """Adopt a cache whose key and grid match; False (nothing adopted) otherwise."""
        try:
            with open(path, encoding="utf-8") as f:
                data = json.load(f)
            if not isinstance(data, dict):
                raise ValueError("expected an object")
            key = None if data.get("key") is None else CostKey.from_dict(data["key"])
            if (data.get("version") != CACHE_VERSION or key != self.key
                    or data.get("draft_shape") != list(self.draft_shape)
                    or (data["context_step"], data["context_intervals"]) != (self.context_step, self.context_intervals)):
                log.info("Live cost cache %s is for another setup; measuring again.", path)
                return False
            cells: Dict[Tuple[int, int, int], Cell] = {}
            for b, w, i, us, n in data["cells"]:
                bad = (any(type(v) is not int for v in (b, w, i, n)) or b <= 0 or n <= 0
                       or not 0 <= i < self.context_intervals or w not in (DRAFT_WIDTH, *self.widths(b))
                       or isinstance(us, bool) or not math.isfinite(us) or us <= 0 or (b, w, i) in cells)
                if bad:
                    raise ValueError("invalid or duplicate timing cell")
                cells[b, w, i] = Cell(us, n)
        except (OSError, ValueError, TypeError, KeyError) as e:
            log.info("Live cost cache %s is unavailable or invalid (%s); measuring again.", path, e)
            return False
        self.cells = cells
        return True

    def cache_path(self, cache_dir: str) -> str:
        assert self.key is not None
        return os.path.join(cache_dir, f"{self.key.digest}.json")
