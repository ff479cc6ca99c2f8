"""Cost calibration of a TokenSpeed host's own draft and target steps, measured while it serves.

A measurement run serves ``batch_size`` identical greedy requests. ``MeasurePolicy`` gives every decode round a fixed
shape: the full depth at one draft width and one verify width, both cycled round-robin over the batch size's sweep
(``draft_widths``: the draft query lengths the calibration grid times; ``verify_widths``: the verify buckets), so every
cell of the sweep comes up in turn as the contexts grow. The host times each round's draft step and verify forward and
hands them to ``CostMeasurement.record``; samples are bucketed by context (``context_step`` apart, up to
``context_stop``) and the median of each cell's samples is kept. Once every (width, context) cell of both models has
``samples`` timings, ``write`` stores them as raw whole-step records and runs the same fits as this package's own
engine calibration (``core.calibration.fit_step_timings``), giving the ``cost/bs_<N>`` tables the round policy prices
with. Only rounds at the measured batch size count, and a prefill (a batch change) restarts the cycle. The reference's
TokenSpeed path measures the same way (``eagle_harness/tokenspeed/measurement.py``).
"""

from __future__ import annotations

import statistics
from typing import Dict, List, Optional, Tuple

from eagle4_b200.core.calibration import AttentionShape, CalibrationPaths, MeasureParams, StepTiming, fit_step_timings
from eagle4_b200.core.limits import ComputeIntensity, draft_query_lens, verify_buckets


def draft_widths(batch_size: int, intensity: ComputeIntensity, node_top_k: int) -> List[int]:
    return [w for w in draft_query_lens(batch_size, intensity) if w <= node_top_k]


def verify_widths(batch_size: int, intensity: ComputeIntensity) -> List[int]:
    return sorted(verify_buckets(batch_size, intensity))


class MeasurePolicy:
    """Fixed round shapes for a measurement run: (draft width, verify width) pairs cycled round-robin."""

    def __init__(self, batch_size: int, intensity: ComputeIntensity, node_top_k: int):
        self.batch_size = batch_size
        self.drafts = draft_widths(batch_size, intensity, node_top_k)
        self.verifies = verify_widths(batch_size, intensity)
        self.round = 0

    def restart(self) -> None:
        """A prefill started a new batch: the cycle starts over."""
        self.round = 0

    def next_round(self, batch_size: int) -> Optional[Tuple[int, int]]:
        """The round's (draft width, verify width), or None for a batch that is not the measured size."""
        if batch_size != self.batch_size:
            return None
        i = self.round
        self.round += 1
        return self.drafts[i % len(self.drafts)], self.verifies[i % len(self.verifies)]


class CostMeasurement:
    """Collects timed draft steps ("slm") and verify forwards ("llm") per (width, context bucket) and fits them."""

    def __init__(self, data_path: str, *, batch_size: int, intensity: ComputeIntensity, node_top_k: int,
                 verify_num: int, context_step: int, context_stop: int, draft: AttentionShape,
                 target: AttentionShape, samples: int = 3):
        self.paths = CalibrationPaths(data_path)
        self.params = MeasureParams(context_step=context_step, context_stop=context_stop, batch_size=batch_size,
                                    verify_num=verify_num, node_top_k=node_top_k, loop_top_m=verify_num,
                                    repeat_cnt=samples)
        self.intensity = intensity
        self.shapes = {"slm": draft, "llm": target}
        self.widths = {"slm": draft_widths(batch_size, intensity, node_top_k),
                       "llm": verify_widths(batch_size, intensity)}
        self.contexts = list(range(context_step, context_stop + 1, context_step))
        self.samples = samples
        self.cells: Dict[Tuple[str, int, int], List[float]] = {}

    def _bucket(self, context: int) -> Optional[int]:
        for c in self.contexts:
            if context <= c:
                return c
        return None

    def record(self, model: str, batch_size: int, width: int, context: int, time_us: float) -> bool:
        """One timed step of ``model`` ("slm" draft, "llm" target); False when it falls outside the sweep."""
        bucket = self._bucket(context)
        if batch_size != self.params.batch_size or bucket is None or width not in self.widths[model]:
            return False
        self.cells.setdefault((model, width, bucket), []).append(float(time_us))
        return True

    def missing(self) -> List[Tuple[str, int, int]]:
        return [(m, w, c) for m in ("slm", "llm") for w in self.widths[m] for c in self.contexts
                if len(self.cells.get((m, w, c), ())) < self.samples]

    @property
    def complete(self) -> bool:
        return not self.missing()

    def write(self, *, tp_size: int = 1) -> str:
        """Fit the cells into ``cost/bs_<N>``; every cell needs its samples."""
        gaps = self.missing()
        if gaps:
            raise ValueError(f"{len(gaps)} (model, width, context) cells lack samples, e.g. {gaps[:3]}")
        timings = {m: [StepTiming(w, c, statistics.median(self.cells[(m, w, c)]))
                       for w in self.widths[m] for c in self.contexts] for m in ("slm", "llm")}
        fit_step_timings(self.paths, self.params, self.intensity, (self.shapes["slm"], timings["slm"]),
                         (self.shapes["llm"], timings["llm"]), tp_size=tp_size)
        return self.paths.cost
