"""Offline calibration: raw timing records, the robust cost fits and the calibration directory layout.

Layout under a calibration ``data_path`` (identical to the reference's, so existing directories load and the fitted
files are byte-identical for the same raw timings; reference ``eagle_harness/core/calibration.py:1-16``)::

    config/measure_config.json                   MeasureParams of the batch being measured
    test/bs_<N>/{model,cache}_{slm,llm}/*.jsonl  raw timings, one record per line
    cost/bs_<N>/{cache,query,model}_{slm,llm}/   fitted costs (json)

``slm`` is the draft model, ``llm`` the target. The fits:

* ``cache``: attention time per layer, per cache-length interval and query length (robust mean of the records);
* ``query``: the rest of a forward, per query length (step time minus the fitted attention of every layer);
* ``model``: ``query + cache * layers`` per interval, with sliding-window layers capped at their window; these are
  the ``model_interval_<i>.json`` curves the cost model reads.

The robust mean is an iterative z-score filter whose threshold shrinks each pass until the kept values span at most a
convergence fraction of their mean (reference ``calibration.py:198-227``). Engines that time only whole forwards use
:func:`fit_step_timings`: the attention cost per layer is the step's growth over its shortest cache length.
"""

from __future__ import annotations

import json
import logging
import os
from collections import defaultdict
from dataclasses import asdict, dataclass
from typing import Any, Dict, Iterable, List, Sequence, Tuple

import numpy as np

from eagle4_b200.core.limits import ComputeIntensity, draft_query_lens, verify_buckets

log = logging.getLogger(__name__)

DRAFT = "slm"
TARGET = "llm"


# --------------------------------------------------------------------------------------------- records and files
@dataclass
class MeasureRecord:
    """``time_us`` for ``measure_count`` repeats of one (query length, cache length) shape."""

    time_us: int
    measure_count: int = 1
    query_length: int = 1
    cache_length: int = 64
    task_category: str = "cache_llm"
    batch_size: int = 1

    def to_dict(self) -> dict:
        return {"time_intervals": self.time_us, "measure_count": self.measure_count,
                "query_length": self.query_length, "cache_length": self.cache_length,
                "task_category": self.task_category, "batch_size": self.batch_size}

    @classmethod
    def from_dict(cls, d: dict) -> "MeasureRecord":
        return cls(d["time_intervals"], d.get("measure_count", 1), d.get("query_length", 1),
                   d.get("cache_length", 64), d.get("task_category", "cache_llm"), d.get("batch_size", 1))

    @property
    def per_call_us(self) -> float:
        return self.time_us / self.measure_count


def _mkparent(path: str) -> None:
    parent = os.path.dirname(path)
    if parent:
        os.makedirs(parent, exist_ok=True)


def save_jsonl(path: str, records: Iterable[MeasureRecord]) -> None:
    _mkparent(path)
    with open(path, "w", encoding="utf-8") as f:
        f.writelines(json.dumps(r.to_dict(), ensure_ascii=False) + "\n" for r in records)


def load_jsonl(path: str) -> List[dict]:
    """The JSON objects of a JSON-lines file; malformed lines are skipped with a warning."""
    out = []
    with open(path, encoding="utf-8") as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                out.append(json.loads(line))
            except json.JSONDecodeError:
                log.warning("skipping a malformed line in %s", path)
    return out


def _dump(path: str, data: dict) -> None:
    _mkparent(path)
    with open(path, "w", encoding="utf-8") as f:
        json.dump(data, f, indent=4)


def _r4(values: Iterable[float]) -> List[float]:
    return [round(v, 4) for v in values]


# --------------------------------------------------------------------------------------------- parameters / layout
@dataclass
class MeasureParams:
    """The sweep of one batch size's calibration, as stored in ``config/measure_config.json``."""

    context_step: int
    context_stop: int
    batch_size: int
    verify_num: int
    node_top_k: int
    loop_top_m: int
    repeat_cnt: int
    enable_fast_measurement: bool = False
    cache_len: int = 1
    query_llm: int = 1
    query_slm: int = 1


@dataclass(frozen=True)
class CalibrationPaths:
    """Directory layout of one calibration ``data_path``."""

    data_path: str

    @property
    def cost(self) -> str:
        return os.path.join(self.data_path, "cost")

    @property
    def test(self) -> str:
        return os.path.join(self.data_path, "test")

    @property
    def config(self) -> str:
        return os.path.join(self.data_path, "config")

    def raw(self, batch_size: int, kind: str, model: str) -> str:
        return os.path.join(self.test, f"bs_{batch_size}", f"{kind}_{model}")

    def fitted(self, batch_size: int, kind: str, model: str) -> str:
        return os.path.join(self.cost, f"bs_{batch_size}", f"{kind}_{model}")

    def write_measure_params(self, params: MeasureParams) -> None:
        path = os.path.join(self.config, "measure_config.json")
        _mkparent(path)
        with open(path, "w", encoding="utf-8") as f:
            json.dump(asdict(params), f, ensure_ascii=False)
            f.write("\n")


@dataclass(frozen=True)
class CacheSweepPlan:
    """Cache-length grid of one attention sweep (timings below ``kv_step`` are warm-up and dropped by the fits)."""

    kv_start: int
    kv_step: int
    kv_stop: int
    interval_step: int
    num_layers: int

    @classmethod
    def from_params(cls, params: MeasureParams) -> "CacheSweepPlan":
        step, stop = params.context_step, params.context_stop
        if step not in (64, 128, 256, 512, 1024):
            raise ValueError(f"the context step {step} is not one of 64, 128, 256, 512, 1024")
        if not 2048 <= stop <= 128 * 1024:
            raise ValueError(f"the context stop {stop} lies outside 2048..131072")
        if stop % step or not 16 <= stop // step <= 128:
            raise ValueError(f"the context stop {stop} is not 16 to 128 context steps of {step}")
        layers, interval = params.repeat_cnt, step // 32
        if params.enable_fast_measurement:
            interval = step // 16
            intervals = stop // step
            if intervals >= 32 and stop >= 32 * 1024:
                layers = max(layers // 4, 1)
            elif (intervals >= 32 and stop >= 8 * 1024) or stop >= 16 * 1024:
                layers = max(layers // 2, 1)
        return cls(step // 2, step, stop, interval, layers)

    def cache_lengths(self) -> range:
        return range(self.kv_start, self.kv_stop + 1, self.interval_step)


def query_lens(category: str, batch_size: int, intensity: ComputeIntensity, max_query_length: int) -> List[int]:
    """Query lengths a fit reads: the draft's widths for the draft, the verify buckets for the target."""
    if category.endswith(DRAFT):
        return [q for q in draft_query_lens(batch_size, intensity) if q <= max_query_length]
    if category.endswith(TARGET):
        return sorted(q for q in verify_buckets(batch_size, intensity) if q <= max_query_length)
    return list(range(1, max_query_length + 1))


# --------------------------------------------------------------------------------------------- robust mean
def remove_outliers(data: Sequence[float], initial_threshold: float = 6.0, threshold_decrement: float = 0.2,
                    min_threshold: float = 1.0, convergence_threshold: float = 0.2, max_iterations: int = 50,
                    sample_rate: float = 0.75) -> Tuple[float, List[float], bool]:
    """Iterative z-score filter; returns ``(mean, kept values, stable)``.

    Each pass keeps the values within ``threshold`` population standard deviations of the kept values' mean, then
    lowers the threshold. It stops when fewer than ``sample_rate`` of the values are left, or when the kept values
    span at most ``convergence_threshold`` of their mean (the result is stable only in the second case). A set of
    identical values has no spread to normalise by: nothing passes the z test and the set counts as unstable.
    """
    if len(data) == 0:
        raise ValueError("no samples to filter")
    kept = np.asarray(list(data), dtype=np.float64)
    mean = float(np.mean(kept))
    floor = sample_rate * len(kept)
    threshold, spread = initial_threshold, 1.0
    for _ in range(max_iterations):
        with np.errstate(divide="ignore", invalid="ignore"):
            z = np.abs((kept - kept.mean()) / kept.std())
        kept = kept[z < threshold]
        if kept.size:
            mean = float(np.mean(kept))
        if kept.size < floor:
            break
        spread = (kept.max() - kept.min()) / mean
        if mean != 0 and spread <= convergence_threshold:
            break
        threshold = max(threshold - threshold_decrement, min_threshold)
    stable = bool(spread <= convergence_threshold and kept.size >= floor)
    return mean, kept.tolist(), stable


# --------------------------------------------------------------------------------------------- fits
def _max_interval(path: str, prefix: str) -> int:
    ids = []
    for name in os.listdir(path):
        if name.startswith(prefix) and name.endswith(".json"):
            try:
                ids.append(int(name.split("_")[-1].split(".")[0]))
            except ValueError as e:
                raise RuntimeError(f"{name}: the file name does not end in a query length") from e
    if not ids:
        raise FileNotFoundError(f"{path} holds no {prefix}<n>.json timing file")
    return max(ids)


def _records(path: str) -> List[dict]:
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} does not exist")
    return load_jsonl(path)


def fit_cache_costs(category: str, source: str, target: str, *, max_query_length: int, cache_length_start: int,
                    cache_length_step: int, cache_length_stop: int, batch_size: int, intensity: ComputeIntensity,
                    fast: bool = False) -> float:
    """Attention cost per layer for every cache interval and query length; returns the share of unstable cells."""
    samples: Dict[int, Dict[int, List[float]]] = defaultdict(lambda: defaultdict(list))
    for q in query_lens(category, batch_size, intensity, max_query_length):
        for rec in _records(os.path.join(source, f"cache_qo_len_{q}.jsonl")):
            kv = rec["cache_length"]
            if cache_length_start <= kv < cache_length_stop:
                samples[(kv - cache_length_start) // cache_length_step][q].append(
                    rec["time_intervals"] / rec["measure_count"])
    curves: Dict[int, List[float]] = {}
    cells = unstable = 0
    for interval, by_q in samples.items():
        curve = curves.setdefault(interval, [0.0] * max_query_length)
        for q, times in by_q.items():
            mean, _, stable = remove_outliers(times, convergence_threshold=0.25 if fast else 0.35)
            curve[q - 1] = mean
            cells += 1
            unstable += not stable
    instability = unstable / cells if cells else 0.0
    if instability >= (0.20 if fast else 0.25):
        log.warning("%.2f%% of the attention-cost intervals did not settle: the fit may be noisy", instability * 100)
    for interval in range((cache_length_stop - cache_length_start) // cache_length_step):
        curve = curves.get(interval, [0.0] * max_query_length)
        ratio = [round(v / curve[0], 4) for v in curve] if curve and curve[0] > 0 else []
        _dump(os.path.join(target, f"cache_interval_{interval}.json"), {
            "value": _r4(curve), "index": list(range(len(curve))), "ratio": _r4(ratio), "array": _r4(curve),
            "batch_size": batch_size, "max_query_length": max_query_length,
            "cache_length_start": cache_length_start, "cache_length_step": cache_length_step,
            "cache_length_stop": cache_length_stop, "instability_rate": round(instability, 2)})
    return instability


def _cache_curves(path: str) -> Dict[int, list]:
    out = {}
    for i in range(_max_interval(path, "cache_interval_") + 1):
        name = os.path.join(path, f"cache_interval_{i}.json")
        if not os.path.exists(name):
            raise FileNotFoundError(f"the attention-cost fit for interval file {name} is missing")
        with open(name, encoding="utf-8") as f:
            out[i] = json.load(f).get("array", [])
    return out


def fit_query_costs(category: str, model_source: str, cache_source: str, target: str, *, max_query_length: int,
                    cache_length_start: int, cache_length_step: int, cache_layers: int, batch_size: int,
                    intensity: ComputeIntensity, average: bool = False, sliding_window_layers: int = 0,
                    sliding_window: int = 0) -> float:
    """Non-attention cost per query length: each measured step minus the fitted attention of its cache length."""
    cache = _cache_curves(cache_source)
    lens = query_lens(category, batch_size, intensity, max_query_length)
    rest: Dict[int, List[float]] = defaultdict(list)
    swa_interval = max((sliding_window - cache_length_start) // cache_length_step, 0)
    for q in lens:
        for rec in _records(os.path.join(model_source, f"model_qo_len_{q}.jsonl")):
            kv = rec["cache_length"]
            if kv < cache_length_start:
                continue
            interval = (kv - cache_length_start) // cache_length_step
            curve = cache.get(interval)
            if curve is None or len(curve) < q:
                continue
            attn = curve[q - 1]
            value = rec["time_intervals"] / rec["measure_count"] - attn * cache_layers
            if sliding_window_layers > 0 and kv > sliding_window:  # windowed layers stop growing at the window
                value += sliding_window_layers * (attn - cache[swa_interval][q - 1])
            rest[q].append(value)
    fitted = {}
    unstable = 0
    for q in lens:
        if not rest.get(q):
            raise RuntimeError(f"query length {q} has no settled non-attention timing")
        mean, _, stable = remove_outliers(rest[q], convergence_threshold=0.50 if average else 0.30)
        unstable += not stable
        fitted[q] = mean
    instability = unstable / len(lens) if lens else 0.0
    if instability >= 0.30:
        log.warning("%.2f%% of the query lengths did not settle: the non-attention fit may be noisy", instability * 100)
    for q in lens:
        _dump(os.path.join(target, f"query_{q}.json"), {"mean": round(fitted[q], 4), "array": _r4(rest[q]),
                                                        "batch_size": batch_size,
                                                        "instability_rate": round(instability, 4)})
    return instability


def fit_model_costs(category: str, query_source: str, cache_source: str, target: str, *, max_query_length_query: int,
                    max_query_length_cache: int, cache_length_start: int, cache_length_step: int, cache_layers: int,
                    batch_size: int, intensity: ComputeIntensity, sliding_window_layers: int = 0,
                    sliding_window: int = 0) -> None:
    """``model_interval_<i>.json``: query cost plus the attention of every layer, per interval and query length."""
    lens = query_lens(category, batch_size, intensity, max_query_length_query)
    rest = []
    for q in lens:
        name = os.path.join(query_source, f"query_{q}.json")
        if not os.path.exists(name):
            raise FileNotFoundError(f"the non-attention cost fit {name} is missing")
        with open(name, encoding="utf-8") as f:
            rest.append(json.load(f).get("mean", 0.0))
    swa_interval = max(sliding_window // cache_length_step - 1, 0)
    curves: List[list] = []
    for interval in range(_max_interval(cache_source, "cache_interval_") + 1):
        with open(os.path.join(cache_source, f"cache_interval_{interval}.json"), encoding="utf-8") as f:
            cache = json.load(f)
        curve = cache.get("array", [])
        curves.append(curve)
        if not curve or len(curve) != max_query_length_cache:
            raise RuntimeError(f"the attention-cost fit of interval {interval} is unusable")
        windowed = swa_interval > 0 and interval > swa_interval
        costs = []
        for r, q in zip(rest, lens):
            if windowed:
                costs.append(r + curve[q - 1] * (cache_layers - sliding_window_layers)
                             + curves[swa_interval][q - 1] * sliding_window_layers)
            else:
                costs.append(r + curve[q - 1] * cache_layers)
        ratio = [round(v / costs[0], 4) for v in costs] if costs and costs[0] > 0 else []
        _dump(os.path.join(target, f"model_interval_{interval}.json"), {
            "notes": "Estimated model_cost = query_cost + cache_cost", "value": _r4(costs),
            "index": [q - 1 for q in lens], "ratio": ratio, "array_model": _r4(costs), "array_query": _r4(rest),
            "array_cache": _r4(v * cache_layers for v in curve), "batch_size": batch_size,
            "max_query_length_query": max_query_length_query, "max_query_length_cache": max_query_length_cache,
            "cache_length_start": cache_length_start, "cache_length_step": cache_length_step,
            "cache_layers_num": cache_layers, "instability_rate": cache.get("instability_rate", -1.0)})


# --------------------------------------------------------------------------------------------- one batch size
@dataclass(frozen=True)
class AttentionShape:
    """What the fits need of a model: its attention layers and how many of them are sliding-window layers."""

    attention_layers: int
    sliding_window_layers: int = 0
    sliding_window: int = 0


def attention_shape(config: Any) -> AttentionShape:
    """Attention layer counts of an HF text config; layouts the fits cannot read are refused."""
    config = getattr(config, "text_config", config)
    layers = getattr(config, "num_hidden_layers", 0)
    types = getattr(config, "layer_types", None)
    window = getattr(config, "sliding_window", None) or 0
    if types is None:
        if getattr(config, "full_attention_interval", None) or getattr(config, "hybrid_override_pattern", None):
            raise ValueError("a hybrid model config must list its layer_types for calibration")
        windowed = window and getattr(config, "use_sliding_window", True)
        types = ["sliding_attention" if windowed else "full_attention"] * layers
    if len(types) != layers or set(types) - {"full_attention", "sliding_attention", "linear_attention", "mamba"}:
        raise ValueError(f"no attention layout can be read from layer types {types!r}")
    attn = sum(t in ("full_attention", "sliding_attention") for t in types)
    sliding = types.count("sliding_attention")
    if attn < 1 or (sliding and window <= 0):
        raise ValueError("calibration needs at least one attention layer, and a window above zero for sliding ones")
    return AttentionShape(attn, sliding, window)


def save_model_timings(paths: CalibrationPaths, params: MeasureParams, records: Sequence[MeasureRecord]) -> None:
    """Group whole-step timings by model and query length into ``model_qo_len_<q>.jsonl``."""
    groups: Dict[Tuple[str, int], List[MeasureRecord]] = defaultdict(list)
    for rec in records:
        groups[(rec.task_category.split("_")[-1], rec.query_length)].append(rec)
    for (model, q), group in sorted(groups.items()):
        save_jsonl(os.path.join(paths.raw(params.batch_size, "model", model), f"model_qo_len_{q}.jsonl"), group)


def fit_batch(paths: CalibrationPaths, params: MeasureParams, intensity: ComputeIntensity, draft: AttentionShape,
              target: AttentionShape, *, tp_size: int = 1) -> None:
    """All fits of one batch size, the draft before the target at each stage."""
    bs, step = params.batch_size, params.context_step
    grid = dict(cache_length_start=step, cache_length_step=step, batch_size=bs, intensity=intensity)
    for model, max_q in ((DRAFT, params.node_top_k), (TARGET, params.verify_num)):
        fit_cache_costs(f"cache_all_{model}", paths.raw(bs, "cache", model), paths.fitted(bs, "cache", model),
                        max_query_length=max_q, cache_length_stop=params.context_stop,
                        fast=params.enable_fast_measurement, **grid)
    shapes = ((DRAFT, draft, params.node_top_k, params.node_top_k,
               (not params.enable_fast_measurement) or tp_size > 1),
              (TARGET, target, params.loop_top_m, params.verify_num, False))
    for model, shape, max_q, _, average in shapes:
        fit_query_costs(f"query_{model}", paths.raw(bs, "model", model), paths.fitted(bs, "cache", model),
                        paths.fitted(bs, "query", model), max_query_length=max_q,
                        cache_layers=shape.attention_layers, average=average,
                        sliding_window_layers=shape.sliding_window_layers, sliding_window=shape.sliding_window,
                        **grid)
    for model, shape, max_q, max_cache, _ in shapes:
        fit_model_costs(f"model_{model}", paths.fitted(bs, "query", model), paths.fitted(bs, "cache", model),
                        paths.fitted(bs, "model", model), max_query_length_query=max_q,
                        max_query_length_cache=max_cache, cache_layers=shape.attention_layers,
                        sliding_window_layers=shape.sliding_window_layers, sliding_window=shape.sliding_window,
                        **grid)


# --------------------------------------------------------------------------------------------- whole-step timings
@dataclass(frozen=True)
class StepTiming:
    """One timed forward: ``query_length`` tokens per request at ``cache_length``, ``time_us`` microseconds."""

    query_length: int
    cache_length: int
    time_us: float


def attention_growth_records(timings: Sequence[StepTiming], attention_layers: int, category: str,
                             batch_size: int = 1) -> List[MeasureRecord]:
    """Attention cost per layer from whole-step timings: the step's growth over its shortest cache length, per
    attention layer (recorded in nanoseconds per call, at least 1)."""
    out = []
    for q in sorted({t.query_length for t in timings}):
        times = {t.cache_length: t.time_us for t in timings if t.query_length == q}
        base = min(times.values())
        out.extend(MeasureRecord(max(int(1000 * (us - base) / attention_layers), 1), 1000, q, kv, category,
                                 batch_size) for kv, us in times.items())
    return out


def fit_step_timings(paths: CalibrationPaths, params: MeasureParams, intensity: ComputeIntensity,
                     draft: Tuple[AttentionShape, Sequence[StepTiming]],
                     target: Tuple[AttentionShape, Sequence[StepTiming]], *, tp_size: int = 1) -> None:
    """Store one batch size's whole-step timings of the draft and the target as raw records and run every fit."""
    paths.write_measure_params(params)
    bs = params.batch_size
    for model, (shape, timings) in ((DRAFT, draft), (TARGET, target)):
        save_model_timings(paths, params, [MeasureRecord(int(1000 * t.time_us), 1000, t.query_length,
                                                         t.cache_length, f"model_{model}", bs) for t in timings])
        by_q: Dict[int, List[MeasureRecord]] = defaultdict(list)
        for rec in attention_growth_records(timings, shape.attention_layers, f"cache_{model}", bs):
            by_q[rec.query_length].append(rec)
        for q, group in by_q.items():
            save_jsonl(os.path.join(paths.raw(bs, "cache", model), f"cache_qo_len_{q}.jsonl"), group)
    fit_batch(paths, params, intensity, draft[0], target[0], tp_size=tp_size)
