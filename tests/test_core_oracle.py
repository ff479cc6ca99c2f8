"""The core algorithm against the reference's own pure-Python core (identical decisions, prices and fitted files).

``tests/golden/core_golden.json`` holds the reference core's traces (``tests/core_traces.py``: limits, cost-model
decisions over random tables, policy exports, chain stops, draft-tree tensors, live costs and their cache file,
calibration fits as file hashes, outlier filtering, sweep plans, chain-width schedules), written once from the
unmodified reference installed under ``baseline/_ref`` by ``tests/golden/make_core_golden.py``. Every test compares
this package's trace with the golden one, so the comparison runs in a clean checkout; when the reference is installed,
its trace is recomputed live as well (so a stale golden file cannot hide a change on either side).
"""

import json
import logging
import os

import pytest

import core_traces as ct

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "baseline", "_ref")
GOLDEN = os.path.join(HERE, "golden", "core_golden.json")

with open(GOLDEN, encoding="utf-8") as f:
    _GOLDEN = json.load(f)


def _trace(mods, name):
    m = mods
    if name == "limits":
        return ct.limits_trace(m["lim"])
    if name.startswith("cost_model_"):
        return ct.cost_model_trace(m["cm"], m["ct"], m["lim"], int(name.rsplit("_", 1)[1]))
    if name == "tree_policy":
        return ct.tree_policy_trace(m["cm"], m["ct"], m["lim"])
    if name == "chain":
        return ct.chain_trace(m["cm"], m["ct"], m["lim"])
    if name == "draft_tree":
        return ct.draft_tree_trace(m["dt"])
    if name == "live_costs":
        return ct.live_costs_trace(m["lc"], m["lim"])
    if name.startswith("fits_"):
        return ct.fits_trace(m["cal"], m["lim"], name[len("fits_"):])
    if name == "step_fits":
        return ct.step_fits_trace(m["cal"], m["lim"])
    if name == "outliers":
        return ct.outliers_trace(m["cal"])
    if name == "sweep":
        return ct.sweep_trace(m["cal"])
    if name == "chain_widths":
        return ct.chain_width_trace(m["cw"])
    raise KeyError(name)


@pytest.fixture(autouse=True)
def _quiet():
    logging.disable(logging.WARNING)  # clamped-context warnings of the synthetic tables
    yield
    logging.disable(logging.NOTSET)


@pytest.mark.parametrize("name", sorted(_GOLDEN))
def test_matches_reference_golden(name):
    assert _trace(ct.ours(), name) == _GOLDEN[name]


@pytest.mark.parametrize("name", sorted(_GOLDEN))
def test_golden_matches_live_reference(name):
    ref = ct.reference(REF)
    if ref is None:
        pytest.skip("reference package not installed under baseline/_ref (the golden comparison above still ran)")
    assert _trace(ref, name) == _GOLDEN[name]


def test_live_cost_cache_interoperates(tmp_path):
    """A cache written by this package loads in the reference and vice versa (skipped without the reference)."""
    ref = ct.reference(REF)
    if ref is None:
        pytest.skip("reference package not installed under baseline/_ref")
    ours = ct.ours()
    widths = lambda b: ours["lim"].verify_buckets(b, ours["lim"].ComputeIntensity.HIGH)  # noqa: E731
    kw = dict(gpu="NVIDIA B200", gpu_count=1, model="m:1", draft="d:2", engine="e", dtype="bf16")
    a = ours["lc"].LiveCosts(widths, key=ours["lc"].CostKey(**kw))
    for i in range(50):
        a.record(1, 0 if i % 3 == 0 else 16, 100 * i, 1000.0 + i)
    path = str(tmp_path / "c.json")
    a.save(path)
    b = ref["lc"].LiveCosts(widths, key=ref["lc"].CostKey(**kw))
    assert b.load(path) and b.to_dict() == a.to_dict()
    b.save(path)
    c = ours["lc"].LiveCosts(widths, key=ours["lc"].CostKey(**kw))
    assert c.load(path) and c.to_dict() == a.to_dict()
