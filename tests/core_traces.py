"""Deterministic traces of the core algorithm's decisions and files, computed through a module namespace.

Each trace takes the modules to exercise (this package's ``eagle4_b200.core`` modules, or the reference's
``eagle_harness.core`` modules with the same names) and returns plain JSON data: the decisions, prices and fitted
files the two implementations must agree on. ``tests/golden/core_golden.json`` holds the traces of the reference
(written by ``tests/golden/make_core_golden.py`` from the unmodified reference under ``baseline/_ref``), so the
comparison runs in a clean checkout; when the reference is installed the tests also recompute its traces live.
"""

from __future__ import annotations

import json
import os
import random
import shutil
import tempfile

import numpy as np
import torch


def jsonable(x):
    """``x`` after a JSON round trip (tuples become lists, float values stay exact)."""
    return json.loads(json.dumps(x))


def digest(x) -> str:
    """SHA-256 of ``x``'s canonical JSON (exact floats): stands for a large table in the golden file."""
    import hashlib

    return hashlib.sha256(json.dumps(jsonable(x), sort_keys=True).encode()).hexdigest()


# ------------------------------------------------------------------------------------------------ cost tables
def _curves(rng, widths, draft_ratio):
    base = rng.uniform(8000, 12000)
    tv = [base * (1 + 0.02 * (w - 1) ** 0.8 + rng.uniform(-0.01, 0.01)) for w in widths]
    tv[0] = base
    dv = [base / draft_ratio]
    return tv, dv


def tables(ct, rng, bss=(1, 4, 8, 32, 128, 512), widths=(1, 8, 16, 32), ratio=20.0, intervals=3):
    out = {}
    for bs in bss:
        ivs, ratios = [], []
        for _ in range(intervals):
            scale = 1 + bs / 64
            tv, dv = _curves(rng, widths, ratio)
            tv = [v * scale ** (0.3 * (w > 1)) for v, w in zip(tv, widths)]
            tgt = ct.CostCurve(tuple(tv), tuple(round(v / tv[0], 4) for v in tv), tuple(w - 1 for w in widths), (), ())
            dr = ct.CostCurve(tuple(dv), (1.0,), (0,), (), ())
            ivs.append(ct.IntervalCost(tgt, dr))
            ratios.append(round(tv[0] / dv[0], 4))
        out[bs] = ct.BatchCostTable(bs, 1024, 1024, widths[-1], widths[-1], 1, tuple(ivs), tuple(ratios))
    return out


# ------------------------------------------------------------------------------------------------ traces
def limits_trace(lim) -> dict:
    out = {"verify": [], "draft": [], "nearest": [], "span": []}
    for bs in (1, 2, 3, 7, 8, 9, 33, 64, 65, 512):
        for it in ("high_intensity", "low_intensity", "chain_intensity"):
            ci = lim.ComputeIntensity(it)
            out["verify"].append(list(lim.verify_buckets(bs, ci)))
            out["draft"].append(list(lim.draft_query_lens(bs, ci)))
    for bs in range(1, 600, 7):
        out["nearest"].append(lim.nearest_cost_batch_size(bs, lim.COST_BATCH_SIZES))
    for args in [(4, 12, 16, 1), (1, 15, 16, 1), (8, 31, 64, 4), (1, 6, 16, 16)]:
        out["span"].append(lim.req_to_token_span(*args))
    out["cost_batch_sizes"] = list(lim.COST_BATCH_SIZES)
    return jsonable(out)


def cost_model_trace(cm, ct, lim, seed: int) -> list:
    rng = random.Random(seed)
    ratio = rng.choice([7.0, 15.0, 25.0, 40.0])
    t = tables(ct, rng, ratio=ratio)
    it = rng.choice(["high_intensity", "low_intensity"])
    model = cm.CostModel(t, cm.CostModelParams(), lim.ComputeIntensity(it), 4, 12, 16)
    out = []
    for _ in range(60):
        bs = rng.choice([1, 2, 5, 8, 16, 40, 200, 512])
        ctx = rng.randint(0, 5000)
        v = model.verify_cost(bs, ctx)
        row = model.draft_cost_row(bs, ctx)
        rec = {"verify": [v.value, v.index, v.threshold], "row": [row.batch_size_ratio, row.adjust_cost_ratio],
               "widths": []}
        for depth in range(12):
            deltas = sorted(rng.uniform(0, 3) for _ in range(5))
            past = model.history_verify_num(bs)
            d = model.tree_width(depth, bs, past, row, deltas)
            rec["widths"].append([past, d.width, d.verify_num, bool(d.stop)])
        scores = [1.001]
        for _ in range(40):
            scores.append(scores[-1] + rng.uniform(0, 0.9) * (0.97 ** len(scores)))
        req = rng.choice([16, 32, 8])
        lag = rng.random() < 0.5
        rec["paged"] = list(model.verify_num_paged(scores, req, bs, ctx, lagged=lag))
        vn = rng.choice([1, 4, 8, 16])
        model.record_verify_num(bs, vn)
        rec["count"] = model.verify_count(bs, 40)
        out.append(rec)
    return jsonable(out)


def tree_policy_trace(cm, ct, lim) -> dict:
    rng = random.Random(11)
    model = cm.CostModel(tables(ct, rng, ratio=18.0), cm.CostModelParams(), lim.ComputeIntensity.HIGH, 4, 12, 16)
    a = model.tree_policy_costs()
    batches = []
    for x in a.batches:
        batches.append({"bs": x.cost_batch_size,
                        "intervals": [[list(i.depth_thresholds), list(i.verify_cost_deltas), i.verify_tier]
                                      for i in x.intervals]})
    return jsonable({"floors": a.history_floors, "initial": a.initial_widths, "batches": digest(batches),
                     "first": batches[0]})


def chain_trace(cm, ct, lim) -> dict:
    rng = random.Random(5)
    widths = (1, 2, 4, 6, 8, 10, 12, 14, 16)
    model = cm.CostModel(tables(ct, rng, widths=widths, ratio=30.0), cm.CostModelParams(), lim.ComputeIntensity.CHAIN,
                         1, 15, 16)
    stops = []
    for bs in (1, 3, 16, 100, 512):
        for depth in range(15):
            d = [0.0, rng.uniform(0, 2)]
            stops.append(model.chain_stop(depth, bs, d))
    a = model.chain_policy_costs()
    costs = [[[list(vars(t).values()) for t in ix] for ix in x.intervals] for x in a.batches]
    return jsonable({"rounds": bool(model.chain_rounds), "stops": stops, "costs": digest(costs), "first": costs[0]})


def draft_tree_trace(dt) -> dict:
    k, depth, bs, H = 4, 6, 3, 8
    tree = dt.DraftTree(dt.TreeShape(k, depth), bs, H, torch.float32, torch.device("cpu"), max_verify=16)
    g = torch.Generator().manual_seed(0)
    p0, t0, h0 = torch.rand(bs, k, generator=g), torch.randint(0, 100, (bs, k), generator=g), torch.rand(bs, H)
    tree.stage_root(bs, p0, t0, h0)
    tree.begin(bs)
    out = {"deltas": []}
    for step in range(1, depth):
        p = torch.rand(bs * k, k, generator=g)
        tk = torch.randint(0, 100, (bs * k, k), generator=g)
        hh = torch.rand(bs * k, H, generator=g)
        tree.step(bs, step, p, tk, hh)
        out["deltas"].append(tree.deltas.tolist())
    for name in ("scores", "tokens", "parents", "front_scores", "best"):
        out[name] = getattr(tree, name).tolist()
    for count in (7, 15):
        a = tree.verify_rows_reference(bs, depth, count)
        r = tree.rank_reference(bs, depth, count)
        out[f"verify_{count}"] = [a[0].tolist(), a[1].tolist()]
        out[f"rank_{count}"] = [r[0].tolist(), r[1].tolist()]
    return jsonable(out)


def live_costs_trace(lc, lim) -> dict:
    widths = lambda b: lim.verify_buckets(b, lim.ComputeIntensity.HIGH)  # noqa: E731
    key = lc.CostKey(gpu="NVIDIA B200", gpu_count=1, model="m:1", draft="d:2", engine="e", dtype="bf16")
    live = lc.LiveCosts(widths, key=key)
    rng = random.Random(3)
    seeds = []
    for _ in range(400):
        b = rng.choice([1, 8, 32])
        w = live.seed_width(b)
        seeds.append(w)
        width = w if w is not None else rng.choice(widths(b) + [0])
        ctx = rng.randint(0, 9000)
        us = rng.uniform(100, 20000) * (5 if rng.random() < 0.02 else 1)
        live.record(b, width, ctx, us)
        if rng.random() < 0.2:
            live.record(b, 0, ctx, us / 20)
    t = live.tables(also=(4, 16))
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "c.json")
        live.save(path)
        with open(path, encoding="utf-8") as f:
            saved = json.load(f)
    return jsonable({"digest": key.digest, "seeds": seeds, "state": live.to_dict(),
                     "priced": [live.priced(b) for b in (1, 4, 8, 16, 32)],
                     "tables": {str(b): [list(t[b].model_ratio), [list(iv.target.value) for iv in t[b].intervals]]
                                for b in sorted(t)},
                     "saved": saved})


# ------------------------------------------------------------------------------------------------ calibration
def _raw(cal_ours, lim_ours, root, bs, intensity, rng, *, step=256, stop=4096, top_k=4, verify=16, loop_top_m=16,
         layers=16):
    """Synthetic raw timings (written with this package's writer: both sides fit the same files)."""
    paths = cal_ours.CalibrationPaths(root)
    params = cal_ours.MeasureParams(context_step=step, context_stop=stop, batch_size=bs, verify_num=verify,
                                    node_top_k=top_k, loop_top_m=loop_top_m, repeat_cnt=8)
    paths.write_measure_params(params)
    lens = {"slm": [q for q in lim_ours.draft_query_lens(bs, intensity) if q <= top_k],
            "llm": [q for q in lim_ours.verify_buckets(bs, intensity) if q <= max(verify, loop_top_m)]}
    for model, qs in lens.items():
        for q in qs:
            recs_c, recs_m = [], []
            for kv in range(step // 2, stop + 1, step // 32):
                for _ in range(3):
                    attn = (2.0 + 0.001 * kv * (1 + 0.05 * q)) * rng.uniform(0.9, 1.1)
                    if rng.random() < 0.05:
                        attn *= 5  # an outlier
                    recs_c.append(cal_ours.MeasureRecord(int(attn * 8), 8, q, kv, f"cache_{model}", bs))
                    model_us = (9000 + 30 * q) * rng.uniform(0.97, 1.03) + attn * layers
                    recs_m.append(cal_ours.MeasureRecord(int(model_us * 4), 4, q, kv, f"model_{model}", bs))
            cal_ours.save_jsonl(os.path.join(paths.raw(bs, "cache", model), f"cache_qo_len_{q}.jsonl"), recs_c)
            cal_ours.save_jsonl(os.path.join(paths.raw(bs, "model", model), f"model_qo_len_{q}.jsonl"), recs_m)
    return params


def _tree(root):
    """File name -> SHA-256 of the bytes of every file under ``root`` (fitted files must be byte-identical)."""
    import hashlib

    out = {}
    for d, _, names in os.walk(root):
        for n in names:
            with open(os.path.join(d, n), "rb") as f:
                out[os.path.relpath(os.path.join(d, n), root)] = hashlib.sha256(f.read()).hexdigest()
    return out


def fits_trace(cal, lim, intensity: str) -> dict:
    """The fitted cost directory (file name -> content hash) of synthetic raw timings for batch sizes 1, 8 and 32."""
    from eagle4_b200.core import calibration as cal_ours
    from eagle4_b200.core import limits as lim_ours

    with tempfile.TemporaryDirectory() as d:
        raw_root, fit_root = os.path.join(d, "raw"), os.path.join(d, "fit")
        os.makedirs(fit_root)
        for bs in (1, 8, 32):
            params = _raw(cal_ours, lim_ours, raw_root, bs, lim_ours.ComputeIntensity(intensity), random.Random(bs))
            shutil.copytree(os.path.join(raw_root, "test"), os.path.join(fit_root, "test"), dirs_exist_ok=True)
            mp = cal.MeasureParams(**{k: getattr(params, k) for k in params.__dataclass_fields__})
            cal.fit_batch(cal.CalibrationPaths(fit_root), mp, lim.ComputeIntensity(intensity), cal.AttentionShape(1),
                          cal.AttentionShape(16, 4, 1024))
        return _tree(os.path.join(fit_root, "cost"))


def step_fits_trace(cal, lim) -> dict:
    rng = random.Random(3)
    high = lim.ComputeIntensity.HIGH
    params = cal.MeasureParams(256, 4096, 4, 16, 4, 16, 8)
    d = [cal.StepTiming(q, kv, 300 + q + kv * 0.01 * rng.uniform(0.99, 1.01))
         for q in lim.draft_query_lens(4, high) if q <= 4 for kv in range(128, 4097, 128)]
    t = [cal.StepTiming(q, kv, 9000 + 20 * q + kv * 0.2 * rng.uniform(0.99, 1.01))
         for q in lim.verify_buckets(4, high) if q <= 16 for kv in range(128, 4097, 128)]
    with tempfile.TemporaryDirectory() as root:
        cal.fit_step_timings(cal.CalibrationPaths(root), params, high, (cal.AttentionShape(1), d),
                             (cal.AttentionShape(16), t))
        return _tree(root)


def outliers_trace(cal) -> list:
    rng = np.random.default_rng(0)
    out = []
    for n in (1, 2, 5, 40, 200):
        for spread in (0.0, 0.05, 0.5):
            data = list(100 * (1 + spread * rng.standard_normal(n)))
            if n > 5:
                data[0] *= 8
            for conv in (0.2, 0.35):
                a = cal.remove_outliers(data, convergence_threshold=conv)
                flag = a[2].item() if hasattr(a[2], "item") else a[2]
                out.append([float(a[0]), [float(x) for x in a[1]], flag])
    return jsonable(out)


def sweep_trace(cal) -> list:
    out = []
    for step, stop, fast in ((256, 4096, False), (1024, 65536, True), (512, 16384, True), (64, 2048, False)):
        p = cal.MeasureParams(step, stop, 1, 16, 4, 16, 8, enable_fast_measurement=fast)
        out.append(dict(cal.CacheSweepPlan.from_params(p).__dict__))
    return jsonable(out)


def chain_width_trace(cw) -> list:
    rng = random.Random(5)
    out = []
    for _ in range(30):
        n = rng.randint(3, 15)
        drafts = 1000
        counts = sorted((rng.randint(0, drafts) for _ in range(n)), reverse=True)
        prof = cw.AcceptProfile.from_counts(drafts, counts)
        rounds = {b: {w: rng.uniform(5000, 30000) * (1 + 0.02 * w * b / 8) for w in range(0, 17)}
                  for b in (1, 4, 16, 64, 256)}
        rec = [cw.served_width_schedule(rounds, prof, 16, 512, allow_no_spec=allow) for allow in (False, True)]
        tree = {b: {w: (rng.uniform(5000, 30000) * (1 + 0.05 * w * b / 8), rng.uniform(1, 1 + w / 4),
                        rng.randint(1, 200)) for w in (1, 4, 8, 16)} for b in (1, 8, 32, 64, 128, 256)}
        rec.append(cw.served_tree_schedule(tree, 16, 512))
        out.append(rec)
    return jsonable(out)


def all_traces(mods) -> dict:
    """Every trace through ``mods`` (a dict of the modules ``cm ct lim lc dt cal cw``)."""
    m = mods
    out = {"limits": limits_trace(m["lim"])}
    for seed in range(6):
        out[f"cost_model_{seed}"] = cost_model_trace(m["cm"], m["ct"], m["lim"], seed)
    out["tree_policy"] = tree_policy_trace(m["cm"], m["ct"], m["lim"])
    out["chain"] = chain_trace(m["cm"], m["ct"], m["lim"])
    out["draft_tree"] = draft_tree_trace(m["dt"])
    out["live_costs"] = live_costs_trace(m["lc"], m["lim"])
    for it in ("high_intensity", "chain_intensity"):
        out[f"fits_{it}"] = fits_trace(m["cal"], m["lim"], it)
    out["step_fits"] = step_fits_trace(m["cal"], m["lim"])
    out["outliers"] = outliers_trace(m["cal"])
    out["sweep"] = sweep_trace(m["cal"])
    out["chain_widths"] = chain_width_trace(m["cw"])
    return out


def ours():
    from eagle4_b200.core import calibration, chain_width, cost_model, cost_table, draft_tree, limits, live_costs

    return {"cm": cost_model, "ct": cost_table, "lim": limits, "lc": live_costs, "dt": draft_tree,
            "cal": calibration, "cw": chain_width}


def reference(ref_dir: str):
    """The reference's core modules from ``ref_dir`` (None when it is not installed there)."""
    import sys

    if not os.path.isdir(os.path.join(ref_dir, "eagle_harness")):
        return None
    sys.path.insert(0, ref_dir)
    try:
        import eagle_harness.core.calibration as cal
        import eagle_harness.core.chain_width as cw
        import eagle_harness.core.cost_model as cm
        import eagle_harness.core.cost_table as ct
        import eagle_harness.core.draft_tree as dt
        import eagle_harness.core.limits as lim
        import eagle_harness.core.live_costs as lc
    finally:
        sys.path.remove(ref_dir)
    return {"cm": cm, "ct": ct, "lim": lim, "lc": lc, "dt": dt, "cal": cal, "cw": cw}
