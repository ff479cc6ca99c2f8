"""Command line: ``python -m eagle4_b200.cli calibrate|check`` (console script ``eagle4-b200``).

``calibrate`` measures this package's engine on the local GPU (target verify forwards and draft steps over a context
sweep, one CUDA graph per timed shape), fits the cost tables into a fresh directory and prints the serving config
that uses them (reference ``eagle_harness/cli.py:268-345``, which drives an SGLang or vLLM server instead; the
settings and output layout are the same: ``settings.json``, the calibration ``data_path`` and ``serve.sh``).
With ``--tp N`` the command supervises N workers (one per GPU, ``torch.distributed.run``) in a process group of its
own and ends the group on a failure, an interrupt or ``--timeout``; ``serve.sh`` is written only when they succeed.
``check`` reports the serving hosts this package plugs into and, with ``--kernels``, loads the native library.
"""

from __future__ import annotations

import argparse
import json
import shlex
import sys
from pathlib import Path
from typing import List, Optional


def _positive(value: str) -> int:
    n = int(value)
    if n < 1:
        raise argparse.ArgumentTypeError("must be a positive integer")
    return n


def _sizes(value: str) -> List[int]:
    try:
        sizes = sorted({_positive(v) for v in value.split(",")})
    except (ValueError, argparse.ArgumentTypeError) as e:
        raise argparse.ArgumentTypeError("use comma-separated positive integers, such as 1,8") from e
    if sizes[-1] > 512:
        raise argparse.ArgumentTypeError("batch sizes must not exceed 512")
    return sizes


def _model_args(args) -> dict:
    return {"model": args.model, "draft": args.draft}


def build_llm(model: str, draft: Optional[str], *, max_batch: int, max_len: int, tree, device="cuda",
              config=None, tp=None, dtype=None, temperature: float = 0.0, seed: int = 0,
              kv_tokens: Optional[int] = None):
    """A named synthetic shape (random weights) or a checkpoint directory pair; ``tp``: this rank's
    :class:`~eagle4_b200.parallel.tp.TensorParallel` (the weights are sharded over its group)."""
    import torch

    from eagle4_b200.api import LLM, NAMED, from_pretrained

    dtype = dtype or torch.bfloat16
    if model in NAMED:
        return LLM.synthetic(model, device=device, tree=tree, max_batch=max_batch, max_len=max_len, config=config,
                             tp=tp, dtype=dtype, temperature=temperature, sample_seed=seed, kv_tokens=kv_tokens)
    return from_pretrained(model, draft, device=device, tree=tree, max_batch=max_batch, max_len=max_len,
                           config=config, tp=tp, dtype=dtype, temperature=temperature, sample_seed=seed,
                           kv_tokens=kv_tokens)


def serve_config(output: Path) -> dict:
    return {"mode": "serve", "data_path": str(output)}


def _serve_command(args) -> str:
    serve = ["--model", args.model] + (["--draft", args.draft] if args.draft else []) + \
        ["--config", json.dumps(serve_config(args.output))]
    if args.tp > 1:
        launch = ["python", "-m", "torch.distributed.run", "--nnodes", "1", "--nproc-per-node", str(args.tp),
                  "--master-addr", "127.0.0.1", "-m", "eagle4_b200.serve"]
    else:
        launch = ["python", "-m", "eagle4_b200.serve"]
    return " ".join(shlex.quote(x) for x in launch + serve)


def _worker_args(args) -> List[str]:
    """The calibrate arguments of one tensor-parallel worker (the same measurement, run as one rank)."""
    out = ["calibrate", "--model", args.model, "--output", str(args.output), "--tp", str(args.tp), "--worker",
           "--batch-sizes", ",".join(map(str, args.batch_sizes)), "--context-step", str(args.context_step),
           "--context-stop", str(args.context_stop), "--repeats", str(args.repeats), "--steps", str(args.steps),
           "--top-k", str(args.top_k), "--draft-tokens", str(args.draft_tokens), "--kind", args.kind]
    if args.draft:
        out += ["--draft", args.draft]
    if args.package:
        out.append("--package")
    return out


def _measure(args, tp=None) -> dict:
    """Build the engine (this rank's shard under ``tp``), measure, fit and optionally package; returns the cost
    model's problems per batch size."""
    import torch

    from eagle4_b200.api import TreeSpec
    from eagle4_b200.core.live_costs import CostKey
    from eagle4_b200.runtime.calibrate import calibrate

    world, rank = (tp.world, tp.rank) if tp is not None else (1, 0)
    tree = TreeSpec(args.steps, 1 if args.kind == "chain" else args.top_k, args.draft_tokens)
    llm = build_llm(args.model, args.draft, max_batch=max(args.batch_sizes), max_len=args.context_stop + 256,
                    tree=tree, tp=tp)
    key = CostKey(gpu=torch.cuda.get_device_name(), gpu_count=world, model=args.model, draft=str(args.draft or ""),
                  engine="eagle4_b200", dtype="bfloat16")
    if args.kind == "chain":
        from eagle4_b200.runtime.calibrate import calibrate_chain

        calibrate_chain(llm.engine, str(args.output), batch_sizes=args.batch_sizes, key=key)
        problems = {}
    else:
        problems = calibrate(llm.engine, str(args.output), batch_sizes=args.batch_sizes,
                             context_step=args.context_step, context_stop=args.context_stop, repeats=args.repeats,
                             key=key)
    if args.package and rank == 0:
        from eagle4_b200.core.cost_profiles import write_profile

        # the directory doubles as a packaged profile: matched by device, TP size and the models' shapes
        tcfg, dcfg = _full_configs(args) if world > 1 else (llm.target.cfg, llm.draft.cfg)
        write_profile(str(args.output), devices=[torch.cuda.get_device_name()], tp_size=world,
                      target_config=tcfg.to_hf(), draft_config=dcfg.to_hf())
    return problems


def _full_configs(args):
    """The whole (unsharded) target and draft configs of ``--model`` / ``--draft``."""
    from eagle4_b200.api import NAMED
    from eagle4_b200.models.configs import TargetConfig
    from eagle4_b200.models.eagle4_config import draft_config_from_hf

    if args.model in NAMED:
        tcfg = NAMED[args.model][0]()
        return tcfg, NAMED[args.model][1](tcfg)
    tcfg = TargetConfig.from_hf(json.loads((Path(args.model) / "config.json").read_text()))
    if not args.draft:
        return tcfg, None
    dcfg = draft_config_from_hf(json.loads((Path(args.draft) / "config.json").read_text()),
                                target_vocab_size=tcfg.vocab_size, target_num_layers=tcfg.num_layers)
    return tcfg, dcfg


def _report(problems: dict) -> None:
    for b, p in problems.items():
        if p:
            print(f"batch size {b}: the cost model refuses these costs ({p}); rounds there keep the fixed shape")


def _calibrate_worker(args) -> int:
    """One rank of a tensor-parallel calibration (launched by the supervising ``calibrate --tp N``)."""
    import datetime
    import os

    import torch
    import torch.distributed as dist

    from eagle4_b200.parallel.tp import TensorParallel

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    if dist.get_world_size() != args.tp:
        raise RuntimeError(f"launched with {dist.get_world_size()} ranks for --tp {args.tp}")
    tp = TensorParallel(max_rows=max(256, max(args.batch_sizes) * args.draft_tokens), max_cols=8192)
    try:
        problems = _measure(args, tp)
        if tp.rank == 0:
            _report(problems)
    finally:
        tp.close()
        dist.destroy_process_group()
    return 0


def _calibrate_tp(args) -> int:
    """Supervise ``--tp N`` workers (one per GPU) in a process group of their own: the group is ended on a failure,
    a time-out or an interrupt; measurements written so far stay; ``serve.sh`` is written only on success."""
    import torch

    from eagle4_b200.runtime.supervise import supervise, torchrun

    cmd = torchrun(args.tp, "eagle4_b200.cli", _worker_args(args))
    if args.dry_run:
        print(json.dumps(_settings(args), indent=2))
        print(" ".join(shlex.quote(x) for x in cmd))
        print(_serve_command(args))
        return 0
    if torch.cuda.device_count() < args.tp:
        raise RuntimeError(f"--tp {args.tp} needs {args.tp} GPUs; {torch.cuda.device_count()} are visible")
    args.output.mkdir(parents=True, exist_ok=False)
    (args.output / "settings.json").write_text(json.dumps(_settings(args), indent=2) + "\n")
    out = supervise(cmd, timeout=args.timeout)
    if out.timed_out:
        print(f"eagle4-b200: calibration passed --timeout {args.timeout:g} s and was stopped; partial measurements "
              f"remain in {args.output}", file=sys.stderr)
        return out.code
    if out.interrupted:
        print(f"eagle4-b200: interrupted; partial measurements remain in {args.output}.", file=sys.stderr)
        return out.code
    if not out.ok:
        print(f"eagle4-b200: calibration workers failed (exit code {out.code}); partial measurements remain in "
              f"{args.output}", file=sys.stderr)
        return out.code
    return _finish(args)


def _settings(args) -> dict:
    return {k: str(v) if isinstance(v, Path) else v for k, v in vars(args).items() if k not in ("func", "worker")}


def _finish(args) -> int:
    command = _serve_command(args)
    (args.output / "serve.sh").write_text("#!/bin/sh\nset -eu\nexec " + command + "\n")
    print(f"Calibration saved in {args.output}. Serve with:\nsh {shlex.quote(str(args.output / 'serve.sh'))}")
    return 0


def _calibrate(args) -> int:
    import torch

    args.output = (args.output or Path("eagle4-calibration")).resolve()
    if args.worker:
        return _calibrate_worker(args)
    if args.tp > 1:
        return _calibrate_tp(args)
    if not torch.cuda.is_available() and not args.dry_run:
        raise RuntimeError("calibration times the GPU; no CUDA device is visible")
    if args.dry_run:
        print(json.dumps(_settings(args), indent=2))
        print(_serve_command(args))
        return 0
    args.output.mkdir(parents=True, exist_ok=False)
    (args.output / "settings.json").write_text(json.dumps(_settings(args), indent=2) + "\n")
    _report(_measure(args))
    return _finish(args)


def _plan(args) -> int:
    from eagle4_b200.runtime.memory import B200_GB, plan

    tcfg, dcfg = _full_configs(args)
    p = plan(tcfg, dcfg, tp=args.tp, max_batch=args.max_batch, max_len=args.max_len, kv_tokens=args.kv_tokens,
             tree=tuple(int(v) for v in args.tree.split(",")), reserve_gb=args.reserve_gb,
             prefill_chunk=args.prefill_chunk)
    summary = p.summary(args.gpu_gb or round(B200_GB, 1))
    print(json.dumps(summary, indent=2))
    return 0 if summary["fits"] else 1


def calibration_report(data: Path, max_verify_width: int = 16, target_is_moe: bool = False) -> dict:
    """What a calibration directory holds and what serve mode would take from it."""
    from eagle4_b200.core.chain_width import chain_widths, load_accept_profile, load_round_times, load_tree_rounds
    from eagle4_b200.core.chain_width import served_tree_schedule
    from eagle4_b200.core.cost_table import cost_model_problem, load_cost_tables
    from eagle4_b200.core.limits import ComputeIntensity, max_batch_size
    from eagle4_b200.core.live_costs import read_key

    data = Path(data)
    if not data.is_dir():
        raise OSError(f"{data} is not a directory")
    key = read_key(str(data))
    out: dict = {"data_path": str(data), "key": key.to_dict() if key else None}
    tables = load_cost_tables(str(data / "cost")) if (data / "cost").is_dir() else {}
    out["cost_tables"] = {
        str(b): {"contexts": [t.cache_length_start, t.cache_length_start + t.cache_length_step * t.max_interval_id],
                 "intervals": len(t.intervals), "problem": cost_model_problem(t, target_is_moe=target_is_moe)}
        for b, t in sorted(tables.items())}
    limit = max_batch_size(ComputeIntensity.CHAIN)
    profile = load_accept_profile(str(data))
    out["accept_profile"] = None if profile is None else {
        "max_width": profile.max_width, "expected_tokens": {w: round(profile.expected_tokens(w), 3)
                                                            for w in range(1, profile.max_width + 1)}}
    out["chain_round_times"] = sorted(load_round_times(str(data)) or {})
    out["chain_schedule"] = chain_widths(str(data), max_verify_width, limit, allow_no_spec=True) \
        if profile is not None else None
    rounds = load_tree_rounds(str(data))
    out["tree_rounds"] = sorted(rounds) if rounds else []
    out["tree_schedule"] = served_tree_schedule(rounds, max_verify_width, max_batch_size(ComputeIntensity.HIGH)) \
        if rounds else None
    out["profile"] = (data / "profile.json").is_file()
    return out


def _report_dir(args) -> int:
    rep = calibration_report(args.data, args.max_verify_width, args.moe_target)
    print(json.dumps(rep, indent=2))
    bad = [b for b, t in rep["cost_tables"].items() if t["problem"]]
    return 1 if bad else 0


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(prog="eagle4-b200", description="EAGLE-4 speculative decoding on B200.")
    sub = ap.add_subparsers(dest="command", required=True)
    cal = sub.add_parser("calibrate", formatter_class=argparse.ArgumentDefaultsHelpFormatter,
                         help="measure and fit cost tables for this GPU and model pair")
    cal.add_argument("--model", required=True, help="named synthetic shape (e.g. qwen3.8-27b) or target directory")
    cal.add_argument("--draft", help="draft checkpoint directory (named shapes bring their own draft)")
    cal.add_argument("--output", type=Path, help="fresh directory (default: ./eagle4-calibration)")
    cal.add_argument("--batch-sizes", type=_sizes, default=[1, 8])
    cal.add_argument("--context-step", type=_positive, default=256)
    cal.add_argument("--context-stop", type=_positive, default=4096)
    cal.add_argument("--repeats", type=_positive, default=10)
    cal.add_argument("--steps", type=_positive, default=12)
    cal.add_argument("--top-k", type=_positive, default=4)
    cal.add_argument("--draft-tokens", type=_positive, default=16)
    cal.add_argument("--kind", choices=("tree", "chain"), default="tree",
                     help="tree: cost tables from timed forwards; chain: served chain rounds and acceptance")
    cal.add_argument("--dry-run", action="store_true", help="print settings and the serving command only")
    cal.add_argument("--package", action="store_true",
                     help="also write profile.json so the directory can ship as a packaged cost profile")
    cal.add_argument("--tp", type=_positive, default=1,
                     help="tensor-parallel GPUs: one worker per GPU under torch.distributed.run, supervised")
    cal.add_argument("--timeout", type=float, help="seconds before a --tp calibration is stopped (default: none)")
    cal.add_argument("--worker", action="store_true", help=argparse.SUPPRESS)
    cal.set_defaults(func=_calibrate)
    pl = sub.add_parser("plan", formatter_class=argparse.ArgumentDefaultsHelpFormatter,
                        help="device memory of a serving configuration per GPU, and the KV tokens that fit")
    pl.add_argument("--model", required=True, help="named synthetic shape or target directory")
    pl.add_argument("--draft", help="draft checkpoint directory (named shapes bring their own draft)")
    pl.add_argument("--tp", type=_positive, default=1)
    pl.add_argument("--max-batch", type=_positive, default=8)
    pl.add_argument("--max-len", type=_positive, default=8192)
    pl.add_argument("--kv-tokens", type=_positive, help="KV token budget (default: every row at max-len)")
    pl.add_argument("--tree", default="12,4,16", help="steps,top_k,draft_tokens")
    pl.add_argument("--gpu-gb", type=float, help="memory budget per GPU in GB (default: a B200's)")
    pl.add_argument("--reserve-gb", type=float, default=4.0, help="decode activations, graph pools, buffers, context")
    pl.add_argument("--prefill-chunk", type=_positive, default=8192, help="the server's --prefill-chunk")
    pl.set_defaults(func=_plan)
    rep = sub.add_parser("report", formatter_class=argparse.ArgumentDefaultsHelpFormatter,
                         help="summarise a calibration directory: setup, tables, schedules, cost-model checks")
    rep.add_argument("data", type=Path, help="calibration directory (data_path)")
    rep.add_argument("--max-verify-width", type=_positive, default=16)
    rep.add_argument("--moe-target", action="store_true", help="check the tables as for a mixture-of-experts target")
    rep.set_defaults(func=_report_dir)
    chk = sub.add_parser("check", help="report the serving hosts and the native library")
    chk.add_argument("--kernels", action="store_true", help="also load the native CUDA library")
    chk.set_defaults(func=lambda a: __import__("eagle4_b200.compat", fromlist=["main"]).main(
        ["--kernels"] if a.kernels else []))
    args = ap.parse_args(argv)
    try:
        return args.func(args)
    except (ValueError, OSError, RuntimeError) as e:
        print(f"eagle4-b200: {e}", file=sys.stderr)
        return 1
    except KeyboardInterrupt:
        print("eagle4-b200: interrupted; partial measurements remain in the output directory.", file=sys.stderr)
        return 130


if __name__ == "__main__":
    raise SystemExit(main())
