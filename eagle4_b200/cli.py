"""Command line: ``python -m eagle4_b200.cli calibrate|check`` (console script ``eagle4-b200``).

``calibrate`` measures this package's engine on the local GPU (target verify forwards and draft steps over a context
sweep, one CUDA graph per timed shape), fits the cost tables into a fresh directory and prints the serving config
that uses them (reference ``eagle_harness/cli.py:268-345``, which drives an SGLang or vLLM server instead; the
settings and output layout are the same: ``settings.json``, the calibration ``data_path`` and ``serve.sh``).
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
              config=None, tp=None, dtype=None):
    """A named synthetic shape (random weights) or a checkpoint directory pair; ``tp``: this rank's
    :class:`~eagle4_b200.parallel.tp.TensorParallel` (the weights are sharded over its group)."""
    import torch

    from eagle4_b200.api import LLM, NAMED, from_pretrained

    dtype = dtype or torch.bfloat16
    if model in NAMED:
        return LLM.synthetic(model, device=device, tree=tree, max_batch=max_batch, max_len=max_len, config=config,
                             tp=tp, dtype=dtype)
    return from_pretrained(model, draft, device=device, tree=tree, max_batch=max_batch, max_len=max_len,
                           config=config, tp=tp, dtype=dtype)


def serve_config(output: Path) -> dict:
    return {"mode": "serve", "data_path": str(output)}


def _calibrate(args) -> int:
    import torch

    from eagle4_b200.api import TreeSpec
    from eagle4_b200.core.live_costs import CostKey
    from eagle4_b200.runtime.calibrate import calibrate

    if not torch.cuda.is_available() and not args.dry_run:
        raise RuntimeError("calibration times the GPU; no CUDA device is visible")
    args.output = (args.output or Path("eagle4-calibration")).resolve()
    settings = {k: str(v) if isinstance(v, Path) else v for k, v in vars(args).items() if k != "func"}
    command = f"python -m eagle4_b200.serve --model {shlex.quote(args.model)}" + (
        f" --draft {shlex.quote(args.draft)}" if args.draft else "") + \
        f" --config {shlex.quote(json.dumps(serve_config(args.output)))}"
    if args.dry_run:
        print(json.dumps(settings, indent=2))
        print(command)
        return 0
    args.output.mkdir(parents=True, exist_ok=False)
    (args.output / "settings.json").write_text(json.dumps(settings, indent=2) + "\n")
    tree = TreeSpec(args.steps, 1 if args.kind == "chain" else args.top_k, args.draft_tokens)
    llm = build_llm(args.model, args.draft, max_batch=max(args.batch_sizes), max_len=args.context_stop + 256,
                    tree=tree)
    key = CostKey(gpu=torch.cuda.get_device_name(), gpu_count=1, model=args.model, draft=str(args.draft or ""),
                  engine="eagle4_b200", dtype="bfloat16")
    if args.kind == "chain":
        from eagle4_b200.runtime.calibrate import calibrate_chain

        calibrate_chain(llm.engine, str(args.output), batch_sizes=args.batch_sizes, key=key)
        problems = {}
    else:
        problems = calibrate(llm.engine, str(args.output), batch_sizes=args.batch_sizes,
                             context_step=args.context_step, context_stop=args.context_stop, repeats=args.repeats,
                             key=key)
    if args.package:
        from eagle4_b200.core.cost_profiles import write_profile

        # the directory doubles as a packaged profile: matched by device, TP size and the models' shapes
        write_profile(str(args.output), devices=[torch.cuda.get_device_name()], tp_size=1,
                      target_config=llm.target.cfg.to_hf(), draft_config=llm.draft.cfg.to_hf())
    bad = {b: p for b, p in problems.items() if p}
    for b, p in bad.items():
        print(f"batch size {b}: the cost model refuses these costs ({p}); rounds there keep the fixed shape")
    (args.output / "serve.sh").write_text("#!/bin/sh\nset -eu\nexec " + command + "\n")
    print(f"Calibration saved in {args.output}. Serve with:\nsh {shlex.quote(str(args.output / 'serve.sh'))}")
    return 0


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
    cal.set_defaults(func=_calibrate)
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
