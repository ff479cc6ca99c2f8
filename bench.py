#!/usr/bin/env python
"""Headline benchmark: EAGLE-4 output tokens/s and speedup over plain decoding.

Config (the benchmark plan's config 2): a Qwen3.8-27B-shaped hybrid target (64 layers, 3 GDN : 1 gated attention,
hidden 5120, vocab 248320) in bf16 with random-init weights, a one-layer EAGLE-4 draft head (H 5120, 40x128 heads,
FFN 16384, rank-128 candidate head), tree steps 12 / top-k 4 / 16 draft tokens, batch 1 per GPU, a 1024-token
uniform-random prompt and 256 greedy output tokens. One step = one whole generation (prefill + 256 tokens).

  python bench.py --gpus N --steps K --warmup W            # this framework
  python bench.py --impl reference ...                     # the reference's own serving path

With N > 1 (launched by torch.distributed.run) the ranks serve one batch together with tensor parallelism (TP = N,
strong scaling; ``--parallelism dp`` runs data-parallel replicas instead). The tensor-parallel collectives are the
fused peer-memory kernels (``--tp-backend torch`` measures the NCCL all-reduce baseline). The device time is the max
over ranks. Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

MODEL_NAMES = {
    "qwen3.8-27b": "Qwen3.8-27B-shaped hybrid (64 layers, 3 GDN:1 attention) + 1-layer EAGLE-4 draft",
    "nemotron-h-8b": "Nemotron-H-style Mamba2/attention hybrid (52 layers) + 1-layer EAGLE-4 draft",
    "llama-3.1-8b": "Llama-3.1-8B-shaped dense target + 1-layer EAGLE-3 draft (32000-token draft vocabulary)",
}
BASELINE_TPS = 302.7  # SGLang TP1, one request, EAGLE-4 tokens/s on 1x B300 (reference docs/support-matrix.md:258-259)
METRIC = "EAGLE-4 output tok/s and speedup vs plain decode, batch 1–512, TP 1/2/4/8"


REF_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")


def _version(module: str):
    """``(installed version or None, import error or None)`` of an engine module, without importing it twice."""
    import importlib
    import importlib.metadata as md

    try:
        mod = importlib.import_module(module)
    except Exception as e:  # noqa: BLE001 - any import failure means the engine cannot serve here
        return None, f"{type(e).__name__}: {e}"[:120]
    try:
        return md.version(module), None
    except md.PackageNotFoundError:
        return getattr(mod, "__version__", "unknown"), None


def reference_probe() -> dict:
    """What the reference's own serving path needs, checked on this machine: the unmodified reference package from
    ``baseline/_ref`` (imported through its public API) and the engines it plugs into (its ``pyproject.toml`` names
    hook-carrying SGLang, TokenSpeed, or vLLM >= 0.32). Returns the findings and, when it cannot generate, why."""
    found = {"baseline_ref": os.path.isdir(REF_DIR)}
    if found["baseline_ref"] and REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        import eagle_harness  # noqa: F401
        from eagle_harness.core.config import parse_harness_config

        parse_harness_config('{"mode": "serve"}')  # the reference's public config entry point works
        import importlib.metadata as md

        try:
            found["eagle_harness"] = md.version("eagle-harness")
        except md.PackageNotFoundError:
            found["eagle_harness"] = "imported"
        found["eagle_harness_path"] = os.path.dirname(eagle_harness.__file__)
    except Exception as e:  # noqa: BLE001
        found["eagle_harness"] = None
        found["eagle_harness_error"] = f"{type(e).__name__}: {e}"[:160]
    engines = {}
    for mod in ("sglang", "vllm", "tokenspeed"):
        ver, err = _version(mod)
        engines[mod] = ver if ver else f"missing ({err})"
    found["engines"] = engines
    usable = []
    if not engines["sglang"].startswith("missing"):
        usable.append("sglang")
    if not engines["tokenspeed"].startswith("missing"):
        usable.append("tokenspeed")
    ver = engines["vllm"]
    if not ver.startswith("missing"):
        try:
            major, minor = (int(x) for x in ver.split(".")[:2])
            if (major, minor) >= (0, 32):
                usable.append("vllm")
        except ValueError:
            pass
    found["usable_engines"] = usable
    if found["eagle_harness"] is None:
        found["unavailable"] = "the reference package does not import from baseline/_ref: " + found[
            "eagle_harness_error"]
    elif not usable:
        found["unavailable"] = (
            "eagle-harness imports (" + str(found["eagle_harness"]) + ") but is an engine plugin: generating needs "
            "hook-carrying SGLang or TokenSpeed, or vLLM>=0.32; found " +
            ", ".join(f"{k} {v}" for k, v in engines.items()) + ", so it cannot generate on this box")
    return found


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                self.rows.append([x.strip() for x in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self) -> dict:
        mhz = sorted(float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit())
        mx = max((float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9 for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(mhz)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="qwen3.8-27b")
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--new-tokens", type=int, default=256)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-plain", action="store_true", help="skip the plain-decode arm")
    ap.add_argument("--tree", default="12,4,16", help="steps,top_k,draft_tokens")
    ap.add_argument("--temperature", type=float, default=0.0, help="> 0: sampled trees (tree rejection)")
    ap.add_argument("--parallelism", default="tp", choices=["tp", "dp"])
    ap.add_argument("--tp-backend", default="fused", choices=["fused", "torch"])
    ap.add_argument("--mode", default="serve", choices=["serve", "static"],
                    help="serve: live-cost model sizes each round (default); static: the full 12/4/16 tree")
    ap.add_argument("--sweep", default=None,
                    help="concurrency sweep (benchmark config 3): comma-separated batch sizes, one JSON line each")
    ap.add_argument("--prompt-range", default="256,4096", help="sweep prompt lengths, uniform in [lo, hi]")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        found = reference_probe()
        if rank == 0:
            if "unavailable" in found:
                print(json.dumps({"impl": "reference", "unavailable": found.pop("unavailable"), "probe": found}))
            else:  # an engine with the hooks is installed: its serving path is not wired into this bench
                print(json.dumps({"impl": "reference", "unavailable": "a hook-carrying engine is installed ("
                                  + ", ".join(found["usable_engines"]) + ") but this bench has no launcher for it",
                                  "probe": found}))
        return

    import torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    dev = torch.device("cuda", local)
    tp = None
    tp_mode = world > 1 and args.parallelism == "tp"
    if tp_mode:
        from eagle4_b200.parallel.tp import TensorParallel

        tp = TensorParallel(backend=args.tp_backend, max_rows=max(256, args.prompt), max_cols=8192, device=dev)
    replicas = 1 if tp_mode else world  # independent request streams
    tree = TreeSpec(*(int(v) for v in args.tree.split(",")))
    if args.sweep:
        sweep(args, tree, tp, dev, rank, world, dist)
        return
    llm = LLM.synthetic(args.model, device=dev, seed=0, tree=tree, max_batch=args.batch,
                        max_len=args.prompt + args.new_tokens + 64, config=json.dumps({"mode": args.mode}), tp=tp,
                        temperature=args.temperature, sample_seed=7)
    gen = torch.Generator().manual_seed(1234 + (0 if tp_mode else rank))
    prompts = torch.randint(0, llm.target.cfg.vocab_size, (args.batch, args.prompt), generator=gen).pin_memory()
    eng = llm.engine
    if tp_mode:  # a crashed or hung rank is named between rounds, before the next round's collectives
        from eagle4_b200.parallel.health import process_group_heartbeat

        eng.heartbeat = process_group_heartbeat()

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def device_timed(speculative: bool):
        dev_prompts = prompts.to(dev)
        for _ in range(args.warmup):
            eng.generate(dev_prompts, args.new_tokens, speculative=speculative)
        barrier()
        torch.cuda.synchronize()
        eng.stats.__init__()
        if getattr(eng, "tree_choice", None) is not None:
            eng.tree_choice.served.clear()  # the share below counts the timed rounds only
        native.LAUNCHES[0] = 0
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            s.record()
            outs = [eng.generate(dev_prompts, args.new_tokens, speculative=speculative) for _ in range(args.steps)]
            e.record()
            torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(s.elapsed_time(e))
        toks = sum(len(o) for out in outs for o in out)
        return ms, toks, clk.summary(), native.LAUNCHES[0], eng.stats.mean_accept, outs

    spec_ms, spec_tok, clocks, launches, accept, spec_out = device_timed(True)
    plain_ms = plain_tok = None
    if not args.no_plain:
        plain_ms, plain_tok, _, _, _, plain_out = device_timed(False)
        same = plain_out[0] == spec_out[0] if args.temperature == 0 else None  # sampled: distributions, not ids
    else:
        same = None

    # end to end through the public API: pinned prompt H2D and generated ids D2H inside the timed region
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_tok = 0
    for _ in range(args.steps):
        out = llm.generate(prompts, args.new_tokens, speculative=True)
        e2e_tok += out.numel()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    native.check_errors(dev)

    total_tok = spec_tok * replicas
    value = total_tok / (spec_ms / 1e3)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(spec_ms / args.steps, 3),
        "higher_is_better": True,
        # tensor parallelism splits the same batch over the GPUs (N = 1 included: total work fixed); data-parallel
        # replicas each serve their own batch
        "scaling": "weak" if args.parallelism == "dp" and world > 1 else "strong",
        "vs_baseline": round(value / BASELINE_TPS, 4),
        "dtype": "bf16",
        "data": "synthetic: uniform-random prompt ids, random-init N(0,0.02) weights of the named shapes",
        "config": {
            "model": MODEL_NAMES.get(args.model, args.model),
            "temperature": args.temperature,
            "global_batch": args.batch * replicas, "seq_len": args.prompt, "new_tokens": args.new_tokens,
            "tree": {"steps": tree.steps, "top_k": tree.top_k, "draft_tokens": tree.draft_tokens,
                     "mode": args.mode, "last_round_depth": eng.last_depth, "last_round_width": eng.last_width},
            "parallelism": f"tp{world}" if tp_mode else (f"dp{world}" if world > 1 else "tp1"),
            "tp_collectives": (args.tp_backend if tp_mode else None),
            "l2": "inputs larger than L2: every forward streams the 54 GB of target weights",
        },
        "speculative_tok_s": round(value, 2),
        "plain_tok_s": round(plain_tok * replicas / (plain_ms / 1e3), 2) if plain_ms else None,
        "speedup_vs_plain": round((spec_tok / spec_ms) / (plain_tok / plain_ms), 4) if plain_ms else None,
        "mean_accepted_per_round": round(accept, 3),
        "served_choice": ({"native_round_share": round(eng.tree_choice.share(eng.tree_choice.NATIVE), 3),
            "rule": "per batch bucket: speculate or decode natively, whichever served more tokens per us "
                    "(settled rounds only: no eager run or graph capture inside the period)"}
            if getattr(eng, "tree_choice", None) is not None else None),
        "spec_equals_plain": same,
        "clocks": clocks,
        "e2e": {"value": round(e2e_tok * replicas / e2e_s, 2), "unit": "tokens/s",
                "h2d_bytes_per_step": int(prompts.numel() * prompts.element_size()),
                "d2h_bytes_per_step": int(args.batch * args.new_tokens * 8)},
        "gpu_launches": launches,
    }
    if rank == 0:
        print(json.dumps(line))
    eng.graphs.clear()  # graphs may hold NCCL calls (torch backend): release them before the group goes
    torch.cuda.synchronize()
    if tp is not None:
        tp.close()
    if dist is not None:
        dist.destroy_process_group()


def sweep(args, tree, tp, dev, rank: int, world: int, dist) -> None:
    """Benchmark config 3: at each batch size, prompts of uniform-random lengths in ``--prompt-range`` and
    ``--new-tokens`` greedy tokens, speculative (serve mode) and plain decoding. Prints one JSON line per batch size:
    decode tokens/s (device time of the rounds, max over ranks), the prefill time, and end-to-end tokens/s."""
    import torch

    from eagle4_b200.api import LLM

    sizes = [int(v) for v in args.sweep.split(",")]
    lo, hi = (int(v) for v in args.prompt_range.split(","))
    gen = torch.Generator().manual_seed(4321)
    plans = {b: [torch.randint(0, 1 << 30, (int(n),), generator=gen)
                 for n in torch.randint(lo, hi + 1, (b,), generator=gen)] for b in sizes}
    span = max(tree.draft_tokens, tree.steps * tree.top_k) + 1

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for b in sizes:
        line = {"metric": METRIC, "impl": "ours", "n_gpus": world, "batch": b, "dtype": "bf16",
                "data": "synthetic: uniform-random prompt ids, random-init N(0,0.02) weights of the named shapes",
                "config": {"model": MODEL_NAMES.get(args.model, args.model), "global_batch": b,
                           "prompt_range": [lo, hi], "new_tokens": args.new_tokens,
                           "parallelism": f"tp{world}" if tp is not None else "tp1",
                           "tree": {"steps": tree.steps, "top_k": tree.top_k, "draft_tokens": tree.draft_tokens,
                                    "mode": args.mode}}}
        try:
            kv = sum(-(-(int(p.shape[0]) + args.new_tokens + span) // 16) * 16 for p in plans[b])  # whole pages
            llm = LLM.synthetic(args.model, device=dev, seed=0, tree=tree, max_batch=b,
                                max_len=hi + args.new_tokens + 64, config=json.dumps({"mode": args.mode}), tp=tp,
                                kv_tokens=kv)
            prompts = [(p % llm.target.cfg.vocab_size).pin_memory() for p in plans[b]]
            eng = llm.engine
            res = {}
            for kind, spec in (("speculative", True), ("plain", False)):
                for _ in range(max(1, min(args.warmup, 1))):  # graph capture and the served choice's exploration
                    llm.generate(prompts, args.new_tokens, speculative=spec)
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                out = llm.generate(prompts, args.new_tokens, speculative=spec)
                torch.cuda.synchronize()
                e2e = max_over_ranks(time.perf_counter() - t0)
                dec = max_over_ranks(eng.last_timing["decode_ms"])
                pre = max_over_ranks(eng.last_timing["prefill_ms"])
                toks = out.numel()
                res[kind] = {"decode_tok_s": round(toks / (dec / 1e3), 2), "prefill_ms": round(pre, 1),
                             "e2e_tok_s": round(toks / e2e, 2)}
            line.update({"value": res["speculative"]["decode_tok_s"], "unit": "tokens/s (decode rounds)",
                         "speculative": res["speculative"], "plain": res["plain"],
                         "speedup_vs_plain": round(res["speculative"]["decode_tok_s"]
                                                   / res["plain"]["decode_tok_s"], 4),
                         "verify_batch_limit": eng.verify_batch_limit,
                         "native_round_share": (round(eng.tree_choice.share(eng.tree_choice.NATIVE), 3)
                                                if eng.tree_choice is not None else None)})
            eng.graphs.clear()
            del llm, eng
        except torch.cuda.OutOfMemoryError as e:
            line["skipped"] = f"out of device memory at this batch and TP size ({str(e).splitlines()[0][:120]})"
        torch.cuda.empty_cache()
        if rank == 0:
            print(json.dumps(line), flush=True)
    if tp is not None:
        torch.cuda.synchronize()
        tp.close()
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
