"""Warm prefill timing of a named model: one request's prompt through the target and the draft (CUDA events).

    python -m eagle4_b200.profile_prefill [--model qwen3.8-27b] [--prompt 1024] [--warmup 1] [--repeats 3]

Prints one JSON line: the mean warm prefill time and its throughput in tokens/s and TFLOP/s (2 FLOPs per weight per
token of the target's projections, the attention FLOPs not counted). Under a one-pass ncu launch list
(``--metrics gpu__time_duration.sum``) the launches of the timed prefills come after the ``--warmup`` ones; an NVTX
range ``prefill_timed`` marks them.
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser(prog="eagle4_b200.profile_prefill")
    ap.add_argument("--model", default="qwen3.8-27b")
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--repeats", type=int, default=3)
    args = ap.parse_args()
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    llm = LLM.synthetic(args.model, tree=TreeSpec(12, 4, 16), max_len=args.prompt + 128)
    eng = llm.engine
    prompt = torch.randint(0, llm.target.cfg.vocab_size, (args.prompt,))
    for _ in range(args.warmup):
        eng.prefill(0, prompt)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("prefill_timed")
    s.record()
    for _ in range(args.repeats):
        eng.prefill(0, prompt)
    e.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.repeats
    proj = sum(w.numel() for k, w in llm.target.w.items() if k.startswith("l") and w.dim() == 2
               and not k.endswith("conv"))
    native.check_errors()
    print(json.dumps({"model": args.model, "prompt": args.prompt, "prefill_ms": round(ms, 2),
                      "tokens_per_s": round(args.prompt / ms * 1e3, 1),
                      "proj_tflops": round(2 * proj * args.prompt / ms / 1e9, 1)}))


if __name__ == "__main__":
    main()
