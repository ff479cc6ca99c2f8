"""Per-phase GPU timing of the serving loop (CUDA events; NVTX ranges name the phases for profilers).

    python -m eagle4_b200.profile_decode [--model qwen3.8-27b] [--prompt 1024] [--rounds 8] [--eager]

Reports the prefill time, a plain-decode round and a speculative round (graph replays unless ``--eager``), and in
eager mode the split of a speculative round into draft extend, draft steps, verify forward and accept/commit.
"""

from __future__ import annotations

import argparse
import json

import torch


def _t(fn, n: int = 1) -> float:
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(n):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / n


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3.8-27b")
    ap.add_argument("--prompt", type=int, default=1024)
    ap.add_argument("--rounds", type=int, default=8)
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--only", choices=["plain", "spec"], default=None)
    args = ap.parse_args()
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    nvtx = torch.cuda.nvtx
    llm = LLM.synthetic(args.model, tree=TreeSpec(12, 4, 16), max_len=args.prompt + 64 * args.rounds + 128)
    eng = llm.engine
    eng.use_graphs = not args.eager
    prompt = torch.randint(0, llm.target.cfg.vocab_size, (args.prompt,))
    res = {}
    nvtx.range_push("prefill")
    res["prefill_ms"] = _t(lambda: eng.prefill(0, prompt))
    nvtx.range_pop()
    for kind in ("plain", "spec"):
        if args.only and kind != args.only:
            continue
        eng.prefill(0, prompt)
        run = (lambda: eng._spec_round(1, args.prompt)) if kind == "spec" else (lambda: eng._plain(1))
        run()  # first round: eager + capture
        nvtx.range_push(f"{kind}_round")
        res[f"{kind}_round_ms"] = _t(run, args.rounds)
        nvtx.range_pop()
    if args.eager and args.only != "plain":
        eng.prefill(0, prompt)
        eng._spec_round(1, args.prompt)
        parts = {}
        parts["draft_begin_ms"] = _t(lambda: eng._phase_begin(1))
        parts["draft_steps_ms"] = _t(lambda: [eng._phase_step(1, s) for s in range(1, eng.steps)])
        parts["verify_ms"] = _t(lambda: eng._phase_verify(1, eng.verify_tokens))
        res.update(parts)
    native.check_errors()
    print(json.dumps({k: round(v, 3) for k, v in res.items()}))


if __name__ == "__main__":
    main()
