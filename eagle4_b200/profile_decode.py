"""Per-phase GPU timing of the serving loop (CUDA events; NVTX ranges name the phases for profilers).

    python -m eagle4_b200.profile_decode [--model qwen3.8-27b] [--prompt 1024] [--rounds 8] [--eager]
    torchrun --nproc-per-node N -m eagle4_b200.profile_decode --tp-backend fused|torch   # tensor parallel

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
    ap.add_argument("--tp-backend", default="fused", choices=["fused", "torch"])
    ap.add_argument("--row-linear", action="store_true", help="also time one row-parallel projection per shape")
    args = ap.parse_args()
    import os

    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    tp = None
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        from eagle4_b200.parallel.tp import TensorParallel, init_distributed

        init_distributed()
        tp = TensorParallel(backend=args.tp_backend, max_rows=max(256, args.prompt))
    nvtx = torch.cuda.nvtx
    llm = LLM.synthetic(args.model, tree=TreeSpec(12, 4, 16), max_len=args.prompt + 64 * args.rounds + 128, tp=tp)
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
    if args.row_linear:
        from eagle4_b200 import ops

        h = llm.target.cfg.hidden_size
        for t in (1, 16):
            for name in ("l0.out_proj", "l0.down"):
                w = llm.target.w[name]
                x = torch.randn(t, w.shape[1], device=w.device).to(w.dtype)
                r = torch.randn(t, h, device=w.device).to(w.dtype)
                nw = llm.target.w["l0.norm2"]
                if tp is not None:
                    res[f"row_{name}_t{t}_us"] = 1e3 * _t(lambda: tp.row_linear(x, w, r, nw), 200)
                res[f"gemm_{name}_t{t}_us"] = 1e3 * _t(lambda: ops.linear_residual(x, w, r), 200)
    native.check_errors()
    if tp is not None:
        import torch.distributed as dist

        keys = sorted(res)
        t = torch.tensor([res[k] for k in keys], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res = dict(zip(keys, t.tolist()))
        res["world"] = world
        llm.engine.graphs.clear()
        torch.cuda.synchronize()
        tp.close()
        if dist.get_rank() != 0:
            return
    print(json.dumps({k: round(v, 3) for k, v in res.items()}))


if __name__ == "__main__":
    main()
