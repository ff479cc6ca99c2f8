"""Times the hot kernels at a model's shapes with CUDA events (warm-up first; the weights exceed L2 so every
launch streams them from HBM) and reports achieved bandwidth against the measured copy peak.

    python -m eagle4_b200.bench_kernels [--model qwen3.8-27b] [--tokens 1 16 64]
"""

from __future__ import annotations

import argparse
import json
import os

import torch


def _peak_gbs() -> float:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def time_fn(fn, iters: int = 20, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3  # microseconds


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="*", default=[1, 16, 64, 256])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", nargs="*", default=None, help="kernel names to run")
    args = ap.parse_args()
    from eagle4_b200.ops import native

    peak = _peak_gbs()
    dev = torch.device("cuda")
    H, F, V = 5120, 17408, 248320
    shapes = {
        "gdn_in_proj": (16480, H), "gdn_out_proj": (H, 6144), "attn_qkv": (14336, H), "attn_o_proj": (H, 6144),
        "mlp_gate_up": (2 * F, H), "mlp_down": (H, F), "lm_head": (V, H), "draft_gate_up": (32768, H),
        "draft_qkv": (15360, 2 * H),
    }
    rows = []
    for name, (n, k) in shapes.items():
        if args.only and name not in args.only:
            continue
        w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
        for t in args.tokens:
            x = torch.randn(t, k, device=dev).to(torch.bfloat16)
            if name == "mlp_gate_up":
                fn = lambda: native.linear_swiglu(x, w)  # noqa: E731
            elif name == "lm_head":
                fn = lambda: native.lm_head_argmax(x, w)  # noqa: E731
            else:
                fn = lambda: native.linear(x, w)  # noqa: E731
            us = time_fn(fn, args.iters, args.warmup)
            gbs = (n * k * 2 + t * k * 2 + t * n * 2) / (us * 1e-6) / 1e9
            rows.append({"kernel": name, "N": n, "K": k, "T": t, "us": round(us, 2), "GB/s": round(gbs, 1),
                         "frac_of_measured_hbm": round(gbs / peak, 3)})
            print(json.dumps(rows[-1]), flush=True)
        del w
    native.check_errors()


if __name__ == "__main__":
    main()
