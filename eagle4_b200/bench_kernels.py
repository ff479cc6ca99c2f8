"""Times the hot kernels at a model's shapes with CUDA events (warm-up first; the weights exceed L2 so every
launch streams them from HBM) and reports achieved bandwidth against the measured copy peak, plus an MD5 of each
kernel's output on seeded inputs, so two builds can be checked for bit-identical results.

    python -m eagle4_b200.bench_kernels [--tokens 1 16 64 256] [--only mlp_down ...] [--no-hash]
"""

from __future__ import annotations

import argparse
import itertools
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


def _peak_tflops() -> float:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def time_fn(fn, iters: int = 20, warmup: int = 3, graph: bool = True) -> float:
    """Mean device time of one ``fn`` call in microseconds. With ``graph`` the ``iters`` calls are captured in one
    CUDA graph and replayed, so host launch cost does not hide the device time of small kernels."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    if g is not None:
        g.replay()
    else:
        for _ in range(iters):
            fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3  # microseconds


def _md5(out) -> str:
    """MD5 of a kernel's output tensors (their bytes on the host, in order)."""
    import hashlib

    h = hashlib.md5()
    for t in (out if isinstance(out, (tuple, list)) else (out,)):
        h.update(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def fn_first(fn, copies, nxt):
    """``fn``'s output on the first weight copy (the cycle is advanced until it comes round)."""
    for _ in range(len(copies)):
        if next(nxt) is copies[-1]:
            break
    return fn()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="*", default=[1, 16, 64, 256])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", nargs="*", default=None, help="kernel names to run")
    ap.add_argument("--nk", type=int, nargs="*", default=None, help="extra plain GEMM shapes as N K pairs")
    ap.add_argument("--eager", action="store_true", help="time eager calls instead of one captured graph")
    ap.add_argument("--no-hash", action="store_true", help="skip the output MD5")
    args = ap.parse_args()
    torch.manual_seed(0)
    from eagle4_b200.ops import native

    peak = _peak_gbs()
    dev = torch.device("cuda")
    H, F, V = 5120, 17408, 248320
    shapes = {
        "gdn_in_proj": (16480, H), "gdn_out_proj": (H, 6144), "attn_qkv": (14336, H), "attn_o_proj": (H, 6144),
        "mlp_gate_up": (2 * F, H), "mlp_down": (H, F), "lm_head": (V, H), "draft_gate_up": (32768, H),
        "draft_qkv": (15360, 2 * H),
    }
    for i in range(0, len(args.nk or []), 2):
        shapes[f"gemm_{args.nk[i]}x{args.nk[i + 1]}"] = (args.nk[i], args.nk[i + 1])
    rows = []
    for name, (n, k) in shapes.items():
        if args.only is not None and name not in args.only:
            continue
        w0 = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
        # enough weight copies that consecutive calls never find their weights in the 126 MB L2
        copies = [w0] + [w0.clone() for _ in range(-(-256 * 2 ** 20 // (w0.numel() * 2)) - 1)]
        nxt = itertools.cycle(copies)
        for t in args.tokens:
            x = torch.randn(t, k, device=dev).to(torch.bfloat16)
            res = torch.randn(t, n, device=dev).to(torch.bfloat16)
            if name == "mlp_gate_up":
                fn = lambda: native.linear_swiglu(x, next(nxt))  # noqa: E731
            elif name == "lm_head":
                fn = lambda: native.lm_head_argmax(x, next(nxt))  # noqa: E731
            elif name in ("gdn_out_proj", "attn_o_proj", "mlp_down"):  # the block's output projection adds the residual
                fn = lambda: native.linear_residual(x, next(nxt), res)  # noqa: E731
            else:
                fn = lambda: native.linear(x, next(nxt))  # noqa: E731
            us = time_fn(fn, args.iters, args.warmup, not args.eager)
            digest = None if args.no_hash else _md5(fn_first(fn, copies, nxt))
            gbs = (n * k * 2 + t * k * 2 + t * n * 2) / (us * 1e-6) / 1e9
            tflops = 2.0 * n * k * t / (us * 1e-6) / 1e12
            rows.append({"kernel": name, "N": n, "K": k, "T": t, "us": round(us, 2), "GB/s": round(gbs, 1),
                         "frac_of_measured_hbm": round(gbs / peak, 3), "TFLOP/s": round(tflops, 1),
                         "frac_of_measured_bf16": round(tflops / _peak_tflops(), 3), "md5": digest})
            print(json.dumps(rows[-1]), flush=True)
        del w0, copies
    if not args.only or "attn_verify" in args.only:
        rows.extend(_bench_attention(native, args, peak))
    if not args.only or "gdn_verify" in args.only:
        rows.extend(_bench_gdn(native, args, peak))
    native.check_errors()


def _bench_attention(native, args, peak):
    """Tree-verify attention at the Qwen3.8-27B attention shape (24 q / 4 kv heads x 256) for one request with a
    1280-token context and a 16-row chain-shaped tree."""
    dev = torch.device("cuda")
    out = []
    hq, hk, d, page, L = 24, 4, 256, 16, 1280
    bt = torch.arange(96, dtype=torch.int32, device=dev).view(1, 96)
    kc = (torch.randn(96 * page, hk, d, device=dev) * 0.1).to(torch.bfloat16)
    vc = (torch.randn(96 * page, hk, d, device=dev) * 0.1).to(torch.bfloat16)
    for t in args.tokens:
        q = torch.randn(t, hq, d, device=dev).to(torch.bfloat16)
        req = torch.zeros(t, dtype=torch.int32, device=dev)
        cs = torch.zeros(t, dtype=torch.int32, device=dev)
        cl = torch.full((t,), L, dtype=torch.int32, device=dev)
        extra = (L + torch.arange(t, device=dev)).int()[None, :].expand(t, t).contiguous()
        ne = torch.arange(1, t + 1, dtype=torch.int32, device=dev)
        fn = lambda: native.attention(q, kc, vc, bt, page, req, cs, cl, extra, ne, d ** -0.5, max_keys=L + t)  # noqa
        us = time_fn(fn, args.iters, args.warmup, not args.eager)
        kv_bytes = (L + t) * hk * d * 2 * 2
        out.append({"kernel": "attn_verify", "T": t, "context": L, "us": round(us, 2),
                    "GB/s": round(kv_bytes / (us * 1e-6) / 1e9, 1)})
        print(json.dumps(out[-1]), flush=True)
    return out


def _bench_gdn(native, args, peak):
    """GDN tree recurrence at the Qwen3.8-27B shape (16 k / 48 v heads x 128) for one request whose rows form a
    chain (each row replays its path from the committed state)."""
    from eagle4_b200.models.configs import qwen38_27b

    cfg = qwen38_27b()
    dev = torch.device("cuda")
    out = []
    state = torch.randn(1, cfg.gdn_v_heads, cfg.gdn_v_dim, cfg.gdn_k_dim, device=dev) * 0.01
    a_log = torch.rand(cfg.gdn_v_heads, device=dev).log1p()
    dt_bias = torch.ones(cfg.gdn_v_heads, device=dev)
    gnorm = torch.ones(cfg.gdn_v_dim, dtype=torch.bfloat16, device=dev)
    for t in args.tokens:
        conv = torch.randn(t, cfg.gdn_conv_dim, device=dev).to(torch.bfloat16)
        proj = torch.randn(t, cfg.gdn_conv_dim + cfg.gdn_value_dim + 2 * cfg.gdn_v_heads, device=dev).to(torch.bfloat16)
        slot = torch.zeros(t, dtype=torch.int32, device=dev)
        parent = (torch.arange(t, device=dev) - 1).int()
        fn = lambda: native.gdn_mixer(conv, proj, cfg, a_log, dt_bias, gnorm, state, slot, parent, False)  # noqa
        us = time_fn(fn, args.iters, args.warmup, not args.eager)
        out.append({"kernel": "gdn_verify", "T": t, "us": round(us, 2),
                    "state_GB/s": round(state.numel() * 4 * t / (us * 1e-6) / 1e9, 1)})
        print(json.dumps(out[-1]), flush=True)
    return out


if __name__ == "__main__":
    main()
