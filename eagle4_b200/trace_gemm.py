"""Per-CTA timeline of one GEMM launch (globaltimer stamps), to see where a small GEMM's time goes.

    python -m eagle4_b200.trace_gemm --nk 5120 1536 --tokens 1

Prints, over the CTAs, the median and max of: setup (start -> barriers/TMEM ready), first stage landed, last MMA
issued, first accumulator ready in the epilogue, epilogue done and kernel end, all relative to the earliest CTA start.
"""

from __future__ import annotations

import argparse
import json

import torch


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--nk", type=int, nargs="+", default=[5120, 1536])
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--epi", type=int, default=1, help="0 plain, 1 residual")
    args = ap.parse_args()
    from eagle4_b200.ops import native

    dev = torch.device("cuda")
    for i in range(0, len(args.nk), 2):
        n, k = args.nk[i], args.nk[i + 1]
        w = (torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
        x = torch.randn(args.tokens, k, device=dev).to(torch.bfloat16)
        for _ in range(3):
            native._C.gemm_traced(x, w, args.epi)
        tr = native._C.gemm_traced(x, w, args.epi).cpu().double()
        t0 = tr[:, 0].min()
        rel = (tr - t0) / 1e3  # us
        names = ["start", "setup", "first_stage", "last_mma", "first_acc", "epi_done", "end", "last_atomic"]
        out = {"N": n, "K": k, "T": args.tokens, "ctas": tr.shape[0]}
        for j, nm in enumerate(names):
            col = rel[:, j]
            col = col[tr[:, j] > 0]
            if col.numel():
                out[nm] = [round(col.median().item(), 2), round(col.max().item(), 2)]
        slow = torch.argsort(rel[:, 5], descending=True)[:6].tolist()
        out["slowest"] = [[c] + [round(rel[c, j].item(), 2) for j in (2, 3, 4, 7, 5)] for c in slow]
        print(json.dumps(out))


if __name__ == "__main__":
    main()
