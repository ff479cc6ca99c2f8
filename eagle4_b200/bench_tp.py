"""Row-parallel projection timing under tensor parallelism (CUDA graphs of back-to-back calls, max over ranks).

    torchrun --nproc-per-node N -m eagle4_b200.bench_tp [--tokens 1 16 256 2048] [--calls 64]

For the Qwen3.8-27B shapes (o_proj/out_proj ``5120 x 6144/N`` and MLP down ``5120 x 17408/N`` per rank) it reports,
per call: the local GEMM + residual alone (``gemm``: no communication, the floor), the fused GEMM + all-reduce +
residual kernel (``fused``) and the NCCL path (``nccl``: bf16 GEMM, bf16 ``all_reduce``, residual), the bytes one
rank sends over NVLink per call (``nvlink_bytes``, against the all-reduce's algorithmic 2 (w-1)/w of the output:
``algo_bytes``), and the roofline of the fused op: the slower of its weight bytes at the measured HBM copy bandwidth
and its NVLink bytes at the measured 770 GB/s per direction.
"""

from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

HBM_GBS = 6548.2
LINK_GBS = 770.0


def graph_us(fn, calls: int, reps: int = 20) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(calls):
            fn()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) * 1e3 / (reps * calls)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, nargs="+", default=[1, 16, 256, 2048])
    ap.add_argument("--calls", type=int, default=64)
    args = ap.parse_args()
    from eagle4_b200 import ops
    from eagle4_b200.parallel.tp import TensorParallel, init_distributed

    rank, world = init_distributed()
    dev = torch.device("cuda", torch.cuda.current_device())
    fused = TensorParallel(backend="fused", max_rows=256, max_cols=8192, device=dev)
    nccl = TensorParallel(backend="torch", device=dev)
    H = 5120
    g = torch.Generator(device=dev).manual_seed(rank)
    rows = []
    for name, k_total in (("out_proj", 6144), ("down", 17408)):
        k = k_total // world
        w = (torch.randn(H, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        for t in args.tokens:
            x = torch.randn(t, k, generator=g, device=dev).to(torch.bfloat16)
            r = torch.randn(t, H, generator=g, device=dev).to(torch.bfloat16)
            calls = max(4, args.calls * 16 // max(16, t))
            res = {"shape": f"{H}x{k}", "op": name, "tokens": t, "world": world}
            res["gemm_us"] = graph_us(lambda: ops.linear_residual(x, w, r), calls)
            res["fused_us"] = graph_us(lambda: fused.row_linear(x, w, r), calls)
            res["nccl_us"] = graph_us(lambda: nccl.row_linear(x, w, r), calls)
            res["form"] = "one-shot" if t <= fused.two_shot_rows else "two-shot"
            res["nvlink_bytes"] = fused.nvlink_bytes(t, H)
            res["algo_bytes"] = int(2 * (world - 1) / world * t * H * 2)
            weight_us = w.numel() * 2 / (HBM_GBS * 1e3)
            link_us = res["nvlink_bytes"] / (LINK_GBS * 1e3)
            flop_us = 2.0 * t * H * k / (1369.3e12) * 1e6
            res["roofline_us"] = round(max(weight_us, link_us, flop_us), 3)
            res["fused_frac_of_roofline"] = round(res["roofline_us"] / res["fused_us"], 3)
            res["speedup_vs_nccl"] = round(res["nccl_us"] / res["fused_us"], 3)
            rows.append(res)
    # the greedy head: a vocabulary shard's GEMM + argmax, then the cross-rank (max, argmax) exchange
    lm = (torch.randn(248320 // max(world, 8), H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    for t in args.tokens:
        x = torch.randn(t, H, generator=g, device=dev).to(torch.bfloat16)
        res = {"op": "greedy_head", "shape": f"{lm.shape[0]}x{H}", "tokens": t, "world": world}
        res["local_us"] = graph_us(lambda: ops.lm_head_argmax(x, lm), args.calls)
        res["fused_us"] = graph_us(lambda: fused.lm_head_argmax(x, lm, 0), args.calls)
        res["nccl_us"] = graph_us(lambda: nccl.lm_head_argmax(x, lm, 0), args.calls)
        rows.append(res)
    torch.cuda.synchronize()
    fused.close()
    if rank == 0:
        for r in rows:
            print(json.dumps({k: (round(v, 3) if isinstance(v, float) else v) for k, v in r.items()}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
