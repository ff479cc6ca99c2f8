"""Kernel-level comparison with the reference's own kernels, run unmodified from ``baseline/_ref`` on this GPU.

    python -m eagle4_b200.bench_reference [--bs 1 8 64] [--iters 20]

The reference cannot serve end to end here (it is an engine plugin), but its kernels are Triton programs that run
on a B200 as they are. For each op this times the reference's launch and this package's sm_100a kernel on the same
shapes (Qwen3.8-27B: K=4 draft tree of depth 12 over 5120-wide hidden states, GDN 16 key / 48 value heads x 128;
Nemotron-H: Mamba2 128 heads x 64, state 128), both captured in one CUDA graph of ``iters`` calls and timed with
CUDA events after warm-up, and prints one JSON line per op with both times and ``speedup`` (reference / ours).

Where the two designs split the work differently the rows say so: the reference's GDN and Mamba2 tree updates store
a state snapshot per tree node, which its commit then copies, while this package's tree pass walks the tree's chains
without stores and its commit replays the accepted path; so those rows time update + commit on both sides (the
reference's commit as the copy of the accepted node's snapshot).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def graph_us(fn, iters: int) -> float:
    """Mean device time of one ``fn`` call (microseconds), from one CUDA graph of ``iters`` calls."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(5):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / (5 * iters)


def _reference():
    if not os.path.isdir(os.path.join(REF, "eagle_harness")):
        raise SystemExit("the reference is not installed under baseline/_ref")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import eagle_harness.core.draft_tree as rdt
    import eagle_harness.kernels.accept_tail as racc
    import eagle_harness.kernels.gdn_tree_recurrence as rgdn
    import eagle_harness.kernels.mamba2_tree as rmamba

    return rdt, rgdn, rmamba, racc


def bench_tree(rdt, bs: int, iters: int) -> dict:
    """One draft-tree step (expand the frontier, keep the best K, best-set work deltas) and the verify selection."""
    from eagle4_b200.core.draft_tree import DraftTree, TreeShape

    dev = torch.device("cuda")
    k, depth, hid = 4, 12, 5120
    g = torch.Generator(device=dev).manual_seed(bs)
    ref = rdt.DraftTree(rdt.TreeShape(k, depth), bs, hid, torch.bfloat16, dev, max_verify=16)
    ours = DraftTree(TreeShape(k, depth), bs, hid, torch.bfloat16, dev, max_verify=16)
    p0 = torch.rand(bs, k, generator=g, device=dev)
    t0 = torch.randint(0, 248320, (bs, k), generator=g, device=dev)
    h0 = torch.randn(bs, hid, generator=g, device=dev).to(torch.bfloat16)
    steps = []
    for _ in range(1, depth):
        steps.append((torch.rand(bs * k, k, generator=g, device=dev),
                      torch.randint(0, 248320, (bs * k, k), generator=g, device=dev),
                      torch.randn(bs * k, hid, generator=g, device=dev).to(torch.bfloat16)))
    for t in (ref, ours):
        t.stage_root(bs, p0, t0, h0)
        t.begin(bs)
        for s, (p, tk, hh) in enumerate(steps, start=1):
            t.step(bs, s, p, tk, hh)
    same = bool(torch.equal(ref.scores, ours.scores) and torch.equal(ref.tokens, ours.tokens)
                and torch.equal(ref.parents, ours.parents))
    mid = depth // 2
    p, tk, hh = steps[mid - 1]
    out = {"op": "tree_step", "bs": bs, "top_k": k, "depth": depth, "same_tree": same,
           "reference_us": graph_us(lambda: ref.step(bs, mid, p, tk, hh), iters),
           "ours_us": graph_us(lambda: ours.step(bs, mid, p, tk, hh), iters)}
    out["speedup"] = out["reference_us"] / out["ours_us"]
    sel = {"op": "tree_verify_rows", "bs": bs, "count": 15,
           "reference_us": graph_us(lambda: ref.verify_rows(bs, depth, 15), iters),
           "ours_us": graph_us(lambda: ours.verify_rows(bs, depth, 15), iters)}
    sel["speedup"] = sel["reference_us"] / sel["ours_us"]
    return [out, sel]


def _chain_tree(t: int):
    """Parent rows of a 16-node verify tree: a chain of 8 with two side branches (row 0 the root)."""
    parent = [-1] + list(range(0, 7)) + [1, 8, 9, 3, 11, 12, 5, 14]
    return parent[:t]


def bench_gdn(rgdn, iters: int, t: int = 16) -> dict:
    from eagle4_b200.models.configs import qwen38_27b
    from eagle4_b200.ops import native

    cfg = qwen38_27b()
    dev = torch.device("cuda")
    H, HV, K, V = cfg.gdn_k_heads, cfg.gdn_v_heads, cfg.gdn_k_dim, cfg.gdn_v_dim
    g = torch.Generator(device=dev).manual_seed(0)
    bf = lambda *s: torch.randn(*s, generator=g, device=dev).to(torch.bfloat16)  # noqa: E731
    q, k, v = bf(1, t, H, K), bf(1, t, H, K), bf(1, t, HV, V)
    a, b = bf(t, HV), bf(t, HV)
    a_log = torch.rand(HV, device=dev).log1p()
    dt_bias = torch.ones(HV, device=dev)
    pool = torch.randn(2, HV, V, K, device=dev) * 0.01
    snaps = torch.zeros(1, t, HV, V, K, device=dev)
    parents = torch.tensor([_chain_tree(t)], dtype=torch.int32, device=dev)
    idx = torch.zeros(1, dtype=torch.int32, device=dev)
    cu = torch.tensor([0, t], dtype=torch.int32, device=dev)
    out_ref = torch.empty_like(v)

    def ref_call():
        rgdn.gdn_tree_recurrent_update(a_log, dt_bias, q, k, v, a, b, initial_state_source=pool,
                                       initial_state_indices=idx, cu_seqlens=cu, intermediate_states_buffer=snaps,
                                       intermediate_state_indices=idx, retrieve_parent_token=parents, out=out_ref)

    conv = torch.cat([q.view(t, -1), k.view(t, -1), v.view(t, -1)], dim=1).contiguous()
    proj = torch.cat([conv, bf(t, HV * V), b, a], dim=1).contiguous()
    gnorm = torch.ones(V, dtype=torch.bfloat16, device=dev)
    slot = torch.zeros(t, dtype=torch.int32, device=dev)
    par = parents[0].clone()
    rows = torch.tensor([[0, 1, 2, 3]], dtype=torch.int32, device=dev)
    nrows = torch.tensor([4], dtype=torch.int32, device=dev)
    slots = torch.zeros(1, dtype=torch.int64, device=dev)
    cst = torch.zeros(2, cfg.gdn_conv_dim, cfg.conv_kernel - 1, dtype=torch.bfloat16, device=dev)
    st_ours = pool.clone()

    def ours_call():
        native.gdn_mixer(conv, proj, cfg, a_log, dt_bias, gnorm, st_ours, slot, par, False)

    def ours_commit():
        native.gdn_commit_all([conv], [proj], [st_ours], [cst], [a_log], [dt_bias], slots, rows, nrows, cfg)

    def ref_commit():  # the accepted node's snapshot becomes the request's state
        pool[0].copy_(snaps[0, 3])

    r = {"op": "gdn_tree_verify", "rows": t, "heads": f"{H}k/{HV}v x {K}",
         "reference_us": graph_us(ref_call, iters), "reference_commit_us": graph_us(ref_commit, iters),
         "ours_us": graph_us(ours_call, iters), "ours_commit_us": graph_us(ours_commit, iters),
         "note": "reference: tree update storing a state snapshot per node, commit = copy of the accepted node's "
                 "snapshot; ours: chain-walk tree pass (gates and gated RMSNorm fused), commit = replay of the "
                 "4-row accepted path"}
    r["speedup"] = (r["reference_us"] + r["reference_commit_us"]) / (r["ours_us"] + r["ours_commit_us"])
    return r


def bench_mamba(rmamba, iters: int, t: int = 16) -> dict:
    from eagle4_b200.models.configs import nemotron_h_8b
    from eagle4_b200.ops import native

    cfg = nemotron_h_8b()
    H, P, N, G = cfg.mamba_heads, cfg.mamba_head_dim, cfg.mamba_state, cfg.mamba_groups
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(1)
    bf = lambda *s: torch.randn(*s, generator=g, device=dev).to(torch.bfloat16)  # noqa: E731
    xbc = bf(t, H * P + 2 * G * N)
    dt = bf(t, H)
    a_log = torch.rand(H, device=dev).log1p()
    dt_bias = torch.randn(H, device=dev) * 0.1
    dskip = torch.randn(H, device=dev)
    state = torch.randn(t + 1, H, P, N, device=dev) * 0.01
    x = xbc[:, :H * P].view(t, H, P)
    bm = xbc[:, H * P:H * P + G * N].view(t, G, N)
    cm = xbc[:, H * P + G * N:].view(t, G, N)
    out_ref = torch.empty(t, H, P, dtype=torch.bfloat16, device=dev)
    a_neg = -a_log.exp()
    sidx = torch.arange(1, t + 1, dtype=torch.int32, device=dev).view(1, t)
    parents = torch.tensor([_chain_tree(t)], dtype=torch.int32, device=dev)
    qsl = torch.tensor([0, t], dtype=torch.int32, device=dev)
    sidx0 = torch.cat([torch.zeros(1, 1, dtype=torch.int32, device=dev), sidx], dim=1)

    def ref_call():
        rmamba.mamba2_tree_state_update(state, x, dt, a_neg, bm, cm, dskip, dt_bias, out_ref,
                                        state_indices=sidx0[:, 1:], parents=parents, query_start_loc=qsl)

    slot = torch.zeros(t, dtype=torch.int32, device=dev)
    par = parents[0].clone()
    st_ours = state[:1].clone()
    rows = torch.tensor([[0, 1, 2, 3]], dtype=torch.int32, device=dev)
    nrows = torch.tensor([4], dtype=torch.int32, device=dev)
    slots = torch.zeros(1, dtype=torch.int64, device=dev)
    conv = torch.zeros(1, xbc.shape[1], cfg.conv_kernel - 1, dtype=torch.bfloat16, device=dev)

    def ours_call():
        native.mamba_tree(xbc, dt, a_log, dt_bias, dskip, st_ours, slot, par, cfg, False)

    def ours_commit():
        native.mamba_commit(xbc, dt, a_log, dt_bias, dskip, xbc, st_ours, conv, slots, rows, nrows, cfg)

    def ref_commit():  # the accepted node's stored state becomes the request's state
        state[0].copy_(state[4])

    r = {"op": "mamba2_tree_verify", "rows": t, "heads": f"{H} x {P}, state {N}",
         "reference_us": graph_us(ref_call, iters), "reference_commit_us": graph_us(ref_commit, iters),
         "ours_us": graph_us(ours_call, iters), "ours_commit_us": graph_us(ours_commit, iters),
         "note": "reference: tree update storing every node's state, commit = copy of the accepted node's state; "
                 "ours: chain-walk tree pass, commit = replay of the 4-row accepted path"}
    r["speedup"] = (r["reference_us"] + r["reference_commit_us"]) / (r["ours_us"] + r["ours_commit_us"])
    return r


def bench_accept(racc, iters: int, width: int = 16) -> dict:
    """Greedy acceptance of one request's 16-node verify tree (chain-shaped prefix accepted)."""
    from eagle4_b200.ops import native

    dev = torch.device("cuda")
    parent = _chain_tree(width)
    toks = torch.arange(width, dtype=torch.int64, device=dev) + 100
    target = torch.roll(toks, -1).clone()  # the target agrees along the first rows of the chain
    nxt = torch.full((width,), -1, dtype=torch.int64, device=dev)
    sib = torch.full((width,), -1, dtype=torch.int64, device=dev)
    for r in range(1, width):
        p = parent[r]
        if int(nxt[p]) < 0:
            nxt[p] = r
        else:
            c = int(nxt[p])
            while int(sib[c]) >= 0:
                c = int(sib[c])
            sib[c] = r
    seq = torch.tensor([50], dtype=torch.int64, device=dev)
    ocl = torch.arange(width, dtype=torch.int64, device=dev) + 1000
    r2t = torch.arange(4096, dtype=torch.int32, device=dev).view(1, 4096)
    rpi = torch.zeros(1, dtype=torch.int64, device=dev)
    ridx = torch.arange(width, dtype=torch.int64, device=dev).view(1, width)

    def ref_call():
        racc.accept_tail(target.int(), toks.view(1, width), ridx, nxt.view(1, width), sib.view(1, width), seq, ocl,
                         r2t, rpi, width)

    prow = torch.tensor([parent], dtype=torch.int32, device=dev)
    tid = target.view(1, width)
    n = torch.full((1,), width, dtype=torch.int32, device=dev)

    def ours_call():
        native.accept_greedy(tid, toks.view(1, width), prow, n)

    r = {"op": "accept_greedy", "rows": width, "reference_us": graph_us(ref_call, iters),
         "ours_us": graph_us(ours_call, iters)}
    r["speedup"] = r["reference_us"] / r["ours_us"]
    return r


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--bs", type=int, nargs="*", default=[1, 8, 64])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", nargs="*", default=None)
    args = ap.parse_args()
    rdt, rgdn, rmamba, racc = _reference()
    rows = []
    want = lambda name: args.only is None or name in args.only  # noqa: E731
    if want("tree"):
        for bs in args.bs:
            rows.extend(bench_tree(rdt, bs, args.iters))
    if want("gdn"):
        rows.append(bench_gdn(rgdn, args.iters))
    if want("mamba"):
        rows.append(bench_mamba(rmamba, args.iters))
    if want("accept"):
        rows.append(bench_accept(racc, args.iters))
    for r in rows:
        print(json.dumps({k: (round(v, 2) if isinstance(v, float) else v) for k, v in r.items()}), flush=True)


if __name__ == "__main__":
    main()
