"""sm_100a kernels against their fp32/fp64 PyTorch definitions (``eagle4_b200.ops.reference``)."""

import pytest
import torch

from eagle4_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nat():
    from eagle4_b200.ops import native

    return native


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


def _close(a, b, tol):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("T,N,K", [(1, 256, 512), (16, 640, 1024), (37, 1000, 1536), (256, 384, 256),
                                   (300, 512, 768), (16, 16480, 5120)])
def test_gemm_plain(nat, T, N, K):
    x, w = _bf(T, K, seed=1), _bf(N, K, scale=0.05, seed=2)
    y = nat.linear(x, w)
    _close(y, ref.linear(x.cpu().float(), w.cpu().float()), 2e-2)
    nat.check_errors()


def test_gemm_batch_invariant(nat):
    """A row's GEMM result does not depend on the other rows of the launch (plain decode vs tree verify)."""
    K, N = 5120, 2048
    x, w = _bf(64, K, seed=3), _bf(N, K, scale=0.02, seed=4)
    full = nat.linear(x, w)
    for t in (1, 7, 16, 33):
        part = nat.linear(x[:t].contiguous(), w)
        assert torch.equal(part, full[:t])
    single = nat.linear(x[5:6].contiguous(), w)
    assert torch.equal(single, full[5:6])


def test_gemm_epilogues(nat):
    T, K, F = 19, 1024, 512
    x = _bf(T, K, seed=5)
    gu = _bf(2 * F, K, scale=0.05, seed=6)
    _close(nat.linear_swiglu(x, gu), ref.linear_swiglu(x.cpu().float(), gu.cpu().float()), 2e-2)
    w = _bf(768, K, scale=0.05, seed=7)
    r = _bf(T, 768, seed=8)
    _close(nat.linear_residual(x, w, r), ref.linear_residual(x.cpu().float(), w.cpu().float(), r.cpu().float()), 2e-2)
    _close(nat.linear_relu2(x, w), ref.linear_relu2(x.cpu().float(), w.cpu().float()), 3e-2)
    _close(nat.logits(x, w), ref.logits(x.cpu().float(), w.cpu().float()), 1e-2)


@pytest.mark.parametrize("T", [1, 16, 100, 300])
def test_gemm_folded_norm(nat, T):
    """RMSNorm folded into the GEMM: raw rows in, the norm weight multiplied into W's columns, the per-token inverse
    RMS applied in the epilogue; matches norm-then-GEMM, is batch invariant, and works for every epilogue kind."""
    K, N, F = 5120, 1024, 512
    x = _bf(T, K, scale=3.0, seed=40)
    nw = _bf(K, scale=0.1, seed=41)
    w = _bf(N, K, scale=0.05, seed=42)
    wf = ref.fold_norm_weight(w, nw, True)
    eps = 1e-6
    xn = ref.rmsnorm(x.cpu().float(), nw.cpu().float(), eps, True)
    want = ref.linear(xn, w.cpu().float())
    got = nat.linear(x, wf, eps)
    _close(got, want, 2e-2)
    _close(got, ref.linear(x.cpu().float(), wf.cpu().float(), eps), 1e-2)
    single = nat.linear(x[T - 1:].contiguous(), wf, eps)
    assert torch.equal(single, got[T - 1:])
    gu = _bf(2 * F, K, scale=0.05, seed=43)
    guf = ref.fold_norm_weight(gu, nw, True)
    _close(nat.linear_swiglu(x, guf, eps), ref.linear_swiglu(xn, gu.cpu().float()), 3e-2)
    _close(nat.linear_relu2(x, wf, eps), ref.linear_relu2(xn, w.cpu().float()), 3e-2)
    nat.check_errors()


def test_lm_head_argmax(nat):
    T, K, V = 21, 1024, 50000
    x, w = _bf(T, K, seed=9), _bf(V, K, scale=0.05, seed=10)
    ids, best = nat.lm_head_argmax(x, w)
    lg = nat.logits(x, w)
    m, i = lg.max(dim=-1)
    assert torch.equal(ids, i)
    assert torch.equal(best, m)


def test_rmsnorm_and_rows(nat):
    x, w = _bf(9, 5120, seed=11), _bf(5120, scale=0.1, seed=12)
    for off in (False, True):
        _close(nat.rmsnorm(x, w, 1e-6, off), ref.rmsnorm(x.cpu(), w.cpu(), 1e-6, off), 1e-2)
    e, h = _bf(9, 256, seed=13), _bf(9, 256, seed=14)
    we, wh = _bf(256, seed=15), _bf(256, seed=16)
    _close(nat.concat_norms(e, h, we, wh, 1e-6), ref.concat_norms(e.cpu(), h.cpu(), we.cpu(), wh.cpu(), 1e-6), 1e-2)
    o, z, gw = _bf(9, 6, 128, seed=17), _bf(9, 768, seed=18), _bf(128, seed=19)
    _close(nat.gated_rmsnorm(o, z, gw, 1e-6), ref.gated_rmsnorm(o.cpu(), z.cpu(), gw.cpu(), 1e-6), 2e-2)
    ids = torch.randint(0, 1000, (13,), device="cuda")
    table = _bf(1000, 256, seed=20)
    assert torch.equal(nat.embedding(ids, table), table[ids])


def _tree_rows(bs, n, L, page, bt, device):
    """Random tree rows per request (parents before children) -> (parent rows, extra slots, counts, slots)."""
    g = torch.Generator().manual_seed(0)
    prow = torch.full((bs, n), -1, dtype=torch.int64)
    for r in range(1, n):
        prow[:, r] = torch.randint(0, r, (bs,), generator=g)
    depth, mask = ref_rows_meta(prow)
    rowidx = torch.arange(n)
    phys = L[:, None] + rowidx[None, :]
    slots = bt[torch.arange(bs)[:, None], phys // page].long() * page + phys % page
    bits = ((mask[:, :, None] >> rowidx[None, None, :]) & 1).bool()
    n_extra = bits.sum(-1).int()
    order = torch.argsort((~bits).int() * n + rowidx, dim=-1)
    extra = torch.gather(slots[:, None, :].expand(bs, n, n), 2, order).int()
    return prow, depth, extra, n_extra, slots


def ref_rows_meta(prow):
    from eagle4_b200.core.draft_tree import rows_meta

    return rows_meta(prow)


@pytest.mark.parametrize("hq,hk,d", [(6, 1, 256), (16, 2, 128), (4, 2, 64)])
def test_attention_tree_and_exactness(nat, hq, hk, d):
    bs, n, page = 2, 8, 16
    L = torch.tensor([300, 517])
    bt = torch.arange(bs * 64, dtype=torch.int32).view(bs, 64)
    slots_total = bt.numel() * page
    kc, vc = _bf(slots_total, hk, d, seed=21), _bf(slots_total, hk, d, seed=22)
    prow, depth, extra, n_extra, slots = _tree_rows(bs, n, L, page, bt, "cpu")
    q = _bf(bs * n, hq, d, seed=23)
    req = torch.arange(bs).repeat_interleave(n).int()
    cs = torch.zeros(bs * n, dtype=torch.int32)
    cl = L.int().repeat_interleave(n)
    ex, ne = extra.reshape(bs * n, n), n_extra.reshape(-1)
    out = nat.attention(q, kc, vc, bt.cuda(), page, req.cuda(), cs.cuda(), cl.cuda(), ex.cuda(), ne.cuda(), d ** -0.5)
    want = ref.attention(q.cpu(), kc.cpu(), vc.cpu(), bt, page, req, cs, cl, ex, ne, d ** -0.5)
    _close(out, want.reshape(want.shape[0], -1), 2e-2)
    gate = _bf(bs * n, hq * d, seed=24)
    gated = nat.attention(q, kc, vc, bt.cuda(), page, req.cuda(), cs.cuda(), cl.cuda(), ex.cuda(), ne.cuda(),
                          d ** -0.5, gate=gate)
    _close(gated, ref.sigmoid_gate(want.reshape(want.shape[0], -1), gate.cpu()), 2e-2)
    # exactness: a chain row verified in the tree equals the same key sequence as committed context
    b, r = 1, n - 1
    anc = extra[b, r, : n_extra[b, r]]
    # re-lay the ancestors as committed positions L.. (copy KV) and attend with context only
    kc2, vc2 = kc.clone(), vc.clone()
    Lb = int(L[b])
    for j, s in enumerate(anc.tolist()):
        dst = int(bt[b, (Lb + j) // page]) * page + (Lb + j) % page
        kc2[dst] = kc[s]
        vc2[dst] = vc[s]
    one = lambda v: torch.tensor([v], dtype=torch.int32, device="cuda")  # noqa: E731
    solo = nat.attention(q[b * n + r: b * n + r + 1].contiguous(), kc2, vc2, bt.cuda(), page, one(b), one(0),
                         one(Lb + len(anc)), torch.zeros(1, 1, dtype=torch.int32, device="cuda"), one(0), d ** -0.5)
    assert torch.equal(solo[0], out[b * n + r])


def test_gdn_mixer_against_reference(nat):
    from eagle4_b200.models.configs import tiny_hybrid

    cfg = tiny_hybrid()
    T, S = 7, 2
    C = cfg.gdn_conv_dim
    proj = _bf(T, C + cfg.gdn_value_dim + 2 * cfg.gdn_v_heads, seed=30)
    conv = _bf(T, C, seed=32)
    a_log = torch.rand(cfg.gdn_v_heads, device="cuda").log1p()
    dt_bias = torch.ones(cfg.gdn_v_heads, device="cuda")
    gnorm = _bf(cfg.gdn_v_dim, seed=33)
    state = torch.randn(S, cfg.gdn_v_heads, cfg.gdn_v_dim, cfg.gdn_k_dim, device="cuda") * 0.1
    slot = torch.tensor([0, 0, 0, 0, 1, 1, 1], dtype=torch.int32, device="cuda")
    parent = torch.tensor([-1, 0, 0, 1, -1, 4, 5], dtype=torch.int32, device="cuda")
    out = nat.gdn_mixer(conv, proj, cfg, a_log, dt_bias, gnorm, state, slot, parent, False)
    cpu = lambda t: t.cpu().float()  # noqa: E731
    want = ref.gdn_mixer(cpu(conv), cpu(proj), cfg, a_log.cpu(), dt_bias.cpu(), cpu(gnorm), state.cpu().clone(),
                         slot.cpu(), parent.cpu(), False)
    _close(out, want, 3e-2)
    # commit of the paths 0 -> 1 -> 3 and 4 -> 5
    rows = torch.tensor([[0, 1, 3], [4, 5, 0]], dtype=torch.int32, device="cuda")
    nrows = torch.tensor([3, 2], dtype=torch.int32, device="cuda")
    slots = torch.tensor([0, 1], device="cuda")
    st2 = state.clone()
    cst = torch.zeros(S, C, 3, dtype=torch.bfloat16, device="cuda")
    nat.gdn_commit_all([conv], [proj], [st2], [cst], [a_log], [dt_bias], slots, rows, nrows, cfg)
    st_ref = state.cpu().clone()
    cs_ref = torch.zeros(S, C, 3, dtype=torch.bfloat16)
    ref.gdn_commit_all([cpu(conv)], [proj.cpu()], [st_ref], [cs_ref], [a_log.cpu()], [dt_bias.cpu()], slots.cpu(),
                       rows.cpu(), nrows.cpu(), cfg)
    _close(st2, st_ref, 2e-3)
    assert torch.equal(cst.cpu(), cs_ref)
    # plain decode equals tree verify: committing [0, 1] then a one-row verify of row 3 gives its tree output
    st3 = state.clone()
    nat.gdn_commit_all([conv], [proj], [st3], [cst.clone()], [a_log], [dt_bias], slots[:1],
                       torch.tensor([[0, 1]], dtype=torch.int32, device="cuda"),
                       torch.tensor([2], dtype=torch.int32, device="cuda"), cfg)
    solo = nat.gdn_mixer(conv[3:4].contiguous(), proj[3:4].contiguous(), cfg, a_log, dt_bias, gnorm, st3, slot[:1],
                         torch.tensor([-1], dtype=torch.int32, device="cuda"), False)
    assert torch.equal(solo[0], out[3])


@pytest.mark.parametrize("hk,hv,kd", [(4, 4, 64), (2, 6, 128)])
def test_gdn_scan_against_reference(nat, hk, hv, kd):
    """Prefill scan (contiguous rows per request, state updated in place) against the float definition: the mixer
    output and the final state, with one request longer than a 32-token staging tile and key heads shared by several
    value heads."""
    import dataclasses

    from eagle4_b200.models.configs import tiny_hybrid

    cfg = dataclasses.replace(tiny_hybrid(), gdn_k_heads=hk, gdn_v_heads=hv, gdn_k_dim=kd, gdn_v_dim=kd)
    C = cfg.gdn_conv_dim
    lens = (45, 9)
    T = sum(lens)
    proj = _bf(T, C + cfg.gdn_value_dim + 2 * cfg.gdn_v_heads, seed=70)
    conv = _bf(T, C, seed=71)
    a_log = torch.rand(cfg.gdn_v_heads, device="cuda").log1p()
    dt_bias = torch.ones(cfg.gdn_v_heads, device="cuda")
    gnorm = _bf(cfg.gdn_v_dim, seed=72)
    state = torch.randn(3, cfg.gdn_v_heads, cfg.gdn_v_dim, cfg.gdn_k_dim, device="cuda") * 0.1
    slot = torch.tensor([2] * lens[0] + [0] * lens[1], dtype=torch.int32, device="cuda")
    parent = torch.tensor([-1] + list(range(lens[0] - 1)) + [-1] + list(range(lens[0], T - 1)), dtype=torch.int32,
                          device="cuda")
    cpu = lambda t: t.cpu().float()  # noqa: E731
    st_ref = state.cpu().clone()
    want = ref.gdn_mixer(cpu(conv), cpu(proj), cfg, a_log.cpu(), dt_bias.cpu(), cpu(gnorm), st_ref, slot.cpu(),
                         parent.cpu(), True)
    st = state.clone()
    out = nat.gdn_mixer(conv, proj, cfg, a_log, dt_bias, gnorm, st, slot, parent, True)
    _close(out, want, 3e-2)
    _close(st, st_ref, 2e-3)
    nat.check_errors()


def test_conv_tree(nat):
    T, C, S, W = 6, 96, 2, 4
    x, w = _bf(T, C, seed=40), _bf(C, W, seed=41)
    cs = _bf(S, C, W - 1, seed=42)
    slot = torch.tensor([0, 0, 0, 1, 1, 1], dtype=torch.int32, device="cuda")
    parent = torch.tensor([-1, 0, 1, -1, 3, 3], dtype=torch.int32, device="cuda")
    out = nat.causal_conv_tree(x, cs, slot, parent, w)
    want = ref.causal_conv_tree(x.cpu().float(), cs.cpu().float(), slot.cpu(), parent.cpu(), w.cpu().float())
    _close(out, want, 2e-2)


def test_conv_tree_with_bias(nat):
    """Nemotron-H's conv has a bias, added before the SiLU."""
    T, C, S, W = 6, 96, 2, 4
    x, w, b = _bf(T, C, seed=43), _bf(C, W, seed=44), _bf(C, seed=45)
    cs = _bf(S, C, W - 1, seed=46)
    slot = torch.tensor([0, 0, 0, 1, 1, 1], dtype=torch.int32, device="cuda")
    parent = torch.tensor([-1, 0, 1, -1, 3, 3], dtype=torch.int32, device="cuda")
    out = nat.causal_conv_tree(x, cs, slot, parent, w, b)
    want = ref.causal_conv_tree(x.cpu().float(), cs.cpu().float(), slot.cpu(), parent.cpu(), w.cpu().float(),
                                b.cpu().float())
    _close(out, want, 2e-2)


def test_gated_rmsnorm_gate_first_and_group_weights(nat):
    """Nemotron-H's gated norm: rmsnorm(o * silu(z)) with one weight row per group (and the shared-row form)."""
    o, z = _bf(9, 8, 64, seed=47), _bf(9, 512, seed=48)
    for w in (_bf(512, seed=49), _bf(64, seed=50)):
        for first in (False, True):
            _close(nat.gated_rmsnorm(o, z, w, 1e-5, first),
                   ref.gated_rmsnorm(o.cpu().float(), z.cpu().float(), w.cpu().float(), 1e-5, first), 2e-2)


def test_candidate_tail_and_accept(nat):
    h, w = _bf(5, 512, seed=50), _bf(3000, 512, scale=0.1, seed=51)
    idx = torch.randint(0, 3000, (5, 64), device="cuda")
    lg = nat._C.gather_dot(h, w, idx)
    _close(lg, ref.gather_dot(h.cpu(), w.cpu(), idx.cpu()), 1e-3)
    p, ids = nat._C.softmax_topk(lg, idx, 4, 1.0)
    pr, idr = ref.softmax_topk(lg.cpu(), idx.cpu(), 4)
    _close(p, pr, 1e-4)
    assert torch.equal(ids.cpu(), idr)
    tokens = torch.tensor([[5, 7, 8, 9], [1, 2, 3, 4]], device="cuda")
    parent = torch.tensor([[-1, 0, 0, 1], [-1, 0, 1, 2]], device="cuda")
    tid = torch.tensor([[8, 0, 3, 0], [2, 3, 4, 6]], device="cuda")
    n = torch.tensor([4, 4], device="cuda")
    a, c, b = nat.accept_greedy(tid, tokens, parent, n)
    ar, cr, br = ref.accept_greedy(tid.cpu(), tokens.cpu(), parent.cpu(), n.cpu())
    assert torch.equal(c.cpu(), cr) and torch.equal(b.cpu(), br)
    assert torch.equal(a.cpu(), ar)


def test_topk_large_and_tree_kernels(nat):
    g = torch.Generator(device="cuda").manual_seed(60)
    s = torch.randn(5, 248320, generator=g, device="cuda")
    s[0, 1000:1010] = 9.0  # ties go to the lower index
    v, i = nat.topk_rows(s, 128)
    vr, ir = ref.topk_rows(s.cpu(), 128)
    assert torch.equal(v.cpu(), vr) and torch.equal(i.cpu(), ir)
    # tree step / verify rows against the tensor definitions
    from eagle4_b200.core.draft_tree import DraftTree, TreeShape
    from eagle4_b200.ops import tree_ops

    shape = TreeShape(top_k=4, max_depth=6)
    bs, H = 3, 256
    trees = [DraftTree(shape, bs, H, torch.bfloat16, "cuda", max_verify=16) for _ in range(2)]
    probs0 = torch.rand(bs, 4, generator=g, device="cuda")
    toks0 = torch.randint(0, 1000, (bs, 4), generator=g, device="cuda")
    hid0 = _bf(bs, H, seed=61)
    for t in trees:
        t.stage_root(bs, probs0, toks0, hid0)
        t.begin_reference(bs)
    for step in range(1, 5):
        p = torch.rand(bs * 4, 4, generator=g, device="cuda")
        tk = torch.randint(0, 1000, (bs * 4, 4), generator=g, device="cuda")
        hid = _bf(bs * 4, H, seed=70 + step)
        slots = torch.randint(0, 1 << 20, (bs, 4), generator=g, device="cuda")
        for t in trees:
            t.set_step_slots(bs, step, slots)
        trees[0].step_reference(bs, step, p, tk, hid)
        tree_ops.tree_step(trees[1], bs, step, p, tk, hid, deltas=False)
    a, b = trees
    for name in ("scores", "tokens", "parents", "front_scores", "front_tokens", "front_hidden", "ancestors", "best",
                 "best_prev", "layer_top"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    ta, pa = a.verify_rows_reference(bs, 5, 15)
    tb, pb = tree_ops.select_rows(b, bs, 5, 15)
    assert torch.equal(ta, tb) and torch.equal(pa, pb)


@pytest.mark.parametrize("shape", ["tiny", "nemotron"])
def test_mamba_tree_and_commit_against_reference(nat, shape):
    """Mamba2 tree verify (each row's path replayed from the committed state) and the commit of accepted paths
    against the float64 definition; one-row decode after a commit equals the row's tree output bit for bit."""
    import dataclasses

    from eagle4_b200.models.configs import nemotron_h_8b, tiny_nemotron

    cfg = tiny_nemotron() if shape == "tiny" else dataclasses.replace(nemotron_h_8b(), mamba_heads=16)
    H, P, N, G = cfg.mamba_heads, cfg.mamba_head_dim, cfg.mamba_state, cfg.mamba_groups
    conv_dim = cfg.mamba_inner + 2 * G * N
    T, S = 7, 2
    xbc = _bf(T, conv_dim, scale=0.5, seed=40)
    dt = _bf(T, H, seed=41)
    a_log = torch.rand(H, device="cuda").log1p()
    dt_bias = torch.randn(H, device="cuda") * 0.1
    dskip = torch.randn(H, device="cuda")
    state = torch.randn(S, H, P, N, device="cuda") * 0.1
    slot = torch.tensor([0, 0, 0, 0, 1, 1, 1], dtype=torch.int32, device="cuda")
    parent = torch.tensor([-1, 0, 0, 1, -1, 4, 5], dtype=torch.int32, device="cuda")
    out = nat.mamba_tree(xbc, dt, a_log, dt_bias, dskip, state, slot, parent, cfg, False)
    cpu = lambda t: t.cpu().float()  # noqa: E731
    want = ref.mamba_tree(cpu(xbc), cpu(dt), a_log.cpu(), dt_bias.cpu(), dskip.cpu(), state.cpu().clone(),
                          slot.cpu(), parent.cpu(), cfg, False)
    _close(out, want, 2e-2)
    # scan mode (prefill): the state advances in place row by row
    st_scan = state.clone()
    chain = torch.tensor([-1, 0, 1, 2, -1, 4, 5], dtype=torch.int32, device="cuda")
    out_scan = nat.mamba_tree(xbc, dt, a_log, dt_bias, dskip, st_scan, slot, chain, cfg, True)
    st_ref = state.cpu().clone()
    want_scan = ref.mamba_tree(cpu(xbc), cpu(dt), a_log.cpu(), dt_bias.cpu(), dskip.cpu(), st_ref, slot.cpu(),
                               chain.cpu(), cfg, True)
    _close(out_scan, want_scan, 2e-2)
    _close(st_scan, st_ref, 2e-3)
    # commit of the paths 0 -> 1 -> 3 and 4 -> 5
    rows = torch.tensor([[0, 1, 3], [4, 5, 0]], dtype=torch.int32, device="cuda")
    nrows = torch.tensor([3, 2], dtype=torch.int32, device="cuda")
    slots = torch.tensor([0, 1], device="cuda")
    st2 = state.clone()
    conv = torch.zeros(S, conv_dim, cfg.conv_kernel - 1, dtype=torch.bfloat16, device="cuda")
    nat.mamba_commit(xbc, dt, a_log, dt_bias, dskip, xbc, st2, conv, slots, rows, nrows, cfg)
    st_ref = state.cpu().clone()
    conv_ref = torch.zeros(S, conv_dim, cfg.conv_kernel - 1, dtype=torch.bfloat16)
    ref.mamba_commit(cpu(xbc), cpu(dt), a_log.cpu(), dt_bias.cpu(), dskip.cpu(), xbc.cpu(), st_ref, conv_ref,
                     slots.cpu(), rows.cpu(), nrows.cpu(), cfg)
    _close(st2, st_ref, 2e-3)
    assert torch.equal(conv.cpu(), conv_ref)
    # plain decode equals tree verify: commit [0, 1], then verify row 3 alone
    st3 = state.clone()
    nat.mamba_commit(xbc, dt, a_log, dt_bias, dskip, xbc, st3, conv.clone(), slots[:1],
                     torch.tensor([[0, 1]], dtype=torch.int32, device="cuda"),
                     torch.tensor([2], dtype=torch.int32, device="cuda"), cfg)
    solo = nat.mamba_tree(xbc[3:4].contiguous(), dt[3:4].contiguous(), a_log, dt_bias, dskip, st3, slot[:1],
                          torch.tensor([-1], dtype=torch.int32, device="cuda"), cfg, False)
    assert torch.equal(solo[0], out[3])
