"""Sampled-tree kernels on the GPU against their float64 definitions, and the sampled engine."""

import pytest
import torch

from eagle4_b200.core import sampled_tree as st
from eagle4_b200.core.draft_tree import TreeShape

pytestmark = pytest.mark.gpu


def _native():
    from eagle4_b200.ops import native

    return native


def test_sample_children_matches_definition():
    nat = _native()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    r, c, k, cap = 64, 128, 4, 40
    logits = torch.randn(r, c, generator=g, device=dev) * 2
    ids = torch.randint(0, 50000, (r, c), generator=g, device=dev)
    q_store = torch.zeros(r, 1, c, device=dev)
    q_ids = torch.zeros(r, 1, c, dtype=torch.int32, device=dev)
    node_slot = torch.zeros(r, cap, dtype=torch.int32, device=dev)
    ctr = torch.full((1,), 5, dtype=torch.int32, device=dev)
    cp, ct = nat.sample_children(logits, ids, k, 0.7, 123, ctr, 3, None, 1, q_store, q_ids, node_slot, 0)
    q, rp, rt, slots = st.sample_children_reference(logits.cpu(), ids.cpu(), k, 0.7, 123, 5, 3)
    assert (ct.cpu() == rt).float().mean() >= 0.99
    torch.testing.assert_close(q_store[:, 0].cpu().double(), q, rtol=1e-4, atol=1e-6)
    assert torch.equal(q_ids[:, 0].cpu().long(), ids.cpu())
    assert (node_slot[:, :k].cpu().long() == slots).float().mean() >= 0.99


def _random_tree(bs, k, depth2_children, c, v, dev, g):
    """Root -> K depth-1 rows; the first depth-1 node expanded into ``depth2_children`` rows."""
    shape = TreeShape(k, 3)
    n = 1 + k + depth2_children
    parent = torch.full((bs, n), 0, dtype=torch.int32)
    parent[:, 0] = -1
    nodes = torch.full((bs, n), -1, dtype=torch.int64)
    nodes[:, 1:1 + k] = torch.arange(k)
    base = shape.layer_start(2)
    nodes[:, 1 + k:] = base + torch.arange(depth2_children)  # lane 0's children
    parent[:, 1 + k:] = 1
    cap = shape.capacity
    q_store = torch.softmax(torch.randn(bs, 1 + cap, c, generator=g) * 1.5, -1)
    q_ids = torch.stack([torch.stack([torch.randperm(v, generator=g)[:c] for _ in range(1 + cap)]) for _ in range(bs)])
    node_slot = torch.stack([torch.randperm(c, generator=g)[:cap] for _ in range(bs)]).int()
    return n, parent, nodes, q_store.float(), q_ids.int(), node_slot, cap


def test_sampled_accept_matches_definition():
    nat = _native()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(1)
    bs, k, c, v = 6, 3, 16, 400
    n, parent, nodes, q_store, q_ids, node_slot, cap = _random_tree(bs, k, 2, c, v, dev, g)
    agree = 0
    total = 0
    for rnd in range(40):
        logits = torch.randn(bs * n, v, generator=g) * 2
        ctr = torch.full((1,), rnd, dtype=torch.int32, device=dev)
        acc, cnt, bonus = nat.sampled_accept(logits.to(dev), 1.0, parent.to(dev), torch.zeros(bs, n, dtype=torch.int64,
                                             device=dev), nodes.to(dev), q_store.to(dev), q_ids.to(dev),
                                             node_slot.to(dev), k, 9, ctr, 0x10000)
        racc, rcnt, rbonus = st.sampled_walk_reference(logits, 1.0, parent, nodes, q_store, q_ids, node_slot, k, 9,
                                                       rnd, 0x10000)
        for b in range(bs):
            total += 1
            same = int(cnt[b]) == int(rcnt[b]) and int(bonus[b]) == int(rbonus[b]) and torch.equal(
                acc[b, : int(cnt[b])].cpu(), racc[b, : int(rcnt[b])])
            agree += same
    assert agree / total >= 0.97, agree / total


def test_sampled_accept_first_token_distribution():
    nat = _native()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(2)
    k, c, v = 2, 4, 6
    p_logits = torch.tensor([1.0, 0.2, -0.5, 0.8, 0.0, -1.0])
    cand = torch.tensor([0, 1, 3, 5])
    trials = 4000
    logits = p_logits.repeat(trials * 3, 1).to(dev)  # rows: root, child 0, child 1 per trial
    q_logits = torch.tensor([0.5, 2.0, 0.1, -0.3]).repeat(trials, 1).to(dev)
    ids = cand.repeat(trials, 1).to(dev)
    q_store = torch.zeros(trials, 1 + 2, c, device=dev)
    q_ids = torch.zeros(trials, 1 + 2, c, dtype=torch.int32, device=dev)
    node_slot = torch.zeros(trials, 2, dtype=torch.int32, device=dev)
    ctr = torch.zeros(1, dtype=torch.int32, device=dev)
    cp, ct = nat.sample_children(q_logits, ids, k, 1.0, 77, ctr, 0, None, 1, q_store, q_ids, node_slot, 0)
    parent = torch.tensor([[-1, 0, 0]], dtype=torch.int32, device=dev).repeat(trials, 1)
    nodes = torch.tensor([[-1, 0, 1]], device=dev).repeat(trials, 1)
    acc, cnt, bonus = nat.sampled_accept(logits, 1.0, parent, torch.zeros(trials, 3, dtype=torch.int64, device=dev),
                                         nodes, q_store, q_ids, node_slot, k, 77, ctr, 0x10000)
    first = torch.where(cnt > 1, ct.gather(1, (acc[:, 1:2] - 1).clamp(min=0)).squeeze(1), bonus)
    freq = torch.bincount(first.cpu(), minlength=v).double() / trials
    p = torch.softmax(p_logits.double(), -1)
    assert (freq - p).abs().max() < 0.03, (freq, p)


def test_sampled_engine_on_gpu():
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    llm = LLM.synthetic("tiny", device="cuda", tree=TreeSpec(4, 2, 8), max_len=512, temperature=1.0, sample_seed=4)
    prompt = torch.randint(0, 4096, (1, 32), generator=torch.Generator().manual_seed(0))
    a = llm.generate(prompt, 16)
    b = llm.generate(prompt, 16, speculative=False)
    assert a.shape == (1, 16) and b.shape == (1, 16)
    assert int(a.max()) < 4096 and int(b.min()) >= 0
    native.check_errors()


def test_vocab_parallel_kernels_match_the_full_walk():
    """The sparse walk and the shard mass / draw kernels, with the vocabulary split in two shards on one GPU, against
    the full-vocabulary accept kernel."""
    nat = _native()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(5)
    bs, k, c, v = 6, 3, 16, 512
    n, parent, nodes, q_store, q_ids, node_slot, cap = _random_tree(bs, k, 2, c, v, dev, g)
    parent, nodes, q_store, q_ids, node_slot = (t.to(dev) for t in (parent, nodes, q_store, q_ids, node_slot))
    S = q_store.shape[1]
    agree = total = 0
    for rnd in range(30):
        logits = (torch.randn(bs * n, v, generator=g) * 2).to(dev)
        ctr = torch.full((1,), rnd, dtype=torch.int32, device=dev)
        tok0 = torch.zeros(bs, n, dtype=torch.int64, device=dev)
        acc, cnt, bonus = nat.sampled_accept(logits, 0.8, parent, tok0, nodes, q_store, q_ids, node_slot, k, 9, ctr,
                                             0x10000)
        lg = logits * (1.0 / 0.8)
        mx = lg.amax(-1)
        z = torch.exp(lg - mx[:, None]).sum(-1)
        node = nodes.reshape(-1)
        qrow = torch.arange(bs, device=dev).repeat_interleave(n) * S + torch.where(node < 0, 0, node + 1)
        ids = q_ids.reshape(bs * S, c).index_select(0, qrow).long()
        p = (torch.exp(lg.gather(1, ids) - mx[:, None]) / z[:, None]).contiguous()
        sacc, scnt, final, r_final = nat._C.sampled_walk_sparse(p, parent, tok0, nodes, q_store, q_ids, node_slot, k, 9,
                                                             ctr, 0x10000)
        shards = [(0, 256), (256, 512)]
        masses = torch.stack([nat._C.shard_residual_mass(logits[:, lo:hi].contiguous(), lo, 0.8, mx, z, final, nodes,
                                                      q_ids, r_final, S, n) for lo, hi in shards]).contiguous()
        toks = torch.stack([nat._C.shard_draw(logits[:, lo:hi].contiguous(), lo, 0.8, mx, z, final, nodes, q_ids,
                                           r_final, S, n, masses, r, 9, ctr, 0x10000)
                            for r, (lo, hi) in enumerate(shards)])
        assert ((toks >= 0).sum(0) == 1).all(), "exactly one rank draws each token"
        tok = toks.amax(0)
        for b in range(bs):
            total += 1
            agree += int(scnt[b]) == int(cnt[b]) and int(tok[b]) == int(bonus[b]) and torch.equal(
                sacc[b, :int(scnt[b])], acc[b, :int(cnt[b])])
    assert agree / total >= 0.95, agree / total


def test_second_run_same_bits_on_gpu():
    """Fresh engines with the same weights and sampling seed emit the same tokens on the GPU (greedy and sampled)."""
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    prompt = torch.randint(0, 4096, (2, 24), generator=torch.Generator().manual_seed(2))

    def run(temperature):
        llm = LLM.synthetic("tiny", device="cuda", tree=TreeSpec(4, 2, 8), max_batch=2, max_len=256,
                            temperature=temperature, sample_seed=5)
        out = llm.generate(prompt, 12)
        del llm
        return out

    for temperature in (0.0, 1.0):
        assert torch.equal(run(temperature), run(temperature))
    native.check_errors()
