"""Mamba2 hybrids (the Nemotron-H family) on CPU: tree verification of Mamba2 layers (per-node state replayed from
the committed state along each row's path), the commit of the accepted path, and speculative output equal to plain
greedy decoding, including multi-row accepted paths through an oracle draft."""

import torch

from eagle4_b200.api import LLM, TreeSpec
from eagle4_b200.models import configs
from eagle4_b200.ops import reference as R


def _llm(seed=0):
    return LLM.synthetic("tiny-mamba", device="cpu", dtype=torch.float32, seed=seed, tree=TreeSpec(4, 2, 8),
                         max_batch=2, max_len=256)


def test_mamba_hybrid_spec_equals_plain():
    llm = _llm()
    assert any(m == "mamba" for m, _ in llm.target.cfg.layers)
    p = torch.randint(0, 4096, (2, 40), generator=torch.Generator().manual_seed(0))
    spec = llm.generate(p, 24, speculative=True)
    plain = llm.generate(p, 24, speculative=False)
    assert torch.equal(spec, plain)


def test_mamba_hybrid_accepts_oracle_paths():
    """Candidates that are the target's own greedy continuation are accepted along whole paths, so the Mamba2
    commit replays several rows per round and the output still equals plain decoding."""
    llm = _llm(seed=2)
    p = torch.randint(0, 4096, (1, 24), generator=torch.Generator().manual_seed(5))
    ref = llm.generate(p, 20, speculative=False)[0].tolist()
    seq = p[0].tolist() + ref + [0] * 16
    drf = llm.draft

    def candidates(normed, k, pos):
        want = torch.tensor([seq[int(q) + 2] for q in pos])
        ids = torch.stack([want] + [(want + j) % 4096 for j in range(1, k)], dim=1)
        probs = torch.tensor([[0.9] + [0.1 / (k - 1)] * (k - 1)]).expand(normed.shape[0], k)
        return probs, ids

    saved, drf.candidates = drf.candidates, candidates
    llm.engine.stats.__init__()
    out = llm.generate(p, 20, speculative=True)[0].tolist()
    drf.candidates = saved
    assert out == ref
    assert llm.engine.stats.mean_accept > 2.5


def test_mamba_tree_rows_equal_their_chains():
    """A row verified inside a tree gets the output of running its root-to-row path as a chain from the same
    committed state (the tree-verify definition), and the commit of a path equals the scan over it."""
    cfg = configs.tiny_nemotron()
    g = torch.Generator().manual_seed(1)
    H, P, N, G = cfg.mamba_heads, cfg.mamba_head_dim, cfg.mamba_state, cfg.mamba_groups
    conv_dim = cfg.mamba_inner + 2 * G * N
    T = 7
    parent = torch.tensor([-1, 0, 0, 1, 1, 2, 5], dtype=torch.int32)
    xbc = torch.randn(T, conv_dim, generator=g)
    dt = torch.randn(T, H, generator=g)
    a_log, dt_bias, d = torch.rand(H, generator=g), torch.randn(H, generator=g) * 0.1, torch.randn(H, generator=g)
    state = torch.randn(2, H, P, N, generator=g) * 0.1
    slot = torch.ones(T, dtype=torch.int32)
    tree = R.mamba_tree(xbc, dt, a_log, dt_bias, d, state.clone(), slot, parent, cfg, False)
    for r, path in ((6, [0, 2, 5, 6]), (4, [0, 1, 4])):
        chain_state = state.clone()
        out = R.mamba_tree(xbc[path], dt[path], a_log, dt_bias, d, chain_state, slot[:len(path)],
                           torch.arange(-1, len(path) - 1, dtype=torch.int32), cfg, True)
        assert torch.allclose(out[-1], tree[r], atol=1e-6)
        committed = state.clone()
        conv = torch.zeros(2, conv_dim, cfg.conv_kernel - 1)
        R.mamba_commit(xbc, dt, a_log, dt_bias, d, xbc, committed, conv, torch.tensor([1]),
                       torch.tensor([path]), torch.tensor([len(path)]), cfg)
        assert torch.allclose(committed[1], chain_state[1], atol=1e-6)
