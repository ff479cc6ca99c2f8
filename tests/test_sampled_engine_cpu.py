"""Sampled trees on CPU: the float64 definitions of the GPU sampler and the engine's sampled rounds."""

import torch

from eagle4_b200.core import sampled_tree as st


def test_stream_uniforms_are_stable_and_uniform():
    u = st.stream_uniforms(7, 3, 0, range(20000))
    assert torch.all((u > 0) & (u < 1))
    assert abs(u.mean().item() - 0.5) < 0.01
    assert torch.equal(u[:10], st.stream_uniforms(7, 3, 0, range(10)))
    assert not torch.equal(u[:10], st.stream_uniforms(7, 4, 0, range(10)))


def test_gumbel_children_follow_q():
    # first draw frequencies match q (Gumbel-max)
    logits = torch.tensor([[2.0, 1.0, 0.5, -1.0]])
    ids = torch.arange(4)[None]
    counts = torch.zeros(4)
    for rnd in range(4000):
        _, _, ch, _ = st.sample_children_reference(logits, ids, 2, 1.0, 11, rnd, 0)
        counts[ch[0, 0]] += 1
        assert ch[0, 0] != ch[0, 1]
    q = torch.softmax(logits[0].double(), -1)
    assert (counts / counts.sum() - q).abs().max() < 0.03


def test_walk_output_distribution_equals_target():
    # a root with two drafted children: the emitted first token must follow p whatever q is
    v, c, k = 6, 4, 2
    p_logits = torch.tensor([1.0, 0.2, -0.5, 0.8, 0.0, -1.0])
    q_logits = torch.tensor([[0.5, 2.0, 0.1, -0.3]])
    cand = torch.tensor([[0, 1, 3, 5]])
    counts = torch.zeros(v)
    trials = 6000
    for rnd in range(trials):
        q, cp, ct, slots = st.sample_children_reference(q_logits, cand, k, 1.0, 5, rnd, 0)
        q_store = torch.zeros(1, 1 + k, c)
        q_ids = torch.zeros(1, 1 + k, c, dtype=torch.int32)
        q_store[0, 0] = q[0].float()
        q_ids[0, 0] = cand[0].int()
        node_slot = slots.int()
        logits = torch.stack([p_logits, p_logits, p_logits])  # rows: root, child 0, child 1
        parent = torch.tensor([[-1, 0, 0]], dtype=torch.int32)
        nodes = torch.tensor([[-1, 0, 1]])
        acc, cnt, bonus = st.sampled_walk_reference(logits, 1.0, parent, nodes, q_store, q_ids, node_slot, k, 5, rnd,
                                                    0x10000)
        first = int(ct[0, int(acc[0, 1]) - 1]) if cnt[0] > 1 else int(bonus[0])
        counts[first] += 1
    p = torch.softmax(p_logits.double(), -1)
    assert (counts / trials - p).abs().max() < 0.025, (counts / trials, p)


def test_sampled_engine_runs_on_cpu():
    from eagle4_b200.api import LLM, TreeSpec

    llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_len=256,
                        temperature=1.0, sample_seed=3)
    prompt = torch.randint(0, 4096, (1, 24), generator=torch.Generator().manual_seed(0))
    spec = llm.generate(prompt, 10)
    plain = llm.generate(prompt, 10, speculative=False)
    assert spec.shape == (1, 10) and plain.shape == (1, 10)
    assert int(llm.engine.round_ctr[0]) > 0


def test_second_run_same_bits():
    """Two fresh engines with the same weights and seed emit the same tokens, greedy and sampled, speculative and
    plain; another sampling seed draws other tokens."""
    from eagle4_b200.api import LLM, TreeSpec

    prompt = torch.randint(0, 4096, (2, 20), generator=torch.Generator().manual_seed(1))

    def run(temperature, seed, speculative):
        llm = LLM.synthetic("tiny", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=2,
                            max_len=256, temperature=temperature, sample_seed=seed)
        return llm.generate(prompt, 12, speculative=speculative)

    for temperature in (0.0, 0.05):
        for speculative in (True, False):
            assert torch.equal(run(temperature, 3, speculative), run(temperature, 3, speculative))
    assert not torch.equal(run(0.05, 3, True), run(0.05, 4, True))
