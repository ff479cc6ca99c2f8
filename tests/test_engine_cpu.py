"""Config 1 of the benchmark plan on CPU: speculative output equals plain greedy decoding, token for token."""

import torch

from eagle4_b200.models import configs, weights
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.target import TargetModel
from eagle4_b200.runtime.engine import Engine


def _models(seed=0):
    tc = configs.tiny_hybrid()
    dc = configs.tiny_draft(tc)
    tw = weights.init_target(tc, seed=seed)
    dw = weights.init_draft(dc, seed=seed + 1, embed=tw["embed"])
    return TargetModel(tc, tw, aux_layer_ids=dc.aux_layer_ids), DraftModel(dc, dw)


def test_spec_equals_plain_tiny_hybrid():
    tgt, drf = _models()
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, tgt.cfg.vocab_size, (2, 64), generator=g).tolist()
    spec = Engine(tgt, drf, max_reqs=2, max_len=128, steps=4, top_k=2, verify_tokens=8)
    out_spec = spec.generate(prompts, 32, speculative=True)
    plain = Engine(tgt, drf, max_reqs=2, max_len=128, steps=4, top_k=2, verify_tokens=8)
    out_plain = plain.generate(prompts, 32, speculative=False)
    assert out_spec == out_plain
    assert all(len(o) == 32 for o in out_spec)
    assert spec.stats.rounds < 32  # fewer rounds than tokens: every round emits at least one token


def test_spec_accepts_oracle_draft():
    """A draft whose first candidate is the target's true greedy continuation is accepted along whole paths:
    the accept walk, the KV moves and the recurrent-state replay of multi-row paths give plain greedy output."""
    tgt, drf = _models(seed=3)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, tgt.cfg.vocab_size, (1, 16), generator=g).tolist()
    plain = Engine(tgt, drf, max_reqs=1, max_len=96, steps=4, top_k=2, verify_tokens=8)
    ref = plain.generate(prompts, 24, speculative=False)[0]
    seq = prompts[0] + ref + [0] * 16
    cand = drf.candidates

    def candidates(normed, k, pos):
        want = torch.tensor([seq[int(p) + 2] for p in pos])
        ids = torch.stack([want] + [(want + j) % tgt.cfg.vocab_size for j in range(1, k)], dim=1)
        probs = torch.tensor([[0.9] + [0.1 / (k - 1)] * (k - 1)]).expand(normed.shape[0], k)
        return probs, ids

    drf.candidates = candidates
    eng = Engine(tgt, drf, max_reqs=1, max_len=96, steps=4, top_k=2, verify_tokens=8)
    out = eng.generate(prompts, 24, speculative=True)[0]
    drf.candidates = cand
    assert out == ref
    assert eng.stats.mean_accept > 3.0  # depth-4 trees: root + 3 drafted levels + bonus per round
