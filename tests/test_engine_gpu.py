"""The serving loop on the GPU kernels: greedy speculative output equals plain greedy decode, token for token,
on the tiny hybrid in bf16 (every target op is batch-invariant and plain decode is a one-row verify)."""

import pytest
import torch

from eagle4_b200.models import configs, weights
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.target import TargetModel
from eagle4_b200.runtime.engine import Engine

pytestmark = pytest.mark.gpu


def _models(dev="cuda"):
    tc = configs.tiny_hybrid()
    dc = configs.tiny_draft(tc)
    tw = weights.init_target(tc, device=dev, dtype=torch.bfloat16, seed=0)
    dw = weights.init_draft(dc, device=dev, dtype=torch.bfloat16, seed=1, embed=tw["embed"])
    return TargetModel(tc, tw, aux_layer_ids=dc.aux_layer_ids), DraftModel(dc, dw)


def test_gpu_spec_equals_plain():
    from eagle4_b200.ops import native

    tgt, drf = _models()
    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, tgt.cfg.vocab_size, (2, 64), generator=g).tolist()
    spec = Engine(tgt, drf, max_reqs=2, max_len=160, steps=4, top_k=2, verify_tokens=8)
    out_spec = spec.generate(prompts, 48, speculative=True)
    plain = Engine(tgt, drf, max_reqs=2, max_len=160, steps=4, top_k=2, verify_tokens=8)
    out_plain = plain.generate(prompts, 48, speculative=False)
    native.check_errors()
    assert out_spec == out_plain


def test_gpu_matches_cpu_reference_logits():
    """The bf16 GPU forward and the fp32 CPU oracle agree on the same weights: the final hidden states are nearly
    parallel and the GPU's greedy token is within bf16 rounding of the oracle's best logit."""
    from eagle4_b200.models.target import RowBatch, TargetCache

    tgt, _ = _models()
    cpu_w = {k: v.float().cpu() for k, v in tgt.w.items()}
    tcpu = TargetModel(tgt.cfg, cpu_w)
    n = 32
    ids = torch.randint(0, tgt.cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(3))

    def run(model, dev):
        pos = torch.arange(n, device=dev)
        one = lambda v: torch.full((n,), v, dtype=torch.int32, device=dev)  # noqa: E731
        rb = RowBatch(ids=ids.to(dev), pos=pos, req=one(0), write_slot=pos.long(), ctx_start=one(0),
                      ctx_len=(pos + 1).int(), extra=torch.zeros(n, 1, dtype=torch.int32, device=dev),
                      n_extra=one(0), parent=(pos - 1).int(), state_slot=one(0), scan=True)
        cache = TargetCache.allocate(model.cfg, max_reqs=1, max_len=64, page=16, device=dev,
                                     dtype=model.w["embed"].dtype)
        out, _ = model.forward(rb, cache)
        return out[-1:].float().cpu(), model.greedy(out[-1:])[0].cpu()

    hg, tok_g = run(tgt, "cuda")
    hc, _ = run(tcpu, "cpu")
    cos = torch.nn.functional.cosine_similarity(hg, hc).item()
    assert cos > 0.999
    logits = hc @ cpu_w["lm_head"].t()
    assert logits[0, tok_g].item() >= logits.max().item() - 0.05 * logits.abs().max().item()
