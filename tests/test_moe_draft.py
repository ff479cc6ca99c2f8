"""Nemotron-class EAGLE-4 draft structures: the latent ReLU^2 MoE MLP and the attn_norm (eh_proj) input fusion.

The MoE block is checked against the block computed expert by expert (sigmoid router, top-k over bias-corrected
scores, renormalised unbiased weights, routed ReLU^2 experts in the latent space, routed scale before
fc2_latent_proj, ReLU^2 shared expert after: the formula of the reference's
tests/test_eagle4_model.py:370-392), grouped routing against its definition, the config and checkpoint layouts by
round trips, and the engine by speculative == plain greedy decoding."""

import pytest
import torch

from eagle4_b200 import ops
from eagle4_b200.api import LLM, TreeSpec
from eagle4_b200.models import configs, weights
from eagle4_b200.models.eagle4_config import check_supported, draft_config_from_hf
from eagle4_b200.ops import reference as ref


def _block(x, w, moe):
    """The block expert by expert, in float64."""
    x = x.double()
    scores = torch.sigmoid(x @ w["moe_gate"].double().T)
    chosen = torch.topk(scores + w["moe_bias"].double(), moe["top_k"], dim=-1).indices
    wts = torch.gather(scores, -1, chosen)
    wts = wts / wts.sum(-1, keepdim=True)
    latent = x @ w["fc1_latent"].double().T
    routed = torch.zeros_like(latent)
    for t in range(x.shape[0]):
        for j in range(moe["top_k"]):
            e = int(chosen[t, j])
            up = torch.relu(latent[t] @ w["experts_up"][e].double().T) ** 2
            routed[t] += wts[t, j] * (up @ w["experts_down"][e].double().T)
    shared = torch.relu(x @ w["shared_up"].double().T) ** 2 @ w["shared_down"].double().T
    return (moe["scale"] * routed) @ w["fc2_latent"].double().T + shared


def _moe_weights(H=64, E=12, F=40, L=24, S=48, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: (torch.randn(*s, generator=g) * 0.3).to(dtype)  # noqa: E731
    return {"moe_gate": r(E, H).float(), "moe_bias": r(E).float(), "fc1_latent": r(L, H), "fc2_latent": r(H, L),
            "experts_up": r(E, F, L), "experts_down": r(E, L, F), "shared_up": r(S, H), "shared_down": r(H, S)}


def test_latent_moe_block_matches_the_expert_by_expert_formula():
    moe = configs.latent_moe(12, 3, 40, 24, 48, scale=5.0)
    w = _moe_weights()
    x = torch.randn(7, 64, generator=torch.Generator().manual_seed(1))
    got = ops.latent_moe(x, w, moe, torch.zeros(7, 64))
    want = _block(x, w, moe)
    assert torch.allclose(got.double(), want, rtol=2e-4, atol=2e-4 * want.abs().max().item())
    # the expert index mapping is load-bearing: rolling the banks changes the function
    w2 = dict(w, experts_up=w["experts_up"].roll(1, 0))
    assert not torch.allclose(ops.latent_moe(x, w2, moe, torch.zeros(7, 64)), got)


def test_grouped_routing_picks_experts_from_the_best_groups_only():
    g = torch.Generator().manual_seed(2)
    x, gate, bias = torch.randn(9, 16, generator=g), torch.randn(16, 16, generator=g), torch.randn(16, generator=g)
    chosen, w = ref.moe_route(x, gate, bias, top_k=4, n_group=4, topk_group=2)
    biased = torch.sigmoid(x @ gate.T) + bias
    best_groups = biased.view(9, 4, 4).topk(2, dim=-1).values.sum(-1).topk(2, dim=-1).indices
    for t in range(9):
        assert set((chosen[t] // 4).tolist()) <= set(best_groups[t].tolist())
    assert torch.allclose(w.sum(-1), torch.ones(9))
    flat, _ = ref.moe_route(x, gate, bias, top_k=4)
    assert torch.equal(flat, biased.topk(4, dim=-1).indices)


def test_config_round_trip_and_refusals():
    d = configs.tiny_moe_draft(configs.tiny_nemotron())
    hf = d.to_hf()
    back = draft_config_from_hf(hf, target_vocab_size=d.vocab_size)
    assert back.attn_norm and back.moe == d.moe
    for bad in ({"enable_post_mlp_norm": True}, {"moe_architecture": "sparse_swiglu", "hidden_act": "silu"}):
        with pytest.raises(NotImplementedError):
            check_supported({**hf, **bad})


def test_checkpoint_names_round_trip(tmp_path):
    t = configs.tiny_nemotron()
    d = configs.tiny_moe_draft(t)
    w = weights.init_draft(d, seed=3)
    weights.save_draft(str(tmp_path), d, w)
    back = weights.load_draft(str(tmp_path), d, embed=w["embed"])
    for k in ("eh_proj", "pre_attention_layernorm", "moe_gate", "moe_bias", "fc1_latent", "fc2_latent",
              "experts_up", "experts_down", "shared_up", "shared_down", "qkv"):
        assert torch.equal(back[k], w[k]), k
    # released checkpoints spell the layer "midlayer."
    sd = {k.replace("layers.0.", "midlayer."): v for k, v in weights.draft_state_dict(d, w).items()}
    legacy = weights.draft_from_state_dict(d, sd, embed=w["embed"])
    assert torch.equal(legacy["experts_down"], w["experts_down"])


@pytest.mark.parametrize("bs", [1, 3])
def test_moe_draft_speculative_equals_plain(bs):
    llm = LLM.synthetic("tiny-moe", device="cpu", dtype=torch.float32, tree=TreeSpec(4, 2, 8), max_batch=bs,
                        max_len=256)
    g = torch.Generator().manual_seed(bs)
    prompts = [torch.randint(1, 4096, (int(torch.randint(6, 30, (1,), generator=g)),), generator=g)
               for _ in range(bs)]
    spec = llm.generate(prompts, 10)
    plain = llm.generate(prompts, 10, speculative=False)
    assert torch.equal(spec, plain)


def test_moe_draft_shards_replicated():
    from eagle4_b200.parallel.sharding import shard_draft

    d = configs.tiny_moe_draft(configs.tiny_nemotron())
    w = weights.init_draft(d, seed=4)
    loc, sw = shard_draft(d, w, 2, 1)
    assert loc.num_heads == d.num_heads // 2 and loc.moe == d.moe
    assert sw["experts_up"] is w["experts_up"] and sw["eh_proj"] is w["eh_proj"]
