"""The latent-MoE expert kernels (csrc/moe.cu) against the PyTorch definition, their batch invariance, and a
Nemotron-class draft (attn_norm + latent MoE) serving speculative == plain on the GPU."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(T, E, k, L, F, seed=0):
    from eagle4_b200.ops import reference as ref

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(seed)
    latent = (torch.randn(T, L, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    up = (torch.randn(E, F, L, generator=g, device=dev) * L ** -0.5).to(torch.bfloat16)
    down = (torch.randn(E, L, F, generator=g, device=dev) * F ** -0.5).to(torch.bfloat16)
    gate = torch.randn(E, L, generator=g, device=dev)
    bias = torch.randn(E, generator=g, device=dev) * 0.1
    chosen, w = ref.moe_route(latent.float(), gate, bias, k)
    return latent, chosen, w * 2.0, up, down


@pytest.mark.parametrize("shape", [(5, 16, 4, 64, 96), (4, 512, 22, 1024, 2688), (64, 512, 22, 1024, 2688)])
def test_moe_experts_match_definition(shape):
    from eagle4_b200.ops import native
    from eagle4_b200.ops import reference as ref

    latent, chosen, w, up, down = _case(*shape)
    got = native.moe_experts(latent, chosen, w, up, down).float()
    want = ref.moe_experts(latent, chosen, w, up, down).float()
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert err < 2e-2, err
    native.check_errors(latent.device)


def test_moe_experts_rows_do_not_depend_on_the_batch():
    from eagle4_b200.ops import native

    latent, chosen, w, up, down = _case(48, 512, 22, 1024, 2688, seed=3)
    full = native.moe_experts(latent, chosen, w, up, down)
    for t in (0, 17, 47):
        one = native.moe_experts(latent[t:t + 1].contiguous(), chosen[t:t + 1], w[t:t + 1], up, down)
        assert torch.equal(one[0], full[t])


def test_moe_draft_spec_equals_plain_on_gpu():
    from eagle4_b200.api import LLM, TreeSpec
    from eagle4_b200.ops import native

    llm = LLM.synthetic("tiny-moe", device="cuda", tree=TreeSpec(4, 2, 8), max_batch=2, max_len=512)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(1, 4096, (40,), generator=g), torch.randint(1, 4096, (70,), generator=g)]
    spec = llm.generate(prompts, 16)
    plain = llm.generate(prompts, 16, speculative=False)
    assert torch.equal(spec, plain)
    native.check_errors(torch.device("cuda"))
