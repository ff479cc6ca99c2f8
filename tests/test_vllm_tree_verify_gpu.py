"""vLLM's GDN / Mamba2 spec rows through the tree-verify extension on a B200 (this package's kernels, bf16 inputs)
against the same extension on CPU (the float64 definitions): one tree round, the commit of its accepted paths and the
next round."""

import types

import pytest
import torch

from tests.test_vllm_tree_verify import PARENTS, QSL, STATE_INDICES

pytestmark = pytest.mark.gpu
KW = 4


def _case(kind, g):
    from eagle4_b200.plugins.common import GdnShape
    from eagle4_b200.plugins.vllm import tree_verify as tv

    if kind == "gdn":  # head sizes the kernels serve (K 64 / 128)
        shape = GdnShape(2, 4, 64, 64, KW)
        channels, heads, out_dim = shape.gdn_conv_dim, 4, shape.gdn_value_dim
        ssm = torch.randn(12, 4, 64, 64, generator=g) * 0.1
    else:
        shape = tv.MambaShape(4, 64, 128, 2, KW)
        channels, heads, out_dim = shape.mamba_inner + 2 * 2 * 128, 4, shape.mamba_inner
        ssm = torch.randn(12, 4, 64, 128, generator=g) * 0.1
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731 - activations and conv weights are bf16 on the GPU
    params = {"A_log": torch.randn(heads, generator=g) * 0.5, "dt_bias": torch.randn(heads, generator=g) * 0.5,
              "D": torch.randn(heads, generator=g), "weight": bf(torch.randn(channels, KW, generator=g) * 0.5),
              "bias": bf(torch.randn(channels, generator=g) * 0.5) if kind == "mamba2" else None}
    conv = torch.randn(12, channels, KW - 1 + 4, generator=g)
    return shape, channels, heads, out_dim, params, ssm, conv


def _rows(kind, shape, heads, out_dim, params, ssm, conv, x, gate, num_accepted, qsl, state_indices, dev, act):
    common = dict(conv_state=conv, conv_weight=params["weight"].to(dev, act)[:, None, :],
                  conv_bias=None if params["bias"] is None else params["bias"].to(dev, act), activation="silu",
                  state_indices=state_indices.to(dev), num_accepted_tokens=num_accepted.to(dev),
                  query_start_loc=qsl.to(dev), ssm_state=ssm, layer_name="l0",
                  out=torch.zeros(x.shape[0], out_dim, device=dev, dtype=act))
    if kind == "gdn":
        return types.SimpleNamespace(mixed_qkv=x.to(dev, act), a=gate[0].to(dev, act), b=gate[1].to(dev, act),
                                     A_log=params["A_log"].to(dev), dt_bias=params["dt_bias"].to(dev),
                                     num_k_heads=shape.gdn_k_heads, head_k_dim=shape.gdn_k_dim,
                                     num_v_heads=shape.gdn_v_heads, head_v_dim=shape.gdn_v_dim, **common)
    return types.SimpleNamespace(hidden_states_B_C=x.to(dev, act), dt=gate.to(dev, act),
                                 A=-params["A_log"].to(dev).exp(), D=params["D"].to(dev),
                                 dt_bias=params["dt_bias"].to(dev), num_heads=shape.mamba_heads,
                                 head_dim=shape.mamba_head_dim, n_groups=shape.mamba_groups,
                                 ssm_state_size=shape.mamba_state, **common)


@pytest.mark.parametrize("kind", ["gdn", "mamba2"])
def test_tree_round_on_the_gpu_matches_the_cpu_definition(kind):
    from eagle4_b200.ops import native
    from eagle4_b200.plugins.vllm import tree_verify as tv

    g = torch.Generator().manual_seed(7)
    shape, channels, heads, out_dim, params, ssm0, conv0 = _case(kind, g)
    bf = lambda t: t.to(torch.bfloat16).float()  # noqa: E731 - both runs read the same bf16-rounded inputs
    x1, x2 = bf(torch.randn(9, channels, generator=g)), bf(torch.randn(2, channels, generator=g))
    if kind == "gdn":
        gate1 = (bf(torch.randn(9, heads, generator=g)), bf(torch.randn(9, heads, generator=g)))
        gate2 = (bf(torch.randn(2, heads, generator=g)), bf(torch.randn(2, heads, generator=g)))
    else:
        gate1, gate2 = bf(torch.randn(9, heads, generator=g)), bf(torch.randn(2, heads, generator=g))
    outs = {}
    for where in ("cpu", "cuda"):
        dev = torch.device(where)
        act = torch.float32 if where == "cpu" else torch.bfloat16
        # both runs start from the same bf16-rounded values
        ssm, conv = ssm0.clone().to(dev), conv0.to(torch.bfloat16).to(dev, act)
        xs1, xs2 = x1, x2
        ext = tv.TreeVerify()
        tv.stage_tree(PARENTS.to(dev))
        r1 = _rows(kind, shape, heads, out_dim, params, ssm, conv, xs1, gate1, torch.tensor([2, 1], dtype=torch.int32),
                   QSL, STATE_INDICES, dev, act)
        (ext.forward_spec_rows if kind == "gdn" else ext.forward_mamba2_spec_rows)(r1)
        tv.commit_accepted(torch.tensor([[0, 2, 4, -1, -1], [0, 1, -1, -1, -1]], device=dev),
                           torch.tensor([3, 2], device=dev))
        tv.stage_tree(None)
        r2 = _rows(kind, shape, heads, out_dim, params, ssm, conv, xs2, gate2, torch.tensor([3, 2], dtype=torch.int32),
                   torch.tensor([0, 1, 2]), STATE_INDICES, dev, act)
        (ext.forward_spec_rows if kind == "gdn" else ext.forward_mamba2_spec_rows)(r2)
        if where == "cuda":
            torch.cuda.synchronize()
            native.check_errors()
        outs[where] = (r1.out.float().cpu(), r2.out.float().cpu(), ssm.float().cpu())
    for got, want in zip(outs["cuda"], outs["cpu"]):
        err = (got - want).abs().max().item()
        assert err <= 3e-2 * (want.abs().max().item() + 1e-6), err
