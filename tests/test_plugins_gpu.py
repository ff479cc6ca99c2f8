"""The host adapters' GDN tree-verify path on the GPU (sm_100a conv + raw recurrence kernels) vs float64."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_gdn_extension_kernels_match_reference():
    from eagle4_b200.models import configs
    from eagle4_b200.ops import reference as ref
    from eagle4_b200.plugins.sglang.adapter import GdnTreeVerify

    cfg = configs.qwen38_27b()
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(0)
    t, cd, hv = 8, cfg.gdn_conv_dim, cfg.gdn_v_heads
    x = (torch.randn(t, cd, generator=g)).to(torch.bfloat16)
    conv_w = (torch.randn(cd, cfg.conv_kernel, generator=g) * 0.3).to(torch.bfloat16)
    conv_states = (torch.randn(2, cd, cfg.conv_kernel - 1, generator=g)).to(torch.bfloat16)
    ssm = torch.randn(2, hv, cfg.gdn_v_dim, cfg.gdn_k_dim, generator=g) * 0.05
    a = torch.randn(t, hv, generator=g).to(torch.bfloat16)
    b = torch.randn(t, hv, generator=g).to(torch.bfloat16)
    a_log = torch.rand(hv, generator=g).log()
    dt_bias = torch.ones(hv)

    class Layout:
        parent_token = torch.tensor([-1, 0, 1, 1, -1, 0, 1, 2], device=dev)
        query_start_loc = torch.tensor([0, 4, 8], device=dev)
        cache_indices = torch.tensor([1, 0], device=dev)

    class Conv:
        weight = conv_w[:, None, :].to(dev)

    class Layer:
        conv1d = Conv()
        num_k_heads, num_v_heads, head_k_dim, head_v_dim = cfg.gdn_k_heads, hv, cfg.gdn_k_dim, cfg.gdn_v_dim

    Layer.A_log, Layer.dt_bias = a_log.to(dev), dt_bias.to(dev)
    ext = GdnTreeVerify()
    ext.begin_forward(Layout(), in_graph=False)
    conv = ext.conv_update(Layer(), x.to(dev), conv_states.to(dev), Layout.cache_indices, None, None)
    out = ext.recurrent_update(Layer(), conv[:, : cfg.gdn_key_dim], None, None, a.to(dev), b.to(dev), ssm.to(dev),
                               Layout.cache_indices, Layout.query_start_loc, None, None)
    parent = torch.tensor([-1, 0, 1, 1, -1, 4, 5, 6], dtype=torch.int32)
    slots = torch.tensor([1, 1, 1, 1, 0, 0, 0, 0], dtype=torch.int32)
    want_conv = ref.causal_conv_tree(x, conv_states, slots, parent, conv_w)
    gg, beta = ref.gdn_gates(a, b, a_log, dt_bias)
    want = ref.gdn_tree(conv.cpu(), gg, beta, ssm, slots, parent, cfg, False).reshape(t, -1)
    torch.testing.assert_close(conv.cpu().float(), want_conv.float(), atol=3e-2, rtol=3e-2)
    err = (out.cpu().float() - want.float()).abs().max().item()
    assert err <= 3e-2 * max(1.0, want.float().abs().max().item()), err
