"""Host plugins against generated fake hosts: hook checks, refusal on a changed hook, registration, and the
adapters' tree-verify and accept pieces on CPU tensors.

The fakes are written from each adapter's own hook table (every hooked attribute with the listed parameters) plus
the registry behaviour registration needs; the real hosts (hook-carrying SGLang, vLLM >= 0.32, TokenSpeed) are not
installable offline.
"""

import importlib
import sys

import torch

from tests import fake_hosts


def _install(tmp_path, monkeypatch, hooks, extra, top):
    root = tmp_path / "hosts"
    fake_hosts.write_fake_host(str(root), hooks, extra)
    monkeypatch.syspath_prepend(str(root))
    for name in [m for m in sys.modules if m == top or m.startswith(top + ".")]:
        monkeypatch.delitem(sys.modules, name)
    importlib.invalidate_caches()


def test_adapter_overrides_match_hook_tables():
    from eagle4_b200.plugins.sglang.hooks import adapter_problems
    from eagle4_b200.plugins.tokenspeed.hooks import adapter_problems as tokenspeed_problems

    assert adapter_problems() == []
    assert tokenspeed_problems() == []


def test_sglang_registers_on_matching_host(tmp_path, monkeypatch):
    from eagle4_b200.plugins.sglang import hooks

    _install(tmp_path, monkeypatch, hooks.HOOKS, fake_hosts.SGLANG_REGISTRY, "sglang")
    assert hooks.hook_problems() == []
    from eagle4_b200.plugins.sglang import plugin

    assert plugin.register() is True
    from sglang.srt.models.registry import ModelRegistry
    from sglang.srt.speculative.spec_info import SpeculativeAlgorithm

    fn, spec_class, overlap = SpeculativeAlgorithm.from_string("EAGLE_HARNESS")
    assert overlap and spec_class.__name__ == "HarnessSpecAlgo"
    assert fn(None).__name__ == "HarnessWorker"
    assert ModelRegistry.packages == [plugin.MODEL_PACKAGE]
    assert plugin.register() is True  # idempotent


def test_sglang_refuses_changed_hook(tmp_path, monkeypatch):
    from eagle4_b200.plugins.contract import Hook
    from eagle4_b200.plugins.sglang import hooks

    changed = [Hook(h.path, h.params[:-1], h.kind, h.owner, h.optional)
               if h.path.endswith("recurrent_update") else h for h in hooks.HOOKS]
    _install(tmp_path, monkeypatch, changed, fake_hosts.SGLANG_REGISTRY, "sglang")
    problems = hooks.hook_problems()
    assert problems and "recurrent_update" in problems[0]
    from eagle4_b200.plugins.sglang import plugin

    assert plugin.register() is False


def test_vllm_and_tokenspeed_register(tmp_path, monkeypatch):
    from eagle4_b200.plugins.contract import EXISTS, Hook
    from eagle4_b200.plugins.tokenspeed import hooks as th
    from eagle4_b200.plugins.vllm import hooks as vh

    vhooks = [Hook(u.hook.split("|")[0].strip(), (), EXISTS) for u in vh.HOOK_MAP if u.hook]
    vextra = {"vllm": ['__version__ = "0.32.0rc1.dev300"'],
              "vllm.v1.spec_decode.registry": ["REG = {}\ndef register_speculative_method(name, spec, speculator=None):"
                                               "\n    REG[name] = (spec, speculator)"]}
    _install(tmp_path, monkeypatch, vhooks, vextra, "vllm")
    assert vh.missing_hooks() == []
    from eagle4_b200.plugins.vllm import plugin as vp

    assert vp.register() is True
    from vllm.v1.spec_decode.registry import REG

    assert "eagle_harness" in REG
    _install(tmp_path, monkeypatch, list(th.HOOKS) + list(th.RELEASE_HOOKS), {"tokenspeed": ["__version__ = \"0.1.1\""]}, "tokenspeed")
    assert th.contract() == "release" and th.hook_problems() == []
    from eagle4_b200.plugins.tokenspeed import plugin as tp

    assert tp.register() is True


def test_gdn_tree_verify_extension_matches_model_path():
    """The SGLang GDN extension's conv + recurrence on host-layout inputs equals the engine's fused GDN verify."""
    from eagle4_b200 import ops
    from eagle4_b200.models import configs
    from eagle4_b200.ops import reference as ref
    from eagle4_b200.plugins.sglang.adapter import GdnTreeVerify

    cfg = configs.tiny_hybrid()
    g = torch.Generator().manual_seed(0)
    t, cd, hv = 6, cfg.gdn_conv_dim, cfg.gdn_v_heads
    x = torch.randn(t, cd, generator=g)
    conv_w = torch.randn(cd, cfg.conv_kernel, generator=g) * 0.3
    conv_states = torch.randn(2, cd, cfg.conv_kernel - 1, generator=g)
    ssm = torch.randn(2, hv, cfg.gdn_v_dim, cfg.gdn_k_dim, generator=g) * 0.1
    a = torch.randn(t, hv, generator=g)
    b = torch.randn(t, hv, generator=g)
    a_log = torch.rand(hv, generator=g).log()
    dt_bias = torch.ones(hv)

    class Layout:
        parent_token = torch.tensor([-1, 0, 0, -1, 0, 1])  # two requests of 3 rows each
        query_start_loc = torch.tensor([0, 3, 6])
        cache_indices = torch.tensor([1, 0])

    class Conv:
        weight = conv_w[:, None, :]

    class Layer:
        conv1d = Conv()
        num_k_heads, num_v_heads, head_k_dim, head_v_dim = cfg.gdn_k_heads, hv, cfg.gdn_k_dim, cfg.gdn_v_dim

    Layer.A_log, Layer.dt_bias = a_log, dt_bias

    ext = GdnTreeVerify()
    ext.begin_forward(Layout(), in_graph=False)
    conv = ext.conv_update(Layer(), x, conv_states, Layout.cache_indices, None, None)
    q = conv[:, : cfg.gdn_key_dim]
    out = ext.recurrent_update(Layer(), q, None, None, a, b, ssm, Layout.cache_indices, Layout.query_start_loc, None,
                               None)
    parent = torch.tensor([-1, 0, 0, -1, 3, 4], dtype=torch.int32)
    slots = torch.tensor([1, 1, 1, 0, 0, 0], dtype=torch.int32)
    want_conv = ref.causal_conv_tree(x, conv_states, slots, parent, conv_w)
    gg, beta = ref.gdn_gates(a, b, a_log, dt_bias)
    want = ref.gdn_tree(want_conv, gg, beta, ssm, slots, parent, cfg, False).reshape(t, -1)
    torch.testing.assert_close(conv, want_conv)
    torch.testing.assert_close(out, want)
