"""What the eagle_harness method installs in vLLM's speculative config (plugins/vllm/schedule.py): draft-token
schedules per batch-size range (tree buckets, narrowed by served tree rounds; served chain widths with native ranges),
``num_speculative_tokens``, the draft's aux layers, and the worker's check of the calibration data's setup."""

import types

import pytest

from eagle4_b200.core.chain_width import merge_tree_rounds, save_accept_profile, save_round_times
from eagle4_b200.core.limits import ComputeIntensity, max_batch_size, verify_buckets
from eagle4_b200.core.live_costs import CostKey, write_key
from eagle4_b200.plugins.vllm import schedule as sch
from eagle4_b200.plugins.vllm.config import parse_method_config

KEY = CostKey(gpu="NVIDIA B200", gpu_count=1, model="t", draft="d", engine="vllm", dtype="bfloat16")


def _spec(method_config, **kw):
    draft = types.SimpleNamespace(architectures=["LlamaForCausalLMEagle4"],
                                  eagle_config={"eagle_aux_hidden_state_layer_ids": [3, 31, 59]})
    return types.SimpleNamespace(method_config=method_config, draft_model_config=types.SimpleNamespace(hf_config=draft),
                                 num_speculative_tokens=kw.get("k"), num_speculative_tokens_per_batch_size=kw.get("s"))


def test_static_tree_installs_no_schedule_and_the_full_width():
    spec = _spec({"mode": "static", "node_top_k": 4, "tree_depth": 14, "max_verify_width": 16})
    sch.configure_speculative_config(spec)
    assert spec.num_speculative_tokens_per_batch_size is None and spec.num_speculative_tokens == 15
    assert spec.draft_model_config.hf_config.eagle_aux_hidden_state_layer_ids == [4, 32, 60]


def test_serve_tree_schedule_from_verify_buckets():
    spec = _spec({"max_verify_width": 32})
    sch.configure_speculative_config(spec)
    s = spec.num_speculative_tokens_per_batch_size
    limit = max_batch_size(ComputeIntensity.HIGH)
    assert s[0][0] == 1 and s[-1] == (limit + 1, sch.NO_DRAFT_ABOVE, 0)
    for bs in (1, 3, 8, 9, 64, limit):
        k = sch.width_at(s, bs)
        assert k + 1 <= min(max(verify_buckets(bs, ComputeIntensity.HIGH)), 32)
    assert sch.width_at(s, 1) == 31 and spec.num_speculative_tokens == 31
    widths = [k for _, _, k in s]
    assert widths == sorted(widths, reverse=True)  # never wider at a larger batch


def test_served_tree_rounds_narrow_the_schedule(tmp_path):
    # at batch 64 width 8 yields more tokens per microsecond than width 16 in many rounds
    rows = [{"batch_size": b, "width": w, "round_us": us, "accept": acc, "count": 500}
            for b, w, us, acc in ((64, 16, 30000.0, 2.0), (64, 8, 20000.0, 1.9), (1, 16, 15000.0, 3.0),
                                  (1, 8, 12000.0, 2.0))]
    merge_tree_rounds(str(tmp_path), rows)
    write_key(str(tmp_path), KEY)
    method = parse_method_config({"max_verify_width": 16, "data_path": str(tmp_path)})
    widths = sch.verify_widths(method)
    assert sch.width_at(widths, 1) == 16 and sch.width_at(widths, 64) == 8
    sch.check_data_key(_spec({"max_verify_width": 16, "data_path": str(tmp_path)}), KEY)
    with pytest.raises(ValueError, match="another setup"):
        sch.check_data_key(_spec({"max_verify_width": 16, "data_path": str(tmp_path)}),
                           CostKey(**{**KEY.to_dict(), "gpu_count": 8}))


def _chain_data(path):
    save_accept_profile(path, 1000, [800, 600, 450, 300, 200, 120, 60, 30, 10, 5, 2, 1, 0, 0, 0])
    rows = []
    for b, native, plain, w4 in ((1, 9000.0, 10000.0, 11000.0), (64, 20000.0, 30000.0, 60000.0)):
        rows += [{"batch_size": b, "width": 0, "round_us": native, "count": 50},
                 {"batch_size": b, "width": 1, "round_us": plain, "count": 50},
                 {"batch_size": b, "width": 4, "round_us": w4, "count": 50}]
    save_round_times(path, rows)


def test_chain_schedule_with_native_ranges(tmp_path):
    _chain_data(str(tmp_path))
    spec = _spec({"intensity": "chain_intensity", "data_path": str(tmp_path)})
    sch.configure_speculative_config(spec)
    s = spec.num_speculative_tokens_per_batch_size
    assert sch.width_at(s, 1) == 3  # width 4 pays at batch 1: 3 drafts
    assert sch.width_at(s, 64) == 0 and sch.width_at(s, 512) == 0
    native = sch.installed_native_ranges(spec)
    assert native and any(a <= 64 <= b for a, b in native) and not any(a <= 1 <= b for a, b in native)
    assert spec.num_speculative_tokens == 3
    user = _spec({"intensity": "chain_intensity", "data_path": str(tmp_path)}, s=[(1, 512, 2)])
    sch.configure_speculative_config(user)
    assert user.num_speculative_tokens_per_batch_size == [(1, 512, 2)] and sch.installed_native_ranges(user) == []


def test_unpriced_chain_needs_an_explicit_width_and_widths_must_agree():
    with pytest.raises(ValueError, match="no priced chain schedule"):
        sch.configure_speculative_config(_spec({"intensity": "chain_intensity"}))
    spec = _spec({"intensity": "chain_intensity", "max_verify_width": 6})
    sch.configure_speculative_config(spec)
    assert sch.width_at(spec.num_speculative_tokens_per_batch_size, 100) == 5
    with pytest.raises(ValueError, match="disagrees"):
        sch.configure_speculative_config(_spec({"mode": "static", "max_verify_width": 16}, k=7))
    ok = _spec({"mode": "static", "max_verify_width": 16}, k=15)
    sch.configure_speculative_config(ok)


def test_method_spec_configure_fills_the_config():
    from eagle4_b200.plugins.vllm.adapter import HarnessMethodSpec

    spec = _spec({"max_verify_width": 32})
    out = HarnessMethodSpec().configure(spec)
    assert spec.num_speculative_tokens_per_batch_size and out["num_speculative_tokens"] == spec.num_speculative_tokens


def test_speculator_load_checks_layers_and_the_data_key(tmp_path):
    import dataclasses

    from eagle4_b200.models import configs, weights
    from eagle4_b200.models.draft import DraftModel
    from eagle4_b200.plugins.vllm.adapter import HarnessSpeculator

    tc = configs.tiny_hybrid()
    dc = configs.tiny_draft(tc, draft_vocab=4096)
    draft = DraftModel(dc, weights.init_draft(dc, seed=2))

    class QwenGatedDeltaNetAttention:
        pass

    class ShortConv:
        pass

    method = parse_method_config({"mode": "static", "node_top_k": 2, "tree_depth": 4, "max_verify_width": 8})
    HarnessSpeculator().load_model(draft, max_reqs=2, max_len=128, method=method,
                                   linear_layers=[QwenGatedDeltaNetAttention()])
    with pytest.raises(RuntimeError, match="ShortConv"):
        HarnessSpeculator().load_model(draft, max_reqs=2, max_len=128, method=method, linear_layers=[ShortConv()])
    rows = [{"batch_size": 1, "width": 8, "round_us": 9000.0, "accept": 2.0, "count": 10},
            {"batch_size": 1, "width": 4, "round_us": 8000.0, "accept": 1.5, "count": 10}]
    merge_tree_rounds(str(tmp_path), rows)
    write_key(str(tmp_path), KEY)
    keyed = dataclasses.replace(method, harness=dataclasses.replace(method.harness, data_path=str(tmp_path)))
    HarnessSpeculator().load_model(draft, max_reqs=2, max_len=128, method=keyed, key=KEY)
    with pytest.raises(ValueError, match="another setup"):
        HarnessSpeculator().load_model(draft, max_reqs=2, max_len=128, method=keyed,
                                       key=CostKey(**{**KEY.to_dict(), "gpu": "other"}))
