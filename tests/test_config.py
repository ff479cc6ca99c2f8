"""The configuration reader: same keys and defaults as the reference, unknown and removed keys refused by name,
every problem of a configuration reported at once."""

import json

import pytest

from eagle4_b200.core.config import (ConfigError, HarnessConfig, Mode, config_to_dict, harness_config_from_dict,
                                     parse_harness_config)
from eagle4_b200.core.limits import ComputeIntensity


def test_defaults_and_round_trip(tmp_path):
    c = parse_harness_config(None)
    assert c == HarnessConfig() and c.mode is Mode.SERVE and c.intensity is ComputeIntensity.HIGH
    d = config_to_dict(c)
    assert d["cost_model"]["chain_tiny"] == [2.6, 0.24, 0.0] and d["l2_warm"]["down_proj"] is None
    assert harness_config_from_dict(d) == c
    p = tmp_path / "cfg.json"
    p.write_text(json.dumps({"mode": "static", "cost_model": {"threshold": 3}}))
    c2 = parse_harness_config(str(p))
    assert c2.mode is Mode.STATIC and c2.cost_model.threshold == 3.0 and isinstance(c2.cost_model.threshold, float)


def test_default_data_path_fills_serve_mode_only():
    assert parse_harness_config("", default_data_path="/p").data_path == "/p"
    assert parse_harness_config('{"mode": "serve"}', default_data_path="/p").data_path == "/p"
    assert parse_harness_config('{"mode": "static"}', default_data_path="/p").data_path is None
    assert parse_harness_config('{"data_path": "/q"}', default_data_path="/p").data_path == "/q"


def test_unknown_removed_and_mistyped_keys_reported_together():
    with pytest.raises(ConfigError) as e:
        harness_config_from_dict({"ragged": True, "cost_model": {"ragged_draft_relax": 1, "thresh": 2},
                                  "mode": "fast", "max_verify_batch_size": "8",
                                  "l2_warm": {"gate_up_gdn": [0.5]}})
    msg = str(e.value)
    assert len(e.value.problems) == 6
    for part in ("ragged was removed", "cost_model.ragged_draft_relax was removed", "'thresh'",
                 "mode must be one of", "max_verify_batch_size must be an integer", "l2_warm.gate_up_gdn must be"):
        assert part in msg, (part, msg)
    with pytest.raises(ValueError, match="mode: eval was removed"):
        harness_config_from_dict({"mode": "eval"})
    with pytest.raises(ValueError, match="true or false"):
        harness_config_from_dict({"draft_model": {"embed_full": 1}})
    with pytest.raises(ValueError, match="JSON object"):
        parse_harness_config("[1, 2]")
    with pytest.raises(ValueError, match="no valid JSON"):
        parse_harness_config("{bad")
    with pytest.raises(ValueError, match="mode calibrate writes its tables under data_path"):
        harness_config_from_dict({"mode": "calibrate"})
