"""Draft config validation, window resolution and HF -> DraftConfig conversion (the released draft config)."""

import copy
import json
import os

import pytest

from eagle4_b200.models import configs
from eagle4_b200.models.eagle4_config import (check_supported, draft_config_from_hf, resolve_draft_sliding_window,
                                              validate_eagle4_draft_config)

RELEASED = configs.qwen38_draft(configs.qwen38_27b()).to_hf()


def test_released_shape_round_trips():
    dc = draft_config_from_hf(RELEASED)
    assert dc.sliding_window == 4096 and dc.aux_layer_ids == (3, 31, 59)
    assert dc.num_candidates == 128 and dc.rank == 128 and dc.head_dim == 128


def test_unknown_structural_key_refused():
    bad = dict(RELEASED, new_fancy_fusion=True)
    with pytest.raises(ValueError, match="does not implement"):
        validate_eagle4_draft_config(bad)


def test_window_rules():
    c = dict(RELEASED)
    c.pop("layer_types")
    c["use_sliding_window"] = False
    assert resolve_draft_sliding_window(c) is None
    c["use_sliding_window"] = True
    c.pop("sliding_window")
    with pytest.raises(ValueError):
        resolve_draft_sliding_window(c)
    c = dict(RELEASED, layer_types=["full_attention"])
    assert resolve_draft_sliding_window(c) is None


def test_aux_and_head_checks():
    c = copy.deepcopy(RELEASED)
    c["eagle_config"]["eagle_aux_hidden_state_layer_ids"] = [1, 2]
    with pytest.raises(ValueError):
        validate_eagle4_draft_config(c)
    c = dict(RELEASED, efficient_lm_head_config={"type": "svd", "rank": 1})
    with pytest.raises(ValueError):
        validate_eagle4_draft_config(c)
    with pytest.raises(NotImplementedError):
        check_supported(dict(RELEASED, enable_moe=True, hidden_act="silu", scoring_func="sigmoid",
                             topk_method="noaux_tc"))


def test_reference_profile_config_parses():
    """The draft config shipped with the reference's profiles (the package installed under ``baseline/_ref``)."""
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    path = os.path.join(root, "eagle_harness", "core", "profiles", "mi355x-qwen3.8-27b-tp1", "draft_config.json")
    if not os.path.exists(path):
        pytest.skip("the reference package is not installed under baseline/_ref")
    dc = draft_config_from_hf(json.load(open(path)))
    assert dc.hidden_size == 5120 and dc.sliding_window == 4096
