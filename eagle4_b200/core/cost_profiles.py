"""Cost profiles packaged with the library for measured (device, model shape, TP) setups.

A profile directory under ``eagle4_b200/core/profiles/`` holds ``profile.json`` (the device names, TP size and dtype
it was measured on, and the structural shape of the target and draft) and a calibration ``data_path`` layout
(``cost/bs_<N>/...``; optionally ``rounds/*.json`` served choices). A setup selects a profile only when all of that
matches; anything else keeps the caller's ordinary calibration path, since a profile for one model must not price
another (the reference's packaged profiles, ``eagle_harness/core/cost_profiles.py:48-107``, match the whole
``config.json``; here the shape signature is compared, so configs that differ only in metadata still match).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Dict, Mapping, Optional

PROFILES = Path(__file__).parent / "profiles"

TARGET_SHAPE_KEYS = ("hidden_size", "num_hidden_layers", "vocab_size", "intermediate_size", "num_attention_heads",
                     "num_key_value_heads", "head_dim", "layer_types", "linear_num_key_heads",
                     "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim", "linear_conv_kernel_dim",
                     "full_attention_interval", "hybrid_override_pattern", "mamba_num_heads", "mamba_head_dim",
                     "ssm_state_size", "num_experts", "n_routed_experts")
DRAFT_SHAPE_KEYS = ("hidden_size", "num_hidden_layers", "vocab_size", "draft_vocab_size", "intermediate_size",
                    "num_attention_heads", "num_key_value_heads", "head_dim", "target_hidden_size", "sliding_window",
                    "efficient_lm_head_config", "eagle_config")


def shape_signature(config: Mapping[str, Any], keys) -> Dict[str, Any]:
    cfg = dict(config.get("text_config") or config)
    return {k: cfg[k] for k in keys if cfg.get(k) is not None}


def _config(path: str) -> Optional[dict]:
    if not path:
        return None
    p = Path(path)
    p = p / "config.json" if p.is_dir() else p
    if not p.is_file():
        return None
    return json.loads(p.read_text(encoding="utf-8"))


def _matches(profile: Path, *, device_name: str, target: Optional[dict], draft: Optional[dict], tp_size: int,
             dtype: str, quantization: Optional[str]) -> bool:
    meta = json.loads((profile / "profile.json").read_text(encoding="utf-8"))
    if device_name not in meta["devices"] or tp_size != meta["tp_size"] or quantization is not None:
        return False
    if dtype not in ("auto", "bfloat16", "torch.bfloat16", "bf16"):
        return False
    if target is None or draft is None:
        return False
    return (shape_signature(target, TARGET_SHAPE_KEYS) == meta["target_shape"]
            and shape_signature(draft, DRAFT_SHAPE_KEYS) == meta["draft_shape"])


def packaged_cost_profile(*, device_name: str, model_path: str = "", draft_model_path: str = "", tp_size: int,
                          dtype: str, quantization: Optional[str], target_config: Optional[dict] = None,
                          draft_config: Optional[dict] = None) -> Optional[str]:
    """The ``data_path`` of the packaged profile measured on this setup, or None. Configs come from the model
    directories' ``config.json`` or are passed directly."""
    target = target_config if target_config is not None else _config(model_path)
    draft = draft_config if draft_config is not None else _config(draft_model_path)
    if not PROFILES.is_dir():
        return None
    for profile in sorted(PROFILES.iterdir()):
        if (profile / "profile.json").is_file() and _matches(profile, device_name=device_name, target=target,
                                                             draft=draft, tp_size=tp_size, dtype=dtype,
                                                             quantization=quantization):
            return str(profile)
    return None


def packaged_served_choices(kind: str, **setup) -> Optional[Dict[int, int]]:
    """Served choices per batch key of the matching profile (``rounds/choices_<kind>.json``): the verify width for
    ``"chain"``; 1 to speculate or 0 to decode natively for ``"tree"``. None when no profile or no choices."""
    path = packaged_cost_profile(**setup)
    if path is None:
        return None
    f = Path(path) / "rounds" / f"choices_{kind}.json"
    if not f.is_file():
        return None
    return {int(k): int(v) for k, v in json.loads(f.read_text(encoding="utf-8"))[kind].items()}


def write_profile(directory: str, *, devices, tp_size: int, target_config: Mapping[str, Any],
                  draft_config: Mapping[str, Any], notes: str = "") -> str:
    """Write ``profile.json`` of a profile directory (the calibration tables go beside it)."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    meta = {"devices": list(devices), "tp_size": tp_size, "dtype": "bfloat16",
            "target_shape": shape_signature(target_config, TARGET_SHAPE_KEYS),
            "draft_shape": shape_signature(draft_config, DRAFT_SHAPE_KEYS), "notes": notes}
    (d / "profile.json").write_text(json.dumps(meta, indent=1), encoding="utf-8")
    return str(d / "profile.json")
