"""EAGLE-4 draft structure decisions read from a draft config, independent of any engine.

The three position settings of the released configs, any of which turns rotary positions off (NoPE), and the draft
MoE architecture names (reference ``eagle_harness/models/eagle4_structure.py:14-58``). Configs are HF config objects
or plain dicts.
"""

from __future__ import annotations

import copy
from typing import Any, Dict, Optional

LATENT_MOE_ARCHITECTURE = "nemotron_latent_relu2"
SPARSE_MOE_ARCHITECTURE = "sparse_swiglu"


def _get(config: Any, name: str, default=None):
    if isinstance(config, dict):
        return config.get(name, default)
    return getattr(config, name, default)


def draft_moe_architecture(config: Any) -> Optional[str]:
    """The enabled draft MoE architecture, None for a dense draft."""
    if not _get(config, "enable_moe", False):
        return None
    return _get(config, "moe_architecture") or SPARSE_MOE_ARCHITECTURE


def draft_uses_rope(config: Any) -> bool:
    """False when ``use_rope`` is false, ``position_embedding_type`` is ``none`` or ``partial_rotary_factor`` is 0."""
    return not (_get(config, "use_rope", True) is False or _get(config, "position_embedding_type") == "none"
                or _get(config, "partial_rotary_factor") == 0)


def base_layer_overrides(config: Any) -> Dict[str, Any]:
    """Settings for building a Llama base layer whose MLP or rotary embedding is replaced afterwards: a latent-MoE
    draft's MLP is rebuilt (the base layer gets ``silu``), and a NoPE draft needs a one-position rotary table only."""
    out: Dict[str, Any] = {}
    if draft_moe_architecture(config) == LATENT_MOE_ARCHITECTURE:
        out["hidden_act"] = "silu"
    if not draft_uses_rope(config):
        out["max_position_embeddings"] = 1
    return out


def latent_moe_config(config: Any) -> Any:
    """A shallow copy of a validated latent-MoE draft config with the MoE block's defaults filled in."""
    moe = copy.copy(config)
    groups = int(_get(config, "n_group", 1) or 1)
    values = {"mlp_hidden_act": _get(config, "hidden_act"), "mlp_bias": False,
              "n_shared_experts": int(_get(config, "n_shared_experts", 0) or 0), "n_group": groups,
              "topk_group": int(_get(config, "topk_group", groups) or groups),
              "norm_topk_prob": bool(_get(config, "norm_topk_prob", True)),
              "routed_scaling_factor": float(_get(config, "routed_scaling_factor", 1.0))}
    if isinstance(moe, dict):
        moe.update(values)
    else:
        for k, v in values.items():
            setattr(moe, k, v)
    return moe
