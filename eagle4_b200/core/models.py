"""Target model properties the cost policies read (reference ``eagle_harness/core/models.py:7``)."""

from typing import Any

_EXPERT_COUNTS = ("num_experts", "num_local_experts", "n_routed_experts")


def target_is_moe(hf_config: Any) -> bool:
    """True when the text config has routed experts (any expert count above zero); no architecture-name heuristics."""
    config = getattr(hf_config, "text_config", None) or hf_config
    get = config.get if isinstance(config, dict) else (lambda n, d=None: getattr(config, n, d))
    return any((get(n, 0) or 0) > 0 for n in _EXPERT_COUNTS)
