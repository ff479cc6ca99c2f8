"""The ``method_config`` of the ``eagle_harness`` method in vLLM: the harness config keys plus vLLM's tree keys.

``SpeculativeConfig.method_config`` is one JSON object. The tree keys (``max_verify_width`` nodes including the
root, ``node_top_k``, ``tree_depth``), ``depth_stop_gain`` and ``record_rounds`` are read here; every other key is a
harness config key (``core.config``), unknown ones refused there. The key names, defaults and refusals are the
host-facing interface of the reference's vLLM method (``eagle_harness/vllm/config.py:87-140``), so a vLLM launch
command written for one reads the same here.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping, Optional, Union

from eagle4_b200.core.config import HarnessConfig, harness_config_from_dict
from eagle4_b200.core.limits import (MAX_CHAIN_VERIFY_NUM, MAX_VERIFY_NUM, ComputeIntensity, check_shape,
                                     req_to_token_span)

DERIVED = "derived"
TREE_KEYS = ("max_verify_width", "node_top_k", "tree_depth", "depth_stop_gain", "record_rounds")
DEFAULT_TREE = {"node_top_k": 4, "tree_depth": 12}


@dataclass(frozen=True)
class MethodConfig:
    harness: HarnessConfig
    max_verify_width: int   # verify rows per request, the root included
    node_top_k: int
    tree_depth: int
    depth_stop_gain: Union[float, str, None] = DERIVED
    record_rounds: bool = False  # served rounds' periods go to <data_path>/rounds/tree.json
    explicit_width: bool = False  # max_verify_width was set (an unpriced chain may then run at that fixed width)

    @property
    def num_speculative_tokens(self) -> int:
        return self.max_verify_width - 1

    @property
    def lookahead(self) -> int:
        """Block-table slots past the scheduled tokens that one round writes (draft steps or verify rows)."""
        return max(self.num_speculative_tokens,
                   req_to_token_span(self.node_top_k, self.tree_depth, self.max_verify_width, 1))


def _int(name: str, value: Any) -> int:
    if isinstance(value, bool) or not isinstance(value, int):
        raise ValueError(f"method_config.{name} must be an integer, got {value!r}.")
    return value


def parse_method_config(method_config: Optional[Mapping[str, Any]]) -> MethodConfig:
    """Read and check a ``method_config``; bad values and unknown harness keys raise."""
    data = dict(method_config or {})
    tree = {k: data.pop(k) for k in TREE_KEYS if k in data}
    harness = harness_config_from_dict(data)
    chain = harness.intensity is ComputeIntensity.CHAIN
    width = _int("max_verify_width", tree.get("max_verify_width", MAX_CHAIN_VERIFY_NUM if chain else 32))
    top_k = _int("node_top_k", tree.get("node_top_k", 1 if chain else DEFAULT_TREE["node_top_k"]))
    depth = _int("tree_depth", tree.get("tree_depth", MAX_CHAIN_VERIFY_NUM - 1 if chain else DEFAULT_TREE["tree_depth"]))
    if width > (MAX_CHAIN_VERIFY_NUM if chain else MAX_VERIFY_NUM):
        raise NotImplementedError(f"max_verify_width={width} is not served at {harness.intensity.value}.")
    check_shape(harness.intensity, top_k, depth, width, 1)
    gain = tree.get("depth_stop_gain", DERIVED)
    if gain is not None and gain != DERIVED:
        if isinstance(gain, bool) or not isinstance(gain, (int, float)) or gain < 0:
            raise ValueError(f'method_config.depth_stop_gain must be "derived", a number >= 0 or null, got {gain!r}.')
        # a fixed gain parametrises a depth stop evaluated on the device; here the host cost model decides depths
        raise NotImplementedError("a fixed depth_stop_gain needs the device depth stop, which eagle4_b200 does not "
                                  'build: use "derived" (the cost model\'s depth rule) or null (full depth).')
    record = tree.get("record_rounds", False)
    if not isinstance(record, bool):
        raise ValueError(f"method_config.record_rounds must be true or false, got {record!r}.")
    if record and not harness.data_path:
        raise ValueError("method_config.record_rounds writes rounds/tree.json under data_path: set data_path.")
    return MethodConfig(harness, width, top_k, depth, gain, record, "max_verify_width" in tree)
