"""``HarnessConfig``: every option of the EAGLE_HARNESS algorithm in one typed JSON object.

The JSON keys, their defaults and the refusal of unknown and removed keys are the public surface shared with the
reference (``eagle_harness/core/config.py:37-296``, documented keys in ``docs/configuration.md:13-25``). Parsing is
a small typed-dataclass reader of this package's own. Configuration reads no environment variables.
"""

from __future__ import annotations

import dataclasses
import enum
import json
import os
import typing
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, Dict, Mapping, Optional, Tuple

from eagle4_b200.core.cost_model import ChainCoef, CostModel, CostModelParams, depth_loss_ratio
from eagle4_b200.core.cost_table import BatchCostTable, cost_model_problem, load_cost_tables
from eagle4_b200.core.limits import ComputeIntensity

if TYPE_CHECKING:  # pragma: no cover
    from eagle4_b200.core.live_costs import CostKey


class Mode(str, enum.Enum):
    STATIC = "static"  # the fixed --speculative-num-steps / -eagle-topk / -num-draft-tokens tree
    SERVE = "serve"
    CALIBRATE = "calibrate"

    @property
    def uses_cost_model(self) -> bool:
        return self is not Mode.STATIC


class DraftFamily(str, enum.Enum):
    EAGLE4 = "eagle4"
    EAGLE3 = "eagle3"
    EAGLE = "eagle"


@dataclass(frozen=True)
class DraftModelOptions:
    cuda_candidate_kernels: bool = True
    embed_full: bool = True
    embed_triton: bool = True  # kept for config compatibility; lookups here are always this package's CUDA gather


@dataclass(frozen=True)
class L2Warm:
    """Weight prefetches into L2 during verify: ``(share of the weight's bytes, CTAs)`` or None (off)."""

    gate_up_gdn: Optional[Tuple[float, int]] = (0.42, 16)
    gate_up_attention: Optional[Tuple[float, int]] = (0.3, 74)
    down_proj: Optional[Tuple[float, int]] = None
    next_input: Optional[Tuple[float, int]] = None


@dataclass(frozen=True)
class CostModelConfig:
    threshold: float = 2.5
    async_layer_ratio: float = 0.9
    depth_loss_ratio: Optional[float] = None  # None: from the draft family and target
    chain_tiny: Tuple[float, float, float] = (2.60, 0.24, 0.00)
    chain_small: Tuple[float, float, float] = (2.85, 0.24, 0.00)
    chain_medium: Tuple[float, float, float] = (2.54, 0.24, 0.70)
    chain_large: Tuple[float, float, float] = (1.55, 0.24, 0.00)
    chain_scale_tiny: float = 1.25
    chain_tiny_max_bs: int = 2
    chain_scale_small: float = 1.45
    chain_scale_medium: float = 2.00

    def params(self, family_depth_loss: float) -> CostModelParams:
        loss = self.depth_loss_ratio if self.depth_loss_ratio is not None else family_depth_loss
        coefs = tuple(ChainCoef(*c) for c in (self.chain_tiny, self.chain_small, self.chain_medium, self.chain_large))
        return CostModelParams(
            threshold=self.threshold,
            async_layer_ratio=self.async_layer_ratio,
            depth_loss_ratio=loss,
            chain_coef=coefs,
            chain_scale_tiny=self.chain_scale_tiny,
            chain_tiny_max_bs=self.chain_tiny_max_bs,
            chain_scale_small=self.chain_scale_small,
            chain_scale_medium=self.chain_scale_medium,
        )


@dataclass(frozen=True)
class HarnessConfig:
    data_path: Optional[str] = None
    cost_cache: Optional[str] = None
    mode: Mode = Mode.SERVE
    intensity: ComputeIntensity = ComputeIntensity.HIGH
    draft_family: DraftFamily = DraftFamily.EAGLE4
    cost_model: CostModelConfig = field(default_factory=CostModelConfig)
    draft_model: DraftModelOptions = field(default_factory=DraftModelOptions)
    l2_warm: L2Warm = field(default_factory=L2Warm)
    max_verify_batch_size: Optional[int] = None

    def validate(self) -> "HarnessConfig":
        if self.mode is Mode.CALIBRATE and not self.data_path:
            raise ValueError("calibrate mode needs data_path for its output")
        if self.max_verify_batch_size is not None and self.max_verify_batch_size < 1:
            raise ValueError("max_verify_batch_size must be at least 1")
        return self

    @property
    def cost_dir(self) -> str:
        assert self.data_path is not None
        return os.path.join(self.data_path, "cost")

    @property
    def cost_cache_dir(self) -> str:
        return self.cost_cache or os.path.join(os.path.expanduser("~"), ".cache", "eagle-harness", "costs")


def build_cost_model(config: HarnessConfig, *, node_top_k: int, tree_depth: int, verify_num: int,
                     target_is_moe: bool, tables: Optional[Dict[int, BatchCostTable]] = None,
                     key: Optional["CostKey"] = None) -> CostModel:
    """The worker's cost model, from ``tables`` or the offline tables under ``config.data_path``."""
    loss = depth_loss_ratio(config.draft_family.value, target_is_moe=target_is_moe, intensity=config.intensity)
    if tables is None:
        tables = load_cost_tables(config.cost_dir, key)
        for bs, t in sorted(tables.items()):
            problem = cost_model_problem(t, target_is_moe=target_is_moe)
            if problem is not None:
                raise ValueError(f"Cost tables under {config.cost_dir}/bs_{bs} cannot drive the cost model: {problem}.")
    return CostModel(tables=tables, params=config.cost_model.params(loss), intensity=config.intensity,
                     node_top_k=node_top_k, tree_depth=tree_depth, verify_num=verify_num,
                     target_is_moe=target_is_moe)


# Keys removed in eagle-harness 0.1.1; a config that sets one is refused by name.
REMOVED_IN_0_1_1 = (
    "mode: eval",
    "ragged",
    "cost_model.ragged_draft_relax",
    "cost_model.ragged_verify_threshold",
    "draft_model.moe_gate_acc",
)


def _typed(tp: Any, value: Any, where: str) -> Any:
    if dataclasses.is_dataclass(tp):
        if not isinstance(value, Mapping):
            raise ValueError(f"{where}: expected an object, got {type(value).__name__}.")
        return _read(tp, value, where)
    if isinstance(tp, type) and issubclass(tp, enum.Enum):
        try:
            return tp(value)
        except ValueError as e:
            raise ValueError(f"{where}: {value!r} is not one of {', '.join(m.value for m in tp)}.") from e
    origin = typing.get_origin(tp)
    if origin is typing.Union:
        if value is None:
            return None
        inner = [a for a in typing.get_args(tp) if a is not type(None)][0]
        return _typed(inner, value, where)
    if origin is tuple:
        parts = typing.get_args(tp)
        if not isinstance(value, (list, tuple)) or len(value) != len(parts):
            raise ValueError(f"{where}: expected a list of {len(parts)} values.")
        return tuple(_typed(a, v, f"{where}[{i}]") for i, (a, v) in enumerate(zip(parts, value)))
    if tp is bool:
        if not isinstance(value, bool):
            raise ValueError(f"{where}: expected true/false, got {value!r}.")
        return value
    if tp is int:
        if isinstance(value, bool) or not isinstance(value, int):
            raise ValueError(f"{where}: expected an integer, got {value!r}.")
        return value
    if tp is float:
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise ValueError(f"{where}: expected a number, got {value!r}.")
        return float(value)
    if tp is str:
        if not isinstance(value, str):
            raise ValueError(f"{where}: expected a string, got {value!r}.")
        return value
    raise TypeError(f"{where}: unsupported field type {tp!r}.")


def _read(cls: type, data: Mapping[str, Any], where: str) -> Any:
    hints = typing.get_type_hints(cls)
    names = {f.name for f in dataclasses.fields(cls)}
    dotted = [f"{where}.{k}" if where else k for k in data]
    if not where and data.get("mode") == "eval":
        dotted.append("mode: eval")
    removed = [k for k in dotted if k in REMOVED_IN_0_1_1]
    if removed:
        raise ValueError(f"{', '.join(removed)}: removed in eagle-harness 0.1.1 (no engine used it); delete it.")
    unknown = sorted(set(data) - names)
    if unknown:
        raise ValueError(f"{where or 'config'}: unknown keys {unknown}; valid keys are {sorted(names)}.")
    return cls(**{k: _typed(hints[k], v, f"{where}.{k}" if where else k) for k, v in data.items()})


def harness_config_from_dict(data: Mapping[str, Any]) -> HarnessConfig:
    return _read(HarnessConfig, data, "").validate()


def parse_harness_config(value: Optional[str], *, default_data_path: Optional[str] = None) -> HarnessConfig:
    """Inline JSON, or a path to a JSON file; empty means the default serve-mode config."""
    if value is None or not value.strip():
        return harness_config_from_dict({} if default_data_path is None else {"data_path": default_data_path})
    text = value.strip()
    if not text.startswith(("{", "[")):
        with open(os.path.expanduser(text), encoding="utf-8") as f:
            text = f.read()
    try:
        data = json.loads(text)
    except json.JSONDecodeError as e:
        raise ValueError(f"--speculative-algorithm-config is not valid JSON: {e}") from e
    if not isinstance(data, dict):
        raise ValueError("--speculative-algorithm-config must be a JSON object.")
    if default_data_path is not None and data.get("data_path") is None \
            and data.get("mode", Mode.SERVE.value) == Mode.SERVE.value:
        data["data_path"] = default_data_path
    return harness_config_from_dict(data)


def config_to_dict(config: HarnessConfig) -> Dict[str, Any]:
    """Plain JSON data: enums by value, tuples as lists, nested dataclasses as objects."""

    def conv(v: Any) -> Any:
        if dataclasses.is_dataclass(v):
            return {f.name: conv(getattr(v, f.name)) for f in dataclasses.fields(v)}
        if isinstance(v, enum.Enum):
            return v.value
        if isinstance(v, tuple):
            return [conv(x) for x in v]
        return v

    return conv(config)
