"""``HarnessConfig``: every option of the EAGLE_HARNESS algorithm in one typed JSON object.

The JSON keys, their defaults and the refusal of unknown and removed keys are the public surface shared with the
reference (``eagle_harness/core/config.py:37-296``, documented keys in ``docs/configuration.md:13-25``). The reader
is a schema table (one value checker per key) walked once over the JSON object; it collects every problem of a
configuration and reports them together. Configuration reads no environment variables.
"""

from __future__ import annotations

import dataclasses
import enum
import json
import os
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, Callable, Dict, Mapping, Optional, Tuple

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
            raise ValueError("mode calibrate writes its tables under data_path: set it")
        if self.max_verify_batch_size is not None and self.max_verify_batch_size < 1:
            raise ValueError("max_verify_batch_size is below 1")
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
                raise ValueError(f"the cost model refuses the tables under {config.cost_dir}/bs_{bs}: {problem}")
    return CostModel(tables=tables, params=config.cost_model.params(loss), intensity=config.intensity,
                     node_top_k=node_top_k, tree_depth=tree_depth, verify_num=verify_num,
                     target_is_moe=target_is_moe)


# ---------------------------------------------------------------------------------------------------- reading
# Keys the reference removed in 0.1.1. They are part of the public surface: a config that still sets one is refused
# with the key named (a dotted path; "mode: eval" is the removed mode value).
REMOVED_IN_0_1_1 = (
    "mode: eval",
    "ragged",
    "cost_model.ragged_draft_relax",
    "cost_model.ragged_verify_threshold",
    "draft_model.moe_gate_acc",
)


class ConfigError(ValueError):
    """Every problem found in one configuration object, reported together."""

    def __init__(self, problems):
        self.problems = list(problems)
        super().__init__("invalid --speculative-algorithm-config: " + "; ".join(self.problems))


# A value checker returns the converted value or records a problem (and returns None).
_Checker = Callable[[Any, str, list], Any]


def _scalar(kind: str) -> _Checker:
    def check(v: Any, at: str, problems: list) -> Any:
        ok = {
            "bool": isinstance(v, bool),
            "int": isinstance(v, int) and not isinstance(v, bool),
            "float": isinstance(v, (int, float)) and not isinstance(v, bool),
            "str": isinstance(v, str),
        }[kind]
        if not ok:
            problems.append(f"{at} must be {_NOUN[kind]} (found {v!r})")
            return None
        return float(v) if kind == "float" else v

    return check


_NOUN = {"bool": "true or false", "int": "an integer", "float": "a number", "str": "a string"}


def _member(enum_cls) -> _Checker:
    def check(v: Any, at: str, problems: list) -> Any:
        for m in enum_cls:
            if v == m.value:
                return m
        problems.append(f"{at} must be one of {[m.value for m in enum_cls]} (found {v!r})")
        return None

    return check


def _maybe(inner: _Checker) -> _Checker:
    return lambda v, at, problems: None if v is None else inner(v, at, problems)


def _fixed_list(*items: _Checker) -> _Checker:
    def check(v: Any, at: str, problems: list) -> Any:
        if not isinstance(v, (list, tuple)) or len(v) != len(items):
            problems.append(f"{at} must be a list of {len(items)} values (found {v!r})")
            return None
        return tuple(c(x, f"{at}[{i}]", problems) for i, (c, x) in enumerate(zip(items, v)))

    return check


def _object(cls) -> _Checker:
    return lambda v, at, problems: _read_object(cls, v, at, problems)


_F, _I, _B, _S = _scalar("float"), _scalar("int"), _scalar("bool"), _scalar("str")
_CHAIN = _fixed_list(_F, _F, _F)
_PREFETCH = _maybe(_fixed_list(_F, _I))

# Each configuration object's keys and how a JSON value becomes the field's value.
_SCHEMA: Dict[type, Dict[str, _Checker]] = {
    DraftModelOptions: {"cuda_candidate_kernels": _B, "embed_full": _B, "embed_triton": _B},
    L2Warm: {"gate_up_gdn": _PREFETCH, "gate_up_attention": _PREFETCH, "down_proj": _PREFETCH,
             "next_input": _PREFETCH},
    CostModelConfig: {"threshold": _F, "async_layer_ratio": _F, "depth_loss_ratio": _maybe(_F),
                      "chain_tiny": _CHAIN, "chain_small": _CHAIN, "chain_medium": _CHAIN, "chain_large": _CHAIN,
                      "chain_scale_tiny": _F, "chain_tiny_max_bs": _I, "chain_scale_small": _F,
                      "chain_scale_medium": _F},
}
_SCHEMA[HarnessConfig] = {
    "data_path": _maybe(_S), "cost_cache": _maybe(_S), "mode": _member(Mode), "intensity": _member(ComputeIntensity),
    "draft_family": _member(DraftFamily), "cost_model": _object(CostModelConfig),
    "draft_model": _object(DraftModelOptions), "l2_warm": _object(L2Warm), "max_verify_batch_size": _maybe(_I),
}


def _read_object(cls: type, data: Any, at: str, problems: list) -> Any:
    """One configuration object from JSON ``data``; problems go to ``problems`` (None is returned then)."""
    label = at or "the configuration"
    if not isinstance(data, Mapping):
        problems.append(f"{label} must be a JSON object (found {type(data).__name__})")
        return None
    schema = _SCHEMA[cls]
    found = len(problems)
    values = {}
    for key, raw in data.items():
        path = f"{at}.{key}" if at else key
        if path in REMOVED_IN_0_1_1 or (path == "mode" and raw == "eval"):
            name = "mode: eval" if path == "mode" else path
            problems.append(f"{name} was removed in eagle-harness 0.1.1 (no engine turned it on): drop it")
        elif key not in schema:
            problems.append(f"{label} has no key {key!r} (known keys: {', '.join(sorted(schema))})")
        else:
            values[key] = schema[key](raw, path, problems)
    return cls(**values) if len(problems) == found else None


def harness_config_from_dict(data: Mapping[str, Any]) -> HarnessConfig:
    """A validated :class:`HarnessConfig` from a (possibly partial) JSON object; every problem is reported at once
    (:class:`ConfigError`, a ``ValueError``)."""
    problems: list = []
    config = _read_object(HarnessConfig, data, "", problems)
    if problems:
        raise ConfigError(problems)
    return config.validate()


def _load_json_object(value: str) -> dict:
    """The JSON object of ``--speculative-algorithm-config``: inline JSON, or the path of a file holding it."""
    text = value.strip()
    if text[:1] not in ("{", "["):
        with open(os.path.expanduser(text), encoding="utf-8") as f:
            text = f.read()
    try:
        data = json.loads(text)
    except json.JSONDecodeError as e:
        raise ValueError(f"--speculative-algorithm-config holds no valid JSON ({e})") from e
    if not isinstance(data, dict):
        raise ValueError("--speculative-algorithm-config must hold one JSON object")
    return data


def parse_harness_config(value: Optional[str], *, default_data_path: Optional[str] = None) -> HarnessConfig:
    """The configuration from ``--speculative-algorithm-config`` (inline JSON or a file path; empty or None: the
    default serve-mode configuration). ``default_data_path`` (a packaged profile matched to the device) fills an
    absent ``data_path`` of a serve-mode configuration."""
    data = _load_json_object(value) if value is not None and value.strip() else {}
    serve = data.get("mode", Mode.SERVE.value) == Mode.SERVE.value
    if default_data_path is not None and serve and data.get("data_path") is None:
        data = dict(data, data_path=default_data_path)
    return harness_config_from_dict(data)


def config_to_dict(config: HarnessConfig) -> Dict[str, Any]:
    """Plain JSON data: enums by value, tuples as lists, nested configuration objects as dicts."""
    out: Dict[str, Any] = {}
    for f in dataclasses.fields(config):
        v = getattr(config, f.name)
        if dataclasses.is_dataclass(v):
            out[f.name] = config_to_dict(v)
        elif isinstance(v, enum.Enum):
            out[f.name] = v.value
        elif isinstance(v, tuple):
            out[f.name] = json.loads(json.dumps(v))
        else:
            out[f.name] = v
    return out
