"""The TokenSpeed API the TokenSpeed adapter is written against.

Two TokenSpeed lines carry the plugin API: ``capabilities`` (``PLUGIN_CAPABILITIES`` lists additive contracts and
``PLUGIN_API_VERSION`` changes only on breaking ones) and ``release`` (the ``0.1.1+eagle.N`` engines: no capability
set, the API version counts every contract, and the tree policy has private names). The host names are TokenSpeed's
interface, as in reference ``eagle_harness/tokenspeed/hooks.py:40-186``.
"""

from __future__ import annotations

import importlib
from typing import List, NamedTuple, Optional

from eagle4_b200.plugins.contract import EXISTS, OVERRIDE, Hook, override_mismatches, problems

RELEASE_MIN_API_VERSION = 4
CAPABILITY_API_VERSIONS = frozenset({3})
REQUIRED_CAPABILITIES = frozenset({"drafter.algorithm_config", "drafter.aux_hidden_capture", "drafter.tree_layout",
                                   "attention.windowed_tree_lanes", "drafter.round_protocol", "drafter.tree_lanes",
                                   "drafter.tree_policy", "sampling.tree_sampler"})


class TreePolicy(NamedTuple):
    candidates: str
    seed: str
    expand: str
    window: str


PUBLIC_POLICY = TreePolicy("round_candidates", "seed_tree", "expand_tree", "verify_window")
RELEASE_POLICY = TreePolicy("_candidates", "_seed_tree_lanes", "_expand_tree_lanes", "_draft_window")

_EAGLE = "tokenspeed.runtime.execution.drafter.eagle:Eagle"
_BASE = "tokenspeed.runtime.execution.drafter.base:BaseDrafter"
_SAMPLING = "tokenspeed.runtime.sampling.backends.base:SamplingBackend"


def _policy(names: TreePolicy):
    return (Hook(f"{_EAGLE}.{names.seed}", ("bs", "logits_output", "frontier")),
            Hook(f"{_EAGLE}.{names.expand}", ("bs", "step", "logits_output")),
            Hook(f"{_EAGLE}.{names.window}", ("bs", "next_tokens")))


HOOKS = (
    Hook("tokenspeed.runtime.plugins:PLUGIN_API_VERSION", (), EXISTS),
    Hook(f"{_SAMPLING}.bind_tree_sampler", ("factory",)),
    Hook(f"{_SAMPLING}.supports_tree_sampler", (), EXISTS),
    Hook("tokenspeed.runtime.plugins.registry:register_drafter",
         ("algorithm", "drafter_cls", "model_cls", "captures_aux_hidden_states", "uses_tree_layout")),
    Hook("tokenspeed.runtime.plugins.registry:register_model", ("cls", "architectures")),
    Hook("tokenspeed.runtime.configs.model_profile:ModelProfile", (), EXISTS),
    Hook(f"{_BASE}.configure_algorithm", ("algorithm_config",), OVERRIDE,
         "eagle4_b200.plugins.tokenspeed.adapter:HarnessDrafter"),
    Hook("tokenspeed.runtime.execution.drafter:drafter_captures_aux_hidden_states", ("algorithm",)),
    Hook(f"{_EAGLE}.bind_tree", ("tree_spec",)),
    Hook(f"{_EAGLE}.bind_tree_lanes", ("tree_spec",)),
    Hook(f"{_BASE}.prepare_round_sampling", ("sampling_params_list",)),
    Hook(f"{_BASE}.replay_decode_graph", ("graph", "bs", "graph_bs")),
    Hook(f"{_BASE}.finish_round", ("ctx", "graph_bs")),
    Hook(f"{_BASE}.complete_round", (), EXISTS),
    Hook(f"{_BASE}.capture_round_graphs", ("graph_bs", "lo_bs", "stream", "pool")),
    Hook(f"{_BASE}.has_round_graphs", ("graph_bs",)),
    Hook(f"{_BASE}.release_round_graphs", (), EXISTS),
    Hook("tokenspeed.runtime.layers.attention.backends.base:AttentionBackend.begin_tree_lanes", ("bs", "live_bs")),
    Hook("tokenspeed.runtime.layers.attention.backends.paged.tree_verify:TreeDraftInputs.set_frontier", (), EXISTS),
    Hook("tokenspeed.runtime.models.llama_eagle3:LlamaForCausalLMEagle3.exit_logits",
         ("input_ids", "hidden_states", "aux_hidden_states", "ctx"), OVERRIDE,
         "eagle4_b200.plugins.tokenspeed.models:LlamaForCausalLMEagle4"),
    Hook("tokenspeed.runtime.execution.context:ForwardContext.gather_ids", (), EXISTS),
    Hook("tokenspeed.runtime.distributed.comm_ops:all_gather", ("tensor", "group", "dim")),
)
CAPABILITY_HOOKS = _policy(PUBLIC_POLICY)
RELEASE_HOOKS = _policy(RELEASE_POLICY) + (
    Hook("tokenspeed.runtime.layers.attention.backends.paged.trtllm:TRTLLMMHAAttnBackend._tree_lane_window_cascade",
         ("lanes", "step")),)
SAMPLED_HOOKS = (
    Hook("tokenspeed.runtime.sampling.tree_verify:DraftTreeQ.zeros",
         ("rows", "num_slots", "num_candidates", "num_nodes", "device")),
    Hook("tokenspeed.runtime.sampling.tree_verify:TreeVerifyBatch.draft_q", (), EXISTS),
    Hook("tokenspeed.runtime.execution.runtime_states:RuntimeStates.init_draft_tree_q",
         ("num_nodes", "num_slots", "num_candidates")),
    Hook(f"{_SAMPLING}.verifies_draft_tree_q", (), EXISTS),
    Hook(f"{_SAMPLING}.speculative_sampling_pools", (), EXISTS),
)


def contract() -> Optional[str]:
    try:
        plugins = importlib.import_module("tokenspeed.runtime.plugins")
    except ImportError:
        return None
    return "capabilities" if hasattr(plugins, "PLUGIN_CAPABILITIES") else "release"


def tree_policy() -> TreePolicy:
    return RELEASE_POLICY if contract() == "release" else PUBLIC_POLICY


def hook_problems() -> List[str]:
    kind = contract()
    out: List[str] = []
    if kind == "capabilities":
        plugins = importlib.import_module("tokenspeed.runtime.plugins")
        if plugins.PLUGIN_API_VERSION not in CAPABILITY_API_VERSIONS:
            out.append(f"PLUGIN_API_VERSION {plugins.PLUGIN_API_VERSION} is not one of "
                       f"{sorted(CAPABILITY_API_VERSIONS)} (a breaking plugin API change)")
        missing = sorted(REQUIRED_CAPABILITIES - set(plugins.PLUGIN_CAPABILITIES))
        if missing:
            out.append(f"PLUGIN_CAPABILITIES lacks {', '.join(missing)}")
    out += problems(HOOKS + (CAPABILITY_HOOKS if kind == "capabilities" else RELEASE_HOOKS))
    if not out and kind == "release":
        version = importlib.import_module("tokenspeed.runtime.plugins").PLUGIN_API_VERSION
        if version < RELEASE_MIN_API_VERSION:
            out.append(f"PLUGIN_API_VERSION {version} < {RELEASE_MIN_API_VERSION}")
    return out


def sampled_hook_problems() -> List[str]:
    return problems(SAMPLED_HOOKS)


def adapter_problems() -> List[str]:
    """This package's overrides whose signatures differ from the table (checked without TokenSpeed)."""
    return override_mismatches(HOOKS)
