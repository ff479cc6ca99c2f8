"""The vLLM API the vLLM adapter is written against (hook-carrying vLLM builds, ``vllm>=0.32.0rc1.dev283``).

One entry per engine need, with the vLLM attribute that carries it (``" | "`` between alternative locations; empty
when vLLM offers no hook). The attribute names are vLLM's interface, as in reference
``eagle_harness/vllm/adapter.py:43-90``.
"""

from __future__ import annotations

from typing import List, NamedTuple

from eagle4_b200.plugins.contract import EXISTS, Hook, problems

VERIFY_EXTENSION_MODULES = ("vllm.model_executor.layers.mamba.verify_extension",
                            "vllm.model_executor.layers.mamba.gdn.verify_extension")


class HookUse(NamedTuple):
    need: str
    hook: str
    status: str  # "cpu": tested on CPU against fakes; "gpu": needs the host on a GPU; "none": no hook in vLLM


_SPEC = "vllm.v1.worker.gpu.spec_decode.speculator"
HOOK_MAP = (
    HookUse("algorithm registration", "vllm.v1.spec_decode.registry:register_speculative_method", "cpu"),
    HookUse("opaque algorithm config", "vllm.config.speculative:SpeculativeConfig.method_config", "cpu"),
    HookUse("method configure / tree budget", "vllm.v1.spec_decode.registry:SpeculativeMethodSpec.configure", "cpu"),
    HookUse("KV headroom", "vllm.v1.spec_decode.registry:SpeculativeMethodSpec.num_lookahead_tokens", "cpu"),
    HookUse("draft + KV slots", f"{_SPEC}:DraftModelSpeculator.propose", "gpu"),
    HookUse("verify positions and tree mask", f"{_SPEC}:BaseSpeculator.prepare_verify_inputs", "gpu"),
    HookUse("verify accept", f"{_SPEC}:BaseSpeculator.make_rejection_sampler", "gpu"),
    HookUse("accepted-path KV compaction", f"{_SPEC}:BaseSpeculator.post_accept", "gpu"),
    HookUse("GDN tree verify of the spec rows",
            " | ".join(f"{m}:LinearAttnVerifyExtension.forward_spec_rows" for m in VERIFY_EXTENSION_MODULES), "gpu"),
    HookUse("tree attention backend", "vllm.v1.attention.backends.registry:AttentionBackendEnum.CUSTOM", "gpu"),
    HookUse("request admission (no logprobs, text only)", "", "none"),
    HookUse("worker idle / batch released", "", "none"),
)


def _field_ok(path: str) -> bool:
    """A dataclass / pydantic field without a class-level default also counts."""
    from eagle4_b200.plugins.contract import field_names, resolve

    owner, _, name = path.rpartition(".")
    try:
        return name in field_names(resolve(owner))
    except (ImportError, AttributeError):
        return False


def missing_hooks() -> List[str]:
    out = []
    for use in HOOK_MAP:
        if use.hook and problems([Hook(use.hook, (), EXISTS)]) and not _field_ok(use.hook):
            out.append(use.hook)
    return out


hook_problems = missing_hooks


# Optional speculator hooks: vLLM builds that have them call them per scheduled batch; builds without them skip them
# (the method still registers). ``plugins.vllm.batch_policy`` answers both.
OPTIONAL_HOOKS = (
    HookUse("native decode per batch size", f"{_SPEC}:BaseSpeculator.suspend_drafting", "cpu"),
    HookUse("drafts verified per batch size", f"{_SPEC}:BaseSpeculator.verify_budget", "cpu"),
)


def host_speculator_hooks() -> List[str]:
    """The optional hooks this vLLM calls, checked by parameter names against ``batch_policy.SPECULATOR_HOOKS``."""
    import inspect

    from eagle4_b200.plugins.contract import resolve
    from eagle4_b200.plugins.vllm.batch_policy import SPECULATOR_HOOKS

    found = []
    for use in OPTIONAL_HOOKS:
        name = use.hook.rsplit(".", 1)[1]
        try:
            fn = resolve(use.hook)
        except (ImportError, AttributeError):
            continue
        if callable(fn) and tuple(inspect.signature(fn).parameters)[1:] == SPECULATOR_HOOKS[name]:
            found.append(name)
    return found
