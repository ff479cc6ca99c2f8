"""What the ``eagle_harness`` method installs in vLLM's speculative config at configure time.

vLLM sizes a speculative engine before any worker starts: the drafts per request (``num_speculative_tokens``, and per
batch-size range ``num_speculative_tokens_per_batch_size``), the linear-attention state slots it reserves per request
(one per verify row) and the layers whose hidden states the target captures for the draft. The method answers from
the ``method_config`` and the calibration data under ``data_path``:

* **verify widths** per batch-size range (rows per request, the root included): chains take the served chain-width
  schedule (``core.chain_width.chain_widths``: served round periods and the acceptance profile; width 0 decodes that
  range natively); trees take the widest verify bucket of each calibrated batch size (a batch between two calibrated
  sizes takes the larger size's width, which is never wider), narrowed where recorded served tree rounds
  (``rounds/tree.json``) show a narrower width pays;
* the **draft-token schedule** is the widths minus the root, ending with zero drafts above the method's batch limit;
* ``num_speculative_tokens`` defaults to the widest scheduled draft count, not ``max_verify_width - 1``: vLLM keeps
  ``1 + num_speculative_tokens`` state slots for every running request, so a width no batch size verifies would only
  cost memory;
* the draft's **aux layers**: the checkpoint names the target layers whose outputs the draft was trained on; vLLM
  captures the input of the layer it is given, so each id moves up by one.

``check_data_key`` re-derives the schedule with the serving worker's setup key: configure runs in vLLM's API process,
which cannot name the GPU, so each worker refuses calibration data measured elsewhere before serving. The hook names
and the ``(first, last, value)`` range triples are vLLM's; the reference method installs the same things
(``eagle_harness/vllm/config.py:219-330``).
"""

from __future__ import annotations

from typing import Any, List, Sequence, Tuple

from eagle4_b200.core.chain_width import chain_widths, load_tree_rounds, merge_ranges, served_tree_schedule, width_at
from eagle4_b200.core.limits import ComputeIntensity, cost_batch_sizes, max_batch_size, verify_buckets
from eagle4_b200.plugins.vllm.config import MethodConfig, parse_method_config

Schedule = List[Tuple[int, int, int]]
NO_DRAFT_ABOVE = 1 << 16  # the last range of a draft-token schedule: no drafts above the method's batch limit
EAGLE4_ARCH = "LlamaForCausalLMEagle4"


def _ceiling_ranges(per_batch: dict, limit: int) -> Schedule:
    """Ranges covering ``1..limit``: each batch size takes the value of the smallest calibrated size at or above it."""
    sizes = sorted(per_batch)
    rows, first = [], 1
    for b in sizes:
        if b > limit:
            break
        rows.append((first, b, per_batch[b]))
        first = b + 1
    if first <= limit:
        rows.append((first, limit, per_batch[sizes[-1]]))
    return merge_ranges(rows)


def verify_widths(method: MethodConfig, *, key=None) -> Schedule:
    """Verify rows per request for every batch size up to the method's limit (0: decode natively)."""
    h = method.harness
    limit = max_batch_size(h.intensity)
    if h.intensity is ComputeIntensity.CHAIN:
        widths = chain_widths(h.data_path, method.max_verify_width, limit, allow_no_spec=True, key=key) \
            if h.data_path else None
        if widths is None:
            if not method.explicit_width:
                raise ValueError(f"eagle_harness: no priced chain schedule under {h.data_path!r} (an acceptance "
                                 "profile and served round times or cost tables): calibrate the chain, or set "
                                 "max_verify_width for a fixed unpriced chain")
            widths = [(1, limit, method.max_verify_width)]
        return widths
    base = _ceiling_ranges({b: min(max(verify_buckets(b, h.intensity)), method.max_verify_width)
                            for b in cost_batch_sizes(limit)}, limit)
    rounds = load_tree_rounds(h.data_path, key) if h.data_path else None
    measured = served_tree_schedule(rounds, method.max_verify_width, limit) if rounds else None
    if measured is None:
        return base
    cuts = sorted({a for a, _, _ in base} | {a for a, _, _ in measured if a <= limit})
    ends = [c - 1 for c in cuts[1:]] + [limit]
    return merge_ranges((a, e, min(width_at(base, a), width_at(measured, a))) for a, e in zip(cuts, ends))


def draft_token_schedule(widths: Sequence[Tuple[int, int, int]]) -> Schedule:
    """Drafts per request (verify rows minus the root) per batch-size range, none above the last range."""
    rows = [(a, b, max(0, int(w) - 1)) for a, b, w in widths]
    return merge_ranges(rows + [(rows[-1][1] + 1, NO_DRAFT_ABOVE, 0)])


def native_ranges(widths: Sequence[Tuple[int, int, int]]) -> List[Tuple[int, int]]:
    return [(a, b) for a, b, w in widths if w == 0]


def aux_hidden_state_layers(draft_hf_config: Any) -> Tuple[int, ...]:
    """The target layers whose inputs vLLM captures for the draft: the checkpoint's output-layer ids plus one."""
    eagle = getattr(draft_hf_config, "eagle_config", None)
    if eagle is None and isinstance(draft_hf_config, dict):
        eagle = draft_hf_config.get("eagle_config")
    named = (eagle or {}).get("eagle_aux_hidden_state_layer_ids") or ()
    return tuple(int(i) + 1 for i in named)


def configure_speculative_config(spec_config: Any) -> MethodConfig:
    """``SpeculativeMethodSpec.configure``: fill vLLM's speculative config in place; returns the parsed method."""
    method = parse_method_config(getattr(spec_config, "method_config", None))
    draft_model = getattr(spec_config, "draft_model_config", None)
    draft = getattr(draft_model, "hf_config", None)
    if draft is not None and EAGLE4_ARCH in (getattr(draft, "architectures", None) or ()):
        draft.eagle_aux_hidden_state_layer_ids = list(aux_hidden_state_layers(draft))
    if method.harness.mode.uses_cost_model and getattr(spec_config, "num_speculative_tokens_per_batch_size",
                                                       None) is None:
        spec_config.num_speculative_tokens_per_batch_size = draft_token_schedule(verify_widths(method))
    schedule = getattr(spec_config, "num_speculative_tokens_per_batch_size", None)
    widest = method.num_speculative_tokens if not schedule else max(1, max(k for _, _, k in schedule))
    given = getattr(spec_config, "num_speculative_tokens", None)
    if given is None:
        spec_config.num_speculative_tokens = widest
    elif given not in (widest, method.num_speculative_tokens):
        raise ValueError(f"num_speculative_tokens={given} disagrees with method_config.max_verify_width="
                         f"{method.max_verify_width} (they differ by one): set only one of them")
    return method


def installed_native_ranges(spec_config: Any) -> List[Tuple[int, int]]:
    """The batch-size ranges the installed schedule decodes natively (empty when the user set the schedule)."""
    method = parse_method_config(getattr(spec_config, "method_config", None))
    if not method.harness.mode.uses_cost_model:
        return []
    widths = verify_widths(method)
    installed = [tuple(r) for r in getattr(spec_config, "num_speculative_tokens_per_batch_size", None) or ()]
    if installed != draft_token_schedule(widths):
        return []
    return native_ranges(widths)


def check_data_key(spec_config: Any, key) -> None:
    """A serving worker's check that ``data_path`` was measured on its setup (raises otherwise)."""
    method = parse_method_config(getattr(spec_config, "method_config", None))
    if method.harness.mode.uses_cost_model or method.node_top_k > 1:
        verify_widths(method, key=key)
