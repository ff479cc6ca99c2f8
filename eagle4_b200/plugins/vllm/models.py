"""``LlamaForCausalLMEagle4`` for vLLM: the EAGLE-4 draft head as the ``eagle_harness`` method's draft model.

vLLM hands a draft model its config with two keys of its own (``eagle_aux_hidden_state_layer_ids``, the target layers
whose inputs vLLM captures for ``fc``: the checkpoint's output-layer ids plus one, set by the method's configure step,
and ``target_layer_count``); ``check_supported`` drops those and applies this package's
draft validation (unknown structural keys, window rules, the single-layer structures; latent ReLU^2 MoE and
``attn_norm`` are built, the sparse SwiGLU MoE is not). The model's layer runs on this package's kernels:

* ``combine_hidden_states``: ``fc`` over the ``fc_norm``-ed aux hidden states (target features -> draft hidden);
* ``forward_rows(input_ids, positions, hidden_states, attend)``: the draft layer on a set of rows with vLLM's own
  attention: ``attend(q, k, v)`` gets rotated q / k and v, writes them into vLLM's KV cache, attends and returns the
  heads' outputs; returns ``(normed, next hidden)``;
* ``compute_candidates(normed, k)``: the low-rank candidate head's top-``k`` children (probabilities, target ids);
  ``compute_logits(normed)``: the full-vocabulary row (``-inf`` outside the candidates) for vLLM's own samplers.

The speculator (``plugins.vllm.adapter.HarnessSpeculator.load_model``) takes this model or its ``draft``.
Reference counterparts: ``eagle_harness/vllm/models.py:72,145`` (``check_supported``, ``LlamaForCausalLMEagle4``) and
``eagle_harness/vllm/model_rows.py:26`` (row forwards with caller-supplied attention).
"""

from __future__ import annotations

from typing import Any, Callable, Iterable, Optional, Set, Tuple

import torch

from eagle4_b200.models import weights as wmod
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.eagle4_config import check_supported as check_draft_config
from eagle4_b200.models.eagle4_config import draft_config_from_hf
from eagle4_b200.plugins.candidate_logits import Candidates, scatter_to_vocab

VLLM_KEYS = ("eagle_aux_hidden_state_layer_ids", "target_layer_count")


def _hf_dict(config: Any) -> dict:
    if isinstance(config, dict):
        return dict(config)
    return config.to_dict() if hasattr(config, "to_dict") else dict(vars(config))


def check_supported(config: Any) -> dict:
    """Validate a vLLM draft config; returns it as a dict without vLLM's own keys. Unbuilt structures raise."""
    hf = {k: v for k, v in _hf_dict(config).items() if k not in VLLM_KEYS}
    check_draft_config(hf)
    return hf


def _draft_hf_config(vllm_config: Any) -> Any:
    spec = getattr(vllm_config, "speculative_config", None)
    draft = getattr(spec, "draft_model_config", None)
    return getattr(draft, "hf_config", None)


class LlamaForCausalLMEagle4(torch.nn.Module):
    def __init__(self, *, vllm_config: Any = None, prefix: str = "", config: Any = None):
        super().__init__()
        config = config if config is not None else _draft_hf_config(vllm_config)
        if config is None:
            raise ValueError("the EAGLE-4 draft needs its HF config (vllm_config.speculative_config or config=)")
        raw = _hf_dict(config)
        self.cfg = draft_config_from_hf(check_supported(raw))
        aux = raw.get("eagle_aux_hidden_state_layer_ids")
        self.aux_layer_ids: Tuple[int, ...] = tuple(aux) if aux else tuple(self.cfg.aux_layer_ids)
        self.prefix = prefix
        self.draft: Optional[DraftModel] = None

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]], embed: Optional[torch.Tensor] = None
                     ) -> Set[str]:
        """The draft checkpoint's tensors (EAGLE-4 names, ``model.`` / ``midlayer.`` prefixes accepted); ``embed``:
        the target's embedding when the checkpoint has none. Returns the names taken."""
        sd = {name: t for name, t in weights}
        self.draft = DraftModel(self.cfg, wmod.draft_from_state_dict(self.cfg, sd, embed=embed))
        return set(sd)

    def _model(self) -> DraftModel:
        if self.draft is None:
            raise RuntimeError("load_weights first")
        return self.draft

    def combine_hidden_states(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """Target aux hidden states ``[T, num_aux * H_target]`` -> draft hidden ``[T, H]``."""
        return self._model().project(hidden_states)

    def forward_rows(self, input_ids: torch.Tensor, positions: torch.Tensor, hidden_states: torch.Tensor,
                     attend: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
        return self._model().forward_rows(input_ids, positions, hidden_states, attend)

    def compute_candidates(self, normed: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-``k`` children of each row: (probabilities fp32 ``[T, k]``, target ids int64 ``[T, k]``)."""
        return self._model().candidates(normed, k)

    def compute_logits(self, normed: torch.Tensor) -> torch.Tensor:
        """``[T, vocab]`` fp32: the candidates' exact logits, ``-inf`` elsewhere (full-vocabulary heads: all)."""
        ids, logits = self._model().candidate_logits(normed)
        return scatter_to_vocab(Candidates(logits.float(), ids.long()), self.cfg.vocab_size)


EntryClass = [LlamaForCausalLMEagle4]
