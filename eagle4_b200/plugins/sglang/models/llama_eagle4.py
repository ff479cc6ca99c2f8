"""``LlamaForCausalLMEagle4`` for SGLang's model registry: the EAGLE-4 draft head over this package's draft model.

The released draft checkpoint (``config.json`` + safetensors in the EAGLE-4 names) is validated
(``eagle4_b200.models.eagle4_config``) and loaded into the runtime layout; the forward runs this package's draft
layer (fused kernels, its own paged draft KV) and the low-rank candidate head. Besides the forward, SGLang's EAGLE
worker calls a draft model for:

* ``set_embed`` / ``set_embed_and_head``: the target's embedding is shared; the EAGLE-4 draft keeps its own LM head
  (the candidate head re-scores with it), so the target's head is not taken;
* ``candidate_topk``: the children of each row (the softmax over the ``C`` candidates, which is the softmax of the
  ``-inf``-filled full row); ``proposal_candidates``: the whole sparse distribution sampled trees draw from;
* ``get_hot_token_id`` (no reduced vocabulary) and ``get_attention_sliding_window_size`` (SGLang counts the window
  without the current token).

Reference counterpart: ``eagle_harness/sglang/models/llama_eagle4.py:327-500`` (the same config keys, weight names
and host-facing methods).
"""

from __future__ import annotations

from typing import Iterable, Optional, Tuple

import torch

from eagle4_b200.models import weights as wmod
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.eagle4_config import draft_config_from_hf
from eagle4_b200.plugins.candidate_logits import Candidates


class LlamaForCausalLMEagle4(torch.nn.Module):
    def __init__(self, config, quant_config=None, prefix: str = ""):
        super().__init__()
        if quant_config is not None:
            raise NotImplementedError("eagle4_b200 drafts are served in bf16 (no quantization)")
        hf = config.to_dict() if hasattr(config, "to_dict") else dict(config)
        self.cfg = draft_config_from_hf(hf)
        self.draft: Optional[DraftModel] = None
        self._embed: Optional[torch.Tensor] = None

    def _model(self) -> DraftModel:
        if self.draft is None:
            raise RuntimeError("load_weights first")
        return self.draft

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]], embed: Optional[torch.Tensor] = None):
        """The checkpoint's tensors (EAGLE-4 names; missing low-rank factors are rebuilt by SVD); ``embed``: the
        target's embedding when the checkpoint has none (or the one ``set_embed`` gave). Returns the names taken."""
        sd = {name: t for name, t in weights}
        self.draft = DraftModel(self.cfg, wmod.draft_from_state_dict(
            self.cfg, sd, embed=embed if embed is not None else self._embed))
        return set(sd)

    # ---- what SGLang's EAGLE worker shares with the draft
    def set_embed(self, embed: torch.Tensor) -> None:
        """Share the target's embedding table."""
        self._embed = embed
        if self.draft is not None:
            self.draft.w["embed"] = embed

    def set_embed_and_head(self, embed: torch.Tensor, head: torch.Tensor) -> None:
        """Share only the embedding: the draft's candidate head re-scores with the draft's own LM head."""
        self.set_embed(embed)

    def get_hot_token_id(self) -> None:
        """No reduced draft vocabulary (EAGLE-4 drafts emit target ids)."""
        return None

    def get_attention_sliding_window_size(self) -> Optional[int]:
        """The draft's window as SGLang counts it (without the current token), or None."""
        w = self.cfg.sliding_window
        return None if not w else w - 1

    # ---- the forward and the candidate head
    def forward(self, ids, hidden, pos, req, write_slot, ctx_start, ctx_len, extra, n_extra, cache, max_keys=None):
        """Draft rows -> ``(normed, next hidden)`` (the draft layer over its own paged KV cache)."""
        return self._model().forward(ids, hidden, pos, req, write_slot, ctx_start, ctx_len, extra, n_extra, cache,
                                     max_keys)

    def candidates(self, normed: torch.Tensor, k: int):
        return self._model().candidates(normed, k)

    def candidate_topk(self, normed: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-``k`` next tokens of each row: (fp32 probabilities ``[rows, k]``, ids ``[rows, k]``)."""
        return self._model().candidates(normed, k)

    def proposal_candidates(self, normed: torch.Tensor) -> Candidates:
        """The sparse distribution a sampled tree draws from: the ``C`` candidates' exact fp32 logits and ids."""
        ids, logits = self._model().candidate_logits(normed)
        return Candidates(logits.float(), ids.long())


EntryClass = [LlamaForCausalLMEagle4]
