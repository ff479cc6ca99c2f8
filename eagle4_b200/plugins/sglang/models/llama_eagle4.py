"""``LlamaForCausalLMEagle4`` for SGLang's model registry: the EAGLE-4 draft head over this package's draft model.

The released draft checkpoint (``config.json`` + safetensors in the EAGLE-4 names) is validated
(``eagle4_b200.models.eagle4_config``) and loaded into the runtime layout; the forward runs this package's draft
layer (fused kernels, its own paged draft KV) and the low-rank candidate head. Reference counterpart:
``eagle_harness/sglang/models/llama_eagle4.py`` (the same config keys and weight names).
"""

from __future__ import annotations

from typing import Iterable, Optional, Tuple

import torch

from eagle4_b200.models import weights as wmod
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.eagle4_config import draft_config_from_hf


class LlamaForCausalLMEagle4(torch.nn.Module):
    def __init__(self, config, quant_config=None, prefix: str = ""):
        super().__init__()
        if quant_config is not None:
            raise NotImplementedError("eagle4_b200 drafts are served in bf16 (no quantization)")
        hf = config.to_dict() if hasattr(config, "to_dict") else dict(config)
        self.cfg = draft_config_from_hf(hf)
        self.draft: Optional[DraftModel] = None

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]], embed: Optional[torch.Tensor] = None):
        sd = {name: t for name, t in weights}
        self.draft = DraftModel(self.cfg, wmod.draft_from_state_dict(self.cfg, sd, embed=embed))
        return set(sd)

    def forward(self, ids, hidden, pos, req, write_slot, ctx_start, ctx_len, extra, n_extra, cache, max_keys=None):
        """Draft rows -> ``(normed, next hidden)`` (the draft layer over its own paged KV cache)."""
        return self.draft.forward(ids, hidden, pos, req, write_slot, ctx_start, ctx_len, extra, n_extra, cache,
                                  max_keys)

    def candidates(self, normed: torch.Tensor, k: int):
        return self.draft.candidates(normed, k)


EntryClass = [LlamaForCausalLMEagle4]
