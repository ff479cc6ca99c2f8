"""Public entry point for generation: build a target and draft head, then ``LLM.generate``.

    llm = LLM.synthetic("qwen3.8-27b", device="cuda")      # random-init weights of the named shape
    out = llm.generate(prompt_ids, max_new_tokens=256)       # [B, P] int64 (CPU, ideally pinned) -> [B, new]

``generate`` copies the prompts to the device, runs the serving loop (speculative EAGLE rounds, or plain decode) and
returns the generated ids on the host.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from eagle4_b200.core.config import HarnessConfig, parse_harness_config
from eagle4_b200.models import configs, weights
from eagle4_b200.models.draft import DraftModel
from eagle4_b200.models.target import TargetModel
from eagle4_b200.runtime.engine import Engine

NAMED = {
    "tiny": (configs.tiny_hybrid, configs.tiny_draft),
    "qwen3.8-27b": (configs.qwen38_27b, configs.qwen38_draft),
    "nemotron-h-8b": (configs.nemotron_h_8b, lambda t: configs.generic_draft(t, heads=32, kv=8, head_dim=128)),
    "llama-3.1-8b": (configs.llama31_8b, configs.eagle3_llama_draft),
}


@dataclass
class TreeSpec:
    steps: int = 12
    top_k: int = 4
    draft_tokens: int = 16


class LLM:
    def __init__(self, target: TargetModel, draft: Optional[DraftModel], *, tree: TreeSpec = TreeSpec(),
                 max_batch: int = 1, max_len: int = 4096, page: int = 16, config=None):
        """``config``: a ``HarnessConfig``, or the ``--speculative-algorithm-config`` JSON text (inline or a path);
        None is the static tree of ``tree``."""
        if isinstance(config, str):
            config = parse_harness_config(config)
        self.target, self.draft, self.tree = target, draft, tree
        self.engine = Engine(target, draft, max_reqs=max_batch, max_len=max_len, page=page, steps=tree.steps,
                             top_k=tree.top_k, verify_tokens=tree.draft_tokens, config=config)

    @classmethod
    def synthetic(cls, name: str, *, device="cuda", dtype=torch.bfloat16, seed: int = 0, tree: TreeSpec = TreeSpec(),
                  max_batch: int = 1, max_len: int = 4096, draft: bool = True, config=None) -> "LLM":
        """Random-init weights (N(0, 0.02)) of a named architecture; the draft shares the target's embedding."""
        tcfg_fn, dcfg_fn = NAMED[name]
        tcfg = tcfg_fn()
        dcfg = dcfg_fn(tcfg)
        tw = weights.init_target(tcfg, device=device, dtype=dtype, seed=seed)
        target = TargetModel(tcfg, tw, aux_layer_ids=dcfg.aux_layer_ids)
        dm = None
        if draft:
            dw = weights.init_draft(dcfg, device=device, dtype=dtype, seed=seed + 1, embed=tw["embed"])
            dm = DraftModel(dcfg, dw)
        return cls(target, dm, tree=tree, max_batch=max_batch, max_len=max_len, config=config)

    def generate(self, prompt_ids: torch.Tensor, max_new_tokens: int, *, speculative: bool = True) -> torch.Tensor:
        """``prompt_ids [B, P]`` int64 on the host -> generated ids ``[B, max_new_tokens]`` on the host."""
        dev_ids = prompt_ids.to(self.target.device, non_blocking=True)
        out = self.engine.generate(dev_ids, max_new_tokens, speculative=speculative)
        return torch.tensor(out, dtype=torch.int64)
