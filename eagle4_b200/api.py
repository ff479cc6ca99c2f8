"""Public entry point for generation: build a target and draft head, then ``LLM.generate``.

    llm = LLM.synthetic("qwen3.8-27b", device="cuda")      # random-init weights of the named shape
    out = llm.generate(prompt_ids, max_new_tokens=256)       # [B, P] int64 (CPU, ideally pinned) -> [B, new]

``generate`` copies the prompts to the device, runs the serving loop (speculative EAGLE rounds, or plain decode) and
returns the generated ids on the host.
"""

from __future__ import annotations

import dataclasses
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
    "tiny-mamba": (configs.tiny_nemotron, lambda t: dataclasses.replace(configs.tiny_draft(t), aux_layer_ids=(1, 3, 5))),
    # attn_norm input fusion + latent ReLU^2 MoE draft (the Nemotron-class draft structures)
    "tiny-moe": (configs.tiny_nemotron, lambda t: dataclasses.replace(configs.tiny_moe_draft(t),
                                                                      aux_layer_ids=(1, 3, 5))),
    "nemotron-h-8b-moe": (configs.nemotron_h_8b, configs.nemotron_moe_draft),
    "qwen3.8-27b": (configs.qwen38_27b, configs.qwen38_draft),
    "nemotron-h-8b": (configs.nemotron_h_8b, lambda t: configs.generic_draft(t, heads=32, kv=8, head_dim=128)),
    "llama-3.1-8b": (configs.llama31_8b, configs.eagle3_llama_draft),
    # production widths, two layers, tied embeddings: kernel profiling at real shapes within a few GB
    "qwen3.8-27b-2l": (lambda: configs.profile_slice(configs.qwen38_27b()),
                       lambda t: dataclasses.replace(configs.qwen38_draft(t), aux_layer_ids=(0, 1, 1))),
    "nemotron-h-8b-2l": (lambda: configs.profile_slice(configs.nemotron_h_8b(), ("mamba", "attn")),
                         lambda t: dataclasses.replace(configs.generic_draft(t, heads=32, kv=8, head_dim=128),
                                                       aux_layer_ids=(0, 1, 1))),
}


@dataclass
class TreeSpec:
    steps: int = 12
    top_k: int = 4
    draft_tokens: int = 16


class LLM:
    def __init__(self, target: TargetModel, draft: Optional[DraftModel], *, tree: TreeSpec = TreeSpec(),
                 max_batch: int = 1, max_len: int = 4096, page: int = 16, config=None, temperature: float = 0.0,
                 seed: int = 0, kv_tokens: Optional[int] = None):
        """``config``: a ``HarnessConfig``, or the ``--speculative-algorithm-config`` JSON text (inline or a path);
        None is the static tree of ``tree``. ``temperature > 0`` samples (sampled trees with tree rejection)."""
        if isinstance(config, str):
            config = parse_harness_config(config)
        config = _with_packaged_profile(config, target, draft)
        self.target, self.draft, self.tree = target, draft, tree
        self.engine = Engine(target, draft, max_reqs=max_batch, max_len=max_len, page=page, steps=tree.steps,
                             top_k=tree.top_k, verify_tokens=tree.draft_tokens, config=config,
                             temperature=temperature, seed=seed, kv_tokens=kv_tokens)

    @classmethod
    def synthetic(cls, name: str, *, device="cuda", dtype=torch.bfloat16, seed: int = 0, tree: TreeSpec = TreeSpec(),
                  max_batch: int = 1, max_len: int = 4096, draft: bool = True, config=None, tp=None,
                  temperature: float = 0.0, sample_seed: int = 0, kv_tokens: Optional[int] = None) -> "LLM":
        """Random-init weights (N(0, 0.02)) of a named architecture; the draft shares the target's embedding.
        With ``tp`` (a :class:`~eagle4_b200.parallel.tp.TensorParallel`) every rank draws the same full weights and
        keeps its shard."""
        from eagle4_b200.parallel.sharding import shard_draft, shard_target

        tcfg_fn, dcfg_fn = NAMED[name]
        tcfg = tcfg_fn()
        dcfg = dcfg_fn(tcfg)
        world, rank = (tp.world, tp.rank) if tp is not None else (1, 0)
        tw = weights.init_target(tcfg, device=device, dtype=dtype, seed=seed)
        dw = weights.init_draft(dcfg, device=device, dtype=dtype, seed=seed + 1, embed=tw["embed"],
                                lm_head=tw["lm_head"]) if draft else None
        ltcfg, tw = shard_target(tcfg, tw, world, rank)
        target = TargetModel(ltcfg, tw, aux_layer_ids=dcfg.aux_layer_ids, tp=tp)
        dm = None
        if draft:
            ldcfg, dw = shard_draft(dcfg, dw, world, rank)
            dm = DraftModel(ldcfg, dw, tp=tp)
        return cls(target, dm, tree=tree, max_batch=max_batch, max_len=max_len, config=config,
                   temperature=temperature, seed=sample_seed, kv_tokens=kv_tokens)

    def generate(self, prompt_ids, max_new_tokens: int, *, speculative: bool = True) -> torch.Tensor:
        """``prompt_ids [B, P]`` int64 on the host (or a list of 1-D prompts of different lengths) -> generated ids
        ``[B, max_new_tokens]`` on the host."""
        if isinstance(prompt_ids, (list, tuple)):
            dev_ids = [p.to(self.target.device, non_blocking=True) for p in prompt_ids]
            out = self.engine.generate(dev_ids, max_new_tokens, speculative=speculative)
            return torch.tensor(out, dtype=torch.int64)
        dev_ids = prompt_ids.to(self.target.device, non_blocking=True)
        out = self.engine.generate(dev_ids, max_new_tokens, speculative=speculative)
        return torch.tensor(out, dtype=torch.int64)

    def complete(self, prompts, tokenizer=None, *, max_new_tokens: int = 128, stop=(), stop_token_ids=(),
                 ignore_eos: bool = False, speculative: bool = True) -> list:
        """Continuous-batching generation of many requests, each ending on its own stop condition.

        ``prompts``: texts (with ``tokenizer``, a Hugging Face tokenizer) or token-id lists; more prompts than
        ``max_batch`` queue and join the batch as rows free up. Returns one dict per prompt, in order:
        ``token_ids``, ``finish_reason`` (``length`` / ``stop`` / ``eos``) and, with a tokenizer, ``text`` (cut
        before the first stop string that ended it)."""
        from eagle4_b200.runtime.scheduler import RequestParams, Scheduler

        stop = (stop,) if isinstance(stop, str) else tuple(stop)
        if (stop or any(isinstance(p, str) for p in prompts)) and tokenizer is None:
            raise ValueError("text prompts and stop strings need a tokenizer")
        detok = (lambda ids: tokenizer.decode(ids)) if tokenizer is not None else None
        eos = getattr(tokenizer, "eos_token_id", None) if tokenizer is not None else None
        params = RequestParams(max_new_tokens=max_new_tokens, stop_token_ids=tuple(stop_token_ids), eos_token_id=eos,
                               ignore_eos=ignore_eos, stop=stop)
        sched = Scheduler(self.engine, speculative=speculative, detokenize=detok)
        reqs = [sched.submit(list(tokenizer(p)["input_ids"]) if isinstance(p, str) else list(p), params)
                for p in prompts]
        sched.run()
        out = []
        for r in reqs:
            row = {"token_ids": list(r.output), "finish_reason": r.finish_reason}
            if tokenizer is not None:
                text = tokenizer.decode(r.output)
                cuts = [i for i in (text.find(x) for x in stop) if i >= 0] if r.finish_reason == "stop" else []
                row["text"] = text[:min(cuts)] if cuts else text
            out.append(row)
        return out


def _with_packaged_profile(config: Optional[HarnessConfig], target: TargetModel,
                           draft: Optional[DraftModel]) -> Optional[HarnessConfig]:
    """A serve-mode config without calibration data takes the packaged cost profile measured on this setup (same
    GPU, TP size and model shapes), when one ships with the package; anything else is returned unchanged."""
    if config is None or config.data_path or draft is None or not config.mode.uses_cost_model:
        return config
    if target.device.type != "cuda":
        return config
    from eagle4_b200.core.cost_profiles import packaged_cost_profile

    if target.tp is not None and target.tp.world > 1:
        return config  # the packaged profiles are measured on one GPU
    path = packaged_cost_profile(device_name=torch.cuda.get_device_name(target.device), tp_size=1,
                                 dtype="bfloat16", quantization=None, target_config=target.cfg.to_hf(),
                                 draft_config=draft.cfg.to_hf())
    return dataclasses.replace(config, data_path=path) if path else config


def _load_safetensors_dir(path: str, device) -> dict:
    import os

    from safetensors.torch import load_file

    sd = {}
    for name in sorted(os.listdir(path)):
        if name.endswith(".safetensors"):
            sd.update(load_file(os.path.join(path, name), device=str(device)))
    if not sd:
        raise FileNotFoundError(f"no .safetensors files under {path}")
    return sd


def from_pretrained(model_path: str, draft_path: Optional[str] = None, *, device="cuda", dtype=torch.bfloat16,
                    tree: TreeSpec = TreeSpec(), max_batch: int = 1, max_len: int = 4096, config=None,
                    tp=None, temperature: float = 0.0, sample_seed: int = 0, kv_tokens: Optional[int] = None) -> LLM:
    """An :class:`LLM` from a Hugging Face target directory and an EAGLE-4 / EAGLE-3 draft directory (both with
    ``config.json`` and safetensors). Draft configs are validated; structures this package does not build raise.
    With ``tp`` (a :class:`~eagle4_b200.parallel.tp.TensorParallel`) every rank reads the full checkpoints into host
    memory, keeps its shard and moves only that to its GPU."""
    import json
    import os

    from eagle4_b200.models.configs import TargetConfig
    from eagle4_b200.models.eagle4_config import draft_config_from_hf
    from eagle4_b200.parallel.sharding import shard_draft, shard_target

    with open(os.path.join(model_path, "config.json"), encoding="utf-8") as f:
        tcfg = TargetConfig.from_hf(json.load(f))
    dm = None
    aux = (2, tcfg.num_layers // 2, tcfg.num_layers - 3)
    if draft_path is not None:
        with open(os.path.join(draft_path, "config.json"), encoding="utf-8") as f:
            dcfg = draft_config_from_hf(json.load(f), target_vocab_size=tcfg.vocab_size,
                                        target_num_layers=tcfg.num_layers)
        aux = dcfg.aux_layer_ids
    world, rank = (tp.world, tp.rank) if tp is not None else (1, 0)
    sd = {k: v.to(dtype) if v.is_floating_point() else v for k, v in _load_safetensors_dir(model_path, "cpu").items()}
    full = weights.target_from_hf(tcfg, sd)
    del sd
    ltcfg, tw = shard_target(tcfg, full, world, rank)
    tw = {k: v.to(device) for k, v in tw.items()}
    target = TargetModel(ltcfg, tw, aux_layer_ids=aux, tp=tp)
    if draft_path is not None:
        ldcfg, dw = shard_draft(dcfg, weights.load_draft(draft_path, dcfg, device="cpu", dtype=dtype,
                                                         embed=full["embed"]), world, rank)
        dm = DraftModel(ldcfg, {k: v.to(device) for k, v in dw.items()}, tp=tp)
    del full
    return LLM(target, dm, tree=tree, max_batch=max_batch, max_len=max_len, config=config, temperature=temperature,
               seed=sample_seed, kv_tokens=kv_tokens)
