"""EAGLE-4 draft ``config.json`` validation, sliding-window resolution and conversion to ``DraftConfig``.

A released draft config is a Llama config plus EAGLE keys. Structural keys this package does not build are refused,
so a new draft structure can never be served silently wrong. The key sets and the sliding-window activation rule
are those of the released checkpoints (reference ``eagle_harness/models/eagle4_config.py:27-285``):

* window activation: an explicit ``layer_types`` wins, then ``use_sliding_window``, then a positive
  ``sliding_window`` alone; sliding-window drafts are single-layer;
* ``eagle_config`` carries exactly three aux layers; ``efficient_lm_head_config`` is ``low_rank`` or
  ``weighted_low_rank`` with ``rank`` / ``num_candidates`` / ``smooth_factor``.

Configs are plain dicts here (or any object with ``to_dict()``); no engine is needed.
"""

from __future__ import annotations

from numbers import Integral
from typing import Any, Dict, Mapping, Optional, Tuple

from eagle4_b200.models.configs import DraftConfig
from eagle4_b200.models.eagle4_structure import LATENT_MOE_ARCHITECTURE, draft_moe_architecture, draft_uses_rope

EAGLE4_ARCH = "LlamaForCausalLMEagle4"
LAYER_TYPES = ("full_attention", "sliding_attention")
LATENT_MOE = LATENT_MOE_ARCHITECTURE
DENSE_MOE = ("sparse_swiglu",)

STRUCTURAL_KEYS = frozenset({
    "draft_vocab_size", "target_hidden_size", "num_aux_hidden_states", "eagle_config",
    "share_draft_embedding_from_target", "fc_norm", "enable_fc_norm", "bias", "input_fuse_type", "attn_norm",
    "use_rope", "position_embedding_type", "partial_rotary_factor", "rope_is_neox_style", "sliding_window",
    "use_sliding_window", "layer_types", "norm_output", "enable_post_mlp_norm", "enable_moe", "moe_architecture",
    "n_routed_experts", "num_experts_per_tok", "moe_intermediate_size", "n_shared_experts",
    "moe_shared_expert_intermediate_size", "moe_latent_size", "n_group", "topk_group", "norm_topk_prob",
    "routed_scaling_factor", "scoring_func", "topk_method", "expert_bias_update_rate", "moe_router_bias_update_rate",
    "efficient_lm_head_config", "enable_2hs", "enable_defa",
})
NON_STRUCTURAL_KEYS = frozenset({
    "_torchspec_version", "load_balance_loss_alpha", "seq_aux_loss_alpha", "aux_loss_alpha", "moe_seq_aux_loss_coeff",
    "expert_parallel_size", "moe_expert_parallel_size", "moe_initialization", "moe_mtp_layer_index",
    "moe_mtp_source_revision", "moe_router_dtype", "rope_interleave", "max_window_layers", "quantization_config",
})
RUNTIME_KEYS = frozenset({"context_len", "encoder_only", "language_only", "language_model_only"})
DERIVED_HEAD_DIM_KEYS = frozenset({"v_head_dim", "swa_head_dim", "swa_v_head_dim"})
HEAD_KEYS = frozenset({"type", "rank", "num_candidates", "smooth_factor"})

# Llama config attributes (the keys every draft may carry besides the EAGLE ones).
LLAMA_KEYS = frozenset({
    "vocab_size", "max_position_embeddings", "hidden_size", "intermediate_size", "num_hidden_layers",
    "num_attention_heads", "num_key_value_heads", "hidden_act", "initializer_range", "rms_norm_eps",
    "pretraining_tp", "use_cache", "rope_theta", "rope_scaling", "rope_parameters", "attention_bias",
    "attention_dropout", "mlp_bias", "head_dim", "tie_word_embeddings", "bos_token_id", "eos_token_id",
    "pad_token_id", "architectures", "model_type", "torch_dtype", "dtype", "transformers_version",
    "return_dict", "output_hidden_states", "output_attentions", "torchscript", "use_bfloat16",
    "tf_legacy_loss", "pruned_heads", "chunk_size_feed_forward", "is_encoder_decoder", "is_decoder",
    "cross_attention_hidden_size", "add_cross_attention", "tie_encoder_decoder", "finetuning_task", "id2label",
    "label2id", "task_specific_params", "problem_type", "tokenizer_class", "prefix", "sep_token_id",
    "decoder_start_token_id", "name_or_path", "_name_or_path", "_attn_implementation_autoset",
})


def _as_dict(config) -> Dict[str, Any]:
    if isinstance(config, Mapping):
        return dict(config)
    return dict(config.to_dict())


def resolve_draft_sliding_window(config) -> Optional[int]:
    """The draft's attention window, or None (also None for non-EAGLE-4 configs); invalid settings raise."""
    cfg = _as_dict(config)
    if EAGLE4_ARCH not in (cfg.get("architectures") or ()):
        return None
    window = cfg.get("sliding_window")
    if window is not None:
        if isinstance(window, bool) or not isinstance(window, Integral) or window < 1:
            raise ValueError(f"EAGLE4 draft sliding_window must be a positive integer, got {window!r}.")
        window = int(window)
    enabled = cfg.get("use_sliding_window")
    if enabled is not None and not isinstance(enabled, bool):
        raise ValueError(f"EAGLE4 draft use_sliding_window must be a boolean, got {enabled!r}.")
    layers = cfg.get("num_hidden_layers")
    types = cfg.get("layer_types")
    if types is not None:
        if not isinstance(types, (list, tuple)) or len(types) != layers:
            raise ValueError("EAGLE4 draft layer_types must list one entry per draft layer, got "
                             f"{types!r} for num_hidden_layers={layers}.")
        bad = [t for t in types if t not in LAYER_TYPES]
        if bad:
            raise ValueError(f"EAGLE4 draft layer_types supports only {list(LAYER_TYPES)}, got {bad!r}.")
        if "sliding_attention" in types and window is None:
            raise ValueError("EAGLE4 draft layer_types has sliding_attention but no positive sliding_window.")
        enabled = types[0] == "sliding_attention"
    elif enabled is None:
        enabled = window is not None
    if enabled and window is None:
        raise ValueError("EAGLE4 draft use_sliding_window requires a positive sliding_window.")
    if not enabled:
        return None
    if layers != 1:
        raise ValueError(f"EAGLE4 sliding-window drafts must have num_hidden_layers=1, got {layers}.")
    return window


def _expect(cfg: Mapping[str, Any], name: str, allowed: tuple) -> None:
    if name not in cfg:
        return
    v = cfg[name]
    if isinstance(v, bool) or any(isinstance(a, bool) for a in allowed):
        ok = any(v is a for a in allowed)
    else:
        ok = v in allowed
    if not ok:
        raise ValueError(f"EAGLE4 draft config {name}={v!r} is not supported (expected one of {list(allowed)}).")


def validate_eagle4_draft_config(config) -> None:
    """Refuse draft configs whose structure this package does not build."""
    cfg = _as_dict(config)
    keys = set(cfg) - LLAMA_KEYS - RUNTIME_KEYS - DERIVED_HEAD_DIM_KEYS
    unknown = sorted(keys - STRUCTURAL_KEYS - NON_STRUCTURAL_KEYS)
    if unknown:
        raise ValueError(f"EAGLE4 draft config has keys this model does not implement: {unknown}.")
    head_dim = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    for name in sorted(DERIVED_HEAD_DIM_KEYS):
        v = cfg.get(name)
        if v and v != head_dim:
            raise ValueError(f"EAGLE4 draft config {name}={v} differs from head_dim={head_dim}; "
                             "the draft attention uses one head dim for q, k and v.")
    for name in ("fc_norm", "enable_fc_norm", "attn_norm", "use_rope", "norm_output", "enable_post_mlp_norm",
                 "enable_moe", "share_draft_embedding_from_target", "norm_topk_prob"):
        _expect(cfg, name, (True, False))
    for name in ("bias", "attention_bias", "mlp_bias", "enable_2hs", "enable_defa"):
        _expect(cfg, name, (False,))
    _expect(cfg, "rope_is_neox_style", (True,))
    _expect(cfg, "partial_rotary_factor", (None, 0, 1))
    _expect(cfg, "input_fuse_type", ("concat",))
    _expect(cfg, "num_aux_hidden_states", (3,))
    _expect(cfg, "moe_architecture", DENSE_MOE + (LATENT_MOE,))
    eagle = cfg.get("eagle_config") or {}
    extra = set(eagle) - {"use_aux_hidden_state", "eagle_aux_hidden_state_layer_ids"}
    ids = eagle.get("eagle_aux_hidden_state_layer_ids")
    if extra or (ids is not None and len(ids) != 3):
        raise ValueError(f"EAGLE4 draft eagle_config={eagle!r} is not supported: the fc input takes exactly three "
                         "aux hidden states.")
    head = cfg.get("efficient_lm_head_config")
    if head is not None and (not isinstance(head, dict) or head.get("type") not in ("low_rank", "weighted_low_rank")
                             or set(head) - HEAD_KEYS):
        raise ValueError(f"EAGLE4 draft efficient_lm_head_config={head!r} is not supported.")
    moe = draft_moe_architecture(cfg)
    latent = moe == LATENT_MOE
    _expect(cfg, "hidden_act", ("relu2",) if latent else ("silu",))
    if moe is not None:
        _expect(cfg, "scoring_func", ("sigmoid",))
        _expect(cfg, "topk_method", ("noaux_tc",))
    if latent:
        need = ["n_routed_experts", "num_experts_per_tok", "moe_intermediate_size", "moe_latent_size"]
        if cfg.get("n_shared_experts"):
            need.append("moe_shared_expert_intermediate_size")
        missing = [n for n in need if not cfg.get(n)]
        if missing:
            raise ValueError(f"EAGLE4 latent MoE draft config is missing {missing}.")
    single = {"sliding window": resolve_draft_sliding_window(cfg) is not None, "attn_norm": bool(cfg.get("attn_norm")),
              "NoPE": not draft_uses_rope(cfg), "latent MoE": latent}
    used = [k for k, on in single.items() if on]
    if used and cfg.get("num_hidden_layers") != 1:
        raise ValueError(f"EAGLE4 draft structures {used} are implemented for single-layer drafts, got "
                         f"num_hidden_layers={cfg.get('num_hidden_layers')}.")


# Structures the validator accepts that this package's draft model does not build (none of the reference's engine
# adapters builds them either: eagle_harness/models/eagle4_config.py:259-266, sglang/models/llama_eagle4.py:91-100).
UNBUILT = {"enable_post_mlp_norm": True}


def check_supported(config) -> None:
    """Validate, then refuse structures the draft model does not build: the post-MLP norm, the sparse SwiGLU MoE,
    more than one layer. attn_norm (eh_proj input fusion), NoPE and the latent ReLU^2 MoE are built."""
    cfg = _as_dict(config)
    validate_eagle4_draft_config(cfg)
    used = [f"{k}={v!r}" for k, v in UNBUILT.items() if cfg.get(k) == v]
    if used:
        raise NotImplementedError(f"EAGLE-4 drafts with {used} are not built by eagle4_b200.")
    moe = draft_moe_architecture(cfg)
    if moe not in (None, LATENT_MOE):
        raise NotImplementedError(f"EAGLE-4 drafts with the {moe!r} MoE are not built by eagle4_b200 (the latent "
                                  "ReLU^2 MoE is).")
    if cfg.get("num_hidden_layers") != 1:
        raise NotImplementedError(f"EAGLE-4 drafts with {cfg.get('num_hidden_layers')} layers are not built (1 only).")


def _moe_of(cfg: dict) -> Optional[dict]:
    if draft_moe_architecture(cfg) != LATENT_MOE:
        return None
    from eagle4_b200.models.configs import latent_moe

    groups = int(cfg.get("n_group") or 1)
    return latent_moe(int(cfg["n_routed_experts"]), int(cfg["num_experts_per_tok"]), int(cfg["moe_intermediate_size"]),
                      int(cfg["moe_latent_size"]),
                      int(cfg.get("moe_shared_expert_intermediate_size") or 0) if cfg.get("n_shared_experts") else 0,
                      n_group=groups, topk_group=int(cfg.get("topk_group") or groups),
                      norm_topk_prob=bool(cfg.get("norm_topk_prob", True)),
                      scale=float(cfg.get("routed_scaling_factor") or 1.0))


def _default_aux(target_num_layers: Optional[int]) -> Tuple[int, ...]:
    if not target_num_layers:
        raise ValueError("the draft config names no aux layers (eagle_config.eagle_aux_hidden_state_layer_ids): "
                         "give the target's layer count")
    n = int(target_num_layers)
    return (2, n // 2, n - 3)


def draft_config_from_hf(config, *, target_vocab_size: Optional[int] = None,
                         target_num_layers: Optional[int] = None) -> DraftConfig:
    """A ``DraftConfig`` from a released EAGLE-4 (or EAGLE-3) draft ``config.json``. A config that names no aux layers
    (``eagle_config.eagle_aux_hidden_state_layer_ids``; common for EAGLE-3 drafts) takes the usual EAGLE-3 choice for
    a target of ``target_num_layers`` layers: layers 2, L // 2 and L - 3."""
    cfg = _as_dict(config)
    eagle4 = EAGLE4_ARCH in (cfg.get("architectures") or ())
    if eagle4:
        check_supported(cfg)
    hd = cfg.get("head_dim") or cfg["hidden_size"] // cfg["num_attention_heads"]
    rope = cfg.get("rope_parameters") or {}
    eagle = cfg.get("eagle_config") or {}
    ids = eagle.get("eagle_aux_hidden_state_layer_ids")
    vocab = target_vocab_size or cfg["vocab_size"]
    head = cfg.get("efficient_lm_head_config")
    return DraftConfig(
        family="eagle4" if eagle4 else "eagle3",
        hidden_size=cfg["hidden_size"], target_hidden_size=cfg.get("target_hidden_size", cfg["hidden_size"]),
        vocab_size=vocab, draft_vocab_size=cfg.get("draft_vocab_size") or cfg["vocab_size"],
        num_heads=cfg["num_attention_heads"], num_kv_heads=cfg.get("num_key_value_heads", cfg["num_attention_heads"]),
        head_dim=hd, intermediate_size=cfg["intermediate_size"],
        aux_layer_ids=tuple(ids) if ids else _default_aux(target_num_layers),
        rms_norm_eps=cfg.get("rms_norm_eps", 1e-6),
        rope_theta=rope.get("rope_theta", cfg.get("rope_theta", 10000.0)),
        sliding_window=resolve_draft_sliding_window(cfg) if eagle4 else None,
        fc_norm=bool(cfg.get("fc_norm") or cfg.get("enable_fc_norm")), norm_output=bool(cfg.get("norm_output")),
        use_rope=draft_uses_rope(cfg), low_rank=dict(head) if head else None,
        attn_norm=bool(cfg.get("attn_norm")) if eagle4 else False, moe=_moe_of(cfg) if eagle4 else None,
    )
