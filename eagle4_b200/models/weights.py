"""Weights: random initialisation of every architecture (benchmarks run on synthetic weights of the named shapes),
Hugging Face checkpoint mapping into the fused runtime layout, and the EAGLE-4 draft safetensors layout.

Draft checkpoint names accepted (the released layout, ``tests/test_eagle4_model.py:39-63`` and
``sglang/models/llama_eagle4.py:497-592`` in the reference): ``fc.weight`` (or ``fc.linear.weight``),
``fc_norm.{0,1,2}.weight``, ``layers.0.{input_layernorm,hidden_norm,post_attention_layernorm}.weight``,
``layers.0.self_attn.{q,k,v,o}_proj.weight``, ``layers.0.mlp.{gate,up,down}_proj.weight``, ``norm.weight``,
``embed_tokens.weight`` (optional), ``lm_head.weight``, ``efficient_lm_head.weight`` ``[V, r]``,
``efficient_lm_head_down_proj.weight`` ``[r, H]``, ``d2t`` (EAGLE-3 draft-to-target offsets); prefixes ``model.`` and
``midlayer.`` (for ``layers.0.``) are accepted.
"""

from __future__ import annotations

import json
import os
from typing import Dict, Optional

import torch

from eagle4_b200.models.configs import DraftConfig, TargetConfig
from eagle4_b200.ops.reference import interleave_gate_up


def _normal(shape, std, gen, device, dtype):
    if gen is None:  # the meta device: shapes only (memory planning)
        return torch.empty(*shape, device=device, dtype=dtype)
    return (torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)


def _generator(dev: torch.device, seed: int) -> Optional[torch.Generator]:
    return None if dev.type == "meta" else torch.Generator(device=dev).manual_seed(seed)


def init_target(cfg: TargetConfig, *, device="cpu", dtype=torch.float32, seed: int = 0) -> Dict[str, torch.Tensor]:
    """N(0, std) weights in the fused runtime layout; norms at identity, GDN/Mamba2 gates at HF's defaults."""
    dev = torch.device(device)
    gen = _generator(dev, seed)
    std = cfg.init_std
    H = cfg.hidden_size
    one = 0.0 if cfg.norm_offset else 1.0
    w: Dict[str, torch.Tensor] = {}

    def lin(n, k):
        return _normal((n, k), std, gen, dev, dtype)

    def norm(n):
        return torch.full((n,), one, dtype=dtype, device=dev)

    w["embed"] = _normal((cfg.vocab_size, H), std, gen, dev, dtype)
    for i, (mixer, mlp) in enumerate(cfg.layers):
        if mixer is not None:
            w[f"l{i}.norm1"] = norm(H)
        if mixer == "attn":
            qd = cfg.num_heads * cfg.head_dim * (2 if cfg.attn_output_gate else 1)
            w[f"l{i}.qkv"] = lin(qd + 2 * cfg.num_kv_heads * cfg.head_dim, H)
            if cfg.qk_norm:
                w[f"l{i}.q_norm"] = norm(cfg.head_dim)
                w[f"l{i}.k_norm"] = norm(cfg.head_dim)
            w[f"l{i}.o_proj"] = lin(H, cfg.num_heads * cfg.head_dim)
        elif mixer == "gdn":
            rows = cfg.gdn_conv_dim + cfg.gdn_value_dim + 2 * cfg.gdn_v_heads
            w[f"l{i}.in_proj"] = lin(rows, H)
            w[f"l{i}.conv"] = _normal((cfg.gdn_conv_dim, cfg.conv_kernel), 0.5, gen, dev, dtype)
            a = torch.empty(cfg.gdn_v_heads, device=dev).uniform_(1.0, 16.0, generator=gen)
            w[f"l{i}.A_log"] = a.log().float()
            w[f"l{i}.dt_bias"] = torch.ones(cfg.gdn_v_heads, dtype=torch.float32, device=dev)
            w[f"l{i}.gnorm"] = torch.ones(cfg.gdn_v_dim, dtype=dtype, device=dev)
            w[f"l{i}.out_proj"] = lin(H, cfg.gdn_value_dim)
        elif mixer == "mamba":
            rows = cfg.mamba_inner + cfg.mamba_conv_dim + cfg.mamba_heads
            w[f"l{i}.in_proj"] = lin(rows, H)
            w[f"l{i}.conv"] = _normal((cfg.mamba_conv_dim, cfg.conv_kernel), 0.5, gen, dev, dtype)
            a = torch.empty(cfg.mamba_heads, device=dev).uniform_(1.0, 16.0, generator=gen)
            w[f"l{i}.A_log"] = a.log().float()
            w[f"l{i}.dt_bias"] = torch.ones(cfg.mamba_heads, dtype=torch.float32, device=dev)
            w[f"l{i}.D"] = torch.ones(cfg.mamba_heads, dtype=torch.float32, device=dev)
            w[f"l{i}.gnorm"] = torch.ones(cfg.mamba_inner // cfg.mamba_groups, dtype=dtype, device=dev)
            w[f"l{i}.out_proj"] = lin(H, cfg.mamba_inner)
        if mlp is not None:
            w[f"l{i}.norm2"] = norm(H)
            if mlp == "swiglu":
                w[f"l{i}.gate_up"] = lin(2 * cfg.intermediate_size, H)
            else:
                w[f"l{i}.up"] = lin(cfg.intermediate_size, H)
            w[f"l{i}.down"] = lin(H, cfg.intermediate_size)
    w["norm"] = norm(H)
    w["lm_head"] = w["embed"] if cfg.tie_embeddings else _normal((cfg.vocab_size, H), std, gen, dev, dtype)
    return w


def init_draft(cfg: DraftConfig, *, device="cpu", dtype=torch.float32, seed: int = 1,
               lm_head: Optional[torch.Tensor] = None, embed: Optional[torch.Tensor] = None) -> Dict[str, torch.Tensor]:
    """Random draft head in the runtime layout. ``lm_head`` / ``embed`` may be shared from the target (the draft's
    ``embed_tokens`` is optional in released checkpoints and taken from the target)."""
    dev = torch.device(device)
    gen = _generator(dev, seed)
    std = cfg.init_std
    H, Ht = cfg.hidden_size, cfg.target_hidden_size
    w: Dict[str, torch.Tensor] = {}

    def lin(n, k):
        return _normal((n, k), std, gen, dev, dtype)

    ones = lambda n: torch.ones(n, dtype=dtype, device=dev)  # noqa: E731
    if cfg.fc_norm:
        for j in range(cfg.num_aux):
            w[f"fc_norm.{j}"] = ones(Ht)
    w["fc"] = lin(H, cfg.num_aux * Ht)
    w["embed"] = embed if embed is not None else _normal((cfg.vocab_size, H), std, gen, dev, dtype)
    w["input_layernorm"] = ones(H)
    w["hidden_norm"] = ones(H)
    qkv_rows = (cfg.num_heads + 2 * cfg.num_kv_heads) * cfg.head_dim
    if cfg.attn_norm:
        w["eh_proj"] = lin(H, 2 * H)
        w["pre_attention_layernorm"] = ones(H)
    w["qkv"] = lin(qkv_rows, H if cfg.attn_norm else 2 * H)
    w["o_proj"] = lin(H, cfg.num_heads * cfg.head_dim)
    w["post_attention_layernorm"] = ones(H)
    if cfg.moe:
        m = cfg.moe
        E, L, F = m["experts"], m["latent"], m["inter"]
        w["moe_gate"] = _normal((E, H), std, gen, dev, torch.float32)
        w["moe_bias"] = _normal((E,), std, gen, dev, torch.float32)
        w["fc1_latent"] = lin(L, H)
        w["fc2_latent"] = lin(H, L)
        w["experts_up"] = _normal((E, F, L), std, gen, dev, dtype)
        w["experts_down"] = _normal((E, L, F), std, gen, dev, dtype)
        if m.get("shared_inter"):
            w["shared_up"] = lin(m["shared_inter"], H)
            w["shared_down"] = lin(H, m["shared_inter"])
    else:
        w["gate_up"] = lin(2 * cfg.intermediate_size, H)
        w["down"] = lin(H, cfg.intermediate_size)
    w["norm"] = ones(H)
    if lm_head is not None and cfg.draft_vocab_size == lm_head.shape[0]:
        w["lm_head"] = lm_head
    else:
        w["lm_head"] = _normal((cfg.draft_vocab_size, H), std, gen, dev, dtype)
    if cfg.draft_vocab_size != cfg.vocab_size:
        # d2t: draft id -> target id (the first draft_vocab_size target ids, strided over the vocabulary)
        stride = cfg.vocab_size // cfg.draft_vocab_size
        w["d2t"] = (torch.arange(cfg.draft_vocab_size, device=dev) * stride).long()
    if cfg.low_rank and dev.type == "meta":
        w["lr_down"] = torch.empty(cfg.rank, H, device=dev, dtype=dtype)
        w["lr_scores"] = torch.empty(cfg.draft_vocab_size, cfg.rank, device=dev, dtype=dtype)
    elif cfg.low_rank:
        down, scores = low_rank_factors(w["lm_head"], cfg.rank, seed=seed)
        w["lr_down"] = down.to(dtype)
        w["lr_scores"] = scores.to(dtype)
    return w


def low_rank_factors(lm_head: torch.Tensor, rank: int, *, seed: int = 0,
                     token_freq: Optional[torch.Tensor] = None):
    """Rank-``r`` factors of the LM head: ``down [r, H]`` and ``scores [V, r]`` with ``scores @ down ~= lm_head``.

    A randomized SVD (Halko et al. 2011) of the optionally frequency-weighted head; the weighting scales rows by
    ``sqrt(freq)`` before the factorisation and divides it out of ``scores`` afterwards.
    (``eagle_harness/models/low_rank_head.py:67-102`` defines the same factor shapes.)
    """
    w = lm_head.float()
    if token_freq is not None:
        sw = token_freq.float().clamp(min=1e-12).sqrt()[:, None].to(w.device)
        w = w * sw
    torch.manual_seed(seed)
    u, s, v = torch.svd_lowrank(w, q=rank, niter=2)
    scores = u * s[None, :]
    down = v.t().contiguous()
    if token_freq is not None:
        scores = scores / sw
    return down, scores


# ------------------------------------------------------------------------------------------ checkpoints
def _strip(name: str) -> str:
    for p in ("model.",):
        if name.startswith(p):
            name = name[len(p):]
    if name.startswith("midlayer."):
        name = "layers.0." + name[len("midlayer."):]
    if name == "fc.linear.weight":
        name = "fc.weight"
    return name


def draft_state_dict(cfg: DraftConfig, w: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Runtime draft weights in the released safetensors names."""
    H = cfg.hidden_size
    qd, kd = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
    sd = {
        "fc.weight": w["fc"],
        "layers.0.input_layernorm.weight": w["input_layernorm"],
        "layers.0.hidden_norm.weight": w["hidden_norm"],
        "layers.0.self_attn.q_proj.weight": w["qkv"][:qd],
        "layers.0.self_attn.k_proj.weight": w["qkv"][qd: qd + kd],
        "layers.0.self_attn.v_proj.weight": w["qkv"][qd + kd:],
        "layers.0.self_attn.o_proj.weight": w["o_proj"],
        "layers.0.post_attention_layernorm.weight": w["post_attention_layernorm"],
        "norm.weight": w["norm"],
        "lm_head.weight": w["lm_head"],
    }
    if cfg.attn_norm:
        sd["layers.0.eh_proj.weight"] = w["eh_proj"]
        sd["layers.0.pre_attention_layernorm.weight"] = w["pre_attention_layernorm"]
    if cfg.moe:
        p = "layers.0.mlp."
        sd.update({p + "gate.weight": w["moe_gate"], p + "gate.e_score_correction_bias": w["moe_bias"],
                   p + "fc1_latent_proj.weight": w["fc1_latent"], p + "fc2_latent_proj.weight": w["fc2_latent"]})
        for e in range(cfg.moe["experts"]):
            sd[f"{p}experts.{e}.up_proj.weight"] = w["experts_up"][e]
            sd[f"{p}experts.{e}.down_proj.weight"] = w["experts_down"][e]
        if "shared_up" in w:
            sd[p + "shared_experts.up_proj.weight"] = w["shared_up"]
            sd[p + "shared_experts.down_proj.weight"] = w["shared_down"]
    else:
        F = cfg.intermediate_size
        gu = w["gate_up"].view(F // 64, 2, 64, H)
        sd["layers.0.mlp.gate_proj.weight"] = gu[:, 0].reshape(F, H)
        sd["layers.0.mlp.up_proj.weight"] = gu[:, 1].reshape(F, H)
        sd["layers.0.mlp.down_proj.weight"] = w["down"]
    for j in range(cfg.num_aux):
        if f"fc_norm.{j}" in w:
            sd[f"fc_norm.{j}.weight"] = w[f"fc_norm.{j}"]
    if "lr_down" in w:
        sd["efficient_lm_head.weight"] = w["lr_scores"]
        sd["efficient_lm_head_down_proj.weight"] = w["lr_down"]
    if "d2t" in w:
        sd["d2t"] = w["d2t"] - torch.arange(w["d2t"].numel(), device=w["d2t"].device)  # stored as offsets
    return {k: v.contiguous() for k, v in sd.items()}


def draft_from_state_dict(cfg: DraftConfig, sd: Dict[str, torch.Tensor], *, embed: Optional[torch.Tensor] = None
                          ) -> Dict[str, torch.Tensor]:
    """Runtime draft weights from checkpoint tensors (names normalised; factors rebuilt by SVD when missing)."""
    sd = {_strip(k): v for k, v in sd.items()}
    g = lambda n: sd[n]  # noqa: E731
    w: Dict[str, torch.Tensor] = {
        "fc": g("fc.weight"),
        "input_layernorm": g("layers.0.input_layernorm.weight"),
        "hidden_norm": g("layers.0.hidden_norm.weight"),
        "qkv": torch.cat([g("layers.0.self_attn.q_proj.weight"), g("layers.0.self_attn.k_proj.weight"),
                          g("layers.0.self_attn.v_proj.weight")]),
        "o_proj": g("layers.0.self_attn.o_proj.weight"),
        "post_attention_layernorm": g("layers.0.post_attention_layernorm.weight"),
        "norm": g("norm.weight"),
        "lm_head": g("lm_head.weight"),
    }
    if cfg.attn_norm:
        w["eh_proj"] = g("layers.0.eh_proj.weight")
        w["pre_attention_layernorm"] = g("layers.0.pre_attention_layernorm.weight")
    if cfg.moe:
        p = "layers.0.mlp."
        E = cfg.moe["experts"]
        w["moe_gate"] = g(p + "gate.weight").float()
        w["moe_bias"] = g(p + "gate.e_score_correction_bias").float()
        w["fc1_latent"] = g(p + "fc1_latent_proj.weight")
        w["fc2_latent"] = g(p + "fc2_latent_proj.weight")
        w["experts_up"] = torch.stack([g(f"{p}experts.{e}.up_proj.weight") for e in range(E)])
        w["experts_down"] = torch.stack([g(f"{p}experts.{e}.down_proj.weight") for e in range(E)])
        if p + "shared_experts.up_proj.weight" in sd:
            w["shared_up"] = g(p + "shared_experts.up_proj.weight")
            w["shared_down"] = g(p + "shared_experts.down_proj.weight")
    else:
        w["gate_up"] = interleave_gate_up(g("layers.0.mlp.gate_proj.weight"), g("layers.0.mlp.up_proj.weight"))
        w["down"] = g("layers.0.mlp.down_proj.weight")
    for j in range(cfg.num_aux):
        if f"fc_norm.{j}.weight" in sd:
            w[f"fc_norm.{j}"] = sd[f"fc_norm.{j}.weight"]
    if "embed_tokens.weight" in sd:
        w["embed"] = sd["embed_tokens.weight"]
    elif embed is not None:
        w["embed"] = embed
    else:
        raise ValueError("draft checkpoint has no embed_tokens.weight and no target embedding was given")
    if cfg.low_rank:
        if "efficient_lm_head.weight" in sd and "efficient_lm_head_down_proj.weight" in sd:
            w["lr_scores"] = sd["efficient_lm_head.weight"]
            w["lr_down"] = sd["efficient_lm_head_down_proj.weight"]
        else:
            down, scores = low_rank_factors(w["lm_head"], cfg.rank)
            w["lr_down"] = down.to(w["lm_head"].dtype)
            w["lr_scores"] = scores.to(w["lm_head"].dtype)
    if "d2t" in sd:
        d = sd["d2t"].long()
        w["d2t"] = d + torch.arange(d.numel(), device=d.device)
    return w


def save_draft(path: str, cfg: DraftConfig, w: Dict[str, torch.Tensor]) -> None:
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    save_file({k: v.cpu() for k, v in draft_state_dict(cfg, w).items()}, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w", encoding="utf-8") as f:
        json.dump(cfg.to_hf(), f, indent=2)


def load_draft(path: str, cfg: DraftConfig, *, device="cpu", dtype=None, embed=None) -> Dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    sd: Dict[str, torch.Tensor] = {}
    for name in sorted(os.listdir(path)):
        if name.endswith(".safetensors"):
            sd.update(load_file(os.path.join(path, name), device=str(device)))
    if dtype is not None:
        sd = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in sd.items()}
    return draft_from_state_dict(cfg, sd, embed=embed)


def target_from_hf(cfg: TargetConfig, sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Map a Hugging Face Qwen3.5 / Llama / Nemotron-H state dict into the fused runtime layout."""
    if cfg.family == "nemotron_h":
        return _nemotron_from_hf(cfg, sd)
    sd = {k.replace("model.language_model.", "model."): v for k, v in sd.items()}
    g = lambda n: sd[n]  # noqa: E731
    w: Dict[str, torch.Tensor] = {"embed": g("model.embed_tokens.weight"), "norm": g("model.norm.weight")}
    w["lm_head"] = sd.get("lm_head.weight", w["embed"])
    for i, (mixer, mlp) in enumerate(cfg.layers):
        p = f"model.layers.{i}."
        if mixer is not None:
            w[f"l{i}.norm1"] = g(p + "input_layernorm.weight")
        if mixer == "attn":
            q = g(p + "self_attn.q_proj.weight")
            if cfg.attn_output_gate:
                qv = q.view(cfg.num_heads, 2, cfg.head_dim, -1)
                q = torch.cat([qv[:, 0].reshape(-1, q.shape[-1]), qv[:, 1].reshape(-1, q.shape[-1])])
            w[f"l{i}.qkv"] = torch.cat([q, g(p + "self_attn.k_proj.weight"), g(p + "self_attn.v_proj.weight")])
            if cfg.qk_norm:
                w[f"l{i}.q_norm"] = g(p + "self_attn.q_norm.weight")
                w[f"l{i}.k_norm"] = g(p + "self_attn.k_norm.weight")
            w[f"l{i}.o_proj"] = g(p + "self_attn.o_proj.weight")
        elif mixer == "gdn":
            la = p + "linear_attn."
            w[f"l{i}.in_proj"] = torch.cat([g(la + "in_proj_qkv.weight"), g(la + "in_proj_z.weight"),
                                            g(la + "in_proj_b.weight"), g(la + "in_proj_a.weight")])
            w[f"l{i}.conv"] = g(la + "conv1d.weight").squeeze(1)
            w[f"l{i}.A_log"] = g(la + "A_log").float()
            w[f"l{i}.dt_bias"] = g(la + "dt_bias").float()
            w[f"l{i}.gnorm"] = g(la + "norm.weight")
            w[f"l{i}.out_proj"] = g(la + "out_proj.weight")
        if mlp == "swiglu":
            w[f"l{i}.norm2"] = g(p + "post_attention_layernorm.weight")
            w[f"l{i}.gate_up"] = interleave_gate_up(g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight"))
            w[f"l{i}.down"] = g(p + "mlp.down_proj.weight")
    return w


def _nemotron_from_hf(cfg: TargetConfig, sd: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Nemotron-H: one mixer per block (Mamba2 ``M``, attention ``*``, ReLU^2 MLP ``-``) behind the block's RMSNorm.
    The Mamba2 in_proj rows are already ``[z | x B C | dt]``; the conv bias and the gated norm's per-channel weight
    (one row per group) are kept. Checkpoints name the trunk ``backbone.`` (``model.`` after conversion)."""
    sd = {k.replace("backbone.", "model.").replace("model.embedding.", "model.embeddings."): v for k, v in sd.items()}
    g = lambda n: sd[n]  # noqa: E731
    w: Dict[str, torch.Tensor] = {"embed": g("model.embeddings.weight"), "norm": g("model.norm_f.weight")}
    w["lm_head"] = sd.get("lm_head.weight", w["embed"])
    for i, (mixer, mlp) in enumerate(cfg.layers):
        p = f"model.layers.{i}."
        m = p + "mixer."
        if mixer is not None:
            w[f"l{i}.norm1"] = g(p + "norm.weight")
        if mixer == "mamba":
            w[f"l{i}.in_proj"] = g(m + "in_proj.weight")
            w[f"l{i}.conv"] = g(m + "conv1d.weight").squeeze(1)
            if m + "conv1d.bias" in sd:
                w[f"l{i}.conv_bias"] = g(m + "conv1d.bias")
            w[f"l{i}.A_log"] = g(m + "A_log").float()
            w[f"l{i}.D"] = g(m + "D").float()
            w[f"l{i}.dt_bias"] = g(m + "dt_bias").float()
            w[f"l{i}.gnorm"] = g(m + "norm.weight")
            w[f"l{i}.out_proj"] = g(m + "out_proj.weight")
        elif mixer == "attn":
            w[f"l{i}.qkv"] = torch.cat([g(m + "q_proj.weight"), g(m + "k_proj.weight"), g(m + "v_proj.weight")])
            w[f"l{i}.o_proj"] = g(m + "o_proj.weight")
        elif mixer is not None:
            raise ValueError(f"Nemotron-H layer {i}: mixer {mixer!r} is not built")
        if mlp == "relu2":
            w[f"l{i}.norm2"] = g(p + "norm.weight")
            w[f"l{i}.up"] = g(m + "up_proj.weight")
            w[f"l{i}.down"] = g(m + "down_proj.weight")
        elif mlp is not None:
            raise ValueError(f"Nemotron-H layer {i}: MLP {mlp!r} is not built")
    return w
