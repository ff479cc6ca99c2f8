"""Model shapes: target families (Qwen3.5-style GDN hybrid, Nemotron-H-style Mamba2 hybrid, dense Llama) and
draft heads (EAGLE-4, EAGLE-3), plus the named configurations the benchmarks use.

A target is a list of layers; each layer has a token mixer (``gdn``, ``attn``, ``mamba`` or none) and a channel
mixer (``swiglu``, ``relu2`` or none), each behind a pre-norm with a residual add. That one description covers:

* Qwen3.5 hybrids (every layer ``mixer + swiglu``; 3 GDN : 1 gated attention), as in
  ``eagle_harness/core/profiles/mi355x-qwen3.8-27b-tp1/target_config.json``;
* Nemotron-H (every layer a single block: Mamba2, attention or a squared-ReLU MLP);
* Llama (every layer ``attn + swiglu``).
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from typing import List, Optional, Tuple


@dataclass
class TargetConfig:
    family: str  # "qwen3_5" | "qwen3" | "nemotron_h" | "llama"
    hidden_size: int
    vocab_size: int
    layers: List[Tuple[Optional[str], Optional[str]]]  # (mixer, mlp) per layer
    intermediate_size: int
    rms_norm_eps: float = 1e-6
    norm_offset: bool = False  # Qwen3.5 norms scale by (1 + w)
    # attention
    num_heads: int = 0
    num_kv_heads: int = 0
    head_dim: int = 0
    attn_output_gate: bool = False
    qk_norm: bool = False
    rotary_dim: int = 0
    rope_theta: float = 10000.0
    # gated delta net
    gdn_k_heads: int = 0
    gdn_v_heads: int = 0
    gdn_k_dim: int = 0
    gdn_v_dim: int = 0
    conv_kernel: int = 4
    # mamba2
    mamba_heads: int = 0
    mamba_head_dim: int = 0
    mamba_state: int = 0
    mamba_groups: int = 1
    # Mamba2 gated norm: rmsnorm(y * silu(z)) * w as Hugging Face's Nemotron-H computes it (True), or
    # rmsnorm(y) * w * silu(z) (False: the synthetic Nemotron-H-style shapes)
    mamba_gate_first: bool = False
    tie_embeddings: bool = False
    init_std: float = 0.02

    @property
    def num_layers(self) -> int:
        return len(self.layers)

    def layer_ids(self, mixer: str) -> List[int]:
        return [i for i, (m, _) in enumerate(self.layers) if m == mixer]

    @property
    def gdn_key_dim(self) -> int:
        return self.gdn_k_heads * self.gdn_k_dim

    @property
    def gdn_value_dim(self) -> int:
        return self.gdn_v_heads * self.gdn_v_dim

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.gdn_key_dim + self.gdn_value_dim

    @property
    def mamba_inner(self) -> int:
        return self.mamba_heads * self.mamba_head_dim

    @property
    def mamba_conv_dim(self) -> int:
        return self.mamba_inner + 2 * self.mamba_groups * self.mamba_state

    @property
    def is_moe(self) -> bool:
        return False

    def to_json(self) -> str:
        return json.dumps(asdict(self), indent=2)

    @classmethod
    def from_dict(cls, d: dict) -> "TargetConfig":
        d = dict(d)
        d["layers"] = [tuple(x) for x in d["layers"]]
        return cls(**d)

    @classmethod
    def from_hf(cls, hf: dict) -> "TargetConfig":
        """Map a Hugging Face ``config.json`` (Qwen3.5 text config, dense Qwen3, Nemotron-H, Llama). Mixture-of-experts
        targets are refused (not built)."""
        text = hf.get("text_config", hf)
        mt = text.get("model_type", "")
        experts = text.get("num_experts") or text.get("n_routed_experts")
        if "moe" in mt or (experts and mt != "nemotron_h"):  # Nemotron-H names its MoE blocks in the layer pattern
            raise NotImplementedError(f"mixture-of-experts targets ({mt}) are not built by eagle4_b200's own engine; "
                                      "serve them through a host plugin")
        if mt == "qwen3":  # dense Qwen3: attention with q/k norms, full rotary, plain RMSNorm weights
            hd = text.get("head_dim") or text["hidden_size"] // text["num_attention_heads"]
            rope = text.get("rope_parameters", {}) or {}
            return cls(
                family="qwen3", hidden_size=text["hidden_size"], vocab_size=text["vocab_size"],
                layers=[("attn", "swiglu")] * text["num_hidden_layers"], intermediate_size=text["intermediate_size"],
                rms_norm_eps=text.get("rms_norm_eps", 1e-6), num_heads=text["num_attention_heads"],
                num_kv_heads=text["num_key_value_heads"], head_dim=hd, qk_norm=True, rotary_dim=hd,
                rope_theta=rope.get("rope_theta", text.get("rope_theta", 1e6)),
                tie_embeddings=bool(text.get("tie_word_embeddings")),
            )
        if mt.startswith("qwen3"):
            types = text["layer_types"]
            layers = [("gdn" if t == "linear_attention" else "attn", "swiglu") for t in types]
            rope = text.get("rope_parameters", {}) or {}
            prf = rope.get("partial_rotary_factor", text.get("partial_rotary_factor", 1.0))
            return cls(
                family="qwen3_5", hidden_size=text["hidden_size"], vocab_size=text["vocab_size"], layers=layers,
                intermediate_size=text["intermediate_size"], rms_norm_eps=text.get("rms_norm_eps", 1e-6),
                norm_offset=True, num_heads=text["num_attention_heads"], num_kv_heads=text["num_key_value_heads"],
                head_dim=text["head_dim"], attn_output_gate=bool(text.get("attn_output_gate", True)), qk_norm=True,
                rotary_dim=int(text["head_dim"] * prf), rope_theta=rope.get("rope_theta", text.get("rope_theta", 1e7)),
                gdn_k_heads=text["linear_num_key_heads"], gdn_v_heads=text["linear_num_value_heads"],
                gdn_k_dim=text["linear_key_head_dim"], gdn_v_dim=text["linear_value_head_dim"],
                conv_kernel=text.get("linear_conv_kernel_dim", 4), tie_embeddings=bool(hf.get("tie_word_embeddings")),
            )
        if mt == "nemotron_h":
            kind = {"M": ("mamba", None), "*": ("attn", None), "-": (None, "relu2"),
                    "mamba": ("mamba", None), "attention": ("attn", None), "mlp": (None, "relu2")}
            blocks = text.get("hybrid_override_pattern") or text.get("layers_block_type") or []
            unbuilt = sorted({str(b) for b in blocks if b not in kind})
            if unbuilt:
                raise NotImplementedError(f"Nemotron-H blocks {unbuilt} are not built (Mamba2, attention and ReLU^2 "
                                          "MLP blocks are)")
            return cls(
                family="nemotron_h", hidden_size=text["hidden_size"], vocab_size=text["vocab_size"],
                layers=[kind[c] for c in blocks], intermediate_size=text["intermediate_size"],
                mamba_gate_first=bool(text.get("mamba_gate_first", True)),
                tie_embeddings=bool(text.get("tie_word_embeddings")),
                rms_norm_eps=text.get("layer_norm_epsilon", 1e-5), num_heads=text["num_attention_heads"],
                num_kv_heads=text["num_key_value_heads"], head_dim=text.get("head_dim") or
                text["hidden_size"] // text["num_attention_heads"], rotary_dim=0,
                mamba_heads=text["mamba_num_heads"], mamba_head_dim=text["mamba_head_dim"],
                mamba_state=text["ssm_state_size"], mamba_groups=text.get("n_groups", 8),
                conv_kernel=text.get("conv_kernel", 4),
            )
        if mt == "llama":
            hd = text.get("head_dim") or text["hidden_size"] // text["num_attention_heads"]
            return cls(
                family="llama", hidden_size=text["hidden_size"], vocab_size=text["vocab_size"],
                layers=[("attn", "swiglu")] * text["num_hidden_layers"], intermediate_size=text["intermediate_size"],
                rms_norm_eps=text.get("rms_norm_eps", 1e-5), num_heads=text["num_attention_heads"],
                num_kv_heads=text["num_key_value_heads"], head_dim=hd, rotary_dim=hd,
                rope_theta=text.get("rope_theta", 500000.0), tie_embeddings=bool(text.get("tie_word_embeddings")),
            )
        raise ValueError(f"unsupported target model_type {mt!r}")

    def to_hf(self) -> dict:
        """A Hugging Face style ``config.json`` of this shape (the inverse of :meth:`from_hf`)."""
        common = {"hidden_size": self.hidden_size, "vocab_size": self.vocab_size,
                  "num_hidden_layers": self.num_layers, "intermediate_size": self.intermediate_size,
                  "num_attention_heads": self.num_heads, "num_key_value_heads": self.num_kv_heads,
                  "head_dim": self.head_dim, "tie_word_embeddings": self.tie_embeddings}
        if self.family == "qwen3_5":
            return dict(common, model_type="qwen3_5_text", architectures=["Qwen3_5ForCausalLM"],
                        rms_norm_eps=self.rms_norm_eps, attn_output_gate=self.attn_output_gate,
                        layer_types=["linear_attention" if m == "gdn" else "full_attention" for m, _ in self.layers],
                        linear_num_key_heads=self.gdn_k_heads, linear_num_value_heads=self.gdn_v_heads,
                        linear_key_head_dim=self.gdn_k_dim, linear_value_head_dim=self.gdn_v_dim,
                        linear_conv_kernel_dim=self.conv_kernel,
                        rope_parameters={"rope_theta": self.rope_theta,
                                         "partial_rotary_factor": self.rotary_dim / self.head_dim})
        if self.family == "qwen3":
            return dict(common, model_type="qwen3", architectures=["Qwen3ForCausalLM"], rms_norm_eps=self.rms_norm_eps,
                        rope_theta=self.rope_theta)
        if self.family == "nemotron_h":
            sym = {("mamba", None): "M", ("attn", None): "*", (None, "relu2"): "-"}
            return dict(common, model_type="nemotron_h", architectures=["NemotronHForCausalLM"],
                        layer_norm_epsilon=self.rms_norm_eps,
                        hybrid_override_pattern="".join(sym[tuple(x)] for x in self.layers),
                        mamba_num_heads=self.mamba_heads, mamba_head_dim=self.mamba_head_dim,
                        ssm_state_size=self.mamba_state, n_groups=self.mamba_groups, conv_kernel=self.conv_kernel,
                        mamba_gate_first=self.mamba_gate_first)
        return dict(common, model_type="llama", architectures=["LlamaForCausalLM"], rms_norm_eps=self.rms_norm_eps,
                    rope_theta=self.rope_theta)


@dataclass
class DraftConfig:
    """One-layer EAGLE-4 / EAGLE-3 draft head."""

    family: str  # "eagle4" | "eagle3"
    hidden_size: int
    target_hidden_size: int
    vocab_size: int  # target vocabulary (ids the draft emits)
    draft_vocab_size: int  # rows of the draft LM head (< vocab_size means a d2t map)
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    aux_layer_ids: Tuple[int, ...]
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e7
    sliding_window: Optional[int] = 4096
    fc_norm: bool = True
    norm_output: bool = True
    use_rope: bool = True
    low_rank: Optional[dict] = None  # {"type": "low_rank", "rank": r, "num_candidates": c}
    init_std: float = 0.02
    # MTP-style input fusion: eh_proj maps concat(normed embed, normed hidden) to H; that projection is the
    # attention residual and its RMSNorm (pre_attention_layernorm) feeds q/k/v
    attn_norm: bool = False
    # latent ReLU^2 MoE MLP (Nemotron-H block): {"experts", "top_k", "inter", "latent", "shared_inter",
    # "n_group", "topk_group", "norm_topk_prob", "scale"}; None is the dense SwiGLU MLP
    moe: Optional[dict] = None

    @property
    def num_aux(self) -> int:
        return len(self.aux_layer_ids)

    @property
    def rank(self) -> int:
        return int(self.low_rank["rank"]) if self.low_rank else 0

    @property
    def num_candidates(self) -> int:
        return int(self.low_rank["num_candidates"]) if self.low_rank else 0

    def to_hf(self) -> dict:
        """The draft ``config.json`` in the released EAGLE-4 layout."""
        d = {
            "architectures": ["LlamaForCausalLMEagle4" if self.family == "eagle4" else "LlamaForCausalLMEagle3"],
            "model_type": "llama", "hidden_size": self.hidden_size, "target_hidden_size": self.target_hidden_size,
            "vocab_size": self.vocab_size, "draft_vocab_size": self.draft_vocab_size,
            "num_attention_heads": self.num_heads, "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim, "intermediate_size": self.intermediate_size, "num_hidden_layers": 1,
            "rms_norm_eps": self.rms_norm_eps, "rope_parameters": {"rope_theta": self.rope_theta,
                                                                   "rope_type": "default"},
            "eagle_config": {"eagle_aux_hidden_state_layer_ids": list(self.aux_layer_ids),
                             "use_aux_hidden_state": True},
            "num_aux_hidden_states": self.num_aux, "fc_norm": self.fc_norm, "norm_output": self.norm_output,
            "hidden_act": "silu", "tie_word_embeddings": False,
        }
        if self.sliding_window:
            d.update(sliding_window=self.sliding_window, use_sliding_window=True, layer_types=["sliding_attention"])
        else:
            d.update(use_sliding_window=False, layer_types=["full_attention"])
        if self.low_rank:
            d["efficient_lm_head_config"] = dict(self.low_rank)
        if self.attn_norm:
            d["attn_norm"] = True
        if self.moe:
            m = self.moe
            d.update(enable_moe=True, moe_architecture="nemotron_latent_relu2", hidden_act="relu2",
                     n_routed_experts=m["experts"], num_experts_per_tok=m["top_k"], moe_intermediate_size=m["inter"],
                     moe_latent_size=m["latent"], n_shared_experts=1 if m.get("shared_inter") else 0,
                     moe_shared_expert_intermediate_size=m.get("shared_inter") or None, n_group=m.get("n_group", 1),
                     topk_group=m.get("topk_group", 1), norm_topk_prob=bool(m.get("norm_topk_prob", True)),
                     routed_scaling_factor=float(m.get("scale", 1.0)), scoring_func="sigmoid",
                     topk_method="noaux_tc")
        return d


# ------------------------------------------------------------------------------------------------ named shapes
def qwen38_27b() -> TargetConfig:
    """Qwen3.8-27B-shaped hybrid: 64 layers, GDN:attention 3:1 (the packaged target config's dimensions)."""
    types = ["attn" if (i + 1) % 4 == 0 else "gdn" for i in range(64)]
    return TargetConfig(
        family="qwen3_5", hidden_size=5120, vocab_size=248320, layers=[(t, "swiglu") for t in types],
        intermediate_size=17408, norm_offset=True, num_heads=24, num_kv_heads=4, head_dim=256,
        attn_output_gate=True, qk_norm=True, rotary_dim=64, rope_theta=1e7, gdn_k_heads=16, gdn_v_heads=48,
        gdn_k_dim=128, gdn_v_dim=128, conv_kernel=4,
    )


def profile_slice(target: TargetConfig, mixers=("gdn", "attn")) -> TargetConfig:
    """A few layers of a target at its real widths (one per mixer kind, tied embeddings): every per-layer kernel runs
    at the production shapes while the weights stay a few GB (for profiler captures)."""
    import dataclasses

    layers = [next(l for l in target.layers if l[0] == m) for m in mixers]
    return dataclasses.replace(target, layers=layers, tie_embeddings=True)


def qwen38_draft(target: TargetConfig) -> DraftConfig:
    """The released EAGLE-4 draft shape for Qwen3.8-27B (H=5120, 40x128 heads, FFN 16384, window 4096)."""
    return DraftConfig(
        family="eagle4", hidden_size=5120, target_hidden_size=target.hidden_size, vocab_size=target.vocab_size,
        draft_vocab_size=target.vocab_size, num_heads=40, num_kv_heads=40, head_dim=128, intermediate_size=16384,
        aux_layer_ids=(3, 31, 59), sliding_window=4096, rope_theta=1e7,
        low_rank={"type": "low_rank", "rank": 128, "num_candidates": 128},
    )


def tiny_hybrid() -> TargetConfig:
    """The CPU plumbing target: 4 layers (3 GDN + 1 attention), hidden 256, vocab 4096."""
    return TargetConfig(
        family="qwen3_5", hidden_size=256, vocab_size=4096,
        layers=[("gdn", "swiglu"), ("gdn", "swiglu"), ("gdn", "swiglu"), ("attn", "swiglu")],
        intermediate_size=512, norm_offset=True, num_heads=4, num_kv_heads=2, head_dim=64, attn_output_gate=True,
        qk_norm=True, rotary_dim=16, rope_theta=1e7, gdn_k_heads=4, gdn_v_heads=4, gdn_k_dim=64, gdn_v_dim=64,
        conv_kernel=4,
    )


def tiny_draft(target: TargetConfig, draft_vocab: int = 1024) -> DraftConfig:
    return DraftConfig(
        family="eagle4", hidden_size=target.hidden_size, target_hidden_size=target.hidden_size,
        vocab_size=target.vocab_size, draft_vocab_size=draft_vocab, num_heads=4, num_kv_heads=4, head_dim=64,
        intermediate_size=512, aux_layer_ids=(1, 2, 3), sliding_window=None, rope_theta=1e7,
        low_rank={"type": "low_rank", "rank": 32, "num_candidates": 32},
    )


def latent_moe(experts: int, top_k: int, inter: int, latent: int, shared_inter: int, *, n_group: int = 1,
               topk_group: int = 1, norm_topk_prob: bool = True, scale: float = 1.0) -> dict:
    return {"experts": experts, "top_k": top_k, "inter": inter, "latent": latent, "shared_inter": shared_inter,
            "n_group": n_group, "topk_group": topk_group, "norm_topk_prob": norm_topk_prob, "scale": scale}


def tiny_moe_draft(target: TargetConfig) -> DraftConfig:
    """CPU-sized EAGLE-4 draft with both Nemotron draft structures: attn_norm input fusion and a latent ReLU^2 MoE
    (16 experts, 4 per token in 2 groups, latent 64, shared expert)."""
    import dataclasses

    return dataclasses.replace(tiny_draft(target), attn_norm=True,
                               moe=latent_moe(16, 4, 96, 64, 128, n_group=2, topk_group=2, scale=2.5))


def nemotron_moe_draft(target: TargetConfig) -> DraftConfig:
    """A Nemotron-class EAGLE-4 draft shape: attn_norm fusion and a latent ReLU^2 MoE MLP (512 experts, 22 per token,
    latent 1024, expert FFN 2688, shared expert 5376, routed scale 5)."""
    import dataclasses

    return dataclasses.replace(generic_draft(target), attn_norm=True,
                               moe=latent_moe(512, 22, 2688, 1024, 5376, scale=5.0))


def tiny_nemotron() -> TargetConfig:
    """A CPU-sized Nemotron-H-style hybrid: Mamba2 and squared-ReLU blocks with one attention layer (hidden 256,
    Mamba2 8 heads of 32 with state 16 in 2 groups, conv 4, vocab 4096): the Mamba2 tree-verify path in tests."""
    layers: List[Tuple[Optional[str], Optional[str]]] = [("mamba", None), (None, "relu2"), ("mamba", None),
                                                         ("attn", None), ("mamba", None), (None, "relu2")]
    return TargetConfig(
        family="nemotron_h", hidden_size=256, vocab_size=4096, layers=layers, intermediate_size=512,
        rms_norm_eps=1e-5, num_heads=4, num_kv_heads=2, head_dim=64, rotary_dim=0, mamba_heads=8,
        mamba_head_dim=32, mamba_state=16, mamba_groups=2, conv_kernel=4,
    )


def nemotron_h_8b() -> TargetConfig:
    """Nemotron-H-style: 52 layers of single blocks, attention at every 7th layer, Mamba2 128x64 heads, state 128."""
    layers: List[Tuple[Optional[str], Optional[str]]] = []
    for i in range(52):
        if i % 7 == 6:
            layers.append(("attn", None))
        elif i % 2 == 0:
            layers.append(("mamba", None))
        else:
            layers.append((None, "relu2"))
    return TargetConfig(
        family="nemotron_h", hidden_size=4096, vocab_size=131072, layers=layers, intermediate_size=21504,
        rms_norm_eps=1e-5, num_heads=32, num_kv_heads=8, head_dim=128, rotary_dim=0, mamba_heads=128,
        mamba_head_dim=64, mamba_state=128, mamba_groups=8, conv_kernel=4,
    )


def llama31_8b() -> TargetConfig:
    return TargetConfig(
        family="llama", hidden_size=4096, vocab_size=128256, layers=[("attn", "swiglu")] * 32,
        intermediate_size=14336, rms_norm_eps=1e-5, num_heads=32, num_kv_heads=8, head_dim=128, rotary_dim=128,
        rope_theta=500000.0,
    )


def eagle3_llama_draft(target: TargetConfig) -> DraftConfig:
    return DraftConfig(
        family="eagle3", hidden_size=target.hidden_size, target_hidden_size=target.hidden_size,
        vocab_size=target.vocab_size, draft_vocab_size=32000, num_heads=32, num_kv_heads=8, head_dim=128,
        intermediate_size=14336, aux_layer_ids=(2, target.num_layers // 2, target.num_layers - 3),
        sliding_window=None, rope_theta=500000.0, fc_norm=False, norm_output=False, low_rank=None,
    )


def generic_draft(target: TargetConfig, heads: int = 32, kv: int = 8, head_dim: int = 128,
                  ffn: Optional[int] = None) -> DraftConfig:
    n = target.num_layers
    return DraftConfig(
        family="eagle4", hidden_size=target.hidden_size, target_hidden_size=target.hidden_size,
        vocab_size=target.vocab_size, draft_vocab_size=target.vocab_size, num_heads=heads, num_kv_heads=kv,
        head_dim=head_dim, intermediate_size=ffn or target.intermediate_size,
        aux_layer_ids=(2, n // 2, n - 3), sliding_window=4096, rope_theta=1e7,
        low_rank={"type": "low_rank", "rank": 128, "num_candidates": 128},
    )
