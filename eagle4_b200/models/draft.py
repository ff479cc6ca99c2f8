"""EAGLE-4 (and EAGLE-3) one-layer draft head.

Forward of a set of draft rows, as the reference's SGLang port defines it
(``eagle_harness/sglang/models/llama_eagle4.py:166-336``):

1. target features: ``fc_norm_j`` on each of the aux hidden states, concatenated, through ``fc`` (``n*H_t -> H``);
   rows that already carry a draft hidden state skip this;
2. ``qkv(cat(input_layernorm(embed), hidden_norm(hidden)))`` (``2H`` in), RoPE, attention over the draft KV (the
   frozen committed window plus the row's tree ancestors);
3. ``residual = hidden + o_proj(attn)``; ``summed = residual + down(swiglu(gate_up(post_norm(residual))))``;
4. ``normed = norm(summed)`` feeds the head; the next step's hidden is ``normed`` when ``norm_output`` else ``summed``.

Candidate head (EAGLE-4): low-rank scores ``(h @ down^T) @ scores^T`` select the top ``C`` ids; their exact logits
``lm_head[id] . h`` in fp32 feed a softmax over the ``C`` candidates (equal to the full-vocabulary softmax of the
-inf-filled row); the top ``K`` of it are the children. EAGLE-3: full draft-vocabulary softmax and a ``d2t`` map.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, Optional, Tuple

import torch

from eagle4_b200 import ops
from eagle4_b200.models.configs import DraftConfig


@dataclass
class DraftCache:
    block_table: torch.Tensor
    page: int
    k: torch.Tensor  # [slots, Hkv, D]
    v: torch.Tensor

    @classmethod
    def allocate(cls, cfg: DraftConfig, block_table: torch.Tensor, page: int, device, dtype,
                 pages: Optional[int] = None) -> "DraftCache":
        """Draft KV for the target's block table: ``pages`` physical pages (default: one per table entry)."""
        slots = (block_table.numel() if pages is None else pages) * page
        k = torch.zeros(slots, cfg.num_kv_heads, cfg.head_dim, dtype=dtype, device=device)
        return cls(block_table, page, k, torch.zeros_like(k))


class _AttnShape:
    """The attention fields ``ops.qkv_prepare`` reads, for the draft layer."""

    def __init__(self, cfg: DraftConfig):
        self.num_heads = cfg.num_heads
        self.num_kv_heads = cfg.num_kv_heads
        self.head_dim = cfg.head_dim
        self.attn_output_gate = False
        self.rms_norm_eps = cfg.rms_norm_eps
        self.norm_offset = False
        self.rotary_dim = cfg.head_dim if cfg.use_rope else 0
        self.rope_theta = cfg.rope_theta


class DraftModel:
    def __init__(self, cfg: DraftConfig, weights: Dict[str, torch.Tensor], *, tp=None):
        """``cfg`` / ``weights``: this rank's shard under tensor parallelism (``tp``; the head is replicated)."""
        self.cfg = cfg
        self.w = weights
        self.tp = tp
        self.attn_shape = _AttnShape(cfg)
        self.device = weights["fc"].device

    def project(self, aux: torch.Tensor) -> torch.Tensor:
        """Target aux hidden states ``[T, n*H_t]`` -> draft hidden ``[T, H]``."""
        cfg, w = self.cfg, self.w
        if cfg.fc_norm:
            ht = cfg.target_hidden_size
            parts = [ops.rmsnorm(aux[:, j * ht:(j + 1) * ht], w[f"fc_norm.{j}"], cfg.rms_norm_eps, False)
                     for j in range(cfg.num_aux)]
            aux = torch.cat(parts, dim=-1)
        return ops.linear(aux, w["fc"])

    def forward(self, ids: torch.Tensor, hidden: torch.Tensor, pos: torch.Tensor, req: torch.Tensor,
                write_slot: torch.Tensor, ctx_start: torch.Tensor, ctx_len: torch.Tensor, extra: torch.Tensor,
                n_extra: torch.Tensor, cache: DraftCache, max_keys: Optional[int] = None
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Returns ``(normed [T, H], next hidden [T, H])``."""
        x, res = self.layer_input(ids, hidden)
        qkv = ops.linear(x, self.w["qkv"])
        q, _ = ops.qkv_prepare(qkv, self.attn_shape, pos, write_slot, cache.k, cache.v, None, None)
        o = ops.attention(q, cache.k, cache.v, cache.block_table, cache.page, req, ctx_start, ctx_len, extra,
                          n_extra, self.cfg.head_dim ** -0.5, max_keys)
        return self.layer_output(o, res)

    def write_kv(self, ids: torch.Tensor, hidden: torch.Tensor, pos: torch.Tensor, write_slot: torch.Tensor,
                 cache: DraftCache) -> None:
        """Only the rows' draft KV: the layer input, the q/k/v projection and the rotated k and v written to
        ``write_slot``, without the attention, the MLP or the head. A single-layer draft's KV at a position depends
        on that position's input alone, so the KV equals what ``forward`` writes; rows whose outputs are never read
        (a prompt's leading rows) need nothing else. Reference counterpart: ``kv_only_prefill``
        (``eagle_harness/sglang/draft_kv.py:39``)."""
        x, _ = self.layer_input(ids, hidden)
        qkv = ops.linear(x, self.w["qkv"])
        ops.qkv_prepare(qkv, self.attn_shape, pos, write_slot, cache.k, cache.v, None, None)

    def forward_rows(self, ids: torch.Tensor, pos: torch.Tensor, hidden: torch.Tensor,
                     attend: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
        """``forward`` with the host's attention: ``attend(q, k, v)`` gets the rows' rotated ``q [T, Hq, D]``, rotated
        ``k`` and ``v [T, Hkv, D]`` (the host writes them into its own KV cache and attends) and returns
        ``[T, Hq, D]``. Returns ``(normed, next hidden)`` like ``forward``."""
        cfg = self.cfg
        x, res = self.layer_input(ids, hidden)
        qkv = ops.linear(x, self.w["qkv"])
        t = qkv.shape[0]
        # RoPE goes through the same kernel as the engine's rows: it writes the rotated k and the v of row i to slot i
        k = torch.empty(t, cfg.num_kv_heads, cfg.head_dim, dtype=qkv.dtype, device=qkv.device)
        v = torch.empty_like(k)
        slots = torch.arange(t, device=qkv.device)
        q, _ = ops.qkv_prepare(qkv, self.attn_shape, pos, slots, k, v, None, None)
        return self.layer_output(attend(q, k, v).reshape(t, -1), res)

    def layer_input(self, ids: torch.Tensor, hidden: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """``(q/k/v projection input, attention residual)`` of the draft layer for token ids and hidden rows."""
        cfg, w = self.cfg, self.w
        eps = cfg.rms_norm_eps
        e = ops.embedding(ids, w["embed"])
        x = ops.concat_norms(e, hidden, w["input_layernorm"], w["hidden_norm"], eps)
        res = hidden
        if cfg.attn_norm:  # eh_proj input fusion: the projection is the attention residual, its norm feeds q/k/v
            res = ops.linear(x, w["eh_proj"])
            x = ops.rmsnorm(res, w["pre_attention_layernorm"], eps, False)
        return x, res

    def layer_output(self, o: torch.Tensor, res: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Attention output ``[T, Hq, D]`` and residual -> ``(normed, next hidden)``: o_proj, MLP (dense or latent
        MoE), final norm."""
        cfg, w = self.cfg, self.w
        eps = cfg.rms_norm_eps
        if self.tp is not None:
            residual, x = self.tp.row_linear(o, w["o_proj"], res, w["post_attention_layernorm"], eps)
            if cfg.moe:  # the MoE is replicated on every rank: no collective after it
                summed = ops.latent_moe(x, w, cfg.moe, residual)
                normed = ops.rmsnorm(summed, w["norm"], eps, False)
            else:
                summed, normed = self.tp.row_linear(ops.linear_swiglu(x, w["gate_up"]), w["down"], residual,
                                                    w["norm"], eps)
        else:
            residual = ops.linear_residual(o, w["o_proj"], res)
            x = ops.rmsnorm(residual, w["post_attention_layernorm"], eps, False)
            if cfg.moe:
                summed = ops.latent_moe(x, w, cfg.moe, residual)
            else:
                summed = ops.linear_residual(ops.linear_swiglu(x, w["gate_up"]), w["down"], residual)
            normed = ops.rmsnorm(summed, w["norm"], eps, False)
        return normed, (normed if cfg.norm_output else summed)

    def candidates(self, normed: torch.Tensor, k: int, pos: Optional[torch.Tensor] = None
                   ) -> Tuple[torch.Tensor, torch.Tensor]:
        """Top-``k`` children per row: ``(probs fp32 [T, k], target token ids int64 [T, k])``. ``pos`` (the rows'
        positions) is unused by the learned head; position-aware proposers that replace this method read it."""
        cfg, w = self.cfg, self.w
        if cfg.low_rank:
            probs, ids = ops.candidate_head(normed, w["lr_down"], w["lr_scores"], w["lm_head"],
                                            cfg.num_candidates, k)
        else:
            probs, ids = ops.full_head_topk(normed, w["lm_head"], k)
        if "d2t" in w:
            ids = w["d2t"][ids]
        return probs, ids

    def candidate_logits(self, normed: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Candidate ids and their exact fp32 logits (the distribution sampled trees draw from)."""
        cfg, w = self.cfg, self.w
        if cfg.low_rank:
            ids, logit = ops.candidate_logits(normed, w["lr_down"], w["lr_scores"], w["lm_head"], cfg.num_candidates)
        else:
            logit = ops.logits(normed, w["lm_head"])
            ids = torch.arange(logit.shape[1], device=logit.device).expand_as(logit)
        if "d2t" in w:
            ids = w["d2t"][ids]
        return ids, logit
